"""Fused LM-head cross-entropy (nl_lce_fwd / nl_lce_bwd) vs the oracle.

Loss within 1e-3 absolute; dX / dW within 1e-2 of the
oracle normwise (max|err| / max|ref|), the oracle using the same bf16 GEMM
operands."""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import ops  # noqa: E402
from nlearn_b200.kernels import cross_entropy as CE  # noqa: E402
from nlearn_b200 import _lib  # noqa: E402

G = Path(__file__).resolve().parent / "golden"


def nrel(a, b):
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-12))


def run(X, W, t, dev, chunk=None):
    Xt = torch.from_numpy(X).to(dev).requires_grad_()
    Wt = torch.from_numpy(W).to(dev).requires_grad_()
    tt = torch.from_numpy(t).to(dev)
    if chunk:  # target vocabulary chunk of the backward (NLEARN_LCE_CHUNK)
        old = CE._LCE_CHUNK_ENV
        CE._LCE_CHUNK_ENV = str(chunk)
    try:
        loss = CE.linear_cross_entropy(Xt, Wt, tt)
        loss.backward()
    finally:
        if chunk:
            CE._LCE_CHUNK_ENV = old
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return loss.item(), Xt.grad.cpu().numpy(), Wt.grad.cpu().numpy()


@pytest.mark.parametrize("M,D,V", [(256, 64, 2050), (512, 256, 12000)])
def test_check_lce_cases(cuda, M, D, V):
    g = dict(np.load(G / f"lce_{M}_{D}_{V}.npz"))
    rng = np.random.default_rng(0)  # check_lce.py:33-37
    X = (rng.standard_normal((M, D)) * 0.1).astype(np.float32)
    W = (rng.standard_normal((D, V)) * 0.05).astype(np.float32)
    t = rng.integers(0, V, (M,)).astype(np.int32)
    loss, dX, dW = run(X, W, t, cuda)
    assert abs(loss - float(g["loss"])) < 1e-3          # the reference's own loss
    lr, _, dXr, dWr = ops.linear_cross_entropy(X, W, t, bf16_operands=True)
    assert abs(loss - lr) < 1e-3
    assert nrel(dX, dXr) < 1e-2 and nrel(dW, dWr) < 1e-2
    assert nrel(dX, g["dX"]) < 2e-2                     # vs reference f32 gradients
    assert nrel(dW[:, :256], g["dW_cols"]) < 2e-2


@pytest.mark.parametrize("chunk", [64, 8192])
def test_model_vocab(cuda, chunk):
    # BASELINE head: D=512, V=50257 (unpadded W, ragged last tile), M sub-sampled
    rng = np.random.default_rng(1)
    M, D, V = 512 if chunk == 64 else 1024, 512, 50257
    X = rng.standard_normal((M, D)).astype(np.float32)
    W = (rng.standard_normal((D, V)) * 0.02).astype(np.float32)
    t = rng.integers(0, V, (M,)).astype(np.int32)
    loss, dX, dW = run(X, W, t, cuda, chunk=chunk)
    lr, _, dXr, dWr = ops.linear_cross_entropy(X, W, t, bf16_operands=True)
    assert abs(loss - lr) < 1e-3
    assert nrel(dX, dXr) < 1e-2 and nrel(dW, dWr) < 1e-2


def test_full_size_properties(cuda):
    # M=16384 (the config): loss consistent with a materialised-logit CE of the
    # same bf16 operands, and gradient rows of dlogits sum to ~0 => dX . 1 small
    torch.manual_seed(0)
    M, D, V = 16384, 512, 50257
    X = torch.randn(M, D, device=cuda).bfloat16()
    W = (torch.randn(D, V, device=cuda) * 0.02).bfloat16()
    t = torch.randint(0, V, (M,), device=cuda, dtype=torch.int32)
    loss = CE.linear_cross_entropy(X, W, t).item()
    logits = X.float() @ W.float()
    ref = torch.nn.functional.cross_entropy(logits, t.long()).item()
    assert abs(loss - ref) < 1e-3


def test_bwd_ex_writes_bf16_dx(cuda):
    """nl_lce_bwd_ex storing a bf16 dX (no zeroed f32 buffer, no cast) gives
    the accumulating nl_lce_bwd's dX rounded to bf16, and the same dW."""
    torch.manual_seed(4)
    M, D, V = 2048, 512, 50257
    Vp = (V + 63) // 64 * 64
    X = torch.randn(M, D, device=cuda).bfloat16()
    W = (torch.randn(D, Vp, device=cuda) * 0.02).bfloat16()[:, :V]
    t = torch.randint(0, V, (M,), device=cuda, dtype=torch.int32)
    loss, lse = CE.lce_fwd_raw(X, W, t)
    dW1 = torch.zeros(D, Vp, device=cuda)[:, :V]
    dX1, _ = CE.lce_bwd_raw(X, W, t, lse, dW=dW1, dw_accumulate=True)
    dW2 = torch.zeros(D, Vp, device=cuda)[:, :V]
    dX2 = CE.lce_bwd_bf16_dx(X, W, t, lse, dW=dW2)
    torch.cuda.synchronize()
    assert dX2.dtype == torch.bfloat16
    assert nrel(dX2.float().cpu().numpy(), dX1.cpu().numpy()) < 1e-2
    assert nrel(dW2.cpu().numpy(), dW1.cpu().numpy()) < 1e-5
    assert _lib.device_error() == 0
