"""The reference's remaining kernel checks, restated against the B200 kernels
on the same seeded inputs (iree_metal/kernels/test/ in the nlearn tree):

* validate_gemm.py:10-21      1024^3 GEMM, N(0,1)*0.1 inputs (seed 0), atol 2e-2;
* check_gemm_bf16.py:16-28    the three bf16 cases, through the golden fixtures;
* check_ce.py:15-26           fused CE at the training shape (4096, 50257), seed 0;
* grad_check_flash.py:13-46   attention gradients at the training seq 512
                              (64, 512, 64), N(0,1)*0.1 inputs (seed 0), loss = sum(O).

The reference ran its GEMM and attention checks in fp16; the B200 kernels take
bf16, so the inputs are the same numbers rounded to bf16 and the bars are the
north-star ones (max|err| / max|ref| <= 1e-2 for attention gradients; CE loss
within 1e-3 absolute).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from nlearn_b200 import _lib  # noqa: E402
from nlearn_b200 import attention as A  # noqa: E402
from nlearn_b200.kernels import cross_entropy as CE  # noqa: E402
from nlearn_b200.kernels.gemm import gemm  # noqa: E402

G = Path(__file__).resolve().parent / "golden"


def test_validate_gemm_1024(cuda):
    np.random.seed(0)  # validate_gemm.py:11-13
    a = (np.random.randn(1024, 1024) * 0.1).astype(np.float16)
    b = (np.random.randn(1024, 1024) * 0.1).astype(np.float16)
    ref = a.astype(np.float32) @ b.astype(np.float32)
    At = torch.from_numpy(a.astype(np.float32)).to(cuda).bfloat16()
    Bt = torch.from_numpy(b.astype(np.float32)).to(cuda).bfloat16()
    C = gemm(At, Bt).cpu().numpy()
    assert _lib.device_error() == 0
    assert np.allclose(C, ref, atol=2e-2), float(np.abs(C - ref).max())
    # and exactly the f32 product of the bf16 operands, up to summation order
    refb = At.float().cpu().numpy() @ Bt.float().cpu().numpy()
    assert float(np.abs(C - refb).max()) < 1e-4


@pytest.mark.parametrize("name", ["gemm_small", "gemm_medium", "gemm_large"])
def test_check_gemm_bf16_golden(cuda, name):
    g = dict(np.load(G / f"{name}.npz"))
    At = torch.from_numpy(g["A"]).to(cuda).bfloat16()
    Bt = torch.from_numpy(g["B"]).to(cuda).bfloat16()
    C = gemm(At, Bt).cpu().numpy()
    assert _lib.device_error() == 0
    np.testing.assert_allclose(C, g["C"], rtol=1e-5, atol=1e-5 * np.abs(g["C"]).max())


def test_check_ce_training_shape(cuda):
    M, V = 4096, 50257  # check_ce.py:15-19
    rng = np.random.default_rng(0)
    logits = torch.from_numpy(rng.standard_normal((M, V)).astype(np.float32)).to(cuda)
    tgt = torch.from_numpy(rng.integers(0, V, (M,)).astype(np.int32)).to(cuda)
    x = logits.clone().requires_grad_()
    loss = CE.cross_entropy(x, tgt)
    loss.backward()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    l64 = logits.double()
    ref = torch.nn.functional.cross_entropy(l64, tgt.long())
    assert abs(loss.item() - ref.item()) < 1e-3
    dref = (torch.softmax(l64, -1) - torch.nn.functional.one_hot(tgt.long(), V).double()) / M
    d = x.grad.double()
    rel = ((d - dref).abs().mean() / dref.abs().mean()).item()
    assert rel < 1e-4, rel
    assert torch.isfinite(x.grad).all()


def test_grad_check_flash_seq512(cuda):
    N, S, D = 64, 512, 64  # grad_check_flash.py:13, 35-37
    rng = np.random.default_rng(0)
    mk = lambda: torch.from_numpy((rng.standard_normal((N, S, D)) * 0.1).astype(np.float32)).to(cuda).bfloat16()
    Q, K, V = mk(), mk(), mk()
    # loss = sum(O): dO = 1
    O, L = A._flash_fwd_raw(Q, K, V)
    dO = torch.ones_like(O)
    dQ, dK, dV = A._flash_bwd_raw(Q, K, V, O, L, dO)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    # materialised f32 reference (the script's attn_ref), autograd for the gradients
    q, k, v = (t.float().requires_grad_() for t in (Q, K, V))
    s = q @ k.transpose(1, 2) / D ** 0.5
    s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool, device=cuda), 1), float("-inf"))
    o = torch.softmax(s, -1) @ v
    o.sum().backward()
    assert ((O.float() - o).abs().max() / o.abs().max()).item() < 1e-2
    for name, a, b in (("dQ", dQ, q.grad), ("dK", dK, k.grad), ("dV", dV, v.grad)):
        a = a.float()
        err = ((a - b).abs().max() / b.abs().max()).item()
        mean_rel = ((a - b).abs().mean() / b.abs().mean()).item()
        corr = torch.corrcoef(torch.stack([a.flatten(), b.flatten()]))[0, 1].item()
        assert err < 1e-2 and mean_rel < 1e-2 and corr > 0.999, (name, err, mean_rel, corr)
