"""Flash attention parity on the GPU against the CPU oracle (oracle/ops.py,
pinned to the reference's own outputs) on identical bf16-rounded inputs.

Tolerance: max |kernel - oracle| / max |oracle| <= 1e-2
for O, dQ, dK, dV; L (f32 log-sum-exp) within 2e-2 absolute."""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import ops  # noqa: E402
from nlearn_b200 import attention as A  # noqa: E402
from nlearn_b200 import _lib  # noqa: E402

G = Path(__file__).resolve().parent / "golden"
TOL = 1e-2


def nrel(a, b):
    """max |a - b| / max |b|; the floor keeps exactly-zero references (s == 1,
    where softmax over one key has zero dQ / dK) on an absolute 1e-5 scale."""
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-3))


def bf(x):
    return ops.bf16_round(x)


def run_case(Q, K, V, dO, dev):
    Qt, Kt, Vt, dOt = (torch.from_numpy(x).to(dev).to(torch.bfloat16) for x in (Q, K, V, dO))
    O, L = A._flash_fwd_raw(Qt, Kt, Vt)
    dQ, dK, dV = A._flash_bwd_raw(Qt, Kt, Vt, O, L, dOt)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    f = lambda t: t.float().cpu().numpy()
    return f(O), f(L), f(dQ), f(dK), f(dV)


def check(Q, K, V, dO, dev, tol=TOL):
    Q, K, V, dO = bf(Q), bf(K), bf(V), bf(dO)
    O, L, dQ, dK, dV = run_case(Q, K, V, dO, dev)
    Or, Lr = ops.attention_fwd(Q, K, V)
    dQr, dKr, dVr, _ = ops.attention_bwd(Q, K, V, dO)
    errs = dict(O=nrel(O, Or), dQ=nrel(dQ, dQr), dK=nrel(dK, dKr), dV=nrel(dV, dVr),
                L=float(np.abs(L - Lr).max()))
    assert errs["O"] < tol and errs["dQ"] < tol and errs["dK"] < tol and errs["dV"] < tol, errs
    assert errs["L"] < 2e-2, errs
    assert np.isfinite(dQ).all() and np.isfinite(dK).all() and np.isfinite(dV).all()
    return errs


def test_golden_flash_bwd_128(cuda):
    g = dict(np.load(G / "flash_bwd_128.npz"))
    check(g["Q"], g["K"], g["V"], g["dO"], cuda)


def test_golden_flash_fwd_tiled(cuda):
    g = dict(np.load(G / "flash_fwd_tiled.npz"))
    Q, K, V = bf(g["Q"]), bf(g["K"]), bf(g["V"])
    O, L, *_ = run_case(Q, K, V, np.zeros_like(Q), cuda)
    Or, Lr = ops.attention_fwd(Q, K, V)
    assert nrel(O, Or) < TOL
    assert np.abs(L - Lr).max() < 2e-2
    # and against the reference's own f32 outputs on the unrounded inputs
    assert nrel(O, g["O"]) < 2e-2


# (300, 256): 600 backward work items, several snake-order rounds over the
# persistent CTAs; (2, 4096): the long-context length; (5, 777): ragged tiles
@pytest.mark.parametrize("n,s", [(32, 512), (2, 300), (3, 1), (4, 129), (2, 1024), (300, 256), (2, 4096),
                                 (5, 777)])
def test_shapes(cuda, n, s):
    rng = np.random.default_rng(n * 1000 + s)
    mk = lambda: rng.standard_normal((n, s, 64)).astype(np.float32)
    check(mk(), mk(), mk(), mk(), cuda)


def test_large_logits_stability(cuda):
    # scores of magnitude ~100: exercises the online-max rescale of O
    rng = np.random.default_rng(7)
    mk = lambda sc: (rng.standard_normal((4, 512, 64)) * sc).astype(np.float32)
    check(mk(3.0), mk(3.0), mk(1.0), mk(1.0), cuda, tol=2e-2)


def test_reference_targets_dq_dkdv(cuda):
    rng = np.random.default_rng(11)
    mk = lambda: bf(rng.standard_normal((8, 256, 64)).astype(np.float32))
    Q, K, V, dO = mk(), mk(), mk(), mk()
    t = lambda x: torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    O, L = A._flash_fwd_raw(t(Q), t(K), t(V))
    D = (O.float() * t(dO).float()).sum(-1)
    dQ = A.flash_attention_bwd_dq(t(Q), t(K), t(V), t(dO), L, D)
    dK, dV = A.flash_attention_bwd_dkdv(t(Q), t(K), t(V), t(dO), L, D)
    dQr, dKr, dVr, _ = ops.attention_bwd(Q, K, V, dO)
    f = lambda x: x.float().cpu().numpy()
    assert nrel(f(dQ), dQr) < TOL and nrel(f(dK), dKr) < TOL and nrel(f(dV), dVr) < TOL


def test_autograd_and_torch_reference(cuda):
    # BH=256 (full-model shape) against a torch fp32 reference on the GPU
    torch.manual_seed(0)
    n, s = 256, 512
    Q, K, V = (torch.randn(n, s, 64, device=cuda).bfloat16().requires_grad_() for _ in range(3))
    O = A.attention(Q, K, V)
    g = torch.randn_like(O)
    O.backward(g)
    Qr, Kr, Vr = (x.detach().float().requires_grad_() for x in (Q, K, V))
    Or = torch.nn.functional.scaled_dot_product_attention(Qr, Kr, Vr, is_causal=True)
    Or.backward(g.float())
    r = lambda a, b: ((a.float() - b).abs().max() / b.abs().max()).item()
    assert r(O, Or) < TOL
    assert r(Q.grad, Qr.grad) < TOL and r(K.grad, Kr.grad) < TOL and r(V.grad, Vr.grad) < TOL


def test_deterministic_forward(cuda):
    rng = np.random.default_rng(5)
    mk = lambda: torch.from_numpy(rng.standard_normal((16, 512, 64)).astype(np.float32)).to(cuda).bfloat16()
    Q, K, V = mk(), mk(), mk()
    O1, L1 = A._flash_fwd_raw(Q, K, V)
    O2, L2 = A._flash_fwd_raw(Q, K, V)
    assert torch.equal(O1, O2) and torch.equal(L1, L2)


def test_strided_qkv_layout(cuda):
    # Q/K/V read in place from a fused projection [B, S, 3, H, 64]; O written
    # as [B, S, H, 64]; dQ/dK/dV written back into the [B, S, 3, H, 64] layout.
    from nlearn_b200._lib import lib, ptr, stream_handle, check
    B, S, H = 3, 384, 4
    torch.manual_seed(3)
    qkv = torch.randn(B, S, 3, H, 64, device=cuda).bfloat16()
    dO = torch.randn(B, S, H, 64, device=cuda).bfloat16()
    O = torch.empty(B, S, H, 64, device=cuda, dtype=torch.bfloat16)
    L = torch.empty(B * H, S, device=cuda)
    qs = (3 * H * 64, 64, S * 3 * H * 64)
    os_ = (H * 64, 64, S * H * 64)
    check(lib.nl_flash_attention_fwd_strided(ptr(qkv[:, :, 0]), ptr(qkv[:, :, 1]), ptr(qkv[:, :, 2]), *qs, ptr(O),
                                             *os_, ptr(L), B, H, S, 64, stream_handle()), "fwd_strided")
    dqkv = torch.empty_like(qkv)
    D = torch.empty(B * H, S, device=cuda)
    acc = torch.empty(B * H, S, 64, device=cuda)
    check(lib.nl_flash_attention_bwd_strided(ptr(qkv[:, :, 0]), ptr(qkv[:, :, 1]), ptr(qkv[:, :, 2]), *qs, ptr(O),
                                             ptr(dO), *os_, ptr(L), ptr(D), ptr(dqkv[:, :, 0]), ptr(dqkv[:, :, 1]),
                                             ptr(dqkv[:, :, 2]), ptr(acc), B, H, S, 64, stream_handle()),
          "bwd_strided")
    to_c = lambda x: x.permute(0, 2, 1, 3).reshape(B * H, S, 64).contiguous()
    Qc, Kc, Vc = (to_c(qkv[:, :, i]) for i in range(3))
    Oc, Lc = A._flash_fwd_raw(Qc, Kc, Vc)
    dQc, dKc, dVc = A._flash_bwd_raw(Qc, Kc, Vc, Oc, Lc, to_c(dO))
    torch.cuda.synchronize()
    assert torch.equal(to_c(O), Oc) and torch.equal(L, Lc)
    assert torch.equal(to_c(dqkv[:, :, 1]), dKc) and torch.equal(to_c(dqkv[:, :, 2]), dVc)
    assert ((to_c(dqkv[:, :, 0]).float() - dQc.float()).abs().max() <= 1e-2 * dQc.float().abs().max())


@pytest.mark.parametrize("n,s", [(32, 512), (3, 200)])
def test_f32_reference_targets(cuda, n, s):
    """The three targets on what the reference's wrappers send (f32 Q, K, V,
    dO; attention.py:82-91, 97, 111-128): f32 O, dQ, dK, dV out, converted to
    bf16 tensor-core operands inside the library.  Checked against the f32
    oracle on the unrounded inputs."""
    rng = np.random.default_rng(n + s)
    mk = lambda: rng.standard_normal((n, s, 64)).astype(np.float32)
    Q, K, V, dO = mk(), mk(), mk(), mk()
    t = lambda x: torch.from_numpy(x).to(cuda)
    O, L = A.flash_attention_fwd(t(Q), t(K), t(V))
    assert O.dtype == torch.float32 and L.dtype == torch.float32
    D = (O * t(dO)).sum(-1)                       # attention.py:115, D computed by the caller
    dQ = A.flash_attention_bwd_dq(t(Q), t(K), t(V), t(dO), L, D)
    dK, dV = A.flash_attention_bwd_dkdv(t(Q), t(K), t(V), t(dO), L, D)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert dQ.dtype == dK.dtype == dV.dtype == torch.float32
    Or, Lr = ops.attention_fwd(Q, K, V)
    dQr, dKr, dVr, _ = ops.attention_bwd(Q, K, V, dO)
    f = lambda x: x.cpu().numpy()
    assert nrel(f(O), Or) < TOL and np.abs(f(L) - Lr).max() < 2e-2
    assert nrel(f(dQ), dQr) < TOL and nrel(f(dK), dKr) < TOL and nrel(f(dV), dVr) < TOL


def test_f32_autograd_follows_reference_rule(cuda):
    """_attention_iree_flash with f32 inputs: the fwd target, then D =
    rowsum(dO * O) and the dq / dkdv targets, all f32 at the boundary."""
    torch.manual_seed(1)
    n, s = 16, 256
    Q, K, V = (torch.randn(n, s, 64, device=cuda).requires_grad_() for _ in range(3))
    O = A._attention_iree_flash(Q, K, V)
    assert O.dtype == torch.float32
    g = torch.randn_like(O)
    O.backward(g)
    Qr, Kr, Vr = (x.detach().double().requires_grad_() for x in (Q, K, V))
    Or = torch.nn.functional.scaled_dot_product_attention(Qr, Kr, Vr, is_causal=True)
    Or.backward(g.double())
    r = lambda a, b: ((a.double() - b).abs().max() / b.abs().max()).item()
    assert r(O, Or) < TOL
    assert Q.grad.dtype == torch.float32
    assert r(Q.grad, Qr.grad) < TOL and r(K.grad, Kr.grad) < TOL and r(V.grad, Vr.grad) < TOL


def test_dt_entry_points_reject_bad_workspace_and_dtype(cuda):
    from nlearn_b200._lib import lib, stream_handle, STATUS
    n, s = 2, 64
    assert lib.nl_flash_attention_workspace_bytes(0, n, s, 64, 0) > 0
    assert lib.nl_flash_attention_workspace_bytes(0, n, s, 64, 1) == 0
    assert lib.nl_flash_attention_workspace_bytes(0, n, s, 32, 0) == 0
    x = torch.zeros(n, s, 64, device=cuda)
    L = torch.zeros(n, s, device=cuda)
    st = lib.nl_flash_attention_fwd_dt(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), L.data_ptr(), n, s,
                                       64, 0, None, 0, stream_handle())
    assert STATUS[st] == "NL_ERR_WORKSPACE"
    st = lib.nl_flash_attention_fwd_dt(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), L.data_ptr(), n, s,
                                       64, 7, None, 0, stream_handle())
    assert STATUS[st] == "NL_ERR_DTYPE"
