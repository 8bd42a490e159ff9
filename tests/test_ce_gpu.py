"""Cross-entropy row kernels on the GPU vs the oracle (pinned to the
reference's CE): loss within 1e-3 absolute, dlogits within
1e-5 absolute (f32 out) of the f64 oracle."""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import ops  # noqa: E402
from nlearn_b200.kernels import cross_entropy as CE  # noqa: E402

G = Path(__file__).resolve().parent / "golden"


def test_golden_ce(cuda):
    g = dict(np.load(G / "ce_512x1024.npz"))
    lg = torch.from_numpy(g["logits"]).to(cuda)
    t = torch.from_numpy(g["targets"]).to(cuda)
    loss, lse = CE._ce_fwd_raw(lg, t)
    assert abs(loss.mean().item() - float(g["loss"])) < 1e-4
    d = CE._ce_bwd_raw(lg, t, lse)
    lr, lser = ops.ce_fwd(g["logits"], g["targets"])
    dr = ops.ce_bwd(g["logits"], g["targets"], lser)
    assert np.abs(d.cpu().numpy() - dr).max() < 1e-6
    # autograd through the custom op
    lg2 = lg.clone().requires_grad_()
    CE.cross_entropy(lg2, t).backward()
    assert np.abs(lg2.grad.cpu().numpy() - dr).max() < 1e-6


@pytest.mark.parametrize("M,V,ld", [(64, 50257, 50257), (33, 50257, 50264), (7, 5, 5), (16, 1000, 1003)])
def test_shapes_and_pitch(cuda, M, V, ld):
    rng = np.random.default_rng(M + V)
    x = (rng.standard_normal((M, ld)) * 3).astype(np.float32)
    t = rng.integers(0, V, M).astype(np.int32)
    xt = torch.from_numpy(x).to(cuda)[:, :V]
    tt = torch.from_numpy(t).to(cuda)
    loss, lse, d = CE.ce_fwd_bwd(xt, tt)
    lr, lser = ops.ce_fwd(x[:, :V], t)
    dr = ops.ce_bwd(x[:, :V], t, lser)
    assert np.abs(loss.cpu().numpy() - lr).max() < 1e-3
    assert np.abs(lse.cpu().numpy() - lser).max() < 1e-3
    assert np.abs(d.cpu().numpy() - dr).max() < 1e-5
    l2, s2 = CE._ce_fwd_raw(xt, tt)
    assert torch.allclose(l2, loss) and torch.allclose(s2, lse)


def test_bf16_and_inplace(cuda):
    rng = np.random.default_rng(3)
    M, V = 128, 50264
    x = rng.standard_normal((M, V)).astype(np.float32)
    t = rng.integers(0, V, M).astype(np.int32)
    xb = torch.from_numpy(x).to(cuda).bfloat16()
    tt = torch.from_numpy(t).to(cuda)
    xr = xb.float().cpu().numpy()
    lr, lser = ops.ce_fwd(xr, t)
    dr = ops.ce_bwd(xr, t, lser, scale=0.5)
    loss, lse, d = CE.ce_fwd_bwd(xb, tt, scale=0.5, out=xb)  # in place
    assert d.data_ptr() == xb.data_ptr()
    assert np.abs(loss.cpu().numpy() - lr).max() < 1e-3
    assert np.abs(d.float().cpu().numpy() - dr).max() < 4e-3 * 0.5 + 1e-6


def test_out_of_range_target(cuda):
    x = torch.randn(4, 100, device=cuda)
    t = torch.tensor([0, -1, 100, 5], device=cuda, dtype=torch.int32)
    loss, lse = CE._ce_fwd_raw(x, t)
    assert abs(loss[1].item() - lse[1].item()) < 1e-6 and abs(loss[2].item() - lse[2].item()) < 1e-6
