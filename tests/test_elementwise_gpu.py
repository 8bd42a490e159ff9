"""Training-step tail kernels (nl_layernorm_fwd/bwd, nl_embed_fwd/bwd,
nl_colsum_bf16, nl_adamw_step) against float32 PyTorch references."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from nlearn_b200._lib import lib, ptr, stream_handle, check  # noqa: E402


def rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6)).item()


@pytest.mark.parametrize("M,D", [(16384, 512), (1000, 256), (37, 1024)])
def test_layernorm_fwd_bwd(cuda, M, D):
    torch.manual_seed(M)
    x = torch.randn(M, D, device=cuda).bfloat16()
    g = torch.randn(D, device=cuda)
    b = torch.randn(D, device=cuda)
    y = torch.empty_like(x)
    mean = torch.empty(M, device=cuda)
    rstd = torch.empty(M, device=cuda)
    check(lib.nl_layernorm_fwd(ptr(x), ptr(g), ptr(b), ptr(y), ptr(mean), ptr(rstd), M, D, 1e-5, stream_handle()), "ln")
    xr = x.float().requires_grad_()
    gr, br = g.clone().requires_grad_(), b.clone().requires_grad_()
    yr = torch.nn.functional.layer_norm(xr, (D,), gr, br, 1e-5)
    assert rel(y, yr) < 1e-2
    dy = torch.randn(M, D, device=cuda).bfloat16()
    yr.backward(dy.float())
    dres = torch.ones(M, D, device=cuda)
    dres_bf = torch.empty(M, D, device=cuda, dtype=torch.bfloat16)
    dg = torch.zeros(D, device=cuda)
    db = torch.zeros(D, device=cuda)
    ds = torch.full((D,), 0.5, device=cuda)
    check(lib.nl_layernorm_bwd(ptr(dy), ptr(x), ptr(mean), ptr(rstd), ptr(g), ptr(dres), ptr(dres_bf), ptr(dg),
                               ptr(db), ptr(ds), M, D, 1, stream_handle()), "ln bwd")
    assert rel(ds - 0.5, dres.sum(0)) < 1e-4        # column sums of the new residual gradient, accumulated
    assert rel(dres - 1, xr.grad) < 1e-3
    assert rel(dres_bf, dres) < 1e-2
    assert rel(dg, gr.grad) < 1e-3 and rel(db, br.grad) < 1e-3


def test_embed_and_colsum(cuda):
    V, S, B, D = 1000, 128, 4, 512
    wte = torch.randn(V, D, device=cuda).bfloat16()
    wpe = torch.randn(S, D, device=cuda).bfloat16()
    tok = torch.randint(0, V, (B, S), device=cuda, dtype=torch.int32)
    out = torch.empty(B * S, D, device=cuda, dtype=torch.bfloat16)
    check(lib.nl_embed_fwd(ptr(tok), ptr(wte), ptr(wpe), ptr(out), B * S, S, D, stream_handle()), "embed")
    ref = (wte.float()[tok.long()] + wpe.float()[None]).reshape(-1, D)
    assert rel(out, ref) < 1e-2
    dx = torch.randn(B * S, D, device=cuda)
    dwte = torch.zeros(V, D, device=cuda)
    dwpe = torch.zeros(S, D, device=cuda)
    check(lib.nl_embed_bwd(ptr(tok), ptr(dx), ptr(dwte), ptr(dwpe), B * S, S, D, stream_handle()), "embed bwd")
    rt = torch.zeros(V, D, device=cuda).index_add_(0, tok.reshape(-1).long(), dx)
    assert rel(dwte, rt) < 1e-5 and rel(dwpe, dx.view(B, S, D).sum(0)) < 1e-5
    x = torch.randn(16384, 2048, device=cuda).bfloat16()
    o = torch.ones(2048, device=cuda)
    check(lib.nl_colsum_bf16(ptr(x), ptr(o), 16384, 2048, stream_handle()), "colsum")
    assert rel(o - 1, x.float().sum(0)) < 1e-4


def test_adamw_matches_formula(cuda):
    n = 4096
    p = torch.randn(n, device=cuda)
    g = torch.randn(n, device=cuda)
    m = torch.randn(n, device=cuda) * 0.1
    v = torch.rand(n, device=cuda) * 0.1
    sh = torch.empty(n, device=cuda, dtype=torch.bfloat16)
    lr, b1, b2, eps, wd, t = 1e-3, 0.9, 0.999, 1e-8, 0.1, 7
    hyper = torch.tensor([lr, 1 - b1 ** t, 1 - b2 ** t], device=cuda)
    m2 = b1 * m + (1 - b1) * g
    v2 = b2 * v + (1 - b2) * g * g
    p2 = p - lr * ((m2 / (1 - b1 ** t)) / ((v2 / (1 - b2 ** t)).sqrt() + eps) + wd * p)
    check(lib.nl_adamw_step(ptr(p), ptr(g), ptr(m), ptr(v), ptr(sh), n, ptr(hyper), b1, b2, eps, wd, 1,
                            stream_handle()), "adamw")
    err = dict(p=(p - p2).abs().max().item(), m=(m - m2).abs().max().item(), v=(v - v2).abs().max().item())
    assert err["p"] < 1e-6 and err["m"] < 1e-6 and err["v"] < 1e-6, err
    assert torch.equal(sh, p.bfloat16())
    assert int((g != 0).sum()) == 0      # zero_grad: the gradient is cleared for the next step
