"""Parity at the BASELINE configurations' full sizes.

configs[1] — the bf16 `linear` GEMM sweep at M = bs*seq = 16384, for each of
the five (K, N) model shapes, forward, dX and dW, through the same calls and
epilogues the training step makes (nl_gemm_ex: bf16 store / bias+GELU /
residual forward, dX = dY W^T with W read in place, dW accumulated in f32
from X and dY read MN-major).  The checker is a float32 matmul of the same
bf16 operands on the GPU (TF32 off).

configs[2] — the fused LM-head cross-entropy at M = 16384, D = 512,
V = 50257: loss, dX and dW against a vocabulary-chunked float32 computation
of the same bf16 operands (pass 1: row logsumexp; pass 2: softmax - onehot per
chunk, dX += dl W_c^T, dW_c = X^T dl), the chunked form of
nlearn/kernels/cross_entropy.py:106-167.

Bars (north star): outputs and gradients within max|err| / max|ref| <= 1e-2
of the float32 reference; CE loss within 1e-3 absolute.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

from nlearn_b200 import _lib  # noqa: E402
from nlearn_b200.kernels.gemm import gemm_ex  # noqa: E402
from nlearn_b200.kernels import cross_entropy as CE  # noqa: E402

TOL = 1e-2
M = 16384
SWEEP = [(512, 1536, "qkv"), (512, 512, "proj"), (512, 2048, "ffn_up"), (2048, 512, "ffn_down"),
         (512, 50257, "lm_head")]


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def nrel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-12)).item()


def _bf16(shape, std, gen, dev):
    return (torch.randn(*shape, generator=gen, device=dev) * std).bfloat16()


@pytest.mark.parametrize("K,N,name", SWEEP, ids=[s[2] for s in SWEEP])
def test_gemm_sweep_fwd_dx_dw(cuda, K, N, name):
    """x ~ N(0,1), W ~ N(0,0.02), dY ~ N(0,1); W at the 16-byte
    padded row pitch the model stores (the LM head's 50257 -> 50304)."""
    gen = torch.Generator(device=cuda).manual_seed(K * 7 + N)
    Np = (N + 63) // 64 * 64
    x = _bf16((M, K), 1.0, gen, cuda)
    W = _bf16((K, Np), 0.02, gen, cuda)[:, :N]
    dY = _bf16((M, Np), 1.0, gen, cuda)[:, :N]
    xf, Wf, dYf = x.float(), W.float(), dY.float()

    y_ref = xf @ Wf
    y = gemm_ex(x, W, out_dtype=torch.bfloat16)                                # forward, bf16 store
    assert nrel(y, y_ref) < TOL, ("fwd", nrel(y, y_ref))
    if name == "ffn_up":                                                       # the step's bias+GELU epilogue
        bias = torch.randn(N, generator=gen, device=cuda) * 0.1
        aux = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
        u = gemm_ex(x, W, out_dtype=torch.bfloat16, epilogue=_lib.EPI_BIAS_GELU, bias=bias, aux=aux)
        assert nrel(aux, y_ref + bias) < TOL
        assert nrel(u, torch.nn.functional.gelu(y_ref + bias, approximate="tanh")) < TOL
    if N == 512:                                                               # residual epilogue (proj, ffn_down)
        resid = _bf16((M, N), 1.0, gen, cuda)
        r = gemm_ex(x, W, out_dtype=torch.bfloat16, epilogue=_lib.EPI_RESID, resid=resid)
        assert nrel(r, y_ref + resid.float()) < TOL
    del y, y_ref

    dx_ref = dYf @ Wf.t()
    dx = gemm_ex(dY, W, b_trans=True, out_dtype=torch.bfloat16)                 # dX = dY W^T, W read in place
    assert nrel(dx, dx_ref) < TOL, ("dX", nrel(dx, dx_ref))
    del dx, dx_ref

    dw_ref = xf.t() @ dYf
    dw = torch.zeros(K, Np, device=cuda)[:, :N]
    gemm_ex(x, dY, a_trans=True, out=dw, epilogue=_lib.EPI_ACCUM)              # dW += X^T dY (f32)
    assert nrel(dw, dw_ref) < 1e-4, ("dW", nrel(dw, dw_ref))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


def _chunked_lce_reference(X, W, t, chunk=8192):
    """float32 loss, dX, dW of mean CE(X W) from the bf16 operands, one
    vocabulary chunk at a time (never the whole [M, V] f32 matrix)."""
    Xf = X.float()
    Mr, V = X.shape[0], W.shape[1]
    m = torch.full((Mr,), -float("inf"), device=X.device)
    ssum = torch.zeros(Mr, device=X.device)
    tgt_logit = torch.zeros(Mr, device=X.device)
    rows = torch.arange(Mr, device=X.device)
    for c in range(0, V, chunk):
        lg = Xf @ W[:, c:c + chunk].float()
        cm = torch.maximum(m, lg.max(1).values)
        ssum = ssum * torch.exp(m - cm) + torch.exp(lg - cm[:, None]).sum(1)
        m = cm
        inside = (t >= c) & (t < c + lg.shape[1])
        tgt_logit[inside] = lg[rows[inside], (t[inside] - c).long()]
    lse = m + torch.log(ssum)
    loss = (lse - tgt_logit).mean()
    dX = torch.zeros_like(Xf)
    dW = torch.empty(W.shape, device=X.device)
    for c in range(0, V, chunk):
        Wc = W[:, c:c + chunk].float()
        p = torch.exp(Xf @ Wc - lse[:, None])
        inside = (t >= c) & (t < c + Wc.shape[1])
        p[rows[inside], (t[inside] - c).long()] -= 1.0
        p /= Mr
        dX += p @ Wc.t()
        dW[:, c:c + chunk] = Xf.t() @ p
    return loss.item(), dX, dW


def test_lce_configs2_full_size_grads(cuda):
    """hidden (16384, 512) ~ N(0,1), untied head W (512, 50257)
    ~ N(0, 0.02), int32 targets uniform in [0, 50257)."""
    gen = torch.Generator(device=cuda).manual_seed(2)
    D, V = 512, 50257
    X = _bf16((M, D), 1.0, gen, cuda).requires_grad_()
    W = _bf16((D, V), 0.02, gen, cuda).requires_grad_()
    t = torch.randint(0, V, (M,), generator=gen, device=cuda, dtype=torch.int32)
    loss = CE.linear_cross_entropy(X, W, t)
    loss.backward()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    lr, dXr, dWr = _chunked_lce_reference(X.detach(), W.detach(), t)
    assert abs(loss.item() - lr) < 1e-3, (loss.item(), lr)
    assert nrel(X.grad, dXr) < TOL, nrel(X.grad, dXr)
    assert nrel(W.grad, dWr) < TOL, nrel(W.grad, dWr)


def test_ce_row_kernel_full_size(cuda):
    """The materialised-logit CE kernel (targets `ce_fwd` / `ce_bwd`) at
    (16384, 50257) f32, in place: loss, lse and dlogits / M against torch."""
    gen = torch.Generator(device=cuda).manual_seed(3)
    V = 50257
    logits = torch.randn(M, V, generator=gen, device=cuda) * 2.0
    t = torch.randint(0, V, (M,), generator=gen, device=cuda, dtype=torch.int32)
    lse_ref = torch.logsumexp(logits, 1)
    loss_ref = (lse_ref - logits[torch.arange(M, device=cuda), t.long()])
    p = torch.softmax(logits, 1)
    p[torch.arange(M, device=cuda), t.long()] -= 1.0
    p /= M
    loss, lse, d = CE.ce_fwd_bwd(logits, t, out=logits)
    torch.cuda.synchronize()
    assert abs(loss.mean().item() - loss_ref.mean().item()) < 1e-3
    assert (lse - lse_ref).abs().max().item() < 1e-4
    assert nrel(d, p) < 1e-4
