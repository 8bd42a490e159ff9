"""GEMM parity on the GPU: tcgen05 kernel vs an fp32 matmul of the same
bf16-rounded operands (the reference's own check, check_gemm_bf16.py:16-19),
over every operand layout, ragged M/N/K tails and each fused epilogue."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from nlearn_b200.kernels.gemm import gemm_ex, gemm, linear  # noqa: E402
from nlearn_b200 import _lib  # noqa: E402


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-12)).item()


def _mk(shape, scale, dev, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).to(dev)


SHAPES = [(128, 128, 64), (256, 512, 128), (200, 136, 72), (1000, 1048, 520), (4096, 1536, 512),
          (304, 50264, 64), (16, 24, 8)]


@pytest.mark.parametrize("a_trans", [False, True])
@pytest.mark.parametrize("b_trans", [False, True])
@pytest.mark.parametrize("mnk", SHAPES)
def test_layouts(cuda, a_trans, b_trans, mnk):
    M, N, K = mnk
    A = _mk((K, M) if a_trans else (M, K), 1.0, cuda, 1)
    B = _mk((N, K) if b_trans else (K, N), 0.5, cuda, 2)
    C = gemm_ex(A, B, a_trans=a_trans, b_trans=b_trans)
    ref = (A.float().t() if a_trans else A.float()) @ (B.float().t() if b_trans else B.float())
    torch.cuda.synchronize()
    assert _rel(C, ref) < 1e-5, (mnk, a_trans, b_trans)
    assert _lib.device_error() == 0


def test_bf16_out_and_epilogues(cuda):
    M, N, K = 777, 520, 264
    A = _mk((M, K), 1.0, cuda, 3)
    B = _mk((K, N), 0.3, cuda, 4)
    ref = A.float() @ B.float()
    bias = torch.randn(N, device=cuda)
    C = gemm_ex(A, B, out_dtype=torch.bfloat16)
    assert _rel(C, ref) < 1e-2
    C = gemm_ex(A, B, epilogue=_lib.EPI_BIAS, bias=bias)
    assert _rel(C, ref + bias) < 1e-5
    aux = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    C = gemm_ex(A, B, out_dtype=torch.bfloat16, epilogue=_lib.EPI_BIAS_GELU, bias=bias, aux=aux)
    pre = ref + bias
    assert _rel(aux, pre) < 1e-2
    assert _rel(C, torch.nn.functional.gelu(pre, approximate="tanh")) < 2e-2
    resid = _mk((M, N), 1.0, cuda, 5)
    C = gemm_ex(A, B, out_dtype=torch.bfloat16, epilogue=_lib.EPI_RESID, resid=resid)
    assert _rel(C, ref + resid.float()) < 1e-2
    acc = torch.randn(M, N, device=cuda)
    acc0 = acc.clone()
    gemm_ex(A, B, out=acc, epilogue=_lib.EPI_ACCUM, alpha=0.5)
    assert _rel(acc, acc0 + 0.5 * ref) < 1e-5


def test_split_k_accumulate(cuda):
    # dW-shaped: few output tiles, long reduction -> split-K with float atomics
    M, N, K = 512, 512, 16384
    X = _mk((K, M), 1.0, cuda, 6)  # stored [tokens, in]
    dY = _mk((K, N), 1.0, cuda, 7)
    out = torch.zeros(M, N, device=cuda)
    gemm_ex(X, dY, a_trans=True, out=out, epilogue=_lib.EPI_ACCUM)
    ref = X.float().t() @ dY.float()
    assert _rel(out, ref) < 1e-5


def test_gemm_autograd_and_linear(cuda):
    A = _mk((300, 200), 1.0, cuda, 8).float().requires_grad_()
    B = _mk((200, 100), 1.0, cuda, 9).float().requires_grad_()
    C = gemm(A, B)
    g = torch.randn_like(C)
    C.backward(g)
    Ar = A.detach().clone().requires_grad_()
    Br = B.detach().clone().requires_grad_()
    Cr = Ar.bfloat16().float() @ Br.bfloat16().float()
    Cr.backward(g.bfloat16().float())
    assert _rel(C, Cr) < 1e-5
    assert _rel(A.grad, Ar.grad) < 1e-2
    assert _rel(B.grad, Br.grad) < 1e-2
    x = _mk((4, 64, 512), 1.0, cuda, 10).requires_grad_()
    W = _mk((512, 1536), 0.02, cuda, 11).requires_grad_()
    y = linear(x, W)
    assert y.dtype == torch.bfloat16 and y.shape == (4, 64, 1536)
    assert _rel(y, x.float() @ W.float()) < 1e-2


GEMV_SHAPES = [(1, 512, 512), (3, 1536, 512), (8, 2048, 512), (5, 512, 2048), (2, 200, 72), (7, 64, 8),
               (1, 50257, 512), (4, 4096, 4096)]


@pytest.mark.parametrize("mnk", GEMV_SHAPES)
def test_small_m_gemv_path(cuda, mnk):
    """M <= 8 with row-major operands takes the cluster GEMV kernel (the decode
    step's products); every epilogue it serves against an fp32 reference."""
    M, N, K = mnk
    Np = (N + 63) // 64 * 64                      # padded row pitch (the LM head's W)
    A = _mk((M, K), 1.0, cuda, 11)
    Bfull = _mk((K, Np), 0.5, cuda, 12)
    B = Bfull[:, :N]
    ref = A.float() @ B.float()
    C = gemm_ex(A, B)                              # f32 store
    assert _rel(C, ref) < 1e-5
    bias = torch.randn(N, device=cuda)
    Cb = gemm_ex(A, B, out_dtype=torch.bfloat16, epilogue=_lib.EPI_BIAS, bias=bias)
    assert _rel(Cb, ref + bias) < 1e-2
    resid = torch.randn(M, N, device=cuda).bfloat16()
    Cr = gemm_ex(A, B, out_dtype=torch.bfloat16, epilogue=_lib.EPI_RESID, bias=bias, resid=resid)
    assert _rel(Cr, ref + bias + resid.float()) < 1e-2
    aux = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    Cg = gemm_ex(A, B, out_dtype=torch.bfloat16, epilogue=_lib.EPI_BIAS_GELU, bias=bias, aux=aux)
    pre = ref + bias
    assert _rel(aux, pre) < 1e-2
    assert _rel(Cg, torch.nn.functional.gelu(pre, approximate="tanh")) < 1e-2
    acc = torch.randn(M, N, device=cuda)
    want = acc + 2.0 * ref
    gemm_ex(A, B, out=acc, epilogue=_lib.EPI_ACCUM, alpha=2.0)
    assert _rel(acc, want) < 1e-5
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
