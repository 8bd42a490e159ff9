"""bf16 GEMM operators on the sm_100a tcgen05 kernel — mirror of nlearn.kernels.gemm.

Reference surface (nlearn/kernels/gemm.py):
  * ``gemm(A, B)``   — custom_vjp, C f32 = A.B; dA = dC.B^T, dB = A^T.dC   (61-79)
  * ``matmul(A, B)`` — 2-D x 2-D routed through ``gemm``, else plain matmul  (82-90)
  * ``linear(x, W)`` — flatten leading dims into M, one GEMM, cast to x.dtype (93-115)

Differences that come from the B200 design, not from semantics:
  * the reference pads M,N to 32 and K to 64 for its Metal tiles
    (``_gemm_padded``, 43-58); TMA tiles handle any M/N/K, so only the 16-byte
    row rule remains (K and N rounded up to multiples of 8 where needed);
  * the backward never materialises ``B.T`` / ``A.T`` (gemm.py:74-75): the
    kernel reads either operand K-major or MN-major in place;
  * ``linear`` writes its bf16 output straight from the f32 accumulator.
"""
from __future__ import annotations

import torch

from .._lib import (BF16, EPI_ACCUM, EPI_STORE, F32, check, lib, ptr, stream_handle)

_DT = {torch.float32: F32, torch.bfloat16: BF16}


def _ceil(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("nlearn_b200 GEMM operands must be CUDA tensors (no CPU path)")


def gemm_ex(A: torch.Tensor, B: torch.Tensor, *, a_trans: bool = False, b_trans: bool = False,
            out: torch.Tensor | None = None, out_dtype=torch.float32, alpha: float = 1.0,
            epilogue: int = EPI_STORE, bias: torch.Tensor | None = None, aux: torch.Tensor | None = None,
            resid: torch.Tensor | None = None) -> torch.Tensor:
    """C = alpha * op(A) . op(B) with a fused epilogue.

    ``A`` is stored [M,K] (``a_trans=False``) or [K,M] (``a_trans=True``);
    ``B`` is stored [K,N] (``b_trans=False``) or [N,K] (``b_trans=True``).
    Both bf16, rows contiguous (stride(1) == 1), row pitch a multiple of 8.
    """
    _require_cuda(A, B)
    if A.dtype != torch.bfloat16 or B.dtype != torch.bfloat16:
        raise TypeError("gemm_ex operands must be bfloat16")
    if A.dim() != 2 or B.dim() != 2 or A.stride(1) != 1 or B.stride(1) != 1:
        raise ValueError("gemm_ex operands must be 2-D with unit column stride")
    M, K = (A.shape[1], A.shape[0]) if a_trans else (A.shape[0], A.shape[1])
    Kb, N = (B.shape[1], B.shape[0]) if b_trans else (B.shape[0], B.shape[1])
    if K != Kb:
        raise ValueError(f"inner dimensions differ: {K} vs {Kb}")
    if out is None:
        out = (torch.zeros if epilogue == EPI_ACCUM else torch.empty)((M, N), device=A.device, dtype=out_dtype)
    if out.shape != (M, N) or out.stride(1) != 1:
        raise ValueError(f"out must be [{M},{N}] with unit column stride")
    st = lib.nl_gemm_ex(ptr(A), A.stride(0), int(a_trans), ptr(B), B.stride(0), int(b_trans), ptr(out),
                        out.stride(0), _DT[out.dtype], M, N, K, float(alpha), int(epilogue), ptr(bias), ptr(aux),
                        ptr(resid), stream_handle())
    check(st, "nl_gemm_ex")
    return out


def _pad_cols(x: torch.Tensor, mult: int = 8) -> torch.Tensor:
    """Zero-pad the last dim to a multiple of `mult` (TMA needs 16-byte rows)."""
    c = x.shape[-1]
    cp = _ceil(c, mult)
    if cp == c and x.is_contiguous():
        return x
    out = torch.zeros(*x.shape[:-1], cp, device=x.device, dtype=x.dtype)
    out[..., :c] = x
    return out


def _gemm_raw(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """A[M,K] bf16 @ B[K,N] bf16 -> C[M,N] f32 through ``nl_gemm`` (target `gemm`)."""
    M, K = A.shape
    N = B.shape[1]
    Ap = _pad_cols(A.to(torch.bfloat16))
    Bp = _pad_cols(B.to(torch.bfloat16))
    Kp, Np = Ap.shape[1], Bp.shape[1]
    if Kp != K:
        Bp = torch.cat([Bp, Bp.new_zeros(Kp - K, Np)], 0)
    C = torch.empty(M, Np, device=A.device, dtype=torch.float32)
    check(lib.nl_gemm(ptr(Ap), ptr(Bp), ptr(C), M, Np, Kp, stream_handle()), "nl_gemm")
    return C[:, :N]


def _operand(x: torch.Tensor) -> torch.Tensor:
    """bf16, unit column stride, 16-byte row pitch (copy only when needed)."""
    x = x.to(torch.bfloat16)
    if x.stride(1) != 1 or x.stride(0) % 8 != 0 or x.data_ptr() % 16 != 0:
        x = _pad_cols(x.contiguous())
    return x


class _Gemm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, A, B):
        ctx.save_for_backward(A, B)
        return _gemm_raw(A, B)

    @staticmethod
    def backward(ctx, dC):
        A, B = ctx.saved_tensors
        dCb = _operand(dC)
        Ab, Bb = _operand(A), _operand(B)
        M, K = A.shape
        N = B.shape[1]
        dA = dB = None
        if ctx.needs_input_grad[0]:
            # dA[M,K] = dC[M,N] . B^T : B stored [K,N] is B^T stored "[N',K']" transposed
            # (both padded to the same column count; pad columns are zero)
            dA = gemm_ex(dCb, Bb, b_trans=True).to(A.dtype)
        if ctx.needs_input_grad[1]:
            # dB[K,N] = A^T . dC : A stored [M,K] read MN-major, dC stored [M,N] read MN-major
            dB = gemm_ex(Ab, dCb, a_trans=True)[:K, :N].to(B.dtype)
        return dA, dB


def gemm(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """Differentiable A[M,K] @ B[K,N] -> C[M,N] f32 via the tcgen05 kernel."""
    return _Gemm.apply(A, B)


def matmul(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """``A @ B``: 2-D x 2-D products go to the kernel; other ranks stay a plain
    batched matmul on the device, as reference gemm.py:82-90 routes them.
    CPU tensors raise (there is no CPU path)."""
    _require_cuda(A, B)
    if A.dim() == 2 and B.dim() == 2:
        return gemm(A, B)
    return torch.matmul(A, B)


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, W):
        ctx.save_for_backward(x2, W)
        xb, Wb = _operand(x2), _operand(W)
        y = gemm_ex(xb, Wb, out_dtype=torch.bfloat16 if x2.dtype == torch.bfloat16 else torch.float32)
        return y.to(x2.dtype)

    @staticmethod
    def backward(ctx, dy):
        x2, W = ctx.saved_tensors
        dyb = _operand(dy)
        xb, Wb = _operand(x2), _operand(W)
        dx = dW = None
        if ctx.needs_input_grad[0]:
            dx = gemm_ex(dyb, Wb, b_trans=True,
                         out_dtype=torch.bfloat16 if x2.dtype == torch.bfloat16 else torch.float32).to(x2.dtype)
        if ctx.needs_input_grad[1]:
            dW = gemm_ex(xb, dyb, a_trans=True, epilogue=EPI_ACCUM).to(W.dtype)
        return dx, dW


def linear(x: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
    """``x[..., K] @ W[K, N] -> [..., N]`` as one flattened GEMM, output in x.dtype.
    CPU tensors raise (there is no CPU path)."""
    _require_cuda(x, W)
    if x.dim() >= 2 and W.dim() == 2:
        lead = x.shape[:-1]
        K = x.shape[-1]
        N = W.shape[1]
        if K % 8 == 0 and N % 8 == 0:
            y = _Linear.apply(x.reshape(-1, K), W)
            return y.reshape(*lead, N)
        y = gemm(x.reshape(-1, K), W)
        return y.reshape(*lead, N).to(x.dtype)
    return torch.matmul(x, W)  # other ranks: a plain device matmul, as reference gemm.py:115


__all__ = ["gemm", "matmul", "linear", "gemm_ex"]
