"""Softmax cross-entropy on the sm_100a kernels — mirror of nlearn.kernels.cross_entropy.

Reference surface (nlearn/kernels/cross_entropy.py):
  * ``_ce_fwd_raw(logits, targets) -> (loss[M], lse[M])``   target `ce_fwd` (28-36)
  * ``_ce_bwd_raw(logits, targets, lse) -> dlogits / M``    target `ce_bwd` (39-46)
  * ``cross_entropy(logits, targets)``  mean CE, custom_vjp, flattens (49-81)
  * ``linear_cross_entropy(X, W, targets)`` LM head + CE without the (M, V)
    logits, custom_vjp; backward recomputes the logits (85-170)

``linear_cross_entropy`` runs the fused LM-head kernels (``nl_lce_fwd`` /
``nl_lce_bwd``): the GEMM epilogue reduces each 128x256 logit tile to per-row
(max, sum-exp) partials, and the backward turns each recomputed tile straight
into bf16 dlogits for the dX / dW GEMMs, one vocabulary chunk at a time.
"""
from __future__ import annotations

import os

import torch

from .._lib import BF16, F32, check, lib, ptr, stream_handle

_DT = {torch.float32: F32, torch.bfloat16: BF16}


def _rows(logits: torch.Tensor) -> torch.Tensor:
    if not logits.is_cuda:
        raise ValueError("nlearn_b200 cross-entropy runs on CUDA tensors only (no CPU fallback)")
    if logits.dtype not in _DT:
        logits = logits.float()
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    return logits


def _ce_fwd_raw(logits: torch.Tensor, targets: torch.Tensor):
    """logits[M,V] (f32 or bf16; any row pitch), targets[M] -> (loss[M], lse[M]) f32."""
    lg = _rows(logits)
    M, V = lg.shape
    t = targets.to(torch.int32).contiguous()
    loss = torch.empty(M, device=lg.device, dtype=torch.float32)
    lse = torch.empty(M, device=lg.device, dtype=torch.float32)
    check(lib.nl_ce_fwd(ptr(lg), lg.stride(0), _DT[lg.dtype], ptr(t), ptr(loss), ptr(lse), M, V, stream_handle()),
          "nl_ce_fwd")
    return loss, lse


def _ce_bwd_raw(logits: torch.Tensor, targets: torch.Tensor, lse: torch.Tensor, scale: float | None = None,
                out_dtype=None, out: torch.Tensor | None = None):
    """dlogits = (softmax - onehot) * scale, scale defaulting to 1/M (the reference's)."""
    lg = _rows(logits)
    M, V = lg.shape
    t = targets.to(torch.int32).contiguous()
    if out is None:
        out = torch.empty(M, V, device=lg.device, dtype=out_dtype or lg.dtype)
    sc = (1.0 / M) if scale is None else float(scale)
    check(lib.nl_ce_bwd(ptr(lg), lg.stride(0), _DT[lg.dtype], ptr(t), ptr(lse.float().contiguous()), ptr(out),
                        out.stride(0), _DT[out.dtype], M, V, sc, stream_handle()), "nl_ce_bwd")
    return out


def ce_fwd_bwd(logits: torch.Tensor, targets: torch.Tensor, scale: float | None = None,
               out: torch.Tensor | None = None, out_dtype=None):
    """Fused: loss[M], lse[M] and dlogits from one read of the logits.
    ``out`` may be ``logits`` itself (in-place gradient)."""
    lg = _rows(logits)
    M, V = lg.shape
    t = targets.to(torch.int32).contiguous()
    loss = torch.empty(M, device=lg.device, dtype=torch.float32)
    lse = torch.empty(M, device=lg.device, dtype=torch.float32)
    if out is None:
        out = torch.empty(M, V, device=lg.device, dtype=out_dtype or lg.dtype)
    sc = (1.0 / M) if scale is None else float(scale)
    check(lib.nl_ce_fwd_bwd(ptr(lg), lg.stride(0), _DT[lg.dtype], ptr(t), ptr(loss), ptr(lse), ptr(out),
                            out.stride(0), _DT[out.dtype], M, V, sc, stream_handle()), "nl_ce_fwd_bwd")
    return loss, lse, out


class _CE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets):
        loss, lse = _ce_fwd_raw(logits, targets)
        ctx.save_for_backward(logits, targets, lse)
        return loss.mean()

    @staticmethod
    def backward(ctx, g):
        logits, targets, lse = ctx.saved_tensors
        d = _ce_bwd_raw(logits, targets, lse, scale=None, out_dtype=logits.dtype if logits.dtype in _DT
                        else torch.float32)
        return d * g.to(d.dtype), None


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean softmax cross-entropy; leading dims flattened to (M, V)."""
    V = logits.shape[-1]
    return _CE.apply(logits.reshape(-1, V), targets.reshape(-1))


# Vocabulary chunk of the fused backward (the reference's NLEARN_LCE_CHUNK,
# cross_entropy.py:91), a target width in columns.  Unset, the chunk is as wide
# as a 2 GiB bf16 dlogits buffer allows (the whole vocabulary at M = 16384):
# fewer, larger GEMMs measured fastest on B200.
_LCE_CHUNK_ENV = os.environ.get("NLEARN_LCE_CHUNK")
_LCE_CHUNK_BUDGET = 2 << 30


def _default_chunk(M: int) -> int:
    if _LCE_CHUNK_ENV:
        return max(64, int(_LCE_CHUNK_ENV))
    return max(4096, _LCE_CHUNK_BUDGET // (2 * max(M, 1)))


def _lce_operands(X, W):
    Xb = X.to(torch.bfloat16)
    if Xb.stride(-1) != 1 or Xb.stride(0) % 8 or Xb.data_ptr() % 16:
        Xb = Xb.contiguous()
    Wb = W.to(torch.bfloat16)
    D, V = Wb.shape
    if Wb.stride(-1) != 1 or Wb.stride(0) % 8 or Wb.data_ptr() % 16:
        Vp = (V + 7) // 8 * 8
        Wp = torch.zeros(D, Vp, device=Wb.device, dtype=torch.bfloat16)
        Wp[:, :V] = Wb
        Wb = Wp[:, :V]
    return Xb, Wb


def lce_fwd_raw(Xb, Wb, t):
    """-> loss[M], lse[M] (f32) through nl_lce_fwd."""
    M, D = Xb.shape
    V = Wb.shape[1]
    loss = torch.empty(M, device=Xb.device, dtype=torch.float32)
    lse = torch.empty(M, device=Xb.device, dtype=torch.float32)
    nbytes = lib.nl_lce_workspace_bytes(M, V, 0)
    ws = torch.empty(nbytes, device=Xb.device, dtype=torch.uint8)
    check(lib.nl_lce_fwd(ptr(Xb), Xb.stride(0), ptr(Wb), Wb.stride(0), ptr(t), ptr(loss), ptr(lse), ptr(ws), nbytes,
                         M, D, V, stream_handle()), "nl_lce_fwd")
    return loss, lse


def _balanced_chunk(V: int, target: int) -> int:
    """Chunk width near `target` that splits V into equal parts (a multiple of
    256 columns), so that no thin tail chunk runs at poor GEMM efficiency."""
    n = max(1, round(V / target))
    return min(-(-V // n) + 255, (V + 255)) // 256 * 256 if V > 0 else 256


def lce_bwd_raw(Xb, Wb, t, lse, g=None, dX=None, dW=None, dw_accumulate=False, chunk=None):
    """-> dX f32 [M,D] (accumulated into `dX` if given), dW f32 [D,V] (row pitch of W).
    `chunk` (default NLEARN_LCE_CHUNK) is the target vocabulary chunk width."""
    M, D = Xb.shape
    V = Wb.shape[1]
    chunk = _balanced_chunk(V, chunk or _default_chunk(M))
    if dX is None:
        dX = torch.zeros(M, D, device=Xb.device, dtype=torch.float32)
    if dW is None:
        dW = torch.empty(D, Wb.stride(0), device=Xb.device, dtype=torch.float32)[:, :V]
    gp = None if g is None else g.detach().float().reshape(1).contiguous()
    nbytes = lib.nl_lce_workspace_bytes(M, V, chunk)
    ws = torch.empty(nbytes, device=Xb.device, dtype=torch.uint8)
    check(lib.nl_lce_bwd(ptr(Xb), Xb.stride(0), ptr(Wb), Wb.stride(0), ptr(t), ptr(lse), ptr(gp), 1.0 / M, ptr(dX),
                         ptr(dW), dW.stride(0), int(dw_accumulate), ptr(ws), nbytes, chunk, M, D, V,
                         stream_handle()), "nl_lce_bwd")
    return dX, dW


def lce_bwd_bf16_dx(Xb, Wb, t, lse, dW, dw_accumulate=True):
    """-> dX bf16 [M, D] written (not accumulated) by the LM head's dX GEMM
    (nl_lce_bwd_ex), with dW as lce_bwd_raw: no zeroed f32 dX and no cast
    pass.  Needs one vocabulary chunk (the default at the step's sizes);
    otherwise it accumulates in f32 and casts."""
    M, D = Xb.shape
    V = Wb.shape[1]
    chunk = _balanced_chunk(V, _default_chunk(M))
    if chunk < V:
        dX, _ = lce_bwd_raw(Xb, Wb, t, lse, dW=dW, dw_accumulate=dw_accumulate, chunk=chunk)
        return dX.to(torch.bfloat16)
    dX = torch.empty(M, D, device=Xb.device, dtype=torch.bfloat16)
    nbytes = lib.nl_lce_workspace_bytes(M, V, chunk)
    ws = torch.empty(nbytes, device=Xb.device, dtype=torch.uint8)
    check(lib.nl_lce_bwd_ex(ptr(Xb), Xb.stride(0), ptr(Wb), Wb.stride(0), ptr(t), ptr(lse), None, 1.0 / M, ptr(dX),
                            BF16, 0, ptr(dW), dW.stride(0), int(dw_accumulate), ptr(ws), nbytes, chunk, M, D, V,
                            stream_handle()), "nl_lce_bwd_ex")
    return dX


class _LCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X, W, targets):
        Xb, Wb = _lce_operands(X, W)
        t = targets.reshape(-1).to(torch.int32).contiguous()
        loss, lse = lce_fwd_raw(Xb, Wb, t)
        ctx.save_for_backward(Xb, Wb, t, lse)
        ctx.dtypes = (X.dtype, W.dtype)
        return loss.mean()

    @staticmethod
    def backward(ctx, g):
        Xb, Wb, t, lse = ctx.saved_tensors
        dX, dW = lce_bwd_raw(Xb, Wb, t, lse, g=g)
        return dX.to(ctx.dtypes[0]), dW.to(ctx.dtypes[1]), None


def linear_cross_entropy(X: torch.Tensor, W: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean softmax CE of logits = X[M,D] @ W[D,V] against targets[M], without
    materialising the (M, V) logits (reference cross_entropy.py:131-136)."""
    if not X.is_cuda:
        raise ValueError("nlearn_b200 linear_cross_entropy runs on CUDA tensors only (no CPU fallback)")
    return _LCE.apply(X, W, targets)


__all__ = ["cross_entropy", "linear_cross_entropy", "_ce_fwd_raw", "_ce_bwd_raw", "ce_fwd_bwd", "lce_fwd_raw",
           "lce_bwd_raw", "lce_bwd_bf16_dx"]
