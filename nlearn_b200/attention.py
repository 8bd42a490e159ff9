"""Causal attention on the sm_100a flash kernels — mirror of nlearn.attention.

Reference surface (nlearn/attention.py):
  * ``_flash_fwd_raw(Q, K, V) -> (O, L)``   custom call `flash_attention_fwd` (82-91)
  * ``_attention_iree_flash(Q, K, V)``      custom_vjp; residuals Q,K,V,O,L;
                                            bwd computes D = rowsum(dO*O) then
                                            calls `flash_attention_bwd_dq` and
                                            `flash_attention_bwd_dkdv` (94-131)
  * ``attention(Q, K, V)``                  platform dispatch (188-199)

Here the custom_vjp is a ``torch.autograd.Function`` over the C ABI.  Shapes
are ``(n_heads_total, seq, 64)``.  The three custom-call targets are mirrored
one to one by ``flash_attention_fwd`` / ``flash_attention_bwd_dq`` /
``flash_attention_bwd_dkdv``, which take and return the dtype they are given:
f32 (what the reference's wrappers send, attention.py:97, converted to bf16
tensor-core operands and back inside the library, ``nl_flash_attention_*_dt``)
or bf16.  With f32 inputs ``_attention_iree_flash`` follows the reference's
rule exactly (fwd target; D = rowsum(dO*O); dq and dkdv targets).  With bf16
inputs (the B200 fast path) the backward is ONE fused launch (plus a D/zero
pre-pass and a dQ convert) instead of two kernels that both recompute P.

There is deliberately no CPU / standard-attention fallback: CPU tensors raise.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_handle

HEAD_DIM = 64


def _check(x: torch.Tensor) -> None:
    if not x.is_cuda:
        raise ValueError("nlearn_b200 attention runs on CUDA tensors only (no CPU fallback)")
    if x.dim() != 3 or x.shape[-1] != HEAD_DIM:
        raise ValueError(f"expected (n, s, {HEAD_DIM}), got {tuple(x.shape)}")


def _prep(x: torch.Tensor) -> torch.Tensor:
    _check(x)
    return x.to(torch.bfloat16).contiguous()


def _same(x: torch.Tensor, dtype) -> torch.Tensor:
    """x in `dtype` (f32 or bf16), contiguous, for the dtype-dispatching targets."""
    _check(x)
    return x.to(dtype).contiguous()


def _io_dtype(x: torch.Tensor):
    return torch.float32 if x.dtype == torch.float32 else torch.bfloat16


_NL_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}


def _workspace(target: int, n: int, s: int, dtype, dev) -> tuple:
    nb = lib.nl_flash_attention_workspace_bytes(target, n, s, HEAD_DIM, _NL_DT[dtype])
    ws = torch.empty(max(nb, 1), device=dev, dtype=torch.uint8)
    return ws, nb


def flash_attention_fwd(Q, K, V):
    """Target `flash_attention_fwd` (nlearn/attention.py:82-91): (n,s,64) f32
    or bf16 -> O in the same dtype, L f32 (n,s) = logsumexp of scaled scores."""
    dt = _io_dtype(Q)
    Qc, Kc, Vc = _same(Q, dt), _same(K, dt), _same(V, dt)
    n, s, d = Qc.shape
    O = torch.empty_like(Qc)
    L = torch.empty(n, s, device=Qc.device, dtype=torch.float32)
    ws, nb = _workspace(0, n, s, dt, Qc.device)
    check(lib.nl_flash_attention_fwd_dt(ptr(Qc), ptr(Kc), ptr(Vc), ptr(O), ptr(L), n, s, d, _NL_DT[dt], ptr(ws), nb,
                                        stream_handle()), "nl_flash_attention_fwd_dt")
    return O, L


def flash_attention_bwd_dq(Q, K, V, dO, L, D):
    """Target `flash_attention_bwd_dq` (attention.py:117-121; explicit D):
    dQ in the operands' dtype (f32 or bf16)."""
    dt = _io_dtype(Q)
    Qc, Kc, Vc, dOc = (_same(t, dt) for t in (Q, K, V, dO))
    n, s, d = Qc.shape
    dQ = torch.empty_like(Qc)
    ws, nb = _workspace(1, n, s, dt, Qc.device)
    check(lib.nl_flash_attention_bwd_dq_dt(ptr(Qc), ptr(Kc), ptr(Vc), ptr(dOc), ptr(L.float().contiguous()),
                                           ptr(D.float().contiguous()), ptr(dQ), n, s, d, _NL_DT[dt], ptr(ws), nb,
                                           stream_handle()), "nl_flash_attention_bwd_dq_dt")
    return dQ


def flash_attention_bwd_dkdv(Q, K, V, dO, L, D):
    """Target `flash_attention_bwd_dkdv` (attention.py:122-126; explicit D):
    (dK, dV) in the operands' dtype (f32 or bf16)."""
    dt = _io_dtype(Q)
    Qc, Kc, Vc, dOc = (_same(t, dt) for t in (Q, K, V, dO))
    n, s, d = Qc.shape
    dK, dV = torch.empty_like(Qc), torch.empty_like(Qc)
    ws, nb = _workspace(2, n, s, dt, Qc.device)
    check(lib.nl_flash_attention_bwd_dkdv_dt(ptr(Qc), ptr(Kc), ptr(Vc), ptr(dOc), ptr(L.float().contiguous()),
                                             ptr(D.float().contiguous()), ptr(dK), ptr(dV), n, s, d, _NL_DT[dt],
                                             ptr(ws), nb, stream_handle()), "nl_flash_attention_bwd_dkdv_dt")
    return dK, dV


def _flash_fwd_raw(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor):
    """(n,s,64) -> O (n,s,64) in the input dtype (f32 stays f32, anything else
    runs as bf16), L f32 (n,s) = logsumexp of scaled scores."""
    return flash_attention_fwd(Q, K, V)


def _flash_bwd_raw(Q, K, V, O, L, dO):
    """Fused bf16 backward -> dQ, dK, dV (bf16): one launch computes D, dQ, dK, dV."""
    Qb, Kb, Vb, Ob, dOb = _prep(Q), _prep(K), _prep(V), _prep(O), _prep(dO)
    n, s, d = Qb.shape
    dQ = torch.empty_like(Qb)
    dK = torch.empty_like(Qb)
    dV = torch.empty_like(Qb)
    D = torch.empty(n, s, device=Qb.device, dtype=torch.float32)
    dQacc = torch.empty(n, s, d, device=Qb.device, dtype=torch.float32)
    check(lib.nl_flash_attention_bwd(ptr(Qb), ptr(Kb), ptr(Vb), ptr(Ob), ptr(dOb), ptr(L), ptr(D), ptr(dQ), ptr(dK),
                                     ptr(dV), ptr(dQacc), n, s, d, stream_handle()), "nl_flash_attention_bwd")
    return dQ, dK, dV


class _FlashAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, K, V):
        O, L = _flash_fwd_raw(Q, K, V)
        ctx.save_for_backward(Q, K, V, O, L)
        ctx.in_dtype = Q.dtype
        return O.to(Q.dtype)

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, O, L = ctx.saved_tensors
        dt = ctx.in_dtype
        if O.dtype == torch.float32:
            # the reference's rule (attention.py:111-128): D = rowsum(dO * O),
            # then the dq and dkdv targets on f32 operands
            dOf = dO.float().contiguous()
            D = (dOf * O).sum(-1)
            dQ = flash_attention_bwd_dq(Q, K, V, dOf, L, D)
            dK, dV = flash_attention_bwd_dkdv(Q, K, V, dOf, L, D)
        else:
            dQ, dK, dV = _flash_bwd_raw(Q, K, V, O, L, dO)
        return dQ.to(dt), dK.to(dt), dV.to(dt)


def _attention_flash(Q, K, V):
    """Causal flash attention with O(seq) memory in forward and backward."""
    return _FlashAttention.apply(Q, K, V)


# drop-in name of the reference's custom_vjp (nlearn/attention.py:94)
_attention_iree_flash = _attention_flash


def attention(Q, K, V):
    """Causal attention, Q/K/V (n_heads_total, seq_len, 64) -> same shape."""
    return _attention_flash(Q, K, V)


__all__ = ["attention", "_attention_flash", "_attention_iree_flash", "_flash_fwd_raw", "_flash_bwd_raw",
           "flash_attention_fwd", "flash_attention_bwd_dq", "flash_attention_bwd_dkdv"]
