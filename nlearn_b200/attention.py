"""Causal attention on the sm_100a flash kernels — mirror of nlearn.attention.

Reference surface (nlearn/attention.py):
  * ``_flash_fwd_raw(Q, K, V) -> (O, L)``   custom call `flash_attention_fwd` (82-91)
  * ``_attention_iree_flash(Q, K, V)``      custom_vjp; residuals Q,K,V,O,L;
                                            bwd computes D = rowsum(dO*O) then
                                            calls `flash_attention_bwd_dq` and
                                            `flash_attention_bwd_dkdv` (94-131)
  * ``attention(Q, K, V)``                  platform dispatch (188-199)

Here the custom_vjp is a ``torch.autograd.Function`` over the C ABI
(``nl_flash_attention_fwd`` / ``nl_flash_attention_bwd``).  Shapes are
``(n_heads_total, seq, 64)``.  The reference casts to f32 at the boundary
(attention.py:97) because its Metal target lacks bf16; the B200 kernels take
bf16 operands, so inputs are cast to bf16 and outputs returned in the input
dtype.  The backward is ONE fused launch (plus a D/zero pre-pass and a dQ
convert) instead of two kernels that both recompute P.

There is deliberately no CPU / standard-attention fallback: CPU tensors raise.
"""
from __future__ import annotations

import torch

from ._lib import check, lib, ptr, stream_handle

HEAD_DIM = 64


def _prep(x: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        raise ValueError("nlearn_b200 attention runs on CUDA tensors only (no CPU fallback)")
    if x.dim() != 3 or x.shape[-1] != HEAD_DIM:
        raise ValueError(f"expected (n, s, {HEAD_DIM}), got {tuple(x.shape)}")
    return x.to(torch.bfloat16).contiguous()


def _flash_fwd_raw(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor):
    """(n,s,64) -> O bf16 (n,s,64), L f32 (n,s) = logsumexp of scaled scores."""
    Qb, Kb, Vb = _prep(Q), _prep(K), _prep(V)
    n, s, d = Qb.shape
    O = torch.empty_like(Qb)
    L = torch.empty(n, s, device=Qb.device, dtype=torch.float32)
    check(lib.nl_flash_attention_fwd(ptr(Qb), ptr(Kb), ptr(Vb), ptr(O), ptr(L), n, s, d, stream_handle()),
          "nl_flash_attention_fwd")
    return O, L


def _flash_bwd_raw(Q, K, V, O, L, dO):
    """Fused backward -> dQ, dK, dV (bf16)."""
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


def flash_attention_bwd_dq(Q, K, V, dO, L, D):
    """Reference target `flash_attention_bwd_dq` (explicit D)."""
    Qb, Kb, Vb, dOb = _prep(Q), _prep(K), _prep(V), _prep(dO)
    n, s, d = Qb.shape
    dQ = torch.empty_like(Qb)
    dQacc = torch.empty(n, s, d, device=Qb.device, dtype=torch.float32)
    check(lib.nl_flash_attention_bwd_dq(ptr(Qb), ptr(Kb), ptr(Vb), ptr(dOb), ptr(L.float().contiguous()),
                                        ptr(D.float().contiguous()), ptr(dQ), ptr(dQacc), n, s, d, stream_handle()),
          "nl_flash_attention_bwd_dq")
    return dQ


def flash_attention_bwd_dkdv(Q, K, V, dO, L, D):
    """Reference target `flash_attention_bwd_dkdv` (explicit D)."""
    Qb, Kb, Vb, dOb = _prep(Q), _prep(K), _prep(V), _prep(dO)
    n, s, d = Qb.shape
    dK = torch.empty_like(Qb)
    dV = torch.empty_like(Qb)
    check(lib.nl_flash_attention_bwd_dkdv(ptr(Qb), ptr(Kb), ptr(Vb), ptr(dOb), ptr(L.float().contiguous()),
                                          ptr(D.float().contiguous()), ptr(dK), ptr(dV), n, s, d, stream_handle()),
          "nl_flash_attention_bwd_dkdv")
    return dK, dV


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
        dQ, dK, dV = _flash_bwd_raw(Q, K, V, O, L, dO)
        dt = ctx.in_dtype
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
           "flash_attention_bwd_dq", "flash_attention_bwd_dkdv"]
