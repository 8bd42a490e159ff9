"""CPU oracle for the nlearn hot-path operators — TEST INFRASTRUCTURE ONLY.

A NumPy restatement of what the reference computes, used as the checker by
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py``.  Nothing in the product path (``nlearn_b200``) imports it.

Pinned: ``tests/golden/make_golden.py`` runs the reference's own functions
(its pure-JAX fallbacks under a NumPy stand-in for ``jax.numpy``, and the NumPy
references inside its kernel tests) on the reference tests' seeded inputs;
``tests/test_oracle_golden.py`` checks every function here against those
fixtures.

All paths are relative to the nlearn reference tree.
"""
from __future__ import annotations

import numpy as np

try:
    import ml_dtypes
    _BF16 = ml_dtypes.bfloat16
except ImportError:  # pragma: no cover
    _BF16 = None


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bfloat16, returned as float32."""
    x = np.asarray(x, np.float32)
    if _BF16 is not None:
        return x.astype(_BF16).astype(np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


# --------------------------------------------------------------------- attention
def attention_fwd(Q, K, V):
    """Causal softmax attention with per-row logsumexp.

    Follows ``_attention_standard`` (nlearn/attention.py:138-156): scores =
    Q K^T / sqrt(d), mask ``pos_i >= pos_j``, softmax, times V; and the L
    definition of the flash kernel's test (iree_metal/kernels/test/
    validate_flash_tiled.py:19-29): L = rowmax + log(rowsum(exp(s - rowmax))),
    natural log, of the SCALED scores.  Shapes [n, s, d] -> O [n, s, d], L [n, s].
    """
    Q = np.asarray(Q, np.float32); K = np.asarray(K, np.float32); V = np.asarray(V, np.float32)
    n, s, d = Q.shape
    scale = np.float32(1.0 / np.sqrt(d))
    sc = np.einsum("nid,njd->nij", Q, K) * scale
    mask = np.triu(np.ones((s, s), bool), 1)
    sc = np.where(mask[None], -np.inf, sc)
    mx = sc.max(-1, keepdims=True)
    e = np.exp(sc - mx)
    l = e.sum(-1, keepdims=True)
    O = np.einsum("nij,njd->nid", e / l, V).astype(np.float32)
    L = (mx[..., 0] + np.log(l[..., 0])).astype(np.float32)
    return O, L


def attention_bwd(Q, K, V, dO):
    """Analytic causal-attention backward, as in the reference's flash test
    (iree_metal/kernels/test/validate_flash_bwd.py:30-38):
    dp = dO V^T; ds = p (dp - rowsum(dp p)); dQ = ds K scale; dK = ds^T Q scale;
    dV = p^T dO.  Also returns D = rowsum(dO * O) (nlearn/attention.py:116)."""
    Q = np.asarray(Q, np.float32); K = np.asarray(K, np.float32)
    V = np.asarray(V, np.float32); dO = np.asarray(dO, np.float32)
    n, s, d = Q.shape
    scale = np.float32(1.0 / np.sqrt(d))
    sc = np.einsum("nid,njd->nij", Q, K) * scale
    mask = np.triu(np.ones((s, s), bool), 1)
    sc = np.where(mask[None], -np.inf, sc)
    p = np.exp(sc - sc.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    O = np.einsum("nij,njd->nid", p, V)
    dV = np.einsum("nij,nid->njd", p, dO)
    dp = np.einsum("nid,njd->nij", dO, V)
    ds = p * (dp - (dp * p).sum(-1, keepdims=True))
    dQ = np.einsum("nij,njd->nid", ds, K) * scale
    dK = np.einsum("nij,nid->njd", ds, Q) * scale
    D = (dO * O).sum(-1)
    return dQ.astype(np.float32), dK.astype(np.float32), dV.astype(np.float32), D.astype(np.float32)


# --------------------------------------------------------------------- GEMM
def gemm(A, B):
    """C f32 = A @ B with bf16-rounded operands and f32 accumulation
    (iree_metal/kernels/test/check_gemm_bf16.py:16-19; nlearn/kernels/gemm.py:43-58)."""
    return bf16_round(A) @ bf16_round(B)


def gemm_bwd(A, B, dC):
    """dA = dC B^T, dB = A^T dC (nlearn/kernels/gemm.py:71-76), bf16 operands."""
    A, B, dC = bf16_round(A), bf16_round(B), bf16_round(dC)
    return dC @ B.T, A.T @ dC


# --------------------------------------------------------------------- CE
def ce_fwd(logits, targets):
    """Per-row loss and logsumexp (iree_metal/kernels/cross_entropy.metal:38-68):
    lse = log(sum(exp(row))), loss = lse - row[target]."""
    x = np.asarray(logits, np.float64)
    t = np.asarray(targets, np.int64)
    m = x.max(-1, keepdims=True)
    lse = (m[:, 0] + np.log(np.exp(x - m).sum(-1)))
    loss = lse - x[np.arange(x.shape[0]), t]
    return loss.astype(np.float32), lse.astype(np.float32)


def ce_bwd(logits, targets, lse, scale=None):
    """dlogits = (softmax - onehot) * scale, scale defaulting to 1/M
    (iree_metal/kernels/cross_entropy.metal:81-97)."""
    x = np.asarray(logits, np.float64)
    M = x.shape[0]
    sc = (1.0 / M) if scale is None else scale
    d = np.exp(x - np.asarray(lse, np.float64)[:, None])
    d[np.arange(M), np.asarray(targets, np.int64)] -= 1.0
    return (d * sc).astype(np.float32)


def cross_entropy(logits, targets):
    """Mean softmax CE (nlearn/kernels/cross_entropy.py:71-81)."""
    loss, _ = ce_fwd(np.asarray(logits).reshape(-1, np.shape(logits)[-1]), np.asarray(targets).reshape(-1))
    return float(loss.astype(np.float64).mean())


# --------------------------------------------------------------------- fused LM-head CE
def linear_cross_entropy(X, W, targets, bf16_operands=False):
    """Loss, lse, dX, dW of mean CE over logits = X @ W
    (iree_metal/kernels/test/check_lce.py:14-29 ``ref_np``; chunked semantics
    of nlearn/kernels/cross_entropy.py:106-167 are exact up to rounding, so the
    unchunked form is the oracle).  With ``bf16_operands`` the GEMM operands
    (X, W and dlogits) are rounded to bf16 as the B200 kernels consume them."""
    X = np.asarray(X, np.float32); W = np.asarray(W, np.float32)
    if bf16_operands:
        X, W = bf16_round(X), bf16_round(W)
    t = np.asarray(targets, np.int64)
    M = X.shape[0]
    logits = (X @ W).astype(np.float64)
    m = logits.max(1, keepdims=True)
    z = np.exp(logits - m)
    lse = m[:, 0] + np.log(z.sum(1))
    loss = float((lse - logits[np.arange(M), t]).mean())
    dl = z / z.sum(1, keepdims=True)
    dl[np.arange(M), t] -= 1.0
    dl = (dl / M).astype(np.float32)
    if bf16_operands:
        dl = bf16_round(dl)
    dX = dl @ W.T
    dW = X.T @ dl
    return loss, lse.astype(np.float32), dX.astype(np.float32), dW.astype(np.float32)
