/* nl_ops.h — C ABI of the nlearn-b200 hot-path kernels (sm_100a).
 *
 * These entry points replace the custom-call targets that nlearn's IREE pass
 * lowers to Metal dispatches (iree_metal/patches/08-gemm-dispatch-pass.patch:
 * 230-236 matches the names `flash_attention_fwd`, `flash_attention_bwd_dq`,
 * `flash_attention_bwd_dkdv`, `gemm`, `ce_fwd`, `ce_bwd`), plus the fused
 * additions the B200 path needs.
 *
 * Conventions (all entry points):
 *  - every pointer is a DEVICE pointer owned by the caller; matrices are
 *    row-major with an explicit leading dimension in elements;
 *  - work is enqueued on `stream`; nothing synchronises, nothing allocates
 *    (scratch, where needed, is a caller-provided workspace);
 *  - the return value is an nl_status: 0 on success, negative on a rejected
 *    shape / alignment / dtype or a failed launch.  Kernel-side conditions
 *    (bounded-wait timeouts, position guards) are reported through
 *    nl_get_device_error().
 */
#ifndef NL_OPS_H
#define NL_OPS_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#if defined(__GNUC__)
#define NL_API __attribute__((visibility("default")))
#else
#define NL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  NL_OK = 0,
  NL_ERR_SHAPE = -1,     /* unsupported or inconsistent dimensions          */
  NL_ERR_ALIGN = -2,     /* pointer / leading dimension not 16-byte aligned */
  NL_ERR_LAUNCH = -3,    /* kernel launch failed                            */
  NL_ERR_CUDA = -4,      /* CUDA runtime / driver entry point unavailable   */
  NL_ERR_DTYPE = -5,     /* unsupported dtype code                          */
  NL_ERR_WORKSPACE = -6, /* workspace missing or too small                  */
  NL_ERR_TOO_LARGE = -7  /* problem exceeds a fixed built-in scratch limit   */
} nl_status;

typedef enum { NL_F32 = 0, NL_BF16 = 1 } nl_dtype;

/* GEMM epilogue selector for nl_gemm_ex. */
typedef enum {
  NL_EPI_STORE = 0,     /* C = alpha*A.B                 (C in c_dtype)        */
  NL_EPI_ACCUM = 1,     /* C += alpha*A.B                (C f32; split-K safe) */
  NL_EPI_BIAS = 2,      /* C = alpha*A.B + bias[N]       (bias f32)            */
  NL_EPI_BIAS_GELU = 3, /* aux = A.B + bias; C = gelu_tanh(aux)  (C, aux bf16) */
  NL_EPI_RESID = 4,     /* C = alpha*A.B + bias? + resid (resid in c_dtype)    */
  NL_EPI_DGELU = 5,     /* C = (alpha*A.B) * gelu_tanh'(aux)   (C, aux bf16)   */
  NL_EPI_LCE_STATS = 6, /* internal: fused LM-head CE partial row statistics   */
  NL_EPI_LCE_GRAD = 7   /* internal: fused LM-head CE dlogits (bf16)           */
} nl_epilogue;

/* Library / device introspection. */
NL_API const char* nl_version(void);
/* Reads and clears the device-side error word (1 = a bounded wait timed out,
 * 2 = misaligned shared memory, 3 = a decode position outside the KV cache or
 * the output row).  Synchronises `stream`. */
NL_API int nl_get_device_error(cudaStream_t stream);
/* Kernels launched by this library so far in this process (host-side count). */
NL_API long long nl_launch_count(void);

/* ---------------------------------------------------------------- GEMM
 * Replaces target `gemm` (nlearn/kernels/gemm.py:32-40 `_gemm_raw`;
 * iree_metal/kernels/gemm.metal:48-115): C f32[M,N] = A bf16[M,K] @ B bf16[K,N],
 * all row-major and contiguous.  K, N must be multiples of 8 (16-byte rows);
 * unlike the Metal kernel there is no padding requirement on M/N/K tiles. */
NL_API int nl_gemm(const void* A, const void* B, float* C, int M, int N, int K, cudaStream_t stream);

/* General form used by linear / its backward (nlearn/kernels/gemm.py:67-79
 * `_gemm_fwd`/`_gemm_bwd`) without materialised transposes:
 *   logical A is [M,K]: a_trans=0 -> stored [M,K] (lda>=K); 1 -> stored [K,M] (lda>=M)
 *   logical B is [K,N]: b_trans=0 -> stored [K,N] (ldb>=N); 1 -> stored [N,K] (ldb>=K)
 *   C [M,N] row-major, ldc, dtype c_dtype (NL_F32 / NL_BF16).
 * `bias` (f32[N]), `aux` (bf16 [M,N], ldc) and `resid` ([M,N], ldc, c_dtype)
 * are used by the epilogues that name them and may be NULL otherwise.
 * Leading dimensions of A and B must be multiples of 8 elements. */
NL_API int nl_gemm_ex(const void* A, int lda, int a_trans, const void* B, int ldb, int b_trans, void* C, int ldc,
               int c_dtype, int M, int N, int K, float alpha, int epilogue, const float* bias, void* aux,
               const void* resid, cudaStream_t stream);

/* ---------------------------------------------------------------- cross-entropy
 * Replaces targets `ce_fwd` / `ce_bwd` (nlearn/kernels/cross_entropy.py:28-46;
 * iree_metal/kernels/cross_entropy.metal:38-68, 81-97).  logits [M,V] row-major
 * with row pitch ld (any value >= V), dtype NL_F32 (the reference's) or NL_BF16;
 * targets int32 [M].  A target outside [0,V) contributes loss = lse and no
 * one-hot term.
 *   nl_ce_fwd:     loss[M] = lse - logits[target], lse[M] = logsumexp(row)
 *   nl_ce_bwd:     dlogits = (softmax(row) - onehot) * scale   (reference scale = 1/M)
 *   nl_ce_fwd_bwd: both from one HBM read of the logits; dlogits may alias logits. */
NL_API int nl_ce_fwd(const void* logits, long long ld, int in_dtype, const int* targets, float* loss, float* lse,
                     int M, int V, cudaStream_t stream);
NL_API int nl_ce_bwd(const void* logits, long long ld, int in_dtype, const int* targets, const float* lse,
                     void* dlogits, long long ldd, int out_dtype, int M, int V, float scale, cudaStream_t stream);
NL_API int nl_ce_fwd_bwd(const void* logits, long long ld, int in_dtype, const int* targets, float* loss,
                         float* lse, void* dlogits, long long ldd, int out_dtype, int M, int V, float scale,
                         cudaStream_t stream);

/* ---------------------------------------------------------------- flash attention
 * Causal attention over [n = batch*heads, s, d] row-major tensors, d == 64,
 * scale 1/sqrt(d), any s >= 1.  Q/K/V/O/dO and the gradients are bf16 (the
 * reference casts to f32 at its boundary, nlearn/attention.py:97; on B200 the
 * tensor-core operands are bf16 and the caller casts); L and D are f32 [n,s].
 *
 * Replaces target `flash_attention_fwd` (nlearn/attention.py:82-91;
 * iree_metal/kernels/flash_attention.metal:55-146): O, and L = logsumexp of the
 * scaled scores (natural log) per query row. */
NL_API int nl_flash_attention_fwd(const void* Q, const void* K, const void* V, void* O, float* L, int n, int s,
                                  int d, cudaStream_t stream);

/* Fused backward (one launch for dQ, dK, dV; nlearn/attention.py:111-128 calls
 * the two reference targets below).  Computes D = rowsum(dO*O) into D_ws
 * (f32 [n,s]) and accumulates dQ in dQacc_ws (f32 [n,s,64] scratch, any
 * contents on entry: it is zeroed here). */
NL_API int nl_flash_attention_bwd(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                                  const float* L, float* D_ws, void* dQ, void* dK, void* dV, float* dQacc_ws, int n,
                                  int s, int d, cudaStream_t stream);

/* Replaces target `flash_attention_bwd_dq` (nlearn/attention.py:117-121;
 * flash_attention.metal:168-243): dQ from Q,K,V,dO,L and the given D.
 * dQacc_ws: f32 [n,s,64] scratch. */
NL_API int nl_flash_attention_bwd_dq(const void* Q, const void* K, const void* V, const void* dO, const float* L,
                                     const float* D, void* dQ, float* dQacc_ws, int n, int s, int d,
                                     cudaStream_t stream);

/* Replaces target `flash_attention_bwd_dkdv` (nlearn/attention.py:122-126;
 * flash_attention.metal:265-347): dK, dV from Q,K,V,dO,L and the given D. */
NL_API int nl_flash_attention_bwd_dkdv(const void* Q, const void* K, const void* V, const void* dO,
                                       const float* L, const float* D, void* dK, void* dV, int n, int s, int d,
                                       cudaStream_t stream);

/* Dtype-dispatching forms of the three targets above, taking operands and
 * results in the dtype the reference's custom calls carry them: nlearn's
 * wrappers cast Q, K, V, dO to f32 and receive f32 O, dQ, dK, dV
 * (nlearn/attention.py:82-91, 97, 111-128; the ABI table of
 * iree_metal/patches/08-gemm-dispatch-pass.patch:57-123).  `dtype` (NL_F32 or
 * NL_BF16) applies to Q, K, V, O, dO, dQ, dK, dV; L and D are f32 [n, s].
 * For NL_F32 the library converts to bf16 tensor-core operands and back on
 * `stream` inside `workspace` (caller-owned, 256-byte aligned, at least
 * nl_flash_attention_workspace_bytes(target, n, s, d, dtype) bytes; target
 * 0 = fwd, 1 = bwd_dq, 2 = bwd_dkdv); dQ is widened from the f32 accumulator.
 * An XLA FFI handler registered under each reference target name calls these
 * with the operand order of the table (the handler's scratch allocator
 * provides the workspace). */
NL_API size_t nl_flash_attention_workspace_bytes(int target, int n, int s, int d, int dtype);
NL_API int nl_flash_attention_fwd_dt(const void* Q, const void* K, const void* V, void* O, float* L, int n, int s,
                                     int d, int dtype, void* workspace, size_t ws_bytes, cudaStream_t stream);
NL_API int nl_flash_attention_bwd_dq_dt(const void* Q, const void* K, const void* V, const void* dO, const float* L,
                                        const float* D, void* dQ, int n, int s, int d, int dtype, void* workspace,
                                        size_t ws_bytes, cudaStream_t stream);
NL_API int nl_flash_attention_bwd_dkdv_dt(const void* Q, const void* K, const void* V, const void* dO,
                                          const float* L, const float* D, void* dK, void* dV, int n, int s, int d,
                                          int dtype, void* workspace, size_t ws_bytes, cudaStream_t stream);

/* Allocation-free variant of nl_flash_attention_bwd, for callers that cannot
 * allocate device memory (no workspace argument).  No counterpart in the
 * reference.  Its scratch (dQ accumulator and D) is a fixed array inside the
 * library, sized for n * s <= nl_flash_attention_bwd_noalloc_max_rows()
 * (131072 rows = 32.5 MiB, held on every device that loads the library until
 * the process exits); larger problems return NL_ERR_TOO_LARGE.  The first
 * call on each device resolves the array's device address (make that first
 * call before any stream capture).  All calls share the one array: calls
 * that overlap on the GPU (different streams, threads) race and must be
 * serialised by the caller.  Same results as nl_flash_attention_bwd. */
NL_API long long nl_flash_attention_bwd_noalloc_max_rows(void);
NL_API int nl_flash_attention_bwd_noalloc(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                                          const float* L, void* dQ, void* dK, void* dV, int n, int s, int d,
                                          cudaStream_t stream);

/* Strided forms used by the training step: activations addressed as
 * [B][H][s][64] with element strides (q_s, q_h, q_b) for Q, K, V, dQ, dK, dV
 * and (o_s, o_h, o_b) for O, dO — e.g. Q/K/V read in place from a fused QKV
 * projection [B, s, 3, H, 64] and O written as [B, s, H, 64].  Strides must be
 * multiples of 8 elements.  L, D_ws: f32 [B*H, s]; dQacc_ws: f32 [B*H, s, 64].
 * No reference counterpart: nlearn permutes to (B*H, s, 64) in JAX
 * (nlearn/model.py:175-181) before the contiguous targets above. */
NL_API int nl_flash_attention_fwd_strided(const void* Q, const void* K, const void* V, long long q_s, long long q_h,
                                          long long q_b, void* O, long long o_s, long long o_h, long long o_b,
                                          float* L, int B, int H, int s, int d, cudaStream_t stream);
NL_API int nl_flash_attention_bwd_strided(const void* Q, const void* K, const void* V, long long q_s, long long q_h,
                                          long long q_b, const void* O, const void* dO, long long o_s, long long o_h,
                                          long long o_b, const float* L, float* D_ws, void* dQ, void* dK, void* dV,
                                          float* dQacc_ws, int B, int H, int s, int d, cudaStream_t stream);

/* ---------------------------------------------------------------- training-step tail
 * Memory-bound kernels around the hot path (no reference custom-call: nlearn
 * leaves these to XLA, nlearn/model.py:74-90, 228-241 and train.py:338-339).
 * Activations bf16 row-major [M, D] (D % 256 == 0), statistics / grads f32. */
/* x[m] = wte[tok[m]] + wpe[m % S] (bf16 tables). */
NL_API int nl_embed_fwd(const int* tok, const void* wte, const void* wpe, void* out, int M, int S, int D,
                        cudaStream_t stream);
/* dwte[tok[m]] += dx[m], dwpe[m % S] += dx[m] (f32, atomics). */
NL_API int nl_embed_bwd(const int* tok, const float* dx, float* dwte, float* dwpe, int M, int S, int D,
                        cudaStream_t stream);
/* y = LayerNorm(x; g, b, eps); saves per-row mean, rstd. */
NL_API int nl_layernorm_fwd(const void* x, const float* g, const float* b, void* y, float* mean, float* rstd, int M,
                            int D, float eps, cudaStream_t stream);
/* dres (f32) = (accumulate ? dres : 0) + dLN/dx . dy; dres_bf16 = bf16(dres);
 * dg += sum dy*xhat, db += sum dy; dsum (may be NULL) += column sums of dres
 * (the bias gradient of the residual branch that dres feeds next). */
NL_API int nl_layernorm_bwd(const void* dy, const void* x, const float* mean, const float* rstd, const float* g,
                            float* dres, void* dres_bf16, float* dg, float* db, float* dsum, int M, int D,
                            int accumulate, cudaStream_t stream);
/* out[N] += column sums of bf16 x[M, N] (N % 8 == 0). */
NL_API int nl_colsum_bf16(const void* x, float* out, int M, int N, cudaStream_t stream);
/* AdamW on a flat f32 buffer (optax.adamw semantics); hyper = device
 * f32[3] {lr, 1-b1^t, 1-b2^t}; also writes the bf16 compute copy if non-NULL.
 * zero_grad != 0 clears g after reading it (the next step's accumulating
 * gradient kernels then need no separate zeroing pass).  n % 4 == 0. */
NL_API int nl_adamw_step(float* p, float* g, float* m, float* v, void* shadow_bf16, long long n,
                         const float* hyper, float b1, float b2, float eps, float wd, int zero_grad,
                         cudaStream_t stream);
NL_API int nl_cast_bf16(const float* x, void* y, long long n, cudaStream_t stream);
/* Advance the optimizer step on the device (for CUDA-graph replay): t =
 * ++(*step) (device int32), then hyper[0] = warmup-cosine learning rate at
 * step t-1 (optax.warmup_cosine_decay_schedule(0, peak, warmup, decay_steps,
 * end), as nlearn/train.py:487-505 builds it), hyper[1] = 1 - b1^t,
 * hyper[2] = 1 - b2^t.  No reference counterpart (optax runs on the host). */
NL_API int nl_adamw_schedule(float* hyper, int* step, float peak_lr, int warmup, int decay_steps, float end_lr,
                             float b1, float b2, cudaStream_t stream);

/* Embedding-table rows for the data-parallel exchange and the optimizer (no
 * reference counterpart: optax updates the dense table, nlearn/train.py:338).
 * The token table's gradient is zero on every row that no token of the global
 * batch touched; those rows can be updated (zero-gradient AdamW) as soon as
 * the step starts, and only the touched rows are all-reduced after the
 * backward.  Counts live in device memory, so the kernels need no host sync.
 *   nl_rows_mark:    mark[tok[m]] = 1 for m < M (mark int32 [V], zero on entry)
 *   nl_rows_compact: idx_on = ascending marked rows, idx_off = the others,
 *                    counts[0] = #on, counts[1] = #off; clears mark.  counts
 *                    holds 2 + ceil(V / 1024) int32 (the rest is scratch)
 *   nl_rows_gather:  dst[u] = src[idx[u]] for u < min(*count, max_rows), rows of D f32
 *   nl_rows_scatter: dst[idx[u]] = src[u]
 *   nl_adamw_rows:   nl_adamw_step on rows idx[0 .. *count) of a [rows, D] table
 *                    (g == NULL: zero gradient; zero_grad clears those rows of g) */
NL_API int nl_rows_mark(const int* tok, long long M, int* mark, int V, cudaStream_t stream);
NL_API int nl_rows_compact(int* mark, int V, int* idx_on, int* idx_off, int* counts, cudaStream_t stream);
NL_API int nl_rows_gather(const float* src, const int* idx, const int* count, int D, float* dst, int max_rows,
                          cudaStream_t stream);
NL_API int nl_rows_scatter(const float* src, const int* idx, const int* count, int D, float* dst, int max_rows,
                           cudaStream_t stream);
NL_API int nl_adamw_rows(float* p, float* g, float* m, float* v, void* shadow_bf16, const int* idx,
                         const int* count, int D, int max_rows, const float* hyper, float b1, float b2, float eps,
                         float wd, int zero_grad, cudaStream_t stream);

/* ---------------------------------------------------------------- fused LM-head CE
 * Replaces the jnp-chunked `linear_cross_entropy` (nlearn/kernels/
 * cross_entropy.py:106-167; its custom_vjp 131-170): loss over
 * logits = X[M,D] . W[D,V] (bf16, row-major, ldx/ldw multiples of 8, ldw >= V)
 * without materialising the logits.  Workspace (caller-owned, 256-byte
 * aligned): nl_lce_workspace_bytes(M, V, 0) for the forward,
 * nl_lce_workspace_bytes(M, V, chunk) for the backward. */
NL_API size_t nl_lce_workspace_bytes(int M, int V, int chunk);

/* loss[M] = lse - logit[target], lse[M] (f32). */
NL_API int nl_lce_fwd(const void* X, int ldx, const void* W, int ldw, const int* targets, float* loss, float* lse,
                      void* workspace, size_t ws_bytes, int M, int D, int V, cudaStream_t stream);

/* dlogits = (softmax - onehot) * grad_mul * (*gscale if gscale != NULL), per
 * vocabulary chunk (chunk % 64 == 0):  dX[M,D] f32 += dlogits . W^T (caller
 * zeroes dX, or passes existing gradients to accumulate);
 * dW[D,V] f32 (row pitch lddw) = X^T . dlogits, or += when dw_accumulate. */
NL_API int nl_lce_bwd(const void* X, int ldx, const void* W, int ldw, const int* targets, const float* lse,
                      const float* gscale, float grad_mul, float* dX, float* dW, int lddw, int dw_accumulate,
                      void* workspace, size_t ws_bytes, int chunk, int M, int D, int V, cudaStream_t stream);

/* nl_lce_bwd with the dX output chosen by the caller: dx_accumulate = 0
 * stores dX (no zeroing needed) instead of adding to it, and dx_dtype may then
 * be NL_BF16 when one chunk covers the vocabulary (chunk >= V), which hands the
 * next layer its bf16 gradient directly.  Same reference interface as
 * nl_lce_bwd (nlearn/kernels/cross_entropy.py:131-170). */
NL_API int nl_lce_bwd_ex(const void* X, int ldx, const void* W, int ldw, const int* targets, const float* lse,
                         const float* gscale, float grad_mul, void* dX, int dx_dtype, int dx_accumulate, float* dW,
                         int lddw, int dw_accumulate, void* workspace, size_t ws_bytes, int chunk, int M, int D,
                         int V, cudaStream_t stream);

/* ---------------------------------------------------------------- decode (inference)
 * Replace the reference's generate loop (nlearn/model.py:417-465: full
 * recompute per token, jax.random.categorical sampling) with KV-cache decode
 * steps.  The cache of each layer is its q|k|v rows, [B, S_max, 3*D] bf16
 * (D = H*64), the layout of the prefill's qkv GEMM output.  `pos` is the
 * current position in device memory (int32), read by every kernel of a step
 * and advanced by nl_decode_advance, so a step can be replayed from a graph. */
/* x[b] = wte[tok[b]] + wpe[*pos]  (bf16 tables, bf16 out [B, D]). */
NL_API int nl_decode_embed(const int* tok, const int* pos, const void* wte, const void* wpe, void* x, int B, int D,
                           cudaStream_t stream);
NL_API size_t nl_decode_workspace_bytes(int B, int H, int S_max);
/* o[b, h] = softmax(q k^T / sqrt(d)) v over positions 0..*pos of head h, with
 * q|k|v of position *pos taken from qkv_new [B, 3D] and its k|v row written
 * into the cache.  d == 64.  Workspace: nl_decode_workspace_bytes, zeroed
 * once before first use. */
NL_API int nl_decode_attention(const void* qkv_new, void* cache, void* o, const int* pos, void* workspace,
                               size_t ws_bytes, int B, int H, int S_max, int d, cudaStream_t stream);
/* tok[b] = argmax_j(logits[b, j] / T + Gumbel(seed, *pos, b, j)) for T > 0,
 * argmax_j logits[b, j] for T <= 0; also out[b, *pos + 1] = tok[b] when out
 * is non-NULL. */
NL_API int nl_sample_tokens(const float* logits, long long ldl, int V, float temperature, unsigned long long seed,
                            const int* pos, int* tok, int* out, long long ldo, int B, cudaStream_t stream);
NL_API int nl_decode_advance(int* pos, cudaStream_t stream);
/* C[M, N] = LayerNorm(x)[M, K] . W[K, N] with the nl_gemm_ex epilogues
 * (STORE / ACCUM / BIAS / BIAS_GELU / RESID), the LayerNorm (gamma, beta over
 * K, eps) applied while the small-M kernel stages x; M <= 8, x and W
 * row-major.  Returns NL_ERR_SHAPE for shapes it does not take (the caller
 * then runs nl_layernorm_fwd + nl_gemm_ex).  No reference counterpart (a
 * decode-step fusion). */
NL_API int nl_linear_ln_small(const void* x, long long ldx, const float* gamma, const float* beta, float eps,
                              const void* W, long long ldw, void* C, long long ldc, int c_dtype, int M, int N, int K,
                              int epilogue, const float* bias, void* aux, const void* resid, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NL_OPS_H */
