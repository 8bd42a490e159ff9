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
 *    shape / alignment / dtype or a failed launch.  Kernel-side timeouts of the
 *    bounded waits are reported through nl_get_device_error().
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
  NL_ERR_WORKSPACE = -6  /* workspace missing or too small                  */
} nl_status;

typedef enum { NL_F32 = 0, NL_BF16 = 1 } nl_dtype;

/* GEMM epilogue selector for nl_gemm_ex. */
typedef enum {
  NL_EPI_STORE = 0,     /* C = alpha*A.B                 (C in c_dtype)        */
  NL_EPI_ACCUM = 1,     /* C += alpha*A.B                (C f32; split-K safe) */
  NL_EPI_BIAS = 2,      /* C = alpha*A.B + bias[N]       (bias f32)            */
  NL_EPI_BIAS_GELU = 3, /* aux = A.B + bias; C = gelu_tanh(aux)  (C, aux bf16) */
  NL_EPI_RESID = 4      /* C = alpha*A.B + bias? + resid (resid in c_dtype)    */
} nl_epilogue;

/* Library / device introspection. */
NL_API const char* nl_version(void);
/* Reads and clears the device-side error word (1 = a bounded wait timed out).
 * Synchronises `stream`. */
NL_API int nl_get_device_error(cudaStream_t stream);

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

#ifdef __cplusplus
}
#endif

#endif /* NL_OPS_H */
