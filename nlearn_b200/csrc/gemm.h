// gemm.h — internal entry of the tcgen05 GEMM for other translation units
// (the fused LM-head cross-entropy drives it with its own epilogues).
#pragma once
#include <cuda_runtime.h>
#include <vector_types.h>

namespace nl {

// Extra epilogue inputs for NL_EPI_LCE_STATS / NL_EPI_LCE_GRAD.
struct GemmExtra {
  const int* targets = nullptr;   // [M] global vocabulary index of each row's target
  float2* part = nullptr;         // STATS: [2*ceil(N/256), M] per half-tile (max, sum-exp)
  float* tgt_logit = nullptr;     // STATS: [M] target logit
  const float* lse = nullptr;     // GRAD: [M] logsumexp (natural log)
  const float* gptr = nullptr;    // GRAD: optional device scalar multiplier
  float grad_scale = 1.f;         // GRAD: multiplier (1/M for a mean)
  int v_valid = 0x7fffffff;       // columns >= v_valid are padding
  int col_offset = 0;             // global vocabulary index of column 0
  int force_bn = 0;               // 0 = heuristic, else 128 / 256
};

int gemm_run(const void* A, long long lda, int a_trans, const void* B, long long ldb, int b_trans, void* C,
             long long ldc, int c_dtype, int M, int N, int K, float alpha, int epi, const float* bias, void* aux,
             const void* resid, cudaStream_t stream, const GemmExtra* ex);

// Small-M path (M <= 8, A and B row-major, store / accumulate / bias /
// bias+GELU / residual epilogues): launches and returns a status, or -100 when
// the shape is not one it takes.  gemm_run tries it first.
int gemv_run(const void* A, long long lda, int a_trans, const void* B, long long ldb, int b_trans, void* C,
             long long ldc, int c_dtype, int M, int N, int K, float alpha, int epi, const float* bias, void* aux,
             const void* resid, cudaStream_t stream, const float* ln_g = nullptr, const float* ln_b = nullptr,
             float ln_eps = 0.f);

}  // namespace nl
