// lce.cu — fused LM-head cross-entropy ("linear cross-entropy") on the tcgen05 GEMM.
//
// Replaces nlearn's jnp-chunked linear_cross_entropy (nlearn/kernels/
// cross_entropy.py:106-167): loss = mean_m (lse_m - (X W)[m, t_m]) and its
// gradients dX = dlogits W^T, dW = X^T dlogits with
// dlogits = (softmax(X W) - onehot(t)) * g / M, never holding (M, V) logits.
//
// Forward: ONE GEMM launch over the whole vocabulary whose epilogue reduces
//   each 128x256 logit tile (still in TMEM) to per-row partials (max, sum-exp)
//   and picks the target logit; a small row kernel combines the partials into
//   lse and loss.  No logit is written to memory.
// Backward, per vocabulary chunk of `chunk` columns:
//   1. GEMM recompute of the chunk's logits, epilogue -> bf16 dlogits chunk
//   2. dX (f32) += dlogits_c . W_c^T      (W read K-major in place)
//   3. dW_c     = X^T . dlogits_c         (X and dlogits read MN-major in place)
// Only one (M, chunk) bf16 buffer is live (the reference's _LCE_CHUNK idea, with
// bf16 instead of f32 and no pad copy of W).
#include <cuda_runtime.h>
#include <stddef.h>
#include <cuda_bf16.h>

#include "gemm.h"
#include "host_common.h"
#include "sm100.cuh"

namespace nl {
namespace lce {

constexpr int kTileN = 256;  // the STATS epilogue runs with 256-wide tiles
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Combine the per-half-tile partials (max in natural units, sum of
// exp(x - max)) of each row: a block takes 32 rows; lane = row (coalesced for
// a fixed tile), each of the 8 warps walks every 8th tile, and the 8 running
// (max, sum) pairs of a row are merged through shared memory.
constexpr int kReduceWarps = 8;

__device__ __forceinline__ void lse_merge(float& m, float& s, float pm, float ps) {
  if (pm == -INFINITY) return;
  if (pm > m) {
    s = s * ex2f((m - pm) * kLog2e) + ps;
    m = pm;
  } else {
    s += ps * ex2f((pm - m) * kLog2e);
  }
}

__global__ void __launch_bounds__(32 * kReduceWarps) lce_reduce_kernel(
    const float2* __restrict__ part, const float* __restrict__ tgt_logit, const int* __restrict__ targets,
    float* __restrict__ loss, float* __restrict__ lse, int M, int tiles, int V) {
  griddep_sync();
  __shared__ float2 red[kReduceWarps][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int row = blockIdx.x * 32 + lane;
  float m = -INFINITY, s = 0.f;
  if (row < M) {
#pragma unroll 4
    for (int t = w; t < tiles; t += kReduceWarps) {
      const float2 p = part[(long long)t * M + row];
      lse_merge(m, s, p.x, p.y);
    }
  }
  red[w][lane] = make_float2(m, s);
  __syncthreads();
  if (w != 0 || row >= M) return;
#pragma unroll
  for (int k = 1; k < kReduceWarps; ++k) lse_merge(m, s, red[k][lane].x, red[k][lane].y);
  const float l = m + __log2f(s) * kLn2;
  lse[row] = l;
  const int t = targets[row];
  loss[row] = l - ((t >= 0 && t < V) ? tgt_logit[row] : 0.f);
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Layout {
  size_t part, tgt, dl, total;
};

inline Layout layout(long long M, long long V, long long chunk) {
  Layout L;
  const long long tiles = 2 * ((V + kTileN - 1) / kTileN);  // one partial per tile half
  L.part = 0;
  L.tgt = align256(L.part + static_cast<size_t>(tiles * M) * sizeof(float2));
  L.dl = align256(L.tgt + static_cast<size_t>(M) * sizeof(float));
  L.total = align256(L.dl + static_cast<size_t>(M * (chunk > 0 ? chunk : 0)) * 2);
  return L;
}

}  // namespace lce
}  // namespace nl

using namespace nl;

extern "C" size_t nl_lce_workspace_bytes(int M, int V, int chunk) {
  return lce::layout(M, V, chunk).total;
}

extern "C" int nl_lce_fwd(const void* X, int ldx, const void* W, int ldw, const int* targets, float* loss,
                          float* lse, void* workspace, size_t ws_bytes, int M, int D, int V, cudaStream_t stream) {
  if (M <= 0 || D <= 0 || V <= 0 || ldx < D || ldw < V) return NL_ERR_SHAPE;
  const lce::Layout L = lce::layout(M, V, 0);
  if (!workspace || ws_bytes < L.dl) return NL_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return NL_ERR_ALIGN;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  GemmExtra ex;
  ex.targets = targets;
  ex.part = reinterpret_cast<float2*>(ws + L.part);
  ex.tgt_logit = reinterpret_cast<float*>(ws + L.tgt);
  ex.v_valid = V;
  ex.col_offset = 0;
  ex.force_bn = lce::kTileN;
  int st = gemm_run(X, ldx, 0, W, ldw, 0, nullptr, 0, NL_F32, M, V, D, 1.f, NL_EPI_LCE_STATS, nullptr, nullptr,
                    nullptr, stream, &ex);
  if (st) return st;
  const int tiles = 2 * ((V + lce::kTileN - 1) / lce::kTileN);
  launch_kernel(lce::lce_reduce_kernel, dim3((M + 31) / 32), dim3(32 * lce::kReduceWarps), 0, stream, 1, ex.part,
                ex.tgt_logit, targets, loss, lse, M, tiles, V);
  return launch_status();
}

namespace {
// dX: dx_accumulate -> f32 dX += dl W^T over every chunk; otherwise the first
// chunk stores (in dx_dtype) and later chunks accumulate (f32 only).
int lce_bwd_impl(const void* X, int ldx, const void* W, int ldw, const int* targets, const float* lse,
                 const float* gscale, float grad_mul, void* dX, int dx_dtype, int dx_accumulate, float* dW, int lddw,
                 int dw_accumulate, void* workspace, size_t ws_bytes, int chunk, int M, int D, int V,
                 cudaStream_t stream) {
  if (M <= 0 || D <= 0 || V <= 0 || ldx < D || ldw < V || lddw < V) return NL_ERR_SHAPE;
  if (chunk <= 0 || (chunk & 63)) return NL_ERR_SHAPE;
  if (dx_dtype != NL_F32 && dx_dtype != NL_BF16) return NL_ERR_DTYPE;
  if (dx_dtype == NL_BF16 && (dx_accumulate || chunk < V)) return NL_ERR_DTYPE;
  const lce::Layout L = lce::layout(M, V, chunk);
  if (!workspace || ws_bytes < L.total) return NL_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return NL_ERR_ALIGN;
  void* dl = static_cast<uint8_t*>(workspace) + L.dl;
  const __nv_bfloat16* Wb = static_cast<const __nv_bfloat16*>(W);
  for (int cs = 0; cs < V; cs += chunk) {
    const int vc = (V - cs) < chunk ? (V - cs) : chunk;
    GemmExtra ex;
    ex.targets = targets;
    ex.lse = lse;
    ex.gptr = gscale;
    ex.grad_scale = grad_mul;
    ex.v_valid = vc;
    ex.col_offset = cs;
    int st = gemm_run(X, ldx, 0, Wb + cs, ldw, 0, dl, chunk, NL_BF16, M, vc, D, 1.f, NL_EPI_LCE_GRAD, nullptr,
                      nullptr, nullptr, stream, &ex);
    if (st) return st;
    if (dX) {
      const bool store = !dx_accumulate && cs == 0;
      st = gemm_run(dl, chunk, 0, Wb + cs, ldw, 1, dX, D, store ? dx_dtype : NL_F32, M, D, vc, 1.f,
                    store ? NL_EPI_STORE : NL_EPI_ACCUM, nullptr, nullptr, nullptr, stream, nullptr);
      if (st) return st;
    }
    if (dW) {
      st = gemm_run(X, ldx, 1, dl, chunk, 0, dW + cs, lddw, NL_F32, D, vc, M, 1.f,
                    dw_accumulate ? NL_EPI_ACCUM : NL_EPI_STORE, nullptr, nullptr, nullptr, stream, nullptr);
      if (st) return st;
    }
  }
  return NL_OK;
}
}  // namespace

extern "C" int nl_lce_bwd(const void* X, int ldx, const void* W, int ldw, const int* targets, const float* lse,
                          const float* gscale, float grad_mul, float* dX, float* dW, int lddw, int dw_accumulate,
                          void* workspace, size_t ws_bytes, int chunk, int M, int D, int V, cudaStream_t stream) {
  return lce_bwd_impl(X, ldx, W, ldw, targets, lse, gscale, grad_mul, dX, NL_F32, 1, dW, lddw, dw_accumulate,
                      workspace, ws_bytes, chunk, M, D, V, stream);
}

extern "C" int nl_lce_bwd_ex(const void* X, int ldx, const void* W, int ldw, const int* targets, const float* lse,
                             const float* gscale, float grad_mul, void* dX, int dx_dtype, int dx_accumulate,
                             float* dW, int lddw, int dw_accumulate, void* workspace, size_t ws_bytes, int chunk,
                             int M, int D, int V, cudaStream_t stream) {
  return lce_bwd_impl(X, ldx, W, ldw, targets, lse, gscale, grad_mul, dX, dx_dtype, dx_accumulate, dW, lddw,
                      dw_accumulate, workspace, ws_bytes, chunk, M, D, V, stream);
}
