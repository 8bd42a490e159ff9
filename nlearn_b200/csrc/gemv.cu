// Small-M GEMM (M <= 8): C[M, N] = alpha * A[M, K] . B[K, N], A row-major
// (K contiguous), B row-major (N contiguous) -- the products of one decode
// step at small batch, which are bound by reading B once.  The tcgen05 kernel
// would spend a 128-row tile and its pipeline prologue on them.
//
// A CTA owns 64 columns and a slice of K.  Its 8 warps take every 8th row of
// the slice and each lane a pair of adjacent columns (one 4-byte load of B per
// row, 128 B per warp: coalesced; with an odd N the last pair reads one
// padding column of B's row pitch), with the slice of A staged in shared memory
// as f32; per-thread accumulators are M x 2 floats.  The warps' partials are
// summed in shared memory; the K slices of one column block form a thread-
// block cluster, and the leader CTA adds the other CTAs' partials by reading
// their shared memory over DSMEM (ld.shared::cluster), then applies the fused
// epilogue (store / accumulate / bias / bias + GELU / residual) of nl_gemm_ex.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include "gemm.h"
#include "host_common.h"
#include "sm100.cuh"

namespace nl {
namespace gv {

constexpr int kCols = 64;
constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kMaxCluster = 8;
constexpr int kMaxSlice = 512;  // K rows per CTA (shared memory for A)

struct Params {
  const __nv_bfloat16* A;
  long long lda;
  const __nv_bfloat16* B;
  long long ldb;
  void* C;
  long long ldc;
  int c_bf16, epi;
  float alpha;
  const float* bias;
  __nv_bfloat16* aux;
  const void* resid;
  int M, N, K, kslice;
  const float* ln_g;  // non-null: A is LayerNorm(A) (gamma, beta over K), as the LN kernel rounds it to bf16
  const float* ln_b;
  float ln_eps;
};

__device__ __forceinline__ float gelu(float a) {
  const float t = tanh_approx(0.7978845608028654f * (a + 0.044715f * a * a * a));
  return 0.5f * a * (1.f + t);
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

template <int MM>
__global__ void __launch_bounds__(kThreads) gemv_kernel(Params p) {
  griddep_sync();
  __shared__ float xs[MM][kMaxSlice];
  __shared__ float red[kWarps][MM][kCols];
  __shared__ float part[MM][kCols];
  const int split = blockIdx.x, nsplit = gridDim.x;  // one cluster = the K slices of a column block
  const int c0 = blockIdx.y * kCols;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kbeg = split * p.kslice;
  const int kend = min(p.K, kbeg + p.kslice);
  const int nk = kend > kbeg ? kend - kbeg : 0;

  __shared__ float stat[MM][2];
  if (p.ln_g) {  // per-row mean / rstd over the whole K (two passes), one warp per row
    for (int m = warp; m < MM; m += kWarps) {
      float s1 = 0.f;
      if (m < p.M)
        for (int k = lane; k < p.K; k += 32) s1 += __bfloat162float(p.A[m * p.lda + k]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      const float mean = s1 / p.K;
      float s2 = 0.f;
      if (m < p.M)
        for (int k = lane; k < p.K; k += 32) {
          const float d = __bfloat162float(p.A[m * p.lda + k]) - mean;
          s2 += d * d;
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      if (lane == 0) {
        stat[m][0] = mean;
        stat[m][1] = rsqrtf(s2 / p.K + p.ln_eps);
      }
    }
    __syncthreads();
  }
  for (int i = tid; i < MM * p.kslice; i += kThreads) {
    const int m = i / p.kslice, k = i - m * p.kslice;
    float v = 0.f;
    if (m < p.M && k < nk) {
      v = __bfloat162float(p.A[m * p.lda + kbeg + k]);
      if (p.ln_g) {
        const int kk = kbeg + k;
        v = __bfloat162float(__float2bfloat16_rn((v - stat[m][0]) * stat[m][1] * p.ln_g[kk] + p.ln_b[kk]));
      }
    }
    xs[m][k] = v;
  }
  __syncthreads();

  const int col = c0 + 2 * lane;
  float acc[MM][2];
#pragma unroll
  for (int m = 0; m < MM; ++m) acc[m][0] = acc[m][1] = 0.f;
  if (col < p.N) {
    const __nv_bfloat16* bcol = p.B + col;
    int k = warp;
#pragma unroll 1
    for (; k + 3 * kWarps < nk; k += 4 * kWarps) {
      float2 w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        w[u] = __bfloat1622float2(
            *reinterpret_cast<const __nv_bfloat162*>(bcol + (long long)(kbeg + k + u * kWarps) * p.ldb));
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int m = 0; m < MM; ++m) {
          const float xv = xs[m][k + u * kWarps];
          acc[m][0] = fmaf(xv, w[u].x, acc[m][0]);
          acc[m][1] = fmaf(xv, w[u].y, acc[m][1]);
        }
    }
    for (; k < nk; k += kWarps) {
      const float2 w = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(bcol + (long long)(kbeg + k) * p.ldb));
#pragma unroll
      for (int m = 0; m < MM; ++m) {
        acc[m][0] = fmaf(xs[m][k], w.x, acc[m][0]);
        acc[m][1] = fmaf(xs[m][k], w.y, acc[m][1]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MM; ++m) {
    red[warp][m][2 * lane] = acc[m][0];
    red[warp][m][2 * lane + 1] = acc[m][1];
  }
  __syncthreads();
  for (int i = tid; i < MM * kCols; i += kThreads) {
    const int m = i / kCols, c = i % kCols;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[w][m][c];
    part[m][c] = s;
  }
  if (nsplit > 1) cluster_sync();  // every slice's partials are in its shared memory
  else __syncthreads();
  if (split == 0) {
    for (int i = tid; i < MM * kCols; i += kThreads) {
      const int m = i / kCols, c = i % kCols;
      const int n = c0 + c;
      float v = part[m][c];
      if (nsplit > 1) {
        const uint32_t a = smem_u32(&part[m][c]);
        for (int r = 1; r < nsplit; ++r) v += ld_cluster_f32(mapa_shared(a, r));
      }
      if (m >= p.M || n >= p.N) continue;
      v *= p.alpha;
      const long long off = m * p.ldc + n;
      if (p.bias && (p.epi == NL_EPI_BIAS || p.epi == NL_EPI_BIAS_GELU || p.epi == NL_EPI_RESID)) v += p.bias[n];
      if (p.epi == NL_EPI_RESID && p.resid)
        v += p.c_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.resid)[off])
                      : static_cast<const float*>(p.resid)[off];
      if (p.epi == NL_EPI_BIAS_GELU) {
        p.aux[off] = __float2bfloat16_rn(v);
        v = gelu(v);
      }
      if (p.c_bf16) {
        static_cast<__nv_bfloat16*>(p.C)[off] = __float2bfloat16_rn(v);
      } else {
        float* cf = static_cast<float*>(p.C) + off;
        *cf = (p.epi == NL_EPI_ACCUM) ? *cf + v : v;
      }
    }
  }
  if (nsplit > 1) cluster_sync();  // peers stay resident until the leader has read them
}

}  // namespace gv

// Returns NL_OK after launching, or a negative status; -100 when the shape is
// not one the small-M kernel takes (the caller then uses the tcgen05 GEMM).
int gemv_run(const void* A, long long lda, int a_trans, const void* B, long long ldb, int b_trans, void* C,
             long long ldc, int c_dtype, int M, int N, int K, float alpha, int epi, const float* bias, void* aux,
             const void* resid, cudaStream_t stream, const float* ln_g, const float* ln_b, float ln_eps) {
  static int enabled = -1;
  if (enabled < 0) {
    const char* e = getenv("NL_GEMV");
    enabled = (e && e[0] == '0') ? 0 : 1;
  }
  const bool ok_epi = epi == NL_EPI_STORE || epi == NL_EPI_ACCUM || epi == NL_EPI_BIAS || epi == NL_EPI_BIAS_GELU ||
                      epi == NL_EPI_RESID;
  // column pairs are read as one 4-byte load: an odd N needs one padding
  // column in B's row pitch (the LM head's W is padded to a multiple of 64)
  if (!enabled || M > 8 || a_trans || b_trans || !ok_epi || (ldb & 1) || ldb < N + (N & 1) || K <= 0 ||
      (reinterpret_cast<uintptr_t>(B) & 3))
    return -100;
  const int ncb = (N + gv::kCols - 1) / gv::kCols;
  int ks = (2 * sm_count() + ncb - 1) / ncb;
  if (ks > gv::kMaxCluster) ks = gv::kMaxCluster;
  while ((K + ks - 1) / ks > gv::kMaxSlice) {
    if (ks == gv::kMaxCluster) return -100;  // K too long for the shared-memory slice
    ++ks;
  }
  if (ks > K) ks = K;
  if (ks < 1) ks = 1;
  if (ncb > 65535) return -100;
  gv::Params p;
  p.A = static_cast<const __nv_bfloat16*>(A);
  p.lda = lda;
  p.B = static_cast<const __nv_bfloat16*>(B);
  p.ldb = ldb;
  p.C = C;
  p.ldc = ldc;
  p.c_bf16 = c_dtype == NL_BF16;
  p.epi = epi;
  p.alpha = alpha;
  p.bias = bias;
  p.aux = static_cast<__nv_bfloat16*>(aux);
  p.resid = resid;
  p.M = M;
  p.N = N;
  p.K = K;
  p.kslice = (K + ks - 1) / ks;
  p.ln_g = ln_g;
  p.ln_b = ln_b;
  p.ln_eps = ln_eps;
  const dim3 grid(ks, ncb);
  cudaError_t e;
  if (M == 1) e = launch_kernel(gv::gemv_kernel<1>, grid, dim3(gv::kThreads), 0, stream, ks, p);
  else if (M == 2) e = launch_kernel(gv::gemv_kernel<2>, grid, dim3(gv::kThreads), 0, stream, ks, p);
  else if (M <= 4) e = launch_kernel(gv::gemv_kernel<4>, grid, dim3(gv::kThreads), 0, stream, ks, p);
  else e = launch_kernel(gv::gemv_kernel<8>, grid, dim3(gv::kThreads), 0, stream, ks, p);
  (void)e;
  return launch_status();
}

}  // namespace nl

using namespace nl;

extern "C" int nl_linear_ln_small(const void* x, long long ldx, const float* gamma, const float* beta, float eps,
                                  const void* W, long long ldw, void* C, long long ldc, int c_dtype, int M, int N,
                                  int K, int epilogue, const float* bias, void* aux, const void* resid,
                                  cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || !gamma || !beta) return NL_ERR_SHAPE;
  if (c_dtype != NL_F32 && c_dtype != NL_BF16) return NL_ERR_DTYPE;
  if (epilogue == NL_EPI_BIAS_GELU && (c_dtype != NL_BF16 || aux == nullptr)) return NL_ERR_DTYPE;
  if (epilogue == NL_EPI_ACCUM && c_dtype != NL_F32) return NL_ERR_DTYPE;
  const int st = gemv_run(x, ldx, 0, W, ldw, 0, C, ldc, c_dtype, M, N, K, 1.f, epilogue, bias, aux, resid, stream,
                          gamma, beta, eps);
  return st == -100 ? NL_ERR_SHAPE : st;
}
