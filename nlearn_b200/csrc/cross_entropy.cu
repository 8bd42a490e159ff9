// cross_entropy.cu — fused softmax cross-entropy over materialised logits.
//
// Replaces nlearn's Metal ce_fwd / ce_bwd (iree_metal/kernels/cross_entropy.metal:
// 38-68 and 81-97):
//   fwd: lse = logsumexp(row), loss = lse - row[target]
//   bwd: dlogits = (softmax(row) - onehot(target)) * scale   (reference: scale = 1/M)
// plus a fused fwd+bwd that produces loss, lse and dlogits from ONE read of the
// logits from HBM (the second pass over a row re-reads it from L2) and one
// write — the path's algorithmic minimum.  dlogits may alias logits.
//
// HBM-bound row kernel: one CTA per row, 16-byte vector loads on the aligned
// body of each row (any leading dimension is accepted), online (max, sum-exp)
// per thread in base 2 (ex2.approx), warp-shuffle + shared-memory combine.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>

#include "host_common.h"
#include "sm100.cuh"

namespace nl {
namespace ce {


constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct Stat {
  float m;  // running max, in base-2 units (x * log2 e)
  float s;  // sum of 2^(y - m)
};

__device__ __forceinline__ void stat_add(Stat& a, float y) {
  if (y == -INFINITY) return;
  if (y > a.m) {
    a.s = a.s * ex2_approx(a.m - y) + 1.f;
    a.m = y;
  } else {
    a.s += ex2_approx(y - a.m);
  }
}
__device__ __forceinline__ void stat_add4(Stat& a, float y0, float y1, float y2, float y3) {
  const float mx = fmaxf(fmaxf(y0, y1), fmaxf(y2, y3));
  if (mx == -INFINITY) return;  // fully masked chunk
  if (mx > a.m) {
    a.s *= ex2_approx(a.m - mx);  // a.m == -inf -> 0
    a.m = mx;
  }
  a.s += ex2_approx(y0 - a.m) + ex2_approx(y1 - a.m) + ex2_approx(y2 - a.m) + ex2_approx(y3 - a.m);
}
__device__ __forceinline__ Stat stat_merge(Stat a, Stat b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return a;
  return Stat{m, a.s * ex2_approx(a.m - m) + b.s * ex2_approx(b.m - m)};
}

template <typename T>
__device__ __forceinline__ float ld1(const T* p);
template <>
__device__ __forceinline__ float ld1<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float ld1<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(p[0]); }

template <typename T>
__device__ __forceinline__ void st1(T* p, float v);
template <>
__device__ __forceinline__ void st1<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void st1<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// Elements per 16-byte vector.
template <typename T>
struct Vec { static constexpr int N = 16 / sizeof(T); };

// Row statistics (max, sum-exp) over row[0, V) in base-2 units.
template <int kThreads, typename T>
__device__ Stat row_stat(const T* row, int V) {
  constexpr int VN = Vec<T>::N;
  Stat st{-INFINITY, 0.f};
  const uintptr_t a = reinterpret_cast<uintptr_t>(row);
  int head = static_cast<int>(((16 - (a & 15)) & 15) / sizeof(T));
  if (head > V) head = V;
  for (int i = threadIdx.x; i < head; i += kThreads) stat_add(st, ld1(row + i) * kLog2e);
  const int nvec = (V - head) / VN;
  const uint4* body = reinterpret_cast<const uint4*>(row + head);
  for (int i = threadIdx.x; i < nvec; i += kThreads) {
    uint4 u = __ldg(body + i);
    if constexpr (sizeof(T) == 4) {
      stat_add4(st, __uint_as_float(u.x) * kLog2e, __uint_as_float(u.y) * kLog2e, __uint_as_float(u.z) * kLog2e,
                __uint_as_float(u.w) * kLog2e);
    } else {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
      float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
      float2 f2 = __bfloat1622float2(h[2]), f3 = __bfloat1622float2(h[3]);
      stat_add4(st, f0.x * kLog2e, f0.y * kLog2e, f1.x * kLog2e, f1.y * kLog2e);
      stat_add4(st, f2.x * kLog2e, f2.y * kLog2e, f3.x * kLog2e, f3.y * kLog2e);
    }
  }
  for (int i = head + nvec * VN + threadIdx.x; i < V; i += kThreads) stat_add(st, ld1(row + i) * kLog2e);

  // warp combine
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Stat b{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o)};
    st = stat_merge(st, b);
  }
  __shared__ float sm[kThreads / 32], ss[kThreads / 32];
  __shared__ Stat total;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sm[w] = st.m; ss[w] = st.s; }
  __syncthreads();
  if (w == 0) {
    Stat t = (l < kThreads / 32) ? Stat{sm[l], ss[l]} : Stat{-INFINITY, 0.f};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Stat b{__shfl_xor_sync(0xffffffffu, t.m, o), __shfl_xor_sync(0xffffffffu, t.s, o)};
      t = stat_merge(t, b);
    }
    if (l == 0) total = t;
  }
  __syncthreads();
  return total;
}

// dlogits[v] = (2^(x log2e - lse2) - [v == t]) * scale
template <int kThreads, typename T, typename TO>
__device__ void row_grad(const T* row, TO* drow, int V, int t, float lse2, float scale) {
  for (int i = threadIdx.x; i < V; i += kThreads) {
    // scalar path keeps any leading dimension legal; rows are L2-resident here
    const float p = ex2_approx(ld1(row + i) * kLog2e - lse2);
    st1(drow + i, (p - (i == t ? 1.f : 0.f)) * scale);
  }
}

template <int kThreads, typename T, typename TO>
__device__ void row_grad_vec(const T* row, TO* drow, int V, int t, float lse2, float scale) {
  // vector path when row and drow share 16-byte phase and element size
  constexpr int VN = Vec<T>::N;
  const uintptr_t a = reinterpret_cast<uintptr_t>(row);
  int head = static_cast<int>(((16 - (a & 15)) & 15) / sizeof(T));
  if (head > V) head = V;
  for (int i = threadIdx.x; i < head; i += kThreads) {
    const float p = ex2_approx(ld1(row + i) * kLog2e - lse2);
    st1(drow + i, (p - (i == t ? 1.f : 0.f)) * scale);
  }
  const int nvec = (V - head) / VN;
  const uint4* body = reinterpret_cast<const uint4*>(row + head);
  uint4* dbody = reinterpret_cast<uint4*>(drow + head);
  for (int i = threadIdx.x; i < nvec; i += kThreads) {
    uint4 u = body[i];
    const int v0 = head + i * VN;
    if constexpr (sizeof(T) == 4) {
      float x[4] = {__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w)};
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = (ex2_approx(x[j] * kLog2e - lse2) - (v0 + j == t ? 1.f : 0.f)) * scale;
      dbody[i] = make_uint4(__float_as_uint(x[0]), __float_as_uint(x[1]), __float_as_uint(x[2]), __float_as_uint(x[3]));
    } else {
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        f.x = (ex2_approx(f.x * kLog2e - lse2) - (v0 + 2 * j == t ? 1.f : 0.f)) * scale;
        f.y = (ex2_approx(f.y * kLog2e - lse2) - (v0 + 2 * j + 1 == t ? 1.f : 0.f)) * scale;
        h[j] = __floats2bfloat162_rn(f.x, f.y);
      }
      dbody[i] = u;
    }
  }
  for (int i = head + nvec * VN + threadIdx.x; i < V; i += kThreads) {
    const float p = ex2_approx(ld1(row + i) * kLog2e - lse2);
    st1(drow + i, (p - (i == t ? 1.f : 0.f)) * scale);
  }
}

// mode: 1 = fwd (loss, lse), 2 = bwd (dlogits from given lse), 3 = fused fwd+bwd
template <typename T, typename TO, int MODE, int kThreads>
__global__ void __launch_bounds__(kThreads) ce_kernel(const T* logits, long long ld,
                                                      const int* __restrict__ targets, float* loss, float* lse,
                                                      TO* dlogits, long long ldd, int M, int V, float scale) {
  griddep_sync();
  const int r = blockIdx.x;
  if (r >= M) return;
  const T* row = logits + (long long)r * ld;
  const int t = targets[r];
  const bool tin = (t >= 0 && t < V);
  // read the target logit before any thread may overwrite the row (dlogits
  // is allowed to alias logits)
  const float xt = (threadIdx.x == 0 && tin) ? ld1(row + t) : 0.f;
  float lse2;
  if (MODE & 1) {
    const Stat st = row_stat<kThreads>(row, V);
    lse2 = st.m + __log2f(st.s);
    if (threadIdx.x == 0) {
      const float l = lse2 * kLn2;
      lse[r] = l;
      loss[r] = l - xt;
    }
  } else {
    lse2 = lse[r] * kLog2e;
  }
  if (MODE & 2) {
    TO* drow = dlogits + (long long)r * ldd;
    const bool same_phase = sizeof(T) == sizeof(TO) &&
                            ((reinterpret_cast<uintptr_t>(row) & 15) == (reinterpret_cast<uintptr_t>(drow) & 15));
    if (same_phase) row_grad_vec<kThreads, T, TO>(row, drow, V, tin ? t : -1, lse2, scale);
    else row_grad<kThreads, T, TO>(row, drow, V, tin ? t : -1, lse2, scale);
  }
}

template <int MODE>
int dispatch(const void* logits, long long ld, int in_dtype, const int* targets, float* loss, float* lse,
             void* dlogits, long long ldd, int out_dtype, int M, int V, float scale, cudaStream_t stream) {
  if (M <= 0 || V <= 0 || ld < V || ((MODE & 2) && ldd < V)) return NL_ERR_SHAPE;
  if (in_dtype != NL_F32 && in_dtype != NL_BF16) return NL_ERR_DTYPE;
  if ((MODE & 2) && out_dtype != NL_F32 && out_dtype != NL_BF16) return NL_ERR_DTYPE;
  // The fused form re-reads each row from L2 in its second pass: with one
  // 1024-thread CTA per SM only ~148 rows are in flight, which keeps them
  // L2-resident (a 50k-column f32 row is 200 KB); single-pass forms use
  // 512-thread CTAs, several per SM.
  constexpr int NT = (MODE == 3) ? 1024 : 512;
  dim3 grid(M), block(NT);
#define NL_CE_LAUNCH(T, TO)                                                                                    \
  launch_kernel(ce_kernel<T, TO, MODE, NT>, dim3(grid), dim3(block), 0, stream, 1, reinterpret_cast<const T*>(logits), ld, targets, loss, \
                                                         lse, reinterpret_cast<TO*>(dlogits), ldd, M, V, scale)
  if (in_dtype == NL_F32) {
    if (!(MODE & 2) || out_dtype == NL_F32) NL_CE_LAUNCH(float, float);
    else NL_CE_LAUNCH(float, __nv_bfloat16);
  } else {
    if (!(MODE & 2) || out_dtype == NL_BF16) NL_CE_LAUNCH(__nv_bfloat16, __nv_bfloat16);
    else NL_CE_LAUNCH(__nv_bfloat16, float);
  }
#undef NL_CE_LAUNCH
  return launch_status();
}

}  // namespace ce
}  // namespace nl

extern "C" int nl_ce_fwd(const void* logits, long long ld, int in_dtype, const int* targets, float* loss,
                         float* lse, int M, int V, cudaStream_t stream) {
  return nl::ce::dispatch<1>(logits, ld, in_dtype, targets, loss, lse, nullptr, V, NL_F32, M, V, 0.f, stream);
}

extern "C" int nl_ce_bwd(const void* logits, long long ld, int in_dtype, const int* targets, const float* lse,
                         void* dlogits, long long ldd, int out_dtype, int M, int V, float scale,
                         cudaStream_t stream) {
  return nl::ce::dispatch<2>(logits, ld, in_dtype, targets, nullptr, const_cast<float*>(lse), dlogits, ldd,
                             out_dtype, M, V, scale, stream);
}

extern "C" int nl_ce_fwd_bwd(const void* logits, long long ld, int in_dtype, const int* targets, float* loss,
                             float* lse, void* dlogits, long long ldd, int out_dtype, int M, int V, float scale,
                             cudaStream_t stream) {
  return nl::ce::dispatch<3>(logits, ld, in_dtype, targets, loss, lse, dlogits, ldd, out_dtype, M, V, scale,
                             stream);
}
