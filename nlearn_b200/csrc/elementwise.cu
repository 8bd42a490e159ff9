// elementwise.cu — the memory-bound tail around the hot GEMM / attention / CE
// kernels in the training step: token+position embedding, LayerNorm forward /
// backward, bias-gradient column sums, and the fused AdamW update that also
// refreshes the bf16 compute copy of the weights.
//
// Reference semantics: embeddings nlearn/model.py:74-90 (token + learned
// position table of the BASELINE model), pre-LN LayerNorm with gamma/beta and
// eps 1e-5 (the BASELINE model; iree_metal/kernels/test/bf16_metal_test.py:6-12),
// AdamW as optax.adamw (nlearn/train.py:503-508: b1 0.9, b2 0.999, eps 1e-8,
// decoupled weight decay on every leaf).
//
// All kernels are bandwidth-bound row/element kernels: 16-byte vector access,
// one warp per row for the row reductions, grid-stride loops sized to the SMs.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "host_common.h"
#include "sm100.cuh"

namespace nl {
namespace ew {

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __bfloat1622float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// x[m, :] = wte[tok[m], :] + wpe[m % S, :]   (bf16 tables, bf16 out)
template <int DV>  // D / 256: vectors of 8 per lane
__global__ void embed_fwd_kernel(const int* __restrict__ tok, const __nv_bfloat16* __restrict__ wte,
                                 const __nv_bfloat16* __restrict__ wpe, __nv_bfloat16* __restrict__ out, int M,
                                 int S, int D) {
  griddep_sync();
  const int lane = threadIdx.x & 31;
  for (long long m = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; m < M;
       m += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
    const int t = tok[m];
    const uint4* a = reinterpret_cast<const uint4*>(wte + static_cast<long long>(t) * D);
    const uint4* b = reinterpret_cast<const uint4*>(wpe + static_cast<long long>(m % S) * D);
    uint4* o = reinterpret_cast<uint4*>(out + m * D);
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      float fa[8], fb[8];
      unpack8(a[lane + 32 * j], fa);
      unpack8(b[lane + 32 * j], fb);
#pragma unroll
      for (int i = 0; i < 8; ++i) fa[i] += fb[i];
      o[lane + 32 * j] = pack8(fa);
    }
  }
}

// dwte[tok[m]] += dx[m]; dwpe[m % S] += dx[m]   (f32 gradients, float atomics)
template <int DV>
__global__ void embed_bwd_kernel(const int* __restrict__ tok, const float* __restrict__ dx, float* dwte,
                                 float* dwpe, int M, int S, int D) {
  griddep_sync();
  const int lane = threadIdx.x & 31;
  for (long long m = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; m < M;
       m += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
    const int t = tok[m];
    const float4* g = reinterpret_cast<const float4*>(dx + m * D);
    float4* a = reinterpret_cast<float4*>(dwte + static_cast<long long>(t) * D);
    float4* b = reinterpret_cast<float4*>(dwpe + static_cast<long long>(m % S) * D);
#pragma unroll
    for (int j = 0; j < 2 * DV; ++j) {
      const float4 v = g[lane + 32 * j];
      atomicAdd(a + lane + 32 * j, v);
      atomicAdd(b + lane + 32 * j, v);
    }
  }
}

// y = (x - mean) * rstd * g + b;  per-row mean / rstd saved for the backward.
template <int DV>
__global__ void layernorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ g,
                                     const float* __restrict__ b, __nv_bfloat16* __restrict__ y,
                                     float* __restrict__ mean_out, float* __restrict__ rstd_out, int M, int D,
                                     float eps) {
  griddep_sync();
  const int lane = threadIdx.x & 31;
  // each lane always owns the same 8-column groups: keep gamma / beta in registers
  float gg[DV][8], bb[DV][8];
#pragma unroll
  for (int j = 0; j < DV; ++j) {
    const float4* g4 = reinterpret_cast<const float4*>(g + (lane + 32 * j) * 8);
    const float4* b4 = reinterpret_cast<const float4*>(b + (lane + 32 * j) * 8);
    const float4 g0 = __ldg(g4), g1 = __ldg(g4 + 1), b0 = __ldg(b4), b1 = __ldg(b4 + 1);
    gg[j][0] = g0.x; gg[j][1] = g0.y; gg[j][2] = g0.z; gg[j][3] = g0.w;
    gg[j][4] = g1.x; gg[j][5] = g1.y; gg[j][6] = g1.z; gg[j][7] = g1.w;
    bb[j][0] = b0.x; bb[j][1] = b0.y; bb[j][2] = b0.z; bb[j][3] = b0.w;
    bb[j][4] = b1.x; bb[j][5] = b1.y; bb[j][6] = b1.z; bb[j][7] = b1.w;
  }
  for (long long m = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; m < M;
       m += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + m * D);
    float v[DV][8];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      unpack8(xr[lane + 32 * j], v[j]);
#pragma unroll
      for (int i = 0; i < 8; ++i) sum += v[j][i];
    }
    const float mean = warp_sum(sum) / D;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < DV; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[j][i] - mean;
        q += d * d;
      }
    const float rstd = rsqrtf(warp_sum(q) / D + eps);
    uint4* yr = reinterpret_cast<uint4*>(y + m * D);
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = (v[j][i] - mean) * rstd * gg[j][i] + bb[j][i];
      yr[lane + 32 * j] = pack8(o);
    }
    if (lane == 0) {
      mean_out[m] = mean;
      rstd_out[m] = rstd;
    }
  }
}

// dx = rstd * (g*dy - mean(g*dy) - xhat * mean(g*dy*xhat));  dres += dx (f32),
// dres_bf = bf16(dres);  dg += sum_rows dy*xhat, db += sum_rows dy, and, when
// dsum is given, dsum += sum_rows dres (the bias gradient of the residual
// branch that consumes dres: saves a column-sum pass over it) (atomics).
template <int DV>
__global__ void layernorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                     const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                                     const float* __restrict__ g, float* dres, __nv_bfloat16* dres_bf, float* dg,
                                     float* db, float* dsum, int M, int D, int accumulate) {
  griddep_sync();
  const int lane = threadIdx.x & 31;
  float adg[DV][8], adb[DV][8], ads[DV][8];
#pragma unroll
  for (int j = 0; j < DV; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) adg[j][i] = adb[j][i] = ads[j][i] = 0.f;
  float gg[DV][8];
#pragma unroll
  for (int j = 0; j < DV; ++j) {
    const float4* g4 = reinterpret_cast<const float4*>(g + (lane + 32 * j) * 8);
    const float4 g0 = __ldg(g4), g1 = __ldg(g4 + 1);
    gg[j][0] = g0.x; gg[j][1] = g0.y; gg[j][2] = g0.z; gg[j][3] = g0.w;
    gg[j][4] = g1.x; gg[j][5] = g1.y; gg[j][6] = g1.z; gg[j][7] = g1.w;
  }
  for (long long m = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; m < M;
       m += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
    const float mean = mean_in[m], rstd = rstd_in[m];
    const uint4* xr = reinterpret_cast<const uint4*>(x + m * D);
    const uint4* dyr = reinterpret_cast<const uint4*>(dy + m * D);
    float xh[DV][8], gd[DV][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      float xv[8], dv[8];
      unpack8(xr[lane + 32 * j], xv);
      unpack8(dyr[lane + 32 * j], dv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        xh[j][i] = (xv[i] - mean) * rstd;
        gd[j][i] = dv[i] * gg[j][i];
        s1 += gd[j][i];
        s2 += gd[j][i] * xh[j][i];
        adg[j][i] += dv[i] * xh[j][i];
        adb[j][i] += dv[i];
      }
    }
    const float c1 = warp_sum(s1) / D, c2 = warp_sum(s2) / D;
    float4* rr = reinterpret_cast<float4*>(dres + m * D);
    uint4* rb = reinterpret_cast<uint4*>(dres_bf + m * D);
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      float o[8];
      const float4 r0 = accumulate ? rr[2 * (lane + 32 * j)] : make_float4(0, 0, 0, 0);
      const float4 r1 = accumulate ? rr[2 * (lane + 32 * j) + 1] : make_float4(0, 0, 0, 0);
      const float prev[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o[i] = prev[i] + rstd * (gd[j][i] - c1 - xh[j][i] * c2);
        ads[j][i] += o[i];
      }
      rr[2 * (lane + 32 * j)] = make_float4(o[0], o[1], o[2], o[3]);
      rr[2 * (lane + 32 * j) + 1] = make_float4(o[4], o[5], o[6], o[7]);
      rb[lane + 32 * j] = pack8(o);
    }
  }
  // Block-level reduction of the per-warp gamma / beta partials in shared
  // memory, then one atomic per column per block (few blocks, so the global
  // atomics do not serialise on the D hot addresses).
  __shared__ float red[8][DV * 256];
  const int w = threadIdx.x >> 5;
  const int nsums = dsum ? 3 : 2;
  for (int which = 0; which < nsums; ++which) {
#pragma unroll
    for (int j = 0; j < DV; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        red[w][(lane + 32 * j) * 8 + i] = which == 2 ? ads[j][i] : which ? adb[j][i] : adg[j][i];
    __syncthreads();
    float* dst = which == 2 ? dsum : which ? db : dg;
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
      float t = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) t += red[k][c];
      atomicAdd(dst + c, t);
    }
    __syncthreads();
  }
}

// out[n] (+)= sum_m x[m, n]  for bf16 x [M, N] (N % 8 == 0).  Block = 256
// threads covering 8*32 = 256 columns x 8 row groups; float atomics per block.
__global__ void colsum_kernel(const __nv_bfloat16* __restrict__ x, float* out, int M, int N, int rows_per_block) {
  griddep_sync();
  const int cvec = blockIdx.x * 32 + (threadIdx.x & 31);  // vector of 8 columns
  const int rg = threadIdx.x >> 5;                        // 8 row groups
  if (cvec * 8 >= N) return;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(M, r0 + rows_per_block);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int r = r0 + rg; r < r1; r += 8) {
    float f[8];
    unpack8(reinterpret_cast<const uint4*>(x + static_cast<long long>(r) * N)[cvec], f);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += f[i];
  }
  __shared__ float red[8][32][9];
#pragma unroll
  for (int i = 0; i < 8; ++i) red[rg][threadIdx.x & 31][i] = acc[i];
  __syncthreads();
  if (rg == 0) {
#pragma unroll
    for (int k = 1; k < 8; ++k)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += red[k][threadIdx.x & 31][i];
    atomicAdd(reinterpret_cast<float4*>(out + cvec * 8), make_float4(acc[0], acc[1], acc[2], acc[3]));
    atomicAdd(reinterpret_cast<float4*>(out + cvec * 8 + 4), make_float4(acc[4], acc[5], acc[6], acc[7]));
  }
}

// AdamW (optax.adamw semantics, decoupled decay on all elements):
//   m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2
//   p -= lr * ( (m / bc1) / (sqrt(v / bc2) + eps) + wd * p )
// and the bf16 compute copy is rewritten from the updated master.
// hyper[0..2] = lr, bc1, bc2 live in device memory so that a captured CUDA
// graph picks up each step's schedule value.
__global__ void adamw_kernel(float* __restrict__ p, float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ shadow, long long n4,
                             const float* __restrict__ hyper, float b1, float b2, float eps, float wd,
                             int zero_grad) {
  griddep_sync();
  const float lr = hyper[0], bc1 = hyper[1], bc2 = hyper[2];
  const float ibc1 = 1.f / bc1, ibc2 = 1.f / bc2;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    const float4 gg = reinterpret_cast<const float4*>(g)[i];
    if (zero_grad) reinterpret_cast<float4*>(g)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* P = &pp.x;
    const float* G = &gg.x;
    float* Mm = &mm.x;
    float* Vv = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      Mm[k] = b1 * Mm[k] + (1.f - b1) * G[k];
      Vv[k] = b2 * Vv[k] + (1.f - b2) * G[k] * G[k];
      const float upd = (Mm[k] * ibc1) / (sqrtf(Vv[k] * ibc2) + eps) + wd * P[k];
      P[k] -= lr * upd;
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (shadow) reinterpret_cast<uint2*>(shadow)[i] = make_uint2(pack_bf16x2(pp.x, pp.y), pack_bf16x2(pp.z, pp.w));
  }
}

// One thread: the device-side step counter and this step's AdamW scalars.
__global__ void adamw_schedule_kernel(float* hyper, int* step, float peak, int warmup, int decay_steps, float end,
                                      float b1, float b2) {
  griddep_sync();
  const int t = *step + 1;
  *step = t;
  const int s = t - 1;  // the schedule counts from 0
  float lr;
  if (warmup > 0 && s < warmup) {
    lr = peak * static_cast<float>(s) / static_cast<float>(warmup);
  } else if (decay_steps <= warmup) {
    lr = end;
  } else {
    int k = s - warmup;
    if (k < 0) k = 0;
    if (k > decay_steps - warmup) k = decay_steps - warmup;
    const float frac = static_cast<float>(k) / static_cast<float>(decay_steps - warmup);
    lr = end + (peak - end) * 0.5f * (1.f + cosf(3.14159265358979f * frac));
  }
  hyper[0] = lr;
  hyper[1] = 1.f - powf(b1, static_cast<float>(t));
  hyper[2] = 1.f - powf(b2, static_cast<float>(t));
}

__global__ void cast_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long long n4) {
  griddep_sync();
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(x)[i];
    reinterpret_cast<uint2*>(y)[i] = make_uint2(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w));
  }
}

// ---------------------------------------------------------------- embedding rows
// The token table's gradient is non-zero only on the rows of tokens that occur
// in the (global) batch.  These kernels find those rows once per step (from
// the token ids, known before the forward), so that the exchange and the
// optimizer can treat the two row sets apart: rows no token touched have a
// zero gradient on every rank and can be updated as soon as the step starts;
// only the touched rows wait for the backward and cross NVLink.

// mark[tok[m]] = 1 (mark zeroed beforehand; nl_rows_compact clears it again).
__global__ void rows_mark_kernel(const int* __restrict__ tok, long long M, int* __restrict__ mark, int V) {
  griddep_sync();
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < M;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = tok[i];
    if (t >= 0 && t < V) mark[t] = 1;
  }
}

// Compaction in two passes over chunks of 1024 rows (one CTA per chunk,
// coalesced reads): rows_count_kernel writes each chunk's number of marked
// rows; rows_list_kernel turns the preceding chunks' counts and a block-wide
// ballot scan into positions and writes ascending lists of marked rows
// (idx_on) and unmarked rows (idx_off), counts[0] = #on, counts[1] = #off, and
// clears the marks for the next step.  The lists are the same on every rank
// for the same marks (deterministic order).
__device__ __forceinline__ int block_ballot_scan(bool on, int* warp_tot, int& total) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned b = __ballot_sync(0xffffffffu, on);
  const int before_in_warp = __popc(b & ((1u << lane) - 1u));
  if (lane == 0) warp_tot[warp] = __popc(b);
  __syncthreads();
  if (warp == 0) {
    const int w = warp_tot[lane];
    int inc = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += y;
    }
    warp_tot[lane] = inc - w;
    if (lane == 31) warp_tot[32] = inc;
  }
  __syncthreads();
  total = warp_tot[32];
  return warp_tot[warp] + before_in_warp;
}

__global__ void __launch_bounds__(1024) rows_count_kernel(const int* __restrict__ mark, int V,
                                                          int* __restrict__ chunk_on) {
  griddep_sync();
  __shared__ int warp_tot[33];
  const int r = blockIdx.x * 1024 + threadIdx.x;
  int total;
  block_ballot_scan(r < V && mark[r] != 0, warp_tot, total);
  if (threadIdx.x == 0) chunk_on[blockIdx.x] = total;
}

__global__ void __launch_bounds__(1024) rows_list_kernel(int* __restrict__ mark, int V,
                                                         const int* __restrict__ chunk_on, int* __restrict__ idx_on,
                                                         int* __restrict__ idx_off, int* __restrict__ counts) {
  griddep_sync();
  __shared__ int warp_tot[33];
  __shared__ int base_s[2];
  if (threadIdx.x < 32) {  // marked rows in the chunks before this one, and in all chunks
    int before = 0, all = 0;
    for (int c = threadIdx.x; c < gridDim.x; c += 32) {
      const int v = chunk_on[c];
      all += v;
      before += (c < static_cast<int>(blockIdx.x)) ? v : 0;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      before += __shfl_xor_sync(0xffffffffu, before, o);
      all += __shfl_xor_sync(0xffffffffu, all, o);
    }
    if (threadIdx.x == 0) {
      base_s[0] = before;
      base_s[1] = all;
    }
  }
  const int r = blockIdx.x * 1024 + threadIdx.x;
  const bool on = r < V && mark[r] != 0;
  int total;
  const int pos = block_ballot_scan(on, warp_tot, total);  // (its barriers also publish base_s)
  const int on_before = base_s[0] + pos;
  if (r < V) {
    if (on) {
      idx_on[on_before] = r;
      mark[r] = 0;
    } else {
      idx_off[r - on_before] = r;  // rows before r that are off
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    counts[0] = base_s[1];
    counts[1] = V - base_s[1];
  }
}

// dst[u, :] = src[idx[u], :] for u < *count (one warp per row, float4).
__global__ void rows_gather_kernel(const float* __restrict__ src, const int* __restrict__ idx,
                                   const int* __restrict__ count, int D4, float* __restrict__ dst, int max_rows) {
  griddep_sync();
  const int n = min(*count, max_rows);
  const int lane = threadIdx.x & 31;
  for (int u = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < n; u += (gridDim.x * blockDim.x) >> 5) {
    const float4* s = reinterpret_cast<const float4*>(src) + static_cast<long long>(idx[u]) * D4;
    float4* d = reinterpret_cast<float4*>(dst) + static_cast<long long>(u) * D4;
    for (int c = lane; c < D4; c += 32) d[c] = s[c];
  }
}

// dst[idx[u], :] = src[u, :] for u < *count.
__global__ void rows_scatter_kernel(const float* __restrict__ src, const int* __restrict__ idx,
                                    const int* __restrict__ count, int D4, float* __restrict__ dst, int max_rows) {
  griddep_sync();
  const int n = min(*count, max_rows);
  const int lane = threadIdx.x & 31;
  for (int u = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < n; u += (gridDim.x * blockDim.x) >> 5) {
    const float4* s = reinterpret_cast<const float4*>(src) + static_cast<long long>(u) * D4;
    float4* d = reinterpret_cast<float4*>(dst) + static_cast<long long>(idx[u]) * D4;
    for (int c = lane; c < D4; c += 32) d[c] = s[c];
  }
}

// AdamW (as adamw_kernel) on the rows idx[0 .. *count) of a [rows, D] table;
// g == nullptr means a zero gradient (rows no token touched).
__global__ void adamw_rows_kernel(float* __restrict__ p, float* __restrict__ g, float* __restrict__ m,
                                  float* __restrict__ v, __nv_bfloat16* __restrict__ shadow,
                                  const int* __restrict__ idx, const int* __restrict__ count, int D4, int max_rows,
                                  const float* __restrict__ hyper, float b1, float b2, float eps, float wd,
                                  int zero_grad) {
  griddep_sync();
  const float lr = hyper[0], ibc1 = 1.f / hyper[1], ibc2 = 1.f / hyper[2];
  const long long n = static_cast<long long>(min(*count, max_rows)) * D4;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = static_cast<long long>(idx[i / D4]) * D4 + i % D4;
    float4 pp = reinterpret_cast<float4*>(p)[e];
    const float4 gg = g ? reinterpret_cast<const float4*>(g)[e] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (g && zero_grad) reinterpret_cast<float4*>(g)[e] = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 mm = reinterpret_cast<float4*>(m)[e];
    float4 vv = reinterpret_cast<float4*>(v)[e];
    float* P = &pp.x;
    const float* G = &gg.x;
    float* Mm = &mm.x;
    float* Vv = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      Mm[k] = b1 * Mm[k] + (1.f - b1) * G[k];
      Vv[k] = b2 * Vv[k] + (1.f - b2) * G[k] * G[k];
      const float upd = (Mm[k] * ibc1) / (sqrtf(Vv[k] * ibc2) + eps) + wd * P[k];
      P[k] -= lr * upd;
    }
    reinterpret_cast<float4*>(p)[e] = pp;
    reinterpret_cast<float4*>(m)[e] = mm;
    reinterpret_cast<float4*>(v)[e] = vv;
    if (shadow) reinterpret_cast<uint2*>(shadow)[e] = make_uint2(pack_bf16x2(pp.x, pp.y), pack_bf16x2(pp.z, pp.w));
  }
}

inline int row_grid(long long M) {
  const long long warps = M;
  long long blocks = (warps * 32 + 255) / 256;
  const long long cap = static_cast<long long>(sm_count()) * 8;
  return static_cast<int>(blocks < cap ? blocks : cap);
}

}  // namespace ew
}  // namespace nl

using namespace nl;

extern "C" int nl_embed_fwd(const int* tok, const void* wte, const void* wpe, void* out, int M, int S, int D,
                            cudaStream_t stream) {
  if (M <= 0 || S <= 0 || D % 256) return NL_ERR_SHAPE;
  const auto* a = static_cast<const __nv_bfloat16*>(wte);
  const auto* b = static_cast<const __nv_bfloat16*>(wpe);
  auto* o = static_cast<__nv_bfloat16*>(out);
  const int grid = ew::row_grid(M);
  switch (D / 256) {
    case 1: launch_kernel(ew::embed_fwd_kernel<1>, dim3(grid), dim3(256), 0, stream, 1, tok, a, b, o, M, S, D); break;
    case 2: launch_kernel(ew::embed_fwd_kernel<2>, dim3(grid), dim3(256), 0, stream, 1, tok, a, b, o, M, S, D); break;
    case 4: launch_kernel(ew::embed_fwd_kernel<4>, dim3(grid), dim3(256), 0, stream, 1, tok, a, b, o, M, S, D); break;
    default: return NL_ERR_SHAPE;
  }
  return launch_status();
}

extern "C" int nl_embed_bwd(const int* tok, const float* dx, float* dwte, float* dwpe, int M, int S, int D,
                            cudaStream_t stream) {
  if (M <= 0 || S <= 0 || D % 256) return NL_ERR_SHAPE;
  const int grid = ew::row_grid(M);
  switch (D / 256) {
    case 1: launch_kernel(ew::embed_bwd_kernel<1>, dim3(grid), dim3(256), 0, stream, 1, tok, dx, dwte, dwpe, M, S, D); break;
    case 2: launch_kernel(ew::embed_bwd_kernel<2>, dim3(grid), dim3(256), 0, stream, 1, tok, dx, dwte, dwpe, M, S, D); break;
    case 4: launch_kernel(ew::embed_bwd_kernel<4>, dim3(grid), dim3(256), 0, stream, 1, tok, dx, dwte, dwpe, M, S, D); break;
    default: return NL_ERR_SHAPE;
  }
  return launch_status();
}

extern "C" int nl_layernorm_fwd(const void* x, const float* g, const float* b, void* y, float* mean, float* rstd,
                                int M, int D, float eps, cudaStream_t stream) {
  if (M <= 0 || D % 256) return NL_ERR_SHAPE;
  const auto* xi = static_cast<const __nv_bfloat16*>(x);
  auto* yo = static_cast<__nv_bfloat16*>(y);
  const int grid = ew::row_grid(M);
  switch (D / 256) {
    case 1: launch_kernel(ew::layernorm_fwd_kernel<1>, dim3(grid), dim3(256), 0, stream, 1, xi, g, b, yo, mean, rstd, M, D, eps); break;
    case 2: launch_kernel(ew::layernorm_fwd_kernel<2>, dim3(grid), dim3(256), 0, stream, 1, xi, g, b, yo, mean, rstd, M, D, eps); break;
    case 4: launch_kernel(ew::layernorm_fwd_kernel<4>, dim3(grid), dim3(256), 0, stream, 1, xi, g, b, yo, mean, rstd, M, D, eps); break;
    default: return NL_ERR_SHAPE;
  }
  return launch_status();
}

extern "C" int nl_layernorm_bwd(const void* dy, const void* x, const float* mean, const float* rstd, const float* g,
                                float* dres, void* dres_bf16, float* dg, float* db, float* dsum, int M, int D,
                                int accumulate, cudaStream_t stream) {
  if (M <= 0 || D % 256) return NL_ERR_SHAPE;
  const auto* dyi = static_cast<const __nv_bfloat16*>(dy);
  const auto* xi = static_cast<const __nv_bfloat16*>(x);
  auto* rb = static_cast<__nv_bfloat16*>(dres_bf16);
  int grid = ew::row_grid(M);
  if (grid > 2 * sm_count()) grid = 2 * sm_count();  // few blocks: cheap gamma/beta atomics
  switch (D / 256) {
    case 1:
      launch_kernel(ew::layernorm_bwd_kernel<1>, dim3(grid), dim3(256), 0, stream, 1, dyi, xi, mean, rstd, g, dres, rb, dg, db, dsum, M, D, accumulate);
      break;
    case 2:
      launch_kernel(ew::layernorm_bwd_kernel<2>, dim3(grid), dim3(256), 0, stream, 1, dyi, xi, mean, rstd, g, dres, rb, dg, db, dsum, M, D, accumulate);
      break;
    case 4:
      launch_kernel(ew::layernorm_bwd_kernel<4>, dim3(grid), dim3(256), 0, stream, 1, dyi, xi, mean, rstd, g, dres, rb, dg, db, dsum, M, D, accumulate);
      break;
    default: return NL_ERR_SHAPE;
  }
  return launch_status();
}

extern "C" int nl_colsum_bf16(const void* x, float* out, int M, int N, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || N % 8) return NL_ERR_SHAPE;
  const int rows_per_block = 64;
  dim3 grid((N / 8 + 31) / 32, (M + rows_per_block - 1) / rows_per_block);
  launch_kernel(ew::colsum_kernel, dim3(grid), dim3(256), 0, stream, 1, static_cast<const __nv_bfloat16*>(x), out, M, N, rows_per_block);
  return launch_status();
}

extern "C" int nl_adamw_step(float* p, float* g, float* m, float* v, void* shadow_bf16, long long n,
                             const float* hyper, float b1, float b2, float eps, float wd, int zero_grad,
                             cudaStream_t stream) {
  if (n <= 0 || (n & 3)) return NL_ERR_SHAPE;
  const long long n4 = n / 4;
  long long blocks = (n4 + 255) / 256;
  const long long cap = static_cast<long long>(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  launch_kernel(ew::adamw_kernel, dim3(static_cast<int>(blocks)), dim3(256), 0, stream, 1, p, g, m, v,
                                                                   static_cast<__nv_bfloat16*>(shadow_bf16), n4,
                                                                   hyper, b1, b2, eps, wd, zero_grad);
  return launch_status();
}

extern "C" int nl_adamw_schedule(float* hyper, int* step, float peak_lr, int warmup, int decay_steps, float end_lr,
                                 float b1, float b2, cudaStream_t stream) {
  if (!hyper || !step) return NL_ERR_SHAPE;
  launch_kernel(ew::adamw_schedule_kernel, dim3(1), dim3(1), 0, stream, 1, hyper, step, peak_lr, warmup,
                decay_steps, end_lr, b1, b2);
  return launch_status();
}

extern "C" int nl_cast_bf16(const float* x, void* y, long long n, cudaStream_t stream) {
  if (n <= 0 || (n & 3)) return NL_ERR_SHAPE;
  const long long n4 = n / 4;
  long long blocks = (n4 + 255) / 256;
  const long long cap = static_cast<long long>(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  launch_kernel(ew::cast_bf16_kernel, dim3(static_cast<int>(blocks)), dim3(256), 0, stream, 1, x, static_cast<__nv_bfloat16*>(y), n4);
  return launch_status();
}

extern "C" int nl_rows_mark(const int* tok, long long M, int* mark, int V, cudaStream_t stream) {
  if (M <= 0 || V <= 0 || !tok || !mark) return NL_ERR_SHAPE;
  long long blocks = (M + 255) / 256;
  const long long cap = static_cast<long long>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  launch_kernel(ew::rows_mark_kernel, dim3(static_cast<int>(blocks)), dim3(256), 0, stream, 1, tok, M, mark, V);
  return launch_status();
}

extern "C" int nl_rows_compact(int* mark, int V, int* idx_on, int* idx_off, int* counts, cudaStream_t stream) {
  if (V <= 0 || !mark || !idx_on || !idx_off || !counts) return NL_ERR_SHAPE;
  const int chunks = (V + 1023) / 1024;
  // counts[2 .. 2 + chunks): the marked-row count of each 1024-row chunk
  int* chunk_on = counts + 2;
  launch_kernel(ew::rows_count_kernel, dim3(chunks), dim3(1024), 0, stream, 1, static_cast<const int*>(mark), V,
                chunk_on);
  int st = launch_status();
  if (st) return st;
  launch_kernel(ew::rows_list_kernel, dim3(chunks), dim3(1024), 0, stream, 1, mark, V,
                static_cast<const int*>(chunk_on), idx_on, idx_off, counts);
  return launch_status();
}

namespace {
int rows_grid(int max_rows) {
  long long blocks = (static_cast<long long>(max_rows) * 32 + 255) / 256;
  const long long cap = static_cast<long long>(sm_count()) * 8;
  return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}
}  // namespace

extern "C" int nl_rows_gather(const float* src, const int* idx, const int* count, int D, float* dst, int max_rows,
                              cudaStream_t stream) {
  if (D <= 0 || (D & 3) || max_rows <= 0) return NL_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) return NL_ERR_ALIGN;
  launch_kernel(ew::rows_gather_kernel, dim3(rows_grid(max_rows)), dim3(256), 0, stream, 1, src, idx, count, D / 4,
                dst, max_rows);
  return launch_status();
}

extern "C" int nl_rows_scatter(const float* src, const int* idx, const int* count, int D, float* dst, int max_rows,
                               cudaStream_t stream) {
  if (D <= 0 || (D & 3) || max_rows <= 0) return NL_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) return NL_ERR_ALIGN;
  launch_kernel(ew::rows_scatter_kernel, dim3(rows_grid(max_rows)), dim3(256), 0, stream, 1, src, idx, count, D / 4,
                dst, max_rows);
  return launch_status();
}

extern "C" int nl_adamw_rows(float* p, float* g, float* m, float* v, void* shadow_bf16, const int* idx,
                             const int* count, int D, int max_rows, const float* hyper, float b1, float b2, float eps,
                             float wd, int zero_grad, cudaStream_t stream) {
  if (D <= 0 || (D & 3) || max_rows <= 0 || !idx || !count || !hyper) return NL_ERR_SHAPE;
  const long long n4 = static_cast<long long>(max_rows) * (D / 4);
  long long blocks = (n4 + 255) / 256;
  const long long cap = static_cast<long long>(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  launch_kernel(ew::adamw_rows_kernel, dim3(static_cast<int>(blocks)), dim3(256), 0, stream, 1, p, g, m, v,
                static_cast<__nv_bfloat16*>(shadow_bf16), idx, count, D / 4, max_rows, hyper, b1, b2, eps, wd,
                zero_grad);
  return launch_status();
}
