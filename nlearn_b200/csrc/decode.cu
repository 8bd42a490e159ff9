// Inference path: one-token decode steps over a KV cache.
// A device position outside the cache (or past the output row) is reported
// through the library's device error word (code 3) and nothing is written.
//
// Replaces the reference's generate loop (nlearn/model.py:417-465), which runs
// the whole model on the full token buffer for every new token and samples
// with jax.random.categorical(logits / temperature).  Here the prompt is run
// once (prefill, on the training kernels) and each further token costs one
// decode step: the cache keeps every layer's q|k|v rows in the layout of the
// prefill's qkv GEMM output, [B, S_max, 3*D] bf16, so the strided flash
// forward reads it directly.
//
// Kernels (all read the current position from device memory, so a decode
// step has static shapes and is captured once into a CUDA graph):
//   decode_embed_kernel   x[b] = wte[tok[b]] + wpe[pos]
//   decode_attn_kernel    causal attention of the new query row over positions
//                         0..pos; grid (B*H, position splits of 256); the CTA
//                         that holds position pos appends the new k|v row to
//                         the cache; per-split (max, sum, o) partials are merged
//                         by the last CTA of each head (self-resetting counter)
//   sample_kernel         token = argmax_j(logit_j / T + Gumbel_j) (T > 0) or
//                         argmax_j(logit_j) (T == 0); Gumbel_j = -log(-log(u_j))
//                         with u_j from a counter-based hash (SplitMix64's
//                         finaliser, Steele, Lea & Flood 2014) of
//                         (seed, pos, row, j): the sampled distribution is
//                         categorical(softmax(logits / T)), as in the reference
//   advance_kernel        pos += 1
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "host_common.h"
#include "sm100.cuh"

namespace nl {
namespace dec {

constexpr int HD = 64;
constexpr int kChunk = 256;   // positions per split
constexpr int kThreads = 128;

__global__ void decode_embed_kernel(const int* __restrict__ tok, const int* __restrict__ pos,
                                    const __nv_bfloat16* __restrict__ wte, const __nv_bfloat16* __restrict__ wpe,
                                    __nv_bfloat16* __restrict__ x, int B, int D) {
  griddep_sync();
  const int b = blockIdx.x;
  if (b >= B) return;
  const int t = *pos;
  const __nv_bfloat16* e = wte + static_cast<long long>(tok[b]) * D;
  const __nv_bfloat16* p = wpe + static_cast<long long>(t) * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x)
    x[static_cast<long long>(b) * D + i] = __float2bfloat16_rn(__bfloat162float(e[i]) + __bfloat162float(p[i]));
}

struct AttnParams {
  const __nv_bfloat16* qkv_new;  // [B, 3D] this step's q|k|v rows
  __nv_bfloat16* cache;          // [B, S_max, 3D]
  __nv_bfloat16* o;              // [B, D]
  const int* pos;                // current position (device)
  float* part;                   // [B*H, nsplit, 2 + HD]
  int* count;                    // [B*H], zero between calls (the merging CTA resets it)
  int B, H, S_max, nsplit;
  float scale_log2;              // log2(e) / sqrt(HD)
  int* err;                      // device error word
};

__global__ void __launch_bounds__(kThreads) decode_attn_kernel(AttnParams p) {
  griddep_sync();
  __shared__ float q[HD];
  __shared__ float sc[kChunk];
  __shared__ float red[kThreads / 32][HD];
  __shared__ float wred[kThreads / 32];
  __shared__ int is_last;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int D = p.H * HD;
  const int t = *p.pos;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (t < 0 || t >= p.S_max) {  // no cache row for this position: report, touch nothing
    if (tid == 0 && bh == 0 && split == 0 && p.err) atomicExch(p.err, 3);
    return;
  }
  const long long row_pitch = 3LL * D;
  const __nv_bfloat16* newrow = p.qkv_new + b * row_pitch;
  __nv_bfloat16* cb = p.cache + static_cast<long long>(b) * p.S_max * row_pitch;
  const int c0 = split * kChunk;
  const int c1 = min(c0 + kChunk, t + 1);  // positions [c0, c1)
  float* out = p.part + (static_cast<long long>(bh) * p.nsplit + split) * (2 + HD);

  if (c0 < c1) {
    if (tid < HD) q[tid] = __bfloat162float(newrow[h * HD + tid]);
    // the split holding position t appends this step's k|v row to the cache
    if (t >= c0 && t < c0 + kChunk && tid < 2 * HD) {
      const int part = tid / HD, d = tid % HD;  // 0: k, 1: v
      cb[static_cast<long long>(t) * row_pitch + (1 + part) * D + h * HD + d] = newrow[(1 + part) * D + h * HD + d];
    }
    __syncthreads();
    // scores, one position per thread per pass (base-2, scaled)
    float mloc = -INFINITY;
    for (int j = c0 + tid; j < c1; j += kThreads) {
      const __nv_bfloat16* kr = (j == t) ? newrow + D + h * HD : cb + j * row_pitch + D + h * HD;
      const uint4* k4 = reinterpret_cast<const uint4*>(kr);
      float s = 0.f;
#pragma unroll
      for (int v = 0; v < HD / 8; ++v) {
        const uint4 u = k4[v];
        const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(hh[e]);
          s = fmaf(q[v * 8 + 2 * e], f.x, s);
          s = fmaf(q[v * 8 + 2 * e + 1], f.y, s);
        }
      }
      s *= p.scale_log2;
      sc[j - c0] = s;
      mloc = fmaxf(mloc, s);
    }
    // block max
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
    if (lane == 0) wred[warp] = mloc;
    __syncthreads();
    float m = wred[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) m = fmaxf(m, wred[w]);
    __syncthreads();
    // probabilities and their sum
    float lsum = 0.f;
    for (int j = c0 + tid; j < c1; j += kThreads) {
      const float pr = exp2f(sc[j - c0] - m);
      sc[j - c0] = pr;
      lsum += pr;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (lane == 0) wred[warp] = lsum;
    __syncthreads();
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) l += wred[w];
    // o = sum_j p_j v_j: each warp takes every 4th position, a lane two dims
    float o0 = 0.f, o1 = 0.f;
    for (int j = c0 + warp; j < c1; j += kThreads / 32) {
      const __nv_bfloat16* vr = (j == t) ? newrow + 2 * D + h * HD : cb + j * row_pitch + 2 * D + h * HD;
      const float2 v = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(vr)[lane]);
      const float pr = sc[j - c0];
      o0 = fmaf(pr, v.x, o0);
      o1 = fmaf(pr, v.y, o1);
    }
    red[warp][2 * lane] = o0;
    red[warp][2 * lane + 1] = o1;
    __syncthreads();
    if (tid < HD) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) acc += red[w][tid];
      out[2 + tid] = acc;
    }
    if (tid == 0) {
      out[0] = m;
      out[1] = l;
    }
  } else if (tid == 0) {
    out[0] = -INFINITY;
    out[1] = 0.f;
  }
  // the last split of this head to finish merges all splits
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int done = atomicAdd(p.count + bh, 1);
    is_last = (done == p.nsplit - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* base = p.part + static_cast<long long>(bh) * p.nsplit * (2 + HD);
  float M = -INFINITY;
  for (int s = 0; s < p.nsplit; ++s) M = fmaxf(M, __ldcg(base + s * (2 + HD)));
  if (tid < HD) {
    float L = 0.f, acc = 0.f;
    for (int s = 0; s < p.nsplit; ++s) {
      const float ms = __ldcg(base + s * (2 + HD));
      if (ms == -INFINITY) continue;
      const float w = exp2f(ms - M);
      L += w * __ldcg(base + s * (2 + HD) + 1);
      acc += w * __ldcg(base + s * (2 + HD) + 2 + tid);
    }
    p.o[static_cast<long long>(b) * D + h * HD + tid] = __float2bfloat16_rn(acc / L);
  }
  if (tid == 0) p.count[bh] = 0;
}

// SplitMix64 finaliser (Steele, Lea & Flood, OOPSLA 2014).
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

// One CTA per row: argmax over the vocabulary of logit/T + Gumbel noise.
__global__ void __launch_bounds__(1024) sample_kernel(const float* __restrict__ logits, long long ldl, int V,
                                                     float inv_temp, int greedy, unsigned long long seed,
                                                     const int* __restrict__ pos, int* __restrict__ tok,
                                                     int* __restrict__ out, long long ldo, int* err) {
  griddep_sync();
  __shared__ float bv[32];
  __shared__ int bi[32];
  const int b = blockIdx.x;
  const int t = *pos;
  const float* row = logits + b * ldl;
  const uint64_t key = mix64(seed ^ mix64((static_cast<uint64_t>(t) << 32) ^ static_cast<uint64_t>(b)));
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    float v = row[j];
    if (!greedy) {
      const uint64_t r = mix64(key + static_cast<uint64_t>(j));
      const float u = (static_cast<float>(r >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1), 24 bits
      v = v * inv_temp - logf(-logf(u));
    }
    if (v > best || (v == best && j < bidx)) {
      best = v;
      bidx = j;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
    if (ov > best || (ov == best && oi < bidx)) {
      best = ov;
      bidx = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = bidx;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? bv[lane] : -INFINITY;
    bidx = lane < nw ? bi[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
      if (ov > best || (ov == best && oi < bidx)) {
        best = ov;
        bidx = oi;
      }
    }
    if (lane == 0) {
      tok[b] = bidx;
      if (out) {
        if (t + 1 >= 0 && t + 1 < ldo) out[b * ldo + t + 1] = bidx;
        else if (err) atomicExch(err, 3);  // position past the output row: reported, not written
      }
    }
  }
}

__global__ void advance_kernel(int* pos) {
  griddep_sync();
  *pos += 1;
}

}  // namespace dec
}  // namespace nl

using namespace nl;

extern "C" int nl_decode_embed(const int* tok, const int* pos, const void* wte, const void* wpe, void* x, int B,
                               int D, cudaStream_t stream) {
  if (B <= 0 || D <= 0 || !tok || !pos) return NL_ERR_SHAPE;
  launch_kernel(dec::decode_embed_kernel, dim3(B), dim3(256), 0, stream, 1, tok, pos,
                static_cast<const __nv_bfloat16*>(wte), static_cast<const __nv_bfloat16*>(wpe),
                static_cast<__nv_bfloat16*>(x), B, D);
  return launch_status();
}

extern "C" size_t nl_decode_workspace_bytes(int B, int H, int S_max) {
  const long long nsplit = (S_max + dec::kChunk - 1) / dec::kChunk;
  const size_t part = static_cast<size_t>(B) * H * nsplit * (2 + dec::HD) * sizeof(float);
  return ((part + 255) & ~size_t(255)) + static_cast<size_t>(B) * H * sizeof(int);
}

extern "C" int nl_decode_attention(const void* qkv_new, void* cache, void* o, const int* pos, void* workspace,
                                   size_t ws_bytes, int B, int H, int S_max, int d, cudaStream_t stream) {
  if (d != dec::HD) return NL_ERR_SHAPE;
  if (B <= 0 || H <= 0 || S_max <= 0 || !pos) return NL_ERR_SHAPE;
  if (!workspace || ws_bytes < nl_decode_workspace_bytes(B, H, S_max)) return NL_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(qkv_new) | reinterpret_cast<uintptr_t>(cache) |
       reinterpret_cast<uintptr_t>(workspace)) & 15)
    return NL_ERR_ALIGN;
  const int nsplit = (S_max + dec::kChunk - 1) / dec::kChunk;
  const size_t part_bytes = static_cast<size_t>(B) * H * nsplit * (2 + dec::HD) * sizeof(float);
  dec::AttnParams p;
  p.qkv_new = static_cast<const __nv_bfloat16*>(qkv_new);
  p.cache = static_cast<__nv_bfloat16*>(cache);
  p.o = static_cast<__nv_bfloat16*>(o);
  p.pos = pos;
  p.part = static_cast<float*>(workspace);
  p.count = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + ((part_bytes + 255) & ~size_t(255)));
  p.B = B;
  p.H = H;
  p.S_max = S_max;
  p.nsplit = nsplit;
  p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(dec::HD));
  p.err = device_error_word();
  launch_kernel(dec::decode_attn_kernel, dim3(B * H, nsplit), dim3(dec::kThreads), 0, stream, 1, p);
  return launch_status();
}

extern "C" int nl_sample_tokens(const float* logits, long long ldl, int V, float temperature,
                                unsigned long long seed, const int* pos, int* tok, int* out, long long ldo, int B,
                                cudaStream_t stream) {
  if (B <= 0 || V <= 0 || ldl < V || !pos || !tok) return NL_ERR_SHAPE;
  const int greedy = temperature <= 0.f;
  launch_kernel(dec::sample_kernel, dim3(B), dim3(1024), 0, stream, 1, logits, ldl, V,
                greedy ? 1.f : 1.f / temperature, greedy, seed, pos, tok, out, ldo, device_error_word());
  return launch_status();
}

extern "C" int nl_decode_advance(int* pos, cudaStream_t stream) {
  if (!pos) return NL_ERR_SHAPE;
  launch_kernel(dec::advance_kernel, dim3(1), dim3(1), 0, stream, 1, pos);
  return launch_status();
}
