// gemm.cu — persistent warp-specialised bf16 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces nlearn's Metal `gemm_sg` (iree_metal/kernels/gemm.metal:48-115, C f32 =
// A bf16 . B bf16 with 32x32 simdgroup tiles) and the transposes its backward
// materialises (nlearn/kernels/gemm.py:71-76): either operand may be K-major or
// MN-major in global memory, so dX = dY.W^T and dW = X^T.dY read the forward
// tensors in place.
//
// CTA = 10 warps, one CTA per SM, persistent over output tiles:
//   warp 0      TMA producer: A/B k-blocks (64 deep) into a STAGES-deep ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..9  epilogue (two warps per TMEM lane quarter, half the columns each): tcgen05.ld of the f32 accumulator (one TMEM lane =
//               one output row per thread), fused bias / GELU / residual /
//               accumulate, vectorised stores
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the main loop of tile i+1.  Split-K (for the long-K,
// few-tile dW GEMMs) accumulates with vector float atomics.
#include <stdlib.h>
#include <string.h>

#include "sm100.cuh"
#include "host_common.h"
#include "gemm.h"

namespace nl {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle row of bf16
// 2 control warps + 8 epilogue warps (two per TMEM lane quarter, each taking
// half of the tile's columns) so the epilogue keeps pace with the MMAs.
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr int kStagingBytes = kEpiWarps * 4096;  // one 32x32 f32 block per epilogue warp

struct Params {
  int M, N, K;
  int tiles_m, tiles_n, split_k, kb_per_split, num_kb;
  void* C;
  long long ldc;
  int c_bf16;
  int epi;
  float alpha;
  const float* bias;
  __nv_bfloat16* aux;
  const void* resid;
  int* err;
  // fused LM-head cross-entropy epilogues
  const int* targets;   // [M] target column (global vocab index)
  float2* part;         // LCE_STATS: [2*tiles_n, M] per half-tile (max, sum exp(x-max)), natural units
  float* tgt_logit;     // LCE_STATS: [M] logit of the target column
  const float* lse;     // LCE_GRAD: [M] natural-log logsumexp
  const float* gptr;    // LCE_GRAD: optional device scalar multiplying grad_scale
  float grad_scale;     // LCE_GRAD: dlogits multiplier (1/M for a mean loss)
  int v_valid;          // columns >= v_valid are vocabulary padding (masked)
  int epi_warps;        // 4 or 8 active epilogue warps
  int tma_out;          // 1: outputs leave through staged TMA stores (tmC / tmX valid)
  int group_m;          // M tiles per raster group
  int col_offset;       // global vocab index of this launch's column 0
  int stream_k;         // 1: workers own equal contiguous ranges of (tile, k-block) iterations
};

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;  // 16 KB
  static constexpr int B_BYTES = BN * BK * 2;  // 16 / 32 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + kStagingBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// GELU, tanh form (the BASELINE model's FFN activation) and its derivative.
__device__ __forceinline__ float gelu_tanh(float a) {
  const float t = tanh_approx(0.7978845608028654f * (a + 0.044715f * a * a * a));
  return 0.5f * a * (1.f + t);
}
__device__ __forceinline__ float gelu_tanh_grad(float a) {
  const float t = tanh_approx(0.7978845608028654f * (a + 0.044715f * a * a * a));
  return 0.5f * (1.f + t) + 0.5f * a * (1.f - t * t) * 0.7978845608028654f * (1.f + 3.f * 0.044715f * a * a);
}

// Decode a work unit into (m block, n block, split index) with an M-grouped
// raster so that consecutive CTAs share B panels in L2.
__device__ __forceinline__ void decode_unit(const Params& p, int u, int& mb, int& nb, int& sk) {
  const int tiles = p.tiles_m * p.tiles_n;
  sk = u / tiles;
  int t = u - sk * tiles;
  const int G = p.group_m;
  const int per_group = G * p.tiles_n;
  const int g = t / per_group;
  const int first_m = g * G;
  const int gsz = min(p.tiles_m - first_m, G);
  const int r = t - g * per_group;
  mb = first_m + r % gsz;
  nb = r / gsz;
}

// A CTA's (or CTA pair's) sequence of work: tiles, each with a k-block range.
// Unit mode: units u = worker, worker + workers, ... (tiles x split-K parts).
// Stream-K mode (p.stream_k, accumulating epilogue only): worker w owns the
// contiguous range [w T / W, (w+1) T / W) of the T = tiles x num_kb
// (tile, k-block) iterations, cut at tile boundaries, so every worker does the
// same number of k-blocks whatever the tile count; the partial tiles combine
// through the epilogue's reduce-adds.  Every role of a CTA walks the same
// sequence.
struct Work {
  long long it, end;  // stream-K
  int u, stride;      // unit mode
};
__device__ __forceinline__ Work work_begin(const Params& p, int worker, int workers) {
  Work w{0, 0, worker, workers};
  if (p.stream_k) {
    const long long T = static_cast<long long>(p.tiles_m) * p.tiles_n * p.num_kb;
    w.it = T * worker / workers;
    w.end = T * (worker + 1) / workers;
  }
  return w;
}
__device__ __forceinline__ bool work_next(const Params& p, Work& w, int& mb, int& nb, int& kb0, int& kb1) {
  int sk;
  if (p.stream_k) {
    if (w.it >= w.end) return false;
    const int tile = static_cast<int>(w.it / p.num_kb);
    kb0 = static_cast<int>(w.it - static_cast<long long>(tile) * p.num_kb);
    const long long left = w.end - w.it;
    kb1 = (left < p.num_kb - kb0) ? kb0 + static_cast<int>(left) : p.num_kb;
    w.it += kb1 - kb0;
    decode_unit(p, tile, mb, nb, sk);
    return true;
  }
  if (w.u >= p.tiles_m * p.tiles_n * p.split_k) return false;
  decode_unit(p, w.u, mb, nb, sk);
  kb0 = sk * p.kb_per_split;
  kb1 = min(p.num_kb, kb0 + p.kb_per_split);
  w.u += w.stride;
  return true;
}

constexpr float kLog2e = 1.4426950408889634f;

// Epilogue families, one kernel instantiation each.
constexpr int kEpiGeneric = 0;   // STORE / ACCUM / BIAS / BIAS_GELU / RESID / DGELU
constexpr int kEpiLceStats = 1;  // LCE_STATS
constexpr int kEpiLceGrad = 2;   // LCE_GRAD

// Online (max, sum-exp) of 32 logits of one row, the max kept in base-2 units
// (m = max(x) log2 e, so each term is one FFMA and one MUFU ex2:
// 2^(x log2 e - m)); padding columns (>= v_valid) are skipped, and the target
// logit is picked out only in the chunk that holds it.
__device__ __forceinline__ void lce_stats_chunk(const Params& p, int row, int col0, const float (&v)[32], float& m,
                                                   float& s, float& tl, int t) {
  const int valid = p.v_valid - col0;
  if (valid <= 0) return;
  const int ti = t - col0;
  if (static_cast<unsigned>(ti) < 32u) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i == ti) tl = v[i];
  }
  float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  if (valid >= 32) {
#pragma unroll
    for (int i = 0; i < 32; ++i) mx4[i & 3] = fmaxf(mx4[i & 3], v[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < valid) mx4[i & 3] = fmaxf(mx4[i & 3], v[i]);
  }
  const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * kLog2e;
  if (mx > m) {
    s *= ex2_approx(m - mx);
    m = mx;
  }
  const float nm = -m;
  float s4[4] = {0.f, 0.f, 0.f, 0.f};  // four partial sums: shorter FADD chains
  if (valid >= 32) {
#pragma unroll
    for (int i = 0; i < 32; ++i) s4[i & 3] += ex2_approx(fmaf(v[i], kLog2e, nm));
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < valid) s4[i & 3] += ex2_approx(fmaf(v[i], kLog2e, nm));
  }
  s += (s4[0] + s4[1]) + (s4[2] + s4[3]);
}

// dlogits = (softmax - onehot) * scale for 32 columns, bf16 out; padding -> 0.
__device__ __forceinline__ void lce_grad_chunk(const Params& p, int row, int col0, const float (&v)[32], float lse2,
                                               int t, float scale) {
  if (row >= p.M) return;
  uint32_t pk[16];
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    float d[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = col0 + i + h;
      const float pr = ex2_approx(v[i + h] * kLog2e - lse2);
      d[h] = (c < p.v_valid) ? (pr - (c == t ? 1.f : 0.f)) * scale : 0.f;
    }
    pk[i / 2] = pack_bf16x2(d[0], d[1]);
  }
  __nv_bfloat16* cb = reinterpret_cast<__nv_bfloat16*>(p.C) + (long long)row * p.ldc + col0;
  if (col0 + 32 <= p.N && (p.ldc & 7) == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      reinterpret_cast<uint4*>(cb)[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
  } else {
    for (int i = 0; i < 32 && col0 + i < p.N; ++i) {
      const uint32_t w = pk[i / 2];
      const unsigned short h = (i & 1) ? (w >> 16) : (w & 0xffff);
      cb[i] = __ushort_as_bfloat16(h);
    }
  }
}

// dlogits values (f32) of 32 columns for the staged-store path; padding -> 0.
__device__ __forceinline__ void lce_grad_values(const Params& p, int col0, float (&v)[32], float lse2, int t,
                                                float scale) {
  // (2^(x log2 e - lse log2 e) - [c == t]) * scale: one FFMA, one ex2, one FMUL
  // per column; the one-hot term only in the chunk that holds the target.
  const float nl = -lse2;
  const int valid = p.v_valid - col0;
  if (valid >= 32) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = ex2_approx(fmaf(v[i], kLog2e, nl)) * scale;
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = (i < valid) ? ex2_approx(fmaf(v[i], kLog2e, nl)) * scale : 0.f;
  }
  const int ti = t - col0;
  if (static_cast<unsigned>(ti) < 32u && ti < valid) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i == ti) v[i] -= scale;
  }
}

// Epilogue for one thread: row `row`, 32 consecutive columns from `col0`.
__device__ __forceinline__ void epi_chunk(const Params& p, int row, int col0, float (&v)[32]) {
  if (row >= p.M) return;
  const bool full = (col0 + 32 <= p.N);
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] *= p.alpha;
  const int epi = p.epi;
  if (p.bias && (epi == NL_EPI_BIAS || epi == NL_EPI_BIAS_GELU || epi == NL_EPI_RESID)) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += (col0 + i < p.N) ? __ldg(p.bias + col0 + i) : 0.f;
  }
  const long long off = (long long)row * p.ldc + col0;
  if (epi == NL_EPI_BIAS_GELU) {
    __nv_bfloat16* cb = reinterpret_cast<__nv_bfloat16*>(p.C) + off;
    __nv_bfloat16* ab = p.aux + off;
    const bool vec = full && ((p.ldc & 7) == 0);
    if (vec) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 a, c;
        a.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
        a.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
        a.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
        a.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
        c.x = pack_bf16x2(gelu_tanh(v[8 * j + 0]), gelu_tanh(v[8 * j + 1]));
        c.y = pack_bf16x2(gelu_tanh(v[8 * j + 2]), gelu_tanh(v[8 * j + 3]));
        c.z = pack_bf16x2(gelu_tanh(v[8 * j + 4]), gelu_tanh(v[8 * j + 5]));
        c.w = pack_bf16x2(gelu_tanh(v[8 * j + 6]), gelu_tanh(v[8 * j + 7]));
        reinterpret_cast<uint4*>(ab)[j] = a;
        reinterpret_cast<uint4*>(cb)[j] = c;
      }
    } else {
      for (int i = 0; i < 32 && col0 + i < p.N; ++i) {
        ab[i] = __float2bfloat16_rn(v[i]);
        cb[i] = __float2bfloat16_rn(gelu_tanh(v[i]));
      }
    }
    return;
  }
  if (epi == NL_EPI_DGELU) {
    const __nv_bfloat16* pre = p.aux + off;
    for (int i = 0; i < 32; ++i) v[i] *= (col0 + i < p.N) ? gelu_tanh_grad(__bfloat162float(pre[i])) : 0.f;
  }
  if (epi == NL_EPI_RESID && p.resid) {
    if (p.c_bf16) {
      const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(p.resid) + off;
      for (int i = 0; i < 32; ++i) v[i] += (col0 + i < p.N) ? __bfloat162float(rb[i]) : 0.f;
    } else {
      const float* rf = reinterpret_cast<const float*>(p.resid) + off;
      for (int i = 0; i < 32; ++i) v[i] += (col0 + i < p.N) ? rf[i] : 0.f;
    }
  }
  if (epi == NL_EPI_ACCUM) {
    float* cf = reinterpret_cast<float*>(p.C) + off;
    const bool vec = full && ((p.ldc & 3) == 0);
    if (p.split_k > 1 || p.stream_k) {
      if (vec) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          atomicAdd(reinterpret_cast<float4*>(cf) + j, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
      } else {
        for (int i = 0; i < 32 && col0 + i < p.N; ++i) atomicAdd(cf + i, v[i]);
      }
    } else {
      if (vec) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 o = reinterpret_cast<float4*>(cf)[j];
          o.x += v[4 * j];
          o.y += v[4 * j + 1];
          o.z += v[4 * j + 2];
          o.w += v[4 * j + 3];
          reinterpret_cast<float4*>(cf)[j] = o;
        }
      } else {
        for (int i = 0; i < 32 && col0 + i < p.N; ++i) cf[i] += v[i];
      }
    }
    return;
  }
  // plain store (STORE / BIAS / RESID)
  if (p.c_bf16) {
    __nv_bfloat16* cb = reinterpret_cast<__nv_bfloat16*>(p.C) + off;
    if (full && ((p.ldc & 7) == 0)) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 c;
        c.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
        c.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
        c.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
        c.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
        reinterpret_cast<uint4*>(cb)[j] = c;
      }
    } else {
      for (int i = 0; i < 32 && col0 + i < p.N; ++i) cb[i] = __float2bfloat16_rn(v[i]);
    }
  } else {
    float* cf = reinterpret_cast<float*>(p.C) + off;
    if (full && ((p.ldc & 3) == 0)) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        reinterpret_cast<float4*>(cf)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
      for (int i = 0; i < 32 && col0 + i < p.N; ++i) cf[i] = v[i];
    }
  }
}

// ---------------------------------------------------------------- TMA-store epilogue
// A warp owns a 32-row x 32-column block per chunk.  Row-per-thread stores to
// global memory would touch 32 lines per instruction; instead the block is
// written to this warp's 4 KB staging slot in the swizzled layout a TMA store
// expects (f32: 128 B rows, 128-byte swizzle; bf16: 64 B rows, 64-byte
// swizzle, so 8 consecutive lanes hit 8 distinct bank groups) and one lane
// issues a bulk tensor store (or an atomic bulk reduce-add for accumulating
// epilogues, which also makes split-K safe without per-element atomics).
// Rows >= M and columns >= N of the box are clipped by the TMA unit.
__device__ __forceinline__ void stage_f32(uint8_t* slot, int lane, const float (&v)[32]) {
  const uint32_t base = smem_u32(slot) + lane * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t a = base + ((j ^ (lane & 7)) << 4);
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v[4 * j]), "f"(v[4 * j + 1]),
                 "f"(v[4 * j + 2]), "f"(v[4 * j + 3])
                 : "memory");
  }
}
__device__ __forceinline__ void stage_bf16(uint8_t* slot, int lane, const float (&v)[32]) {
  const uint32_t base = smem_u32(slot) + lane * 64;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t a = base + ((j ^ ((lane >> 1) & 3)) << 4);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(pack_bf16x2(v[8 * j], v[8 * j + 1])),
                 "r"(pack_bf16x2(v[8 * j + 2], v[8 * j + 3])), "r"(pack_bf16x2(v[8 * j + 4], v[8 * j + 5])),
                 "r"(pack_bf16x2(v[8 * j + 6], v[8 * j + 7]))
                 : "memory");
  }
}
// Make the staged block visible to the TMA unit and issue the store from lane 0.
__device__ __forceinline__ void flush_block(const CUtensorMap* m, uint8_t* slot, int lane, int col0, int row0,
                                            bool reduce) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (reduce) tma_reduce_add_2d(m, slot, col0, row0);
    else tma_store_2d(m, slot, col0, row0);
    bulk_commit();
  }
}
// Before rewriting the slot: the previous store must have read it.
__device__ __forceinline__ void slot_reuse_wait(int lane) {
  if (lane == 0) bulk_wait_read_all();
  __syncwarp();
}
// A 32x32 bf16 block fills half of the 4 KB slot, so consecutive blocks
// alternate halves and only the store issued two blocks ago must have read
// its half: the staging of block i overlaps the store of block i-1.
__device__ __forceinline__ uint8_t* half_slot(uint8_t* slot, int lane, uint32_t& nblk) {
  if (lane == 0) bulk_wait_read<1>();
  __syncwarp();
  return slot + ((nblk++ & 1u) << 11);
}

__device__ __forceinline__ void epi_chunk_tma(const Params& p, const CUtensorMap* tmC, const CUtensorMap* tmX,
                                              uint8_t* slot, uint32_t& nblk, int lane, int row, int row0, int col0,
                                              float (&v)[32]) {
  const bool in = row < p.M;
  const int epi = p.epi;
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] *= p.alpha;
  if (p.bias && (epi == NL_EPI_BIAS || epi == NL_EPI_BIAS_GELU || epi == NL_EPI_RESID)) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += (col0 + i < p.N) ? __ldg(p.bias + col0 + i) : 0.f;
  }
  const long long off = (long long)row * p.ldc + col0;
  const bool full = col0 + 32 <= p.N;
  if (epi == NL_EPI_BIAS_GELU) {
    slot_reuse_wait(lane);  // aux = pre-activation, C = gelu(pre): two bf16 halves of the slot
    stage_bf16(slot, lane, v);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
    stage_bf16(slot + 2048, lane, v);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmX, slot, col0, row0);
      tma_store_2d(tmC, slot + 2048, col0, row0);
      bulk_commit();
    }
    return;
  }
  if (epi == NL_EPI_DGELU && in) {
    const __nv_bfloat16* pre = p.aux + off;
    if (full && (p.ldc & 7) == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 u = reinterpret_cast<const uint4*>(pre)[j];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(h[k]);
          v[8 * j + 2 * k] *= gelu_tanh_grad(f.x);
          v[8 * j + 2 * k + 1] *= gelu_tanh_grad(f.y);
        }
      }
    } else {
      for (int i = 0; i < 32; ++i) v[i] *= (col0 + i < p.N) ? gelu_tanh_grad(__bfloat162float(pre[i])) : 0.f;
    }
  }
  if (epi == NL_EPI_RESID && p.resid && in) {
    if (p.c_bf16) {
      const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(p.resid) + off;
      if (full && (p.ldc & 7) == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 u = reinterpret_cast<const uint4*>(rb)[j];
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = __bfloat1622float2(h[k]);
            v[8 * j + 2 * k] += f.x;
            v[8 * j + 2 * k + 1] += f.y;
          }
        }
      } else {
        for (int i = 0; i < 32; ++i) v[i] += (col0 + i < p.N) ? __bfloat162float(rb[i]) : 0.f;
      }
    } else {
      const float* rf = reinterpret_cast<const float*>(p.resid) + off;
      for (int i = 0; i < 32; ++i) v[i] += (col0 + i < p.N) ? rf[i] : 0.f;
    }
  }
  if (p.c_bf16) {
    slot = half_slot(slot, lane, nblk);
    stage_bf16(slot, lane, v);
  } else {
    slot_reuse_wait(lane);
    stage_f32(slot, lane, v);
  }
  flush_block(tmC, slot, lane, col0, row0, epi == NL_EPI_ACCUM);
}

// Epilogue warps (2..9): drain each finished accumulator from TMEM, apply the
// fused epilogue, and release the TMEM buffer by arriving on tempty (a local
// barrier, or the pair leader's via its cluster address).  `unit_rows` is the
// M extent of one work unit (128, or 256 for a CTA pair) and `row_off` this
// CTA's first row inside it.  EK selects the epilogue family at compile time
// (kEpiGeneric / kEpiLceStats / kEpiLceGrad) so that each kernel carries only
// the code of its own family.
template <int BN, int EK>
__device__ __forceinline__ void epilogue_role(const Params& p, uint32_t tmem_base, uint64_t* tfull_bar,
                                              uint32_t tempty0, uint32_t tempty1, bool remote, int unit_rows,
                                              int row_off, const Abort& ab, const CUtensorMap* tmC,
                                              const CUtensorMap* tmX, uint8_t* staging) {
  uint8_t* slot = staging + (warp_id() - 2) * 4096;
  const int warp = warp_id(), lane = lane_id();
  const int cta_unit0 = remote ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int cta_stride = remote ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int q = warp & 3;             // TMEM lane quarter this warp may access
  // with 8 epilogue warps each takes half of the tile's columns; with 4 the
  // warps 6..9 idle and warps 2..5 take all columns
  const int split = p.epi_warps / 4;
  const int half = (warp - 2) >> 2;
  int acc = 0;
  uint32_t acc_ph = 0;
  uint32_t nblk = 0;
  Work wk = work_begin(p, cta_unit0, cta_stride);
  int mb, nb, kb0, kb1;
  while (half < split && work_next(p, wk, mb, nb, kb0, kb1)) {
    if (!mbar_wait(&tfull_bar[acc], acc_ph, ab)) break;
    tc_fence_after();
    const int row = mb * unit_rows + row_off + q * 32 + lane;
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
    int t = -1;
    float lse2 = 0.f, gsc = 0.f, m = -INFINITY, ssum = 0.f, tl = 0.f;
    if (EK != kEpiGeneric && row < p.M) {
      t = p.targets[row] - p.col_offset;
      if (EK == kEpiLceGrad) {
        lse2 = p.lse[row] * kLog2e;
        gsc = p.grad_scale * (p.gptr ? *p.gptr : 1.f);
      }
    }
    // The load of chunk c+1 is in flight while chunk c is processed; the
    // accumulator goes back to the MMA warp as soon as its last chunk is in
    // registers.
    auto release = [&]() {
      tc_fence_before();
      if (remote) mbar_arrive_cluster(acc ? tempty1 : tempty0);
      else mbar_arrive(reinterpret_cast<uint64_t*>(__cvta_shared_to_generic(acc ? tempty1 : tempty0)));
    };
    bool released = false;
    const int c_begin = half * (BN / 32 / split), c_end = (half + 1) * (BN / 32 / split);
    uint32_t r[32];
    if (nb * BN + c_begin * 32 < p.N) tmem_ld32(taddr + c_begin * 32, r);
#pragma unroll 1
    for (int c = c_begin; c < c_end; ++c) {
      const int col0 = nb * BN + c * 32;
      if (col0 >= p.N) break;  // warp-uniform
      tmem_wait_ld_tied(r);
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      if (c + 1 < c_end && col0 + 32 < p.N) {
        tmem_ld32(taddr + (c + 1) * 32, r);
      } else {
        release();
        released = true;
      }
      // TMA-store paths are warp-uniform: rows >= M stage garbage that the store clips
      const int row0 = mb * unit_rows + row_off + q * 32;
      if constexpr (EK == kEpiLceStats) {
        lce_stats_chunk(p, row, col0, v, m, ssum, tl, t);
      } else if constexpr (EK == kEpiLceGrad) {
        if (p.tma_out) {
          lce_grad_values(p, col0, v, lse2, t, gsc);
          uint8_t* h = half_slot(slot, lane, nblk);
          stage_bf16(h, lane, v);
          flush_block(tmC, h, lane, col0, row0, false);
        } else {
          lce_grad_chunk(p, row, col0, v, lse2, t, gsc);
        }
      } else {
        if (p.tma_out) epi_chunk_tma(p, tmC, tmX, slot, nblk, lane, row, row0, col0, v);
        else epi_chunk(p, row, col0, v);
      }
    }
    if (EK == kEpiLceStats && row < p.M) {
      m *= 0.6931471805599453f;  // base-2 max -> natural units
      p.part[(long long)(2 * nb + half) * p.M + row] = make_float2(m, ssum);
      if (split == 1) p.part[(long long)(2 * nb + 1) * p.M + row] = make_float2(-INFINITY, 0.f);
      const int c0 = nb * BN + half * (BN / split);
      if (t >= c0 && t < c0 + BN / split && t < p.N) p.tgt_logit[row] = tl;
    }
    if (!released) release();
    acc ^= 1;
    if (acc == 0) acc_ph ^= 1;
  }
  if (lane == 0) bulk_wait_all();  // stores complete before the CTA retires
}

template <int BN, bool A_MN, bool B_MN, int EK>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX, Params p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES + kStagingBytes);
  uint64_t* full_bar = bars;                       // [STAGES]
  uint64_t* empty_bar = bars + C::STAGES;          // [STAGES]
  uint64_t* tfull_bar = bars + 2 * C::STAGES;      // [2]
  uint64_t* tempty_bar = bars + 2 * C::STAGES + 2; // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * C::STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], p.epi_warps * 32);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_sync();
  Abort ab{abort_flag, p.err};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      Work wk = work_begin(p, blockIdx.x, gridDim.x);
      int mb, nb, kb0, kb1;
      while (ok && work_next(p, wk, mb, nb, kb0, kb1)) {
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1, ab)) { ok = false; break; }
          uint8_t* sA = tiles + s * C::STAGE_BYTES;
          uint8_t* sB = sA + C::A_BYTES;
          mbar_expect_tx(&full_bar[s], C::STAGE_BYTES);
          if (!A_MN) {
            tma_load_2d(&tmA, &full_bar[s], sA, kb * BK, mb * BM);
          } else {
#pragma unroll
            for (int h = 0; h < BM / 64; ++h) tma_load_2d(&tmA, &full_bar[s], sA + h * 8192, mb * BM + h * 64, kb * BK);
          }
          if (!B_MN) {
            tma_load_2d(&tmB, &full_bar[s], sB, kb * BK, nb * BN);
          } else {
#pragma unroll
            for (int h = 0; h < BN / 64; ++h) tma_load_2d(&tmB, &full_bar[s], sB + h * 8192, nb * BN + h * 64, kb * BK);
          }
          if (++s == C::STAGES) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      Work wk = work_begin(p, blockIdx.x, gridDim.x);
      int mb, nb, kb0, kb1;
      while (ok && work_next(p, wk, mb, nb, kb0, kb1)) {
        if (!mbar_wait(&tempty_bar[acc], acc_ph ^ 1, ab)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[s], ph, ab)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(tiles + s * C::STAGE_BYTES);
          const uint32_t b0 = a0 + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sdesc_sw128(a0 + k * 2048, 8192, 1024) : sdesc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b0 + k * 2048, 8192, 1024) : sdesc_sw128(b0 + k * 32, 16, 1024);
            umma_f16_ss(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[s]);
          if (++s == C::STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    epilogue_role<BN, EK>(p, tmem_base, tfull_bar, smem_u32(tempty_bar), smem_u32(tempty_bar + 1), false, BM, 0, ab,
                      &tmC, &tmX, tiles + C::STAGES * C::STAGE_BYTES);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

template <int BN, bool A_MN, bool B_MN, int EK>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& tx, Params& p,
           cudaStream_t stream) {
  using C = Cfg<BN>;
  auto kern = gemm_kernel<BN, A_MN, B_MN, EK>;
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return NL_ERR_LAUNCH;
    configured_dev = dev;
  }
  const int units = p.tiles_m * p.tiles_n * p.split_k;
  const int grid = (p.stream_k || units > sm_count()) ? sm_count() : units;
  launch_kernel(kern, dim3(grid), dim3(kThreads), C::SMEM, stream, 1, ta, tb, tc, tx, p);
  return launch_status();
}


template <int EK>
int launch_layout(int BN, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                  const CUtensorMap& tx, Params& p, cudaStream_t stream) {
  if (BN == 256) {
    if (!a_mn && !b_mn) return launch<256, false, false, EK>(ta, tb, tc, tx, p, stream);
    if (!a_mn && b_mn) return launch<256, false, true, EK>(ta, tb, tc, tx, p, stream);
    if (a_mn && !b_mn) return launch<256, true, false, EK>(ta, tb, tc, tx, p, stream);
    return launch<256, true, true, EK>(ta, tb, tc, tx, p, stream);
  }
  if (!a_mn && !b_mn) return launch<128, false, false, EK>(ta, tb, tc, tx, p, stream);
  if (!a_mn && b_mn) return launch<128, false, true, EK>(ta, tb, tc, tx, p, stream);
  if (a_mn && !b_mn) return launch<128, true, false, EK>(ta, tb, tc, tx, p, stream);
  return launch<128, true, true, EK>(ta, tb, tc, tx, p, stream);
}

// ============================================================== CTA-pair GEMM
// Same roles as gemm_kernel, but a 2-CTA cluster computes 256 x 256 tiles with
// cta_group::2 MMAs (M=256, N=256, K=16) issued by the even CTA.  Each CTA
// loads its 128 rows of A and its 128 columns of B per k-block (32 KB, 6
// stages) and holds the accumulator rows of its own half in its TMEM; every
// load's bytes are counted on the leader's full barrier, and the leader's
// commits arrive on both CTAs' empty / tfull barriers.  Per FLOP this moves
// half the B bytes of the single-CTA 128 x 256 tile through L2.
namespace pair {
constexpr int BM2 = 256, BN2 = 256;
constexpr int A_BYTES = 128 * BK * 2;  // 16 KB: this CTA's rows
constexpr int B_BYTES = 128 * BK * 2;  // 16 KB: this CTA's columns
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int STAGES = 6;
constexpr int TMEM_COLS = 2 * BN2;
constexpr int SMEM = STAGES * STAGE_BYTES + kStagingBytes + 1024 + 256;
}  // namespace pair

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX, Params p) {
  using namespace pair;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES + kStagingBytes);
  uint64_t* full_bar = bars;                    // [STAGES]  (leader's are used)
  uint64_t* empty_bar = bars + STAGES;          // [STAGES]
  uint64_t* tfull_bar = bars + 2 * STAGES;      // [2]
  uint64_t* tempty_bar = bars + 2 * STAGES + 2; // [2]       (leader's are used)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const int unit0 = static_cast<int>(blockIdx.x >> 1), ustride = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 2 * p.epi_warps * 32);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_sync();
  Abort ab{abort_flag, p.err};

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      Work wk = work_begin(p, unit0, ustride);
      int mb, nb, kb0, kb1;
      while (ok && work_next(p, wk, mb, nb, kb0, kb1)) {
        const int arow = mb * BM2 + static_cast<int>(rank) * 128;
        const int bcol = nb * BN2 + static_cast<int>(rank) * 128;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1, ab)) { ok = false; break; }
          uint8_t* sA = tiles + s * STAGE_BYTES;
          uint8_t* sB = sA + A_BYTES;
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[s]), 0);
          if (rank == 0) mbar_expect_tx(&full_bar[s], 2 * STAGE_BYTES);
          if (!A_MN) {
            tma_load_2d_pair(&tmA, fb, sA, kb * BK, arow);
          } else {
            tma_load_2d_pair(&tmA, fb, sA, arow, kb * BK);
            tma_load_2d_pair(&tmA, fb, sA + 8192, arow + 64, kb * BK);
          }
          if (!B_MN) {
            tma_load_2d_pair(&tmB, fb, sB, kb * BK, bcol);
          } else {
            tma_load_2d_pair(&tmB, fb, sB, bcol, kb * BK);
            tma_load_2d_pair(&tmB, fb, sB + 8192, bcol + 64, kb * BK);
          }
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM2, BN2, A_MN ? 1 : 0, B_MN ? 1 : 0);
      const uint32_t peer_empty0 = mapa_shared(smem_u32(&empty_bar[0]), 1);
      const uint32_t own_empty0 = mapa_shared(smem_u32(&empty_bar[0]), 0);
      const uint32_t peer_tfull0 = mapa_shared(smem_u32(&tfull_bar[0]), 1);
      const uint32_t own_tfull0 = mapa_shared(smem_u32(&tfull_bar[0]), 0);
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      Work wk = work_begin(p, unit0, ustride);
      int mb, nb, kb0, kb1;
      while (ok && work_next(p, wk, mb, nb, kb0, kb1)) {
        if (!mbar_wait(&tempty_bar[acc], acc_ph ^ 1, ab)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN2;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[s], ph, ab)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(tiles + s * STAGE_BYTES);
          const uint32_t b0 = a0 + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sdesc_sw128(a0 + k * 2048, 8192, 1024) : sdesc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b0 + k * 2048, 8192, 1024) : sdesc_sw128(b0 + k * 32, 16, 1024);
            umma_f16_ss_pair(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair(own_empty0 + s * 8);
          umma_commit_pair(peer_empty0 + s * 8);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(own_tfull0 + acc * 8);
        umma_commit_pair(peer_tfull0 + acc * 8);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
      }
    }
  } else {
    epilogue_role<BN2, kEpiGeneric>(p, tmem_base, tfull_bar, mapa_shared(smem_u32(&tempty_bar[0]), 0),
                       mapa_shared(smem_u32(&tempty_bar[1]), 0), true, BM2, static_cast<int>(rank) * 128, ab, &tmC,
                       &tmX, tiles + STAGES * STAGE_BYTES);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

template <bool A_MN, bool B_MN>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& tx,
                Params& p, cudaStream_t stream) {
  auto kern = gemm_pair_kernel<A_MN, B_MN>;
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pair::SMEM) != cudaSuccess)
      return NL_ERR_LAUNCH;
    configured_dev = dev;
  }
  const int units = p.tiles_m * p.tiles_n * p.split_k;
  const int pairs = sm_count() / 2;
  const int g = (p.stream_k || units > pairs) ? pairs : units;
  if (launch_kernel(kern, dim3(2 * g), dim3(kThreads), pair::SMEM, stream, 2, ta, tb, tc, tx, p) != cudaSuccess) {
    cudaGetLastError();
    count_launch();
    return NL_ERR_LAUNCH;
  }
  return launch_status();
}

}  // namespace gemm

// Device error word shared by all kernels of this library (per device).
int* device_error_word();

int gemm_run(const void* A, long long lda, int a_trans, const void* B, long long ldb, int b_trans, void* Cp,
             long long ldc, int c_dtype, int M, int N, int K, float alpha, int epi, const float* bias, void* aux,
             const void* resid, cudaStream_t stream, const GemmExtra* ex) {
  using namespace gemm;
  if (M <= 0 || N <= 0 || K < 0) return NL_ERR_SHAPE;
  if (c_dtype != NL_F32 && c_dtype != NL_BF16) return NL_ERR_DTYPE;
  if (epi < NL_EPI_STORE || epi > NL_EPI_LCE_GRAD) return NL_ERR_SHAPE;
  if (epi == NL_EPI_ACCUM && c_dtype != NL_F32) return NL_ERR_DTYPE;
  if (epi == NL_EPI_BIAS_GELU && (c_dtype != NL_BF16 || aux == nullptr)) return NL_ERR_DTYPE;
  if (epi == NL_EPI_DGELU && aux == nullptr) return NL_ERR_DTYPE;
  if (epi >= NL_EPI_LCE_STATS && (ex == nullptr || ex->targets == nullptr)) return NL_ERR_WORKSPACE;
  if (epi == NL_EPI_LCE_STATS && (ex->part == nullptr || ex->tgt_logit == nullptr)) return NL_ERR_WORKSPACE;
  if (epi == NL_EPI_LCE_GRAD && (ex->lse == nullptr || c_dtype != NL_BF16)) return NL_ERR_WORKSPACE;
  if (K == 0) {
    if (epi == NL_EPI_ACCUM) return NL_OK;
    return NL_ERR_SHAPE;
  }
  if (ex == nullptr && M <= 8) {
    const int st = gemv_run(A, lda, a_trans, B, ldb, b_trans, Cp, ldc, c_dtype, M, N, K, alpha, epi, bias, aux,
                            resid, stream);
    if (st != -100) return st;
  }
  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = Cp;
  p.ldc = ldc;
  p.c_bf16 = (c_dtype == NL_BF16);
  p.epi = epi;
  p.alpha = alpha;
  p.bias = bias;
  p.aux = reinterpret_cast<__nv_bfloat16*>(aux);
  p.resid = resid;
  p.err = device_error_word();
  p.num_kb = (K + BK - 1) / BK;
  {
    static int ew = -1;
    if (ew < 0) {
      const char* e = getenv("NL_GEMM_EPI_WARPS");
      ew = (e && atoi(e) == 4) ? 4 : 8;
    }
    p.epi_warps = ew;
    static int grp = -1;
    if (grp < 0) {
      const char* e = getenv("NL_GEMM_GROUP");
      grp = (e && atoi(e) > 0) ? atoi(e) : 16;
    }
    p.group_m = grp;
  }
  if (ex) {
    p.targets = ex->targets;
    p.part = ex->part;
    p.tgt_logit = ex->tgt_logit;
    p.lse = ex->lse;
    p.gptr = ex->gptr;
    p.grad_scale = ex->grad_scale;
    p.v_valid = ex->v_valid;
    p.col_offset = ex->col_offset;
  }

  const bool a_mn = a_trans != 0;
  const bool b_mn = b_trans == 0;
  // Narrow N gets 128-wide tiles (more CTAs); wide N gets 256-wide tiles.
  const int sms = sm_count();
  int BN = 256;
  {
    const long long t256 = (long long)((M + BM - 1) / BM) * ((N + 255) / 256);
    // accumulating GEMMs with a long K fill the machine by splitting K instead
    const bool split_fills = epi == NL_EPI_ACCUM && p.num_kb >= 64;
    if (N <= 128 || (t256 < sms && !split_fills)) BN = 128;
    if (ex && ex->force_bn) BN = ex->force_bn;
    static int fbn = -1;
    if (fbn < 0) {
      const char* e = getenv("NL_GEMM_FORCE_BN");
      fbn = e ? atoi(e) : 0;
    }
    if (fbn == 128 || fbn == 256) BN = fbn;
  }
  // 256 x 256 tiles on CTA pairs wherever 256-wide tiles are chosen and there
  // are enough of them (or a long K to split); NL_GEMM_PAIR=0 disables, 2 forces.
  static int pair_enabled = -1;
  if (pair_enabled < 0) {
    const char* e = getenv("NL_GEMM_PAIR");
    pair_enabled = e ? atoi(e) : 1;  // 0 off, 1 auto, 2 always (256-wide tiles)
  }
  // (measured: pairs win from K >= 1024; at K = 512 the single-CTA kernel is faster)
  bool use_pair = pair_enabled == 1 ? (BN == 256 && p.num_kb >= 16) : (pair_enabled == 2 && BN == 256);
  if (epi >= NL_EPI_LCE_STATS) use_pair = false;  // the LCE epilogues run on single-CTA tiles
  const int workers = use_pair ? sms / 2 : sms;
  const int unit_m = use_pair ? pair::BM2 : BM;
  if (use_pair) {
    const long long t2 = (long long)((M + 255) / 256) * ((N + 255) / 256);
    if (t2 < workers && !(epi == NL_EPI_ACCUM && p.num_kb >= 16)) use_pair = false;
  }
  const int wk = use_pair ? workers : sms;
  const int um = use_pair ? unit_m : BM;
  p.tiles_m = (M + um - 1) / um;
  p.tiles_n = (N + BN - 1) / BN;
  // LM-head statistics GEMM (X small, W wide): one raster group over all M
  // tiles, so the whole of X stays in L2 and each W panel is read from DRAM
  // once (measured: 0.646 -> 0.637 ms at M 16384, N 50257, K 512).
  if (epi == NL_EPI_LCE_STATS && !getenv("NL_GEMM_GROUP") &&
      static_cast<long long>(M) * K * 2 <= (32LL << 20))
    p.group_m = p.tiles_m;
  const int tiles = p.tiles_m * p.tiles_n;
  // Split-K for accumulate-mode GEMMs (the splits combine through the TMA
  // reduce-add): pick the split, at least 8 k-blocks each, that gives the
  // best wave efficiency units / (waves * workers); ties go to fewer splits.
  p.split_k = 1;
  if (epi == NL_EPI_ACCUM && p.num_kb >= 16) {
    double best = 0.0;
    const int smax = p.num_kb / 8 < 32 ? p.num_kb / 8 : 32;
    for (int sk = 1; sk <= smax; ++sk) {
      const long long units = (long long)tiles * sk;
      const long long waves = (units + wk - 1) / wk;
      const double eff = (double)units / (double)(waves * wk);
      if (eff > best + 0.02) {
        best = eff;
        p.split_k = sk;
      }
    }
  }
  // Stream-K for accumulating GEMMs with few output tiles and a long K (the
  // weight gradients, K = tokens): equal k-block ranges per worker instead of
  // whole split-K parts, so no wave is left part-empty.  NL_GEMM_STREAMK=0
  // turns it off, =1 forces it for every accumulating GEMM.
  {
    static int sk_env = -2;
    if (sk_env == -2) {
      const char* e = getenv("NL_GEMM_STREAMK");
      sk_env = e ? atoi(e) : -1;
    }
    // measured on the weight-gradient shapes (K = 16384): stream-K wins where
    // no split-K count fills one wave of workers (512 x 2048: 16 pair tiles,
    // at best 64 of 74 pairs busy: 39.3 -> 34.4 us) and loses where one does
    // (512 x 1536: 12 tiles x 6 parts = 72 of 74: 26.9 -> 28.6 us); with more
    // tiles than workers it spreads each B panel's readers apart in time and
    // loses its L2 reuse (the LM-head weight gradient: 2.10 -> 2.31 ms)
    double one_wave = 0.0;
    for (int sk = 1; sk <= p.num_kb / 8 && static_cast<long long>(tiles) * sk <= wk; ++sk)
      one_wave = static_cast<double>(tiles) * sk / wk;
    const bool want = (epi == NL_EPI_ACCUM) &&
                      (sk_env == 1 || (sk_env != 0 && p.num_kb >= 32 && tiles < wk && one_wave < 0.9));
    if (want) {
      p.stream_k = 1;
      p.split_k = 1;
    }
  }
  p.kb_per_split = (p.num_kb + p.split_k - 1) / p.split_k;
  p.split_k = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;

  CUtensorMap ta, tb;
  int st;
  if (!a_mn) st = make_tmap_bf16_2d(&ta, A, K, M, lda, 64, BM);
  else st = make_tmap_bf16_2d(&ta, A, M, K, lda, 64, BK);
  if (st) return st;
  if (!b_mn) st = make_tmap_bf16_2d(&tb, B, K, N, ldb, 64, use_pair ? 128 : BN);
  else st = make_tmap_bf16_2d(&tb, B, N, K, ldb, 64, BK);
  if (st) return st;
  // Output through staged TMA stores when the output rows are 16-byte aligned.
  CUtensorMap tc, tx;
  memset(&tc, 0, sizeof(tc));
  memset(&tx, 0, sizeof(tx));
  p.tma_out = 0;
  if (Cp != nullptr && epi != NL_EPI_LCE_STATS) {
    bool ok = make_tmap_out_2d(&tc, Cp, p.c_bf16 != 0, N, M, ldc) == NL_OK;
    if (ok && epi == NL_EPI_BIAS_GELU) ok = make_tmap_out_2d(&tx, aux, true, N, M, ldc) == NL_OK;
    p.tma_out = ok ? 1 : 0;
  }

  if (use_pair) {
    if (!a_mn && !b_mn) return launch_pair<false, false>(ta, tb, tc, tx, p, stream);
    if (!a_mn && b_mn) return launch_pair<false, true>(ta, tb, tc, tx, p, stream);
    if (a_mn && !b_mn) return launch_pair<true, false>(ta, tb, tc, tx, p, stream);
    return launch_pair<true, true>(ta, tb, tc, tx, p, stream);
  }
  const int ek = epi == NL_EPI_LCE_STATS ? kEpiLceStats : epi == NL_EPI_LCE_GRAD ? kEpiLceGrad : kEpiGeneric;
  if (ek == kEpiLceStats) return launch_layout<kEpiLceStats>(BN, a_mn, b_mn, ta, tb, tc, tx, p, stream);
  if (ek == kEpiLceGrad) return launch_layout<kEpiLceGrad>(BN, a_mn, b_mn, ta, tb, tc, tx, p, stream);
  return launch_layout<kEpiGeneric>(BN, a_mn, b_mn, ta, tb, tc, tx, p, stream);
}

}  // namespace nl

extern "C" int nl_gemm_ex(const void* A, int lda, int a_trans, const void* B, int ldb, int b_trans, void* C,
                          int ldc, int c_dtype, int M, int N, int K, float alpha, int epilogue, const float* bias,
                          void* aux, const void* resid, cudaStream_t stream) {
  if (epilogue > NL_EPI_DGELU) return NL_ERR_SHAPE;  // LCE epilogues go through nl_lce_*
  return nl::gemm_run(A, lda, a_trans, B, ldb, b_trans, C, ldc, c_dtype, M, N, K, alpha, epilogue, bias, aux,
                      resid, stream, nullptr);
}

extern "C" int nl_gemm(const void* A, const void* B, float* C, int M, int N, int K, cudaStream_t stream) {
  return nl::gemm_run(A, K, 0, B, N, 0, C, N, NL_F32, M, N, K, 1.0f, NL_EPI_STORE, nullptr, nullptr, nullptr,
                      stream, nullptr);
}
