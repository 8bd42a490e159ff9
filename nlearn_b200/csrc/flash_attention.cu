// flash_attention.cu — causal FlashAttention forward + O(seq)-memory backward, sm_100a.
//
// Replaces nlearn's Metal kernels (iree_metal/kernels/flash_attention.metal):
//   fwd       55-146  O = softmax(scale Q K^T + causal) V,  L = m + log(l)  (natural log)
//   bwd_dq   168-243  dQ = scale sum_j p_ij (dP_ij - D_i) K_j
//   bwd_dkdv 265-347  dV = P^T dO,  dK = scale dS^T Q
// with p = exp(scale s - L) recomputed from L, D = rowsum(dO * O)
// (nlearn/attention.py:116).  Layout [n = batch*heads, s, d=64], bf16 Q/K/V/O/dO,
// f32 L and D, scale = 1/sqrt(64) (flash_attention.metal:64).
//
// Forward, one CTA per (head, 128-query tile), 6 warps, 2 CTAs per SM:
//   warp 0     TMA: Q once, K_j / V_j into 2-slot rings
//   warp 1     TMEM alloc (256 cols) + tcgen05.mma issuer:
//                S = Q K_j^T  -> TMEM cols [0,128)    (M=128, N=128, K=64)
//                O += P_j V_j -> TMEM cols [128,192)  (M=128, N=64,  K=128; P read
//                                from TMEM cols [192,256), V from shared memory)
//              S_{j+1} is issued as soon as the softmax warps have pulled S_j
//              into registers, so it overlaps softmax_j.
//   warps 2-5  softmax, one query row per thread: exp2-domain online softmax,
//              O rescale in TMEM (tcgen05.ld/st) when the row max grows,
//              P_j -> bf16 pairs in TMEM (the A operand of the PV MMA).
// Causal tiles above the diagonal are never visited; heavy (late) query tiles
// are scheduled first.
//
// Backward, one CTA per (head, 128-key tile), 14 warps, 1 CTA per SM:
//   warp 0     TMA: K, V once; Q_i / dO_i into 2-slot rings
//   warp 1     TMEM alloc (512 cols) + MMA issuer, per query tile i >= key tile:
//                S^T  = K Q_i^T        cols [0,128)
//                dP^T = V dO_i^T       cols [128,256)
//                dV  += P^T dO_i       cols [256,320)   (A = P^T from TMEM cols [448,512),
//                                                        B = dO_i read MN-major)
//                dK  += dS^T Q_i       cols [320,384)   (B = Q_i  read MN-major)
//                dQ_i = dS K           cols [384,448)   (A = dS^T read MN-major)
//   warps 2-9  one key row per thread, two warps per row quarter splitting the
//              query columns: P^T = exp2(S^T scale log2e - L log2e),
//              dS^T = P^T (dP^T - D); P^T -> bf16 in TMEM, dS^T -> bf16 shared memory
//   warps 10-13 dQ_i tile: TMEM -> swizzled f32 staging -> TMA bulk reduce-add
//              into an f32 accumulator
// followed by a convert kernel dQ = bf16(scale * dQacc).
#include <atomic>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>

#include "host_common.h"
#include "sm100.cuh"

namespace nl {
namespace fa {

constexpr int HD = 64;      // head dim (the reference's MAX_DHEAD, flash_attention.metal:17)
constexpr int BQ = 128;     // query rows per tile
constexpr int BKV = 128;    // key rows per tile
constexpr int TILE = BQ * HD * 2;  // 16 KB bf16 tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Byte offset of element (row r, col k) of a [rows x 128] bf16 matrix stored as
// two K-major SW128 column halves of 16 KB each (the UMMA canonical layout the
// TMA would produce), for 16-byte chunk index c8 = k / 8.
__device__ __forceinline__ uint32_t sw128_off(int r, int c8) {
  return (c8 >> 3) * 16384 + (r >> 3) * 1024 + (r & 7) * 128 + (((c8 & 7) ^ (r & 7)) << 4);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ====================================================================== forward
namespace fwd {
constexpr int kThreads = 6 * 32;
constexpr int OFF_Q = 0;              // 2 slots (the next item's Q loads during this item)
constexpr int OFF_K = 2 * TILE;       // 2 slots
constexpr int OFF_V = 4 * TILE;       // 2 slots
constexpr int OFF_BAR = 6 * TILE;
constexpr int SMEM = OFF_BAR + 256;
constexpr int TMEM_COLS = 256;
constexpr int COL_S = 0, COL_O = 128, COL_P = 192;  // P: 128 bf16 per row packed in 64 columns
}  // namespace fwd

// Activations are addressed as [b][h][s][64] with element strides, so Q/K/V
// can be read straight out of a fused QKV projection and O written in the
// layout the output projection consumes (no permute copies).
struct Strides {
  long long s, h, b;
};

struct FwdParams {
  __nv_bfloat16* O;
  Strides os;
  float* L;
  int n, H, s, nq;
  float sl2;  // scale * log2(e)
  int* err;
};

// Forward work item w (0 .. n*nq-1): query tile qb = nq-1 - w/n (heaviest,
// i.e. latest, query tiles first), head = w % n.  Round k deals items
// k*G .. k*G+G-1 to the G persistent CTAs, forwards in even rounds and
// backwards in odd ones.
__device__ __forceinline__ int fwd_round_item(int k) {
  const int G = static_cast<int>(gridDim.x), b = static_cast<int>(blockIdx.x);
  return k * G + ((k & 1) ? G - 1 - b : b);
}

// Persistent: 2 CTAs per SM, each walking its items with TMEM allocated and
// barriers initialised once.  Ring counters run over the CTA's whole item
// sequence (K/V tiles jg, items it), so the next item's Q and first K/V tiles
// load, and its first S MMA runs, while this item's softmax warps write O.
__global__ void __launch_bounds__(fwd::kThreads, 2)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, FwdParams p) {
  using namespace fwd;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars + 0;   // [2]
  uint64_t* q_empty = bars + 2;  // [2]
  uint64_t* k_full = bars + 4;   // [2]
  uint64_t* k_empty = bars + 6;  // [2]
  uint64_t* v_full = bars + 8;   // [2]
  uint64_t* v_empty = bars + 10; // [2]
  uint64_t* s_full = bars + 12;
  uint64_t* s_free = bars + 13;
  uint64_t* p_full = bars + 14;
  uint64_t* o_done = bars + 15;
  uint64_t* o_free = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int n_items = p.n * p.nq;

  if (smem_u32(smem) & 1023) {  // SW128 tiles need 1 KB alignment
    if (threadIdx.x == 0 && p.err) atomicExch(p.err, 2);
    return;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 128);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(o_free, 128);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  Abort ab{abort_flag, p.err};
  griddep_sync();

  auto item_of = [&](int w, int& qb, int& head) {
    qb = p.nq - 1 - w / p.n;
    head = w % p.n;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA loads
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      bool ok = true;
      int jg = 0;
      for (int it = 0, w = fwd_round_item(0); ok && w < n_items; w = fwd_round_item(++it)) {
        int qb, head;
        item_of(w, qb, head);
        const int bi = head / p.H, hi = head % p.H;
        const int qs = it & 1;
        if (it >= 2 && !mbar_wait(&q_empty[qs], ((it >> 1) - 1) & 1, ab)) break;
        mbar_expect_tx(&q_full[qs], TILE);
        tma_load_4d(&tmQ, &q_full[qs], smem + OFF_Q + qs * TILE, 0, qb * BQ, hi, bi);
        for (int j = 0; j <= qb; ++j, ++jg) {
          const int slot = jg & 1;
          const uint32_t ph = (jg >> 1) & 1;
          if (!mbar_wait(&k_empty[slot], ph ^ 1, ab)) { ok = false; break; }
          mbar_expect_tx(&k_full[slot], TILE);
          tma_load_4d(&tmK, &k_full[slot], smem + OFF_K + slot * TILE, 0, j * BKV, hi, bi);
          if (!mbar_wait(&v_empty[slot], ph ^ 1, ab)) { ok = false; break; }
          mbar_expect_tx(&v_full[slot], TILE);
          tma_load_4d(&tmV, &v_full[slot], smem + OFF_V + slot * TILE, 0, j * BKV, hi, bi);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    // S_j+1 is issued as soon as the softmax warps have pulled S_j into
    // registers (s_free), i.e. while softmax_j runs; the first S of the next
    // item follows the last S of this one the same way.
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(128, 128, 0, 0);
      constexpr uint32_t idO = idesc_bf16_f32(128, 64, 0, 1);
      bool ok = true;
      int jg = 0;   // K/V tiles issued (S MMAs)
      int pg = 0;   // PV MMAs issued
      for (int it = 0, w = fwd_round_item(0); ok && w < n_items; w = fwd_round_item(++it)) {
        int qb, head;
        item_of(w, qb, head);
        const int nkv = qb + 1, qs = it & 1;
        const uint32_t sQ = smem_u32(smem + OFF_Q + qs * TILE);
        if (!mbar_wait(&q_full[qs], (it >> 1) & 1, ab)) break;
        for (int j = 0; j <= nkv; ++j) {
          if (j < nkv) {
            const int slot = jg & 1;
            if (!mbar_wait(&k_full[slot], (jg >> 1) & 1, ab)) { ok = false; break; }
            if (jg > 0 && !mbar_wait(s_free, (jg - 1) & 1, ab)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sK = smem_u32(smem + OFF_K + slot * TILE);
#pragma unroll
            for (int k = 0; k < HD / 16; ++k)
              umma_f16_ss(tmem + COL_S, sdesc_sw128(sQ + k * 32, 16, 1024), sdesc_sw128(sK + k * 32, 16, 1024), idS,
                          k > 0);
            umma_commit(s_full);
            umma_commit(&k_empty[slot]);
            if (j == nkv - 1) umma_commit(&q_empty[qs]);  // the item's last read of Q
            ++jg;
          }
          if (j > 0) {
            const int jj = j - 1, slot = pg & 1;
            if (!mbar_wait(p_full, pg & 1, ab)) { ok = false; break; }
            if (!mbar_wait(&v_full[slot], (pg >> 1) & 1, ab)) { ok = false; break; }
            // the item's first PV overwrites O: the previous item's O must have been read
            if (jj == 0 && it > 0 && !mbar_wait(o_free, (it - 1) & 1, ab)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sV = smem_u32(smem + OFF_V + slot * TILE);
#pragma unroll
            for (int kk = 0; kk < BKV / 16; ++kk)  // P (A operand) read from TMEM, 8 columns per k-step
              umma_f16_ts(tmem + COL_O, tmem + COL_P + kk * 8, sdesc_sw128(sV + kk * 2048, 8192, 1024), idO,
                          (jj > 0 || kk > 0) ? 1u : 0u);
            umma_commit(o_done);
            umma_commit(&v_empty[slot]);
            ++pg;
          }
        }
      }
    }
  } else {
    // ---------------------------------------------------------- softmax warps
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    bool ok = true;
    int jg = 0;
    for (int it = 0, w = fwd_round_item(0); ok && w < n_items; w = fwd_round_item(++it)) {
      int qb, head;
      item_of(w, qb, head);
      const int bi = head / p.H, hi = head % p.H;
      const int nkv = qb + 1;
      const int q = qb * BQ + r;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < nkv; ++j, ++jg) {
        if (!mbar_wait_warp(s_full, jg & 1, ab)) { ok = false; break; }
        tc_fence_after();
        float sv[128];  // raw scores; the softmax scale is folded into the exponent FFMA
        {  // the four 32-column loads of the row in flight together, one wait
          uint32_t u0[32], u1[32], u2[32], u3[32];
          tmem_ld32(trow + COL_S, u0);
          tmem_ld32(trow + COL_S + 32, u1);
          tmem_ld32(trow + COL_S + 64, u2);
          tmem_ld32(trow + COL_S + 96, u3);
          tmem_wait_ld_tied(u0);
          tmem_tie(u1);
          tmem_tie(u2);
          tmem_tie(u3);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            sv[e] = __uint_as_float(u0[e]);
            sv[32 + e] = __uint_as_float(u1[e]);
            sv[64 + e] = __uint_as_float(u2[e]);
            sv[96 + e] = __uint_as_float(u3[e]);
          }
        }
        tc_fence_before();
        mbar_arrive(s_free);
        if (j == qb) {  // diagonal tile: key index > query index is masked
#pragma unroll
          for (int e = 0; e < 128; ++e)
            if (e > r) sv[e] = -INFINITY;
        }
        // row max as 4 independent chains (short dependency chains: one softmax
        // warp per SM sub-partition has little else to hide latency with)
        float mx[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) mx[k] = sv[k];
#pragma unroll
        for (int e = 4; e < 128; ++e) mx[e & 3] = fmaxf(mx[e & 3], sv[e]);
        float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        mt *= p.sl2;  // (scale > 0, so the max commutes with it)
        // Lazy rescale: keep the running max unless the tile's max exceeds it by
        // more than 8 (log2 units).  Then P <= 2^8 and O, l stay in f32 range,
        // and most key tiles after the first skip the O rescale entirely.
        const float m_new = (mt > m + 8.f) ? mt : m;
        float ls[4] = {0.f, 0.f, 0.f, 0.f};  // row sum as 4 independent chains
        uint32_t pk[64];
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          const float a = ex2_approx(fmaf(sv[2 * e], p.sl2, -m_new));
          const float b = ex2_approx(fmaf(sv[2 * e + 1], p.sl2, -m_new));
          ls[e & 3] += a + b;
          pk[e] = pack_bf16x2(a, b);
        }
        const float lt = (ls[0] + ls[1]) + (ls[2] + ls[3]);
        const float alpha = (j > 0) ? ex2_approx(m - m_new) : 0.f;
        if (j > 0) {
          // PV_{j-1} complete: P buffer free, O stable
          if (!mbar_wait_warp(o_done, (jg - 1) & 1, ab)) { ok = false; break; }
          tc_fence_after();
          if (__any_sync(0xffffffffu, alpha < 1.f)) {
            {  // both halves of the O row loaded together, one wait
              uint32_t u0[32], u1[32];
              tmem_ld32(trow + COL_O, u0);
              tmem_ld32(trow + COL_O + 32, u1);
              tmem_wait_ld_tied(u0);
              tmem_tie(u1);
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                u0[e] = __float_as_uint(__uint_as_float(u0[e]) * alpha);
                u1[e] = __float_as_uint(__uint_as_float(u1[e]) * alpha);
              }
              tmem_st32(trow + COL_O, u0);
              tmem_st32(trow + COL_O + 32, u1);
            }
            tmem_wait_st();
          }
        }
        // (j == 0: the previous item's last PV completed before its epilogue,
        // so the P buffer is free)
        l = l * alpha + lt;
        m = m_new;
        {  // P (bf16 pairs) into TMEM columns [COL_P, COL_P + 64) of this row's lane
          uint32_t wv[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) wv[e] = pk[e];
          tmem_st32(trow + COL_P, wv);
#pragma unroll
          for (int e = 0; e < 32; ++e) wv[e] = pk[32 + e];
          tmem_st32(trow + COL_P + 32, wv);
          tmem_wait_st();
        }
        tc_fence_before();
        mbar_arrive(p_full);
      }
      if (!ok || !mbar_wait_warp(o_done, (jg - 1) & 1, ab)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = 1.f / l;
      uint32_t ov[32];
      __nv_bfloat16* orow = p.O + bi * p.os.b + q * p.os.s + hi * p.os.h;
      uint32_t u0[32], u1[32];  // both 32-column halves of the O row in flight, one wait
      tmem_ld32(trow + COL_O, u0);
      tmem_ld32(trow + COL_O + 32, u1);
      tmem_wait_ld_tied(u0);
      tmem_tie(u1);
      tc_fence_before();
      mbar_arrive(o_free);  // O read: the next item's first PV may overwrite it
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint32_t* u = c ? u1 : u0;
#pragma unroll
        for (int e = 0; e < 16; ++e)
          ov[e] = pack_bf16x2(__uint_as_float(u[2 * e]) * inv, __uint_as_float(u[2 * e + 1]) * inv);
        if (q < p.s) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(ov[4 * v], ov[4 * v + 1], ov[4 * v + 2], ov[4 * v + 3]);
        }
      }
      if (q < p.s) p.L[(long long)head * p.s + q] = (m + __log2f(l)) * kLn2;
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ====================================================================== backward
namespace bwd {
constexpr int kThreads = 14 * 32;  // TMA, MMA, 8 P/dS warps, 4 dQ warps
constexpr int OFF_K = 0;          // 2 slots (one per work item in flight)
constexpr int OFF_V = 2 * TILE;   // 2 slots
constexpr int OFF_Q = 4 * TILE;   // 2 slots
constexpr int OFF_DO = 6 * TILE;  // 2 slots
constexpr int OFF_DS = 8 * TILE;  // 32 KB  dS^T [kv rows, q cols]
constexpr int OFF_LD = 10 * TILE;  // L2[2][128], D[2][128] f32
constexpr int OFF_DQS = OFF_LD + 2048;  // dQ staging: 4 warps x two 32x32 f32 boxes (SW128)
constexpr int OFF_BAR = OFF_DQS + 4 * 8192;
constexpr int SMEM = OFF_BAR + 256;
constexpr int TMEM_COLS = 512;
constexpr int COL_S = 0, COL_DP = 128, COL_DV = 256, COL_DK = 320, COL_DQ = 384;
constexpr int COL_PT = 448;  // P^T as bf16 pairs: 128 query columns in 64 TMEM columns
}  // namespace bwd

struct BwdParams {
  const float* L;  // natural-log LSE [n, s]
  const float* D;  // rowsum(dO * O)  [n, s]
  float* dQacc;    // [n, s, 64] f32, zeroed
  __nv_bfloat16* dK;
  __nv_bfloat16* dV;
  Strides gs;  // strides of dK / dV (and dQ)
  int n, H, s, nq;
  float sl2, scale;
  int want_dq, want_dkdv;
  int* err;
};

// Work item w (0 .. n*nq-1) = (key tile jb = w / n, head = w % n): items are
// numbered heaviest first (key tile 0 meets every query tile).  Round k deals
// items k*G .. k*G+G-1 to the G persistent CTAs, forwards in even rounds and
// backwards in odd ones, which evens out the per-CTA work.
__device__ __forceinline__ int bwd_round_item(int k) {
  const int G = static_cast<int>(gridDim.x), b = static_cast<int>(blockIdx.x);
  return k * G + ((k & 1) ? G - 1 - b : b);
}
__device__ __forceinline__ void bwd_item(const BwdParams& p, int w, int& jb, int& head) {
  jb = w / p.n;
  head = w - jb * p.n;
}

// Persistent: one CTA per SM walks its work items; barrier phases run on the
// CTA's item count (K/V slots, dK/dV accumulator) and its running query-tile
// iteration count g (everything per iteration), so the S/dP MMAs of an item
// overlap the dK/dV write-out of the previous one.
__global__ void __launch_bounds__(bwd::kThreads, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                     const __grid_constant__ CUtensorMap tmDQ, BwdParams p) {
  using namespace bwd;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* kv_full = bars + 0;    // [2]
  uint64_t* kv_empty = bars + 2;   // [2]
  uint64_t* qdo_full = bars + 4;   // [2]
  uint64_t* qdo_empty = bars + 6;  // [2]
  uint64_t* s_full = bars + 8;
  uint64_t* st_free = bars + 9;
  uint64_t* ds_full = bars + 10;
  uint64_t* ds_empty = bars + 11;
  uint64_t* dq_full = bars + 12;
  uint64_t* dq_free = bars + 13;
  uint64_t* acc_done = bars + 14;
  uint64_t* acc_free = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* Lbuf = reinterpret_cast<float*>(smem + OFF_LD);  // [2][128]
  float* Dbuf = Lbuf + 256;                               // [2][128]

  const int warp = warp_id(), lane = lane_id();
  const int n_items = p.n * p.nq;

  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0 && p.err) atomicExch(p.err, 2);
    return;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(st_free, 256);
    mbar_init(ds_full, 256);
    mbar_init(ds_empty, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 128);
    mbar_init(acc_done, 1);
    mbar_init(acc_free, 256);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  Abort ab{abort_flag, p.err};
  griddep_sync();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA loads
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
      bool ok = true;
      int g = 0, wi = 0;
      for (int w = bwd_round_item(0); ok && w < n_items; w = bwd_round_item(++wi)) {
        int jb, head;
        bwd_item(p, w, jb, head);
        const int bi = head / p.H, hi = head % p.H;
        const int ks = wi & 1;
        if (wi >= 2 && !mbar_wait(&kv_empty[ks], ((wi >> 1) - 1) & 1, ab)) break;
        mbar_expect_tx(&kv_full[ks], 2 * TILE);
        tma_load_4d(&tmK, &kv_full[ks], smem + OFF_K + ks * TILE, 0, jb * BKV, hi, bi);
        tma_load_4d(&tmV, &kv_full[ks], smem + OFF_V + ks * TILE, 0, jb * BKV, hi, bi);
        for (int i = jb; i < p.nq; ++i, ++g) {
          const int slot = g & 1;
          if (!mbar_wait(&qdo_empty[slot], ((g >> 1) & 1) ^ 1, ab)) { ok = false; break; }
          mbar_expect_tx(&qdo_full[slot], 2 * TILE);
          tma_load_4d(&tmQ, &qdo_full[slot], smem + OFF_Q + slot * TILE, 0, i * BQ, hi, bi);
          tma_load_4d(&tmDO, &qdo_full[slot], smem + OFF_DO + slot * TILE, 0, i * BQ, hi, bi);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    // Software-pipelined over the CTA's iterations g (query tiles of all its
    // items in order): S^T / dP^T of iteration g+1 are issued as soon as the
    // P/dS warps have pulled those of g into registers (st_free), before the
    // dV / dK / dQ products of g, so the tensor pipe computes the next scores
    // while the P/dS warps run the exponentials of the current ones.
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(128, 128, 0, 0);   // S^T, dP^T
      constexpr uint32_t idKV = idesc_bf16_f32(128, 64, 0, 1);   // dV, dK: B MN-major
      constexpr uint32_t idQ = idesc_bf16_f32(128, 64, 1, 1);    // dQ: A and B MN-major
      const uint32_t sDS = smem_u32(smem + OFF_DS);
      // iteration cursor: item index wi, its key tile jb, query-tile offset it
      struct Cur {
        int wi, w, jb, it;
      };
      auto first_of = [&](int wi) {
        Cur c{wi, bwd_round_item(wi), 0, 0};
        if (c.w < n_items) {
          int head;
          bwd_item(p, c.w, c.jb, head);
        }
        return c;
      };
      auto issue_sdp = [&](const Cur& c, int g) -> bool {
        const int ks = c.wi & 1, slot = g & 1;
        if (c.it == 0 && !mbar_wait(&kv_full[ks], (c.wi >> 1) & 1, ab)) return false;
        if (!mbar_wait(&qdo_full[slot], (g >> 1) & 1, ab)) return false;
        if (g > 0 && !mbar_wait(st_free, (g - 1) & 1, ab)) return false;
        tc_fence_after();
        const uint32_t sK = smem_u32(smem + OFF_K + ks * TILE), sV = smem_u32(smem + OFF_V + ks * TILE);
        const uint32_t sQ = smem_u32(smem + OFF_Q + slot * TILE);
        const uint32_t sDO = smem_u32(smem + OFF_DO + slot * TILE);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_f16_ss(tmem + COL_S, sdesc_sw128(sK + k * 32, 16, 1024), sdesc_sw128(sQ + k * 32, 16, 1024), idS,
                      k > 0);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_f16_ss(tmem + COL_DP, sdesc_sw128(sV + k * 32, 16, 1024), sdesc_sw128(sDO + k * 32, 16, 1024), idS,
                      k > 0);
        umma_commit(s_full);
        return true;
      };
      Cur cur = first_of(0);
      bool ok = cur.w < n_items && issue_sdp(cur, 0);
      for (int g = 0; ok && cur.w < n_items; ++g) {
        // the iteration after g
        Cur nxt = cur;
        if (cur.jb + cur.it + 1 < p.nq) {
          ++nxt.it;
        } else {
          nxt = first_of(cur.wi + 1);
        }
        if (nxt.w < n_items && !issue_sdp(nxt, g + 1)) break;
        const int ks = cur.wi & 1, slot = g & 1;
        const uint32_t sK = smem_u32(smem + OFF_K + ks * TILE);
        const uint32_t sQ = smem_u32(smem + OFF_Q + slot * TILE);
        const uint32_t sDO = smem_u32(smem + OFF_DO + slot * TILE);
        if (!mbar_wait(ds_full, g & 1, ab)) break;
        tc_fence_after();
        if (p.want_dkdv) {
          // the previous item's dV / dK must have left TMEM before they restart
          if (cur.it == 0 && cur.wi > 0 && !mbar_wait(acc_free, (cur.wi - 1) & 1, ab)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk) {
            const uint32_t a_off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_f16_ts(tmem + COL_DV, tmem + COL_PT + kk * 8, sdesc_sw128(sDO + kk * 2048, 8192, 1024), idKV,
                        (cur.it > 0 || kk > 0) ? 1u : 0u);
            umma_f16_ss(tmem + COL_DK, sdesc_sw128(sDS + a_off, 16, 1024), sdesc_sw128(sQ + kk * 2048, 8192, 1024),
                        idKV, (cur.it > 0 || kk > 0) ? 1u : 0u);
          }
        }
        if (p.want_dq) {
          if (g > 0 && !mbar_wait(dq_free, (g - 1) & 1, ab)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            umma_f16_ss(tmem + COL_DQ, sdesc_sw128(sDS + kk * 2048, 16384, 1024),
                        sdesc_sw128(sK + kk * 2048, 8192, 1024), idQ, kk > 0 ? 1u : 0u);
          umma_commit(dq_full);
        }
        umma_commit(ds_empty);
        umma_commit(&qdo_empty[slot]);
        if (nxt.wi != cur.wi || nxt.w >= n_items) {  // last query tile of this item
          umma_commit(&kv_empty[ks]);
          umma_commit(acc_done);
        }
        cur = nxt;
      }
    }
  } else if (warp < 10) {
    // ---------------------------------------------------------- P / dS warps
    // two warps per TMEM lane quarter (one key row per thread), each taking
    // half of the 128 query columns
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const int t = (warp - 2) * 32 + lane;  // loader index: threads 0..127 stage L / D
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t sDS = smem_u32(smem + OFF_DS);
    // On a timeout the loops keep iterating without work so that all 256
    // threads still meet at every named barrier (a barrier can not time out).
    bool ok = true;
    int g = 0, wi = 0;
    for (int w = bwd_round_item(0); w < n_items; w = bwd_round_item(++wi)) {
      int jb, head;
      bwd_item(p, w, jb, head);
      const int bi = head / p.H, hi = head % p.H;
      const int kv = jb * BKV + r;
      const float* Lh = p.L + (long long)head * p.s;
      const float* Dh = p.D + (long long)head * p.s;
      float l_next, d_next;
      {
        const int qi = jb * BQ + t;
        l_next = (t < 128 && qi < p.s) ? Lh[qi] * kLog2e : INFINITY;
        d_next = (t < 128 && qi < p.s) ? Dh[qi] : 0.f;
      }
      for (int i = jb; i < p.nq; ++i, ++g) {
        const int buf = g & 1;
        if (t < 128) {
          Lbuf[buf * 128 + t] = l_next;
          Dbuf[buf * 128 + t] = d_next;
        }
        named_bar_sync(1, 256);
        if (i + 1 < p.nq) {
          const int qi = (i + 1) * BQ + t;
          l_next = (t < 128 && qi < p.s) ? Lh[qi] * kLog2e : INFINITY;
          d_next = (t < 128 && qi < p.s) ? Dh[qi] : 0.f;
        }
        if (ok) ok = mbar_wait_warp(s_full, g & 1, ab);
        if (ok && g > 0) ok = mbar_wait_warp(ds_empty, (g - 1) & 1, ab);
        if (!ok) continue;
        tc_fence_after();
        const float* Lb = Lbuf + buf * 128;
        const float* Db = Dbuf + buf * 128;
        // the causal / sequence-end mask is needed only on the diagonal tile
        // and on a ragged last query tile (warp-uniform)
        const bool masked = (i == jb) || ((i + 1) * BQ > p.s);
#pragma unroll 1
        for (int c = 2 * half; c < 2 * half + 2; ++c) {
          uint32_t us[32], ud[32];
          tmem_ld32(trow + COL_S + c * 32, us);
          tmem_ld32(trow + COL_DP + c * 32, ud);
          float nl[32], dcol[32];  // -L (base 2) and D of the 32 query columns: broadcast vector loads
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            const float4 l4 = reinterpret_cast<const float4*>(Lb + c * 32)[v];
            const float4 d4 = reinterpret_cast<const float4*>(Db + c * 32)[v];
            nl[4 * v] = -l4.x; nl[4 * v + 1] = -l4.y; nl[4 * v + 2] = -l4.z; nl[4 * v + 3] = -l4.w;
            dcol[4 * v] = d4.x; dcol[4 * v + 1] = d4.y; dcol[4 * v + 2] = d4.z; dcol[4 * v + 3] = d4.w;
          }
          tmem_wait_ld();
          if (c == 2 * half + 1) {  // this thread's last reads of S^T / dP^T: the MMA warp may overwrite them
            tc_fence_before();
            mbar_arrive(st_free);
          }
          float pv[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) pv[e] = ex2_approx(fmaf(__uint_as_float(us[e]), p.sl2, nl[e]));
          if (masked) {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int qg = i * BQ + c * 32 + e;
              pv[e] = (qg >= kv && qg < p.s) ? pv[e] : 0.f;  // causal (query >= key), in range
            }
          }
          uint32_t pp[16], dd[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            pp[e / 2] = pack_bf16x2(pv[e], pv[e + 1]);
            dd[e / 2] = pack_bf16x2(pv[e] * (__uint_as_float(ud[e]) - dcol[e]),
                                    pv[e + 1] * (__uint_as_float(ud[e + 1]) - dcol[e + 1]));
          }
#pragma unroll
          for (int v = 0; v < 4; ++v)
            st_shared_v4(sDS + sw128_off(r, c * 4 + v), dd[4 * v], dd[4 * v + 1], dd[4 * v + 2], dd[4 * v + 3]);
          // P^T (bf16 pairs) into TMEM: 32 query columns = 16 packed columns
          tmem_st16(trow + COL_PT + c * 16, pp);
        }
        tmem_wait_st();
        tc_fence_before();
        fence_proxy_async_smem();
        mbar_arrive(ds_full);
      }
      if (ok && p.want_dkdv) ok = mbar_wait_warp(acc_done, wi & 1, ab);
      if (ok && p.want_dkdv) {
        tc_fence_after();
        const int which = half;  // half 0 writes dV, half 1 writes dK
        const uint32_t col = (which == 0) ? COL_DV : COL_DK;
        uint32_t u0[32], u1[32];
        tmem_ld32(trow + col, u0);
        tmem_ld32(trow + col + 32, u1);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(acc_free);  // TMEM columns free for the next item
        if (kv < p.s) {
          __nv_bfloat16* dst = (which == 0 ? p.dV : p.dK) + bi * p.gs.b + (long long)kv * p.gs.s + hi * p.gs.h;
          const float mul = (which == 0) ? 1.f : p.scale;
          uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            d4[v] = make_uint4(pack_bf16x2(__uint_as_float(u0[8 * v + 0]) * mul, __uint_as_float(u0[8 * v + 1]) * mul),
                               pack_bf16x2(__uint_as_float(u0[8 * v + 2]) * mul, __uint_as_float(u0[8 * v + 3]) * mul),
                               pack_bf16x2(__uint_as_float(u0[8 * v + 4]) * mul, __uint_as_float(u0[8 * v + 5]) * mul),
                               pack_bf16x2(__uint_as_float(u0[8 * v + 6]) * mul, __uint_as_float(u0[8 * v + 7]) * mul));
#pragma unroll
          for (int v = 0; v < 4; ++v)
            d4[4 + v] =
                make_uint4(pack_bf16x2(__uint_as_float(u1[8 * v + 0]) * mul, __uint_as_float(u1[8 * v + 1]) * mul),
                           pack_bf16x2(__uint_as_float(u1[8 * v + 2]) * mul, __uint_as_float(u1[8 * v + 3]) * mul),
                           pack_bf16x2(__uint_as_float(u1[8 * v + 4]) * mul, __uint_as_float(u1[8 * v + 5]) * mul),
                           pack_bf16x2(__uint_as_float(u1[8 * v + 6]) * mul, __uint_as_float(u1[8 * v + 7]) * mul));
        }
      }
    }
  } else {
    // ---------------------------------------------------------- dQ warps (one query row each)
    // Each warp stages its 32 rows x 64 columns of the dQ tile as two 32 x 32
    // f32 boxes in the swizzled layout of the dQacc tensor map and adds them
    // to dQacc with TMA reduce-adds (rows past s are clipped per head).
    if (p.want_dq) {
      const int quarter = warp & 3;
      const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
      uint8_t* stg = smem + OFF_DQS + (warp - 10) * 8192;
      bool ok = true;
      int g = 0, wi = 0;
      for (int w = bwd_round_item(0); ok && w < n_items; w = bwd_round_item(++wi)) {
        int jb, head;
        bwd_item(p, w, jb, head);
        for (int i = jb; i < p.nq; ++i, ++g) {
          const int q0 = i * BQ + quarter * 32;
          if (!mbar_wait_warp(dq_full, g & 1, ab)) { ok = false; break; }
          tc_fence_after();
          uint32_t u0[32], u1[32];
          tmem_ld32(trow + COL_DQ, u0);
          tmem_ld32(trow + COL_DQ + 32, u1);
          tmem_wait_ld();
          tc_fence_before();
          mbar_arrive(dq_free);
          if (lane == 0) bulk_wait_read_all();  // the previous reduce has read the staging
          __syncwarp();
          const uint32_t b0 = smem_u32(stg) + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            st_shared_v4(b0 + ((j ^ (lane & 7)) << 4), u0[4 * j], u0[4 * j + 1], u0[4 * j + 2], u0[4 * j + 3]);
            st_shared_v4(b0 + 4096 + ((j ^ (lane & 7)) << 4), u1[4 * j], u1[4 * j + 1], u1[4 * j + 2],
                         u1[4 * j + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && q0 < p.s) {
            tma_reduce_add_3d(&tmDQ, stg, 0, q0, head);
            tma_reduce_add_3d(&tmDQ, stg + 4096, 32, q0, head);
            bulk_commit();
          }
        }
      }
      if (lane == 0) bulk_wait_all();
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// D[row] = sum_d dO[row,d] * O[row,d]; optionally zero the dQ accumulator row.
// Eight threads per row (16-byte loads of 8 bf16 each), four rows per warp,
// grid-stride so that each thread keeps several independent loads in flight.
__global__ void bwd_preprocess_kernel(const __nv_bfloat16* __restrict__ O, const __nv_bfloat16* __restrict__ dO,
                                      Strides os, int H, int s, float* __restrict__ D, float* __restrict__ dQacc,
                                      long long rows) {
  griddep_sync();
  const int sub = threadIdx.x & 7;
  for (long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 3; row < rows;
       row += (static_cast<long long>(gridDim.x) * blockDim.x) >> 3) {
    if (O != nullptr) {
      const long long nh = row / s, q = row % s;
      const long long off = (nh / H) * os.b + q * os.s + (nh % H) * os.h + sub * 8;
      const uint4 o = *reinterpret_cast<const uint4*>(O + off);
      const uint4 g = *reinterpret_cast<const uint4*>(dO + off);
      const __nv_bfloat162* oh = reinterpret_cast<const __nv_bfloat162*>(&o);
      const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&g);
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 a = __bfloat1622float2(oh[k]), b = __bfloat1622float2(gh[k]);
        acc += a.x * b.x + a.y * b.y;
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (sub == 0) D[row] = acc;
    }
    if (dQacc) {
      float4* z = reinterpret_cast<float4*>(dQacc + row * HD) + sub * 2;
      z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

// dQ = bf16(scale * dQacc): 8 elements per thread, 16-byte stores into the
// (possibly strided) dQ layout.
__global__ void dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dQ, Strides gs, int H,
                                  int s, float scale, long long n8) {
  griddep_sync();
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i >> 3, c8 = i & 7;
    const long long nh = row / s, q = row % s;
    const long long off = (nh / H) * gs.b + q * gs.s + (nh % H) * gs.h + c8 * 8;
    const float4 a = reinterpret_cast<const float4*>(acc)[2 * i];
    const float4 b = reinterpret_cast<const float4*>(acc)[2 * i + 1];
    *reinterpret_cast<uint4*>(dQ + off) =
        make_uint4(pack_bf16x2(a.x * scale, a.y * scale), pack_bf16x2(a.z * scale, a.w * scale),
                   pack_bf16x2(b.x * scale, b.y * scale), pack_bf16x2(b.z * scale, b.w * scale));
  }
}

static int grid_cap(long long blocks) {
  const long long cap = static_cast<long long>(sm_count()) * 16;
  return static_cast<int>(blocks < cap ? blocks : cap);
}

static int check_common(const void* Q, const void* K, const void* V, int n, int s, int d) {
  if (n <= 0 || s <= 0) return NL_ERR_SHAPE;
  if (d != HD) return NL_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) | reinterpret_cast<uintptr_t>(V)) & 15)
    return NL_ERR_ALIGN;
  return NL_OK;
}

template <typename Kern>
static int set_smem(Kern k, int bytes) {
  static int dev_done = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev_done == dev) return NL_OK;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return NL_ERR_LAUNCH;
  dev_done = dev;
  return NL_OK;
}

}  // namespace fa

int* device_error_word();

// Strided forward: Q/K/V share strides qs, O uses os; L is contiguous [B*H, s].
int flash_fwd(const void* Q, const void* K, const void* V, fa::Strides qs, void* O, fa::Strides os, float* L, int B,
              int H, int s, int d, cudaStream_t stream) {
  using namespace fa;
  if (B <= 0 || H <= 0) return NL_ERR_SHAPE;
  int st = check_common(Q, K, V, B * H, s, d);
  if (st) return st;
  if ((reinterpret_cast<uintptr_t>(O) & 15) || (os.s & 7) || (os.h & 7) || (os.b & 7)) return NL_ERR_ALIGN;
  CUtensorMap tq, tk, tv;
  if ((st = make_tmap_bf16_4d(&tq, Q, s, H, B, qs.s, qs.h, qs.b, BQ))) return st;
  if ((st = make_tmap_bf16_4d(&tk, K, s, H, B, qs.s, qs.h, qs.b, BKV))) return st;
  if ((st = make_tmap_bf16_4d(&tv, V, s, H, B, qs.s, qs.h, qs.b, BKV))) return st;
  FwdParams p{};
  p.O = reinterpret_cast<__nv_bfloat16*>(O);
  p.os = os;
  p.L = L;
  p.n = B * H;
  p.H = H;
  p.s = s;
  p.nq = (s + BQ - 1) / BQ;
  p.sl2 = (1.f / sqrtf(static_cast<float>(HD))) * kLog2e;
  p.err = device_error_word();
  if ((st = set_smem(flash_fwd_kernel, fwd::SMEM))) return st;
  const long long items = static_cast<long long>(p.n) * p.nq;
  if (items > 0x7fffffffLL) return NL_ERR_SHAPE;
  const long long slots = 2LL * sm_count();  // two resident CTAs per SM
  const long long grid = items < slots ? items : slots;
  launch_kernel(flash_fwd_kernel, dim3(static_cast<unsigned>(grid)), dim3(fwd::kThreads), fwd::SMEM, stream, 1, tq, tk, tv, p);
  return launch_status();
}

// Strided backward.  Q/K/V and dQ/dK/dV share strides qs; O/dO use os.
// D (f32 [B*H, s]) and dQacc (f32 [B*H, s, 64]) are caller workspaces; if O is
// non-null, D is computed here from O and dO, otherwise D is an input.
int flash_bwd(const void* Q, const void* K, const void* V, fa::Strides qs, const void* O, const void* dO,
              fa::Strides os, const float* L, float* D, void* dQ, void* dK, void* dV, float* dQacc, int B, int H, int s,
              int d, cudaStream_t stream) {
  using namespace fa;
  if (B <= 0 || H <= 0) return NL_ERR_SHAPE;
  const int n = B * H;
  int st = check_common(Q, K, V, n, s, d);
  if (st) return st;
  if (!dO || !L || !D) return NL_ERR_SHAPE;
  const bool want_dq = dQ != nullptr;
  const bool want_dkdv = dK != nullptr && dV != nullptr;
  if (want_dq && !dQacc) return NL_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(dO) | reinterpret_cast<uintptr_t>(dQ) | reinterpret_cast<uintptr_t>(dK) |
       reinterpret_cast<uintptr_t>(dV) | reinterpret_cast<uintptr_t>(dQacc)) & 15)
    return NL_ERR_ALIGN;
  const long long rows = static_cast<long long>(n) * s;
  if (O || want_dq) {
    const long long threads = rows * 8;
    launch_kernel(bwd_preprocess_kernel, dim3(grid_cap((threads + 255) / 256)), dim3(256), 0, stream, 1, reinterpret_cast<const __nv_bfloat16*>(O), reinterpret_cast<const __nv_bfloat16*>(dO), os, H, s, D,
        want_dq ? dQacc : nullptr, rows);
    if ((st = launch_status())) return st;
  }
  CUtensorMap tq, tk, tv, tdo, tdq;
  if ((st = make_tmap_bf16_4d(&tq, Q, s, H, B, qs.s, qs.h, qs.b, BQ))) return st;
  if ((st = make_tmap_bf16_4d(&tk, K, s, H, B, qs.s, qs.h, qs.b, BKV))) return st;
  if ((st = make_tmap_bf16_4d(&tv, V, s, H, B, qs.s, qs.h, qs.b, BKV))) return st;
  if ((st = make_tmap_bf16_4d(&tdo, dO, s, H, B, os.s, os.h, os.b, BQ))) return st;
  memset(&tdq, 0, sizeof(tdq));
  if (want_dq && (st = make_tmap_f32_rows64_3d(&tdq, dQacc, s, n))) return st;
  BwdParams p{};
  p.L = L;
  p.D = D;
  p.dQacc = dQacc;
  p.dK = reinterpret_cast<__nv_bfloat16*>(dK);
  p.dV = reinterpret_cast<__nv_bfloat16*>(dV);
  p.gs = qs;
  p.n = n;
  p.H = H;
  p.s = s;
  p.nq = (s + BQ - 1) / BQ;
  p.scale = 1.f / sqrtf(static_cast<float>(HD));
  p.sl2 = p.scale * kLog2e;
  p.want_dq = want_dq;
  p.want_dkdv = want_dkdv;
  p.err = device_error_word();
  if ((st = set_smem(flash_bwd_kernel, bwd::SMEM))) return st;
  const long long items = static_cast<long long>(n) * p.nq;
  const long long grid = items < sm_count() ? items : sm_count();
  launch_kernel(flash_bwd_kernel, dim3(static_cast<unsigned>(grid)), dim3(bwd::kThreads), bwd::SMEM, stream, 1, tq, tk, tv, tdo, tdq, p);
  if ((st = launch_status())) return st;
  if (want_dq) {
    const long long n8 = rows * HD / 8;
    launch_kernel(dq_convert_kernel, dim3(grid_cap((n8 + 255) / 256)), dim3(256), 0, stream, 1, dQacc, reinterpret_cast<__nv_bfloat16*>(dQ), qs, H, s, p.scale, n8);
    if ((st = launch_status())) return st;
  }
  return NL_OK;
}

}  // namespace nl

namespace {
// Contiguous [n, s, 64] as the strided form with B = n, H = 1.
inline nl::fa::Strides contiguous(int s) { return nl::fa::Strides{64, 64LL * s, 64LL * s}; }
}  // namespace

extern "C" int nl_flash_attention_fwd(const void* Q, const void* K, const void* V, void* O, float* L, int n, int s,
                                      int d, cudaStream_t stream) {
  return nl::flash_fwd(Q, K, V, contiguous(s), O, contiguous(s), L, n, 1, s, d, stream);
}

extern "C" int nl_flash_attention_bwd(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                                      const float* L, float* D_ws, void* dQ, void* dK, void* dV, float* dQacc_ws,
                                      int n, int s, int d, cudaStream_t stream) {
  if (!O) return NL_ERR_SHAPE;
  return nl::flash_bwd(Q, K, V, contiguous(s), O, dO, contiguous(s), L, D_ws, dQ, dK, dV, dQacc_ws, n, 1, s, d,
                       stream);
}

extern "C" int nl_flash_attention_bwd_dq(const void* Q, const void* K, const void* V, const void* dO,
                                         const float* L, const float* D, void* dQ, float* dQacc_ws, int n, int s,
                                         int d, cudaStream_t stream) {
  if (!dQ) return NL_ERR_SHAPE;
  return nl::flash_bwd(Q, K, V, contiguous(s), nullptr, dO, contiguous(s), L, const_cast<float*>(D), dQ, nullptr,
                       nullptr, dQacc_ws, n, 1, s, d, stream);
}

extern "C" int nl_flash_attention_bwd_dkdv(const void* Q, const void* K, const void* V, const void* dO,
                                           const float* L, const float* D, void* dK, void* dV, int n, int s, int d,
                                           cudaStream_t stream) {
  if (!dK || !dV) return NL_ERR_SHAPE;
  return nl::flash_bwd(Q, K, V, contiguous(s), nullptr, dO, contiguous(s), L, const_cast<float*>(D), nullptr, dK,
                       dV, nullptr, n, 1, s, d, stream);
}

// ----------------------------------------------------------------------------
// Allocation-free backward.  Some callers cannot allocate device memory at the
// point where they run the backward (for example a host framework that hands
// over only its own input / output buffers, or code that runs where
// cudaMalloc is not permitted).  For them the backward's scratch — the f32 dQ
// accumulator [rows, 64] and the f32 D = rowsum(dO*O) vector [rows] — lives in
// this fixed, file-scope device array instead of a caller workspace.
// Limit: rows = n * s <= kNoAllocMaxRows (131072, e.g. 256 heads x 512 or
// 32 heads x 4096), i.e. 32.5 MiB held on every device that loads the library,
// for the life of the process.
constexpr long long kNoAllocMaxRows = 131072;
static __device__ __align__(256) float g_bwd_scratch[kNoAllocMaxRows * (64 + 1)];

namespace {
// Device address of g_bwd_scratch, resolved once per device on that device's
// first call (host code may not use the symbol itself as a pointer).
// Host threads may make their first call on a device concurrently: the cache
// entries are atomics (every thread that resolves the address stores the same
// value, so a lost race costs one extra cudaGetSymbolAddress, nothing more).
float* noalloc_scratch() {
  constexpr int kMaxDev = 64;
  static std::atomic<float*> addr[kMaxDev];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  float* a = addr[dev].load(std::memory_order_acquire);
  if (!a) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_bwd_scratch) != cudaSuccess) return nullptr;
    a = static_cast<float*>(p);
    addr[dev].store(a, std::memory_order_release);
  }
  return a;
}
}  // namespace

extern "C" long long nl_flash_attention_bwd_noalloc_max_rows(void) { return kNoAllocMaxRows; }

extern "C" int nl_flash_attention_bwd_noalloc(const void* Q, const void* K, const void* V, const void* O,
                                              const void* dO, const float* L, void* dQ, void* dK, void* dV, int n,
                                              int s, int d, cudaStream_t stream) {
  if (n <= 0 || s <= 0) return NL_ERR_SHAPE;
  if (static_cast<long long>(n) * s > kNoAllocMaxRows) return NL_ERR_TOO_LARGE;
  if (!O) return NL_ERR_SHAPE;
  float* base = noalloc_scratch();
  if (!base) return NL_ERR_CUDA;
  float* dqacc = base;                                   // [rows, 64], zeroed by the pre-pass
  float* D = base + kNoAllocMaxRows * 64;                // [rows], written by the pre-pass
  return nl::flash_bwd(Q, K, V, contiguous(s), O, dO, contiguous(s), L, D, dQ, dK, dV, dqacc, n, 1, s, d, stream);
}

extern "C" int nl_flash_attention_fwd_strided(const void* Q, const void* K, const void* V, long long q_s,
                                              long long q_h, long long q_b, void* O, long long o_s, long long o_h,
                                              long long o_b, float* L, int B, int H, int s, int d,
                                              cudaStream_t stream) {
  return nl::flash_fwd(Q, K, V, nl::fa::Strides{q_s, q_h, q_b}, O, nl::fa::Strides{o_s, o_h, o_b}, L, B, H, s, d,
                       stream);
}

extern "C" int nl_flash_attention_bwd_strided(const void* Q, const void* K, const void* V, long long q_s,
                                              long long q_h, long long q_b, const void* O, const void* dO,
                                              long long o_s, long long o_h, long long o_b, const float* L,
                                              float* D_ws, void* dQ, void* dK, void* dV, float* dQacc_ws, int B,
                                              int H, int s, int d, cudaStream_t stream) {
  if (!O) return NL_ERR_SHAPE;
  return nl::flash_bwd(Q, K, V, nl::fa::Strides{q_s, q_h, q_b}, O, dO, nl::fa::Strides{o_s, o_h, o_b}, L, D_ws, dQ,
                       dK, dV, dQacc_ws, B, H, s, d, stream);
}

// ----------------------------------------------------------------------------
// Dtype-dispatching forms of the three reference targets.  nlearn's wrappers
// hand `flash_attention_fwd` / `_bwd_dq` / `_bwd_dkdv` f32 operands and expect
// f32 results (nlearn/attention.py:82-91, 97, 111-128).  For NL_F32 the
// operands are converted to bf16 tensor-core operands in the caller's
// workspace on `stream`, the bf16 kernels run, and the results are widened
// back to f32; dQ is taken from the f32 accumulator (scaled) rather than from
// its bf16 rounding.  For NL_BF16 these are the plain entry points.
namespace nl {
namespace fa {

__global__ void cast_f32_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long long n8) {
  griddep_sync();
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(x)[2 * i];
    const float4 b = reinterpret_cast<const float4*>(x)[2 * i + 1];
    reinterpret_cast<uint4*>(y)[i] =
        make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
  }
}

// y = scale * x, x bf16 (src_f32 == nullptr) or f32, y f32; 8 elements per thread.
__global__ void widen_f32_kernel(const __nv_bfloat16* __restrict__ xb, const float* __restrict__ xf,
                                 float* __restrict__ y, float scale, long long n8) {
  griddep_sync();
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 a, b;
    if (xf) {
      a = reinterpret_cast<const float4*>(xf)[2 * i];
      b = reinterpret_cast<const float4*>(xf)[2 * i + 1];
    } else {
      const uint4 v = reinterpret_cast<const uint4*>(xb)[i];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
      const float2 p0 = __bfloat1622float2(h[0]), p1 = __bfloat1622float2(h[1]);
      const float2 p2 = __bfloat1622float2(h[2]), p3 = __bfloat1622float2(h[3]);
      a = make_float4(p0.x, p0.y, p1.x, p1.y);
      b = make_float4(p2.x, p2.y, p3.x, p3.y);
    }
    reinterpret_cast<float4*>(y)[2 * i] = make_float4(a.x * scale, a.y * scale, a.z * scale, a.w * scale);
    reinterpret_cast<float4*>(y)[2 * i + 1] = make_float4(b.x * scale, b.y * scale, b.z * scale, b.w * scale);
  }
}

enum { kTargetFwd = 0, kTargetBwdDq = 1, kTargetBwdDkdv = 2 };

inline size_t ws_align(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Workspace carve-up: `count` bf16 [n, s, 64] tensors, then (dq target) the
// f32 [n, s, 64] accumulator.
size_t dt_workspace_bytes(int target, int n, int s, int d, int dtype) {
  if (n <= 0 || s <= 0 || d != HD || (dtype != NL_F32 && dtype != NL_BF16)) return 0;
  const size_t elems = static_cast<size_t>(n) * s * HD;
  const size_t t16 = ws_align(elems * 2);
  const bool f32 = dtype == NL_F32;
  switch (target) {
    case kTargetFwd: return f32 ? 4 * t16 : 0;
    case kTargetBwdDq: return (f32 ? 5 * t16 : 0) + ws_align(elems * 4);
    case kTargetBwdDkdv: return f32 ? 6 * t16 : 0;
    default: return 0;
  }
}

int cast_in(const void* x, __nv_bfloat16* y, long long elems, cudaStream_t stream) {
  if (reinterpret_cast<uintptr_t>(x) & 15) return NL_ERR_ALIGN;
  const long long n8 = elems / 8;
  launch_kernel(cast_f32_bf16_kernel, dim3(grid_cap((n8 + 255) / 256)), dim3(256), 0, stream, 1,
                static_cast<const float*>(x), y, n8);
  return launch_status();
}

int widen_out(const __nv_bfloat16* xb, const float* xf, void* y, float scale, long long elems, cudaStream_t stream) {
  if (reinterpret_cast<uintptr_t>(y) & 15) return NL_ERR_ALIGN;
  const long long n8 = elems / 8;
  launch_kernel(widen_f32_kernel, dim3(grid_cap((n8 + 255) / 256)), dim3(256), 0, stream, 1, xb, xf,
                static_cast<float*>(y), scale, n8);
  return launch_status();
}

}  // namespace fa
}  // namespace nl

extern "C" size_t nl_flash_attention_workspace_bytes(int target, int n, int s, int d, int dtype) {
  return nl::fa::dt_workspace_bytes(target, n, s, d, dtype);
}

extern "C" int nl_flash_attention_fwd_dt(const void* Q, const void* K, const void* V, void* O, float* L, int n,
                                         int s, int d, int dtype, void* workspace, size_t ws_bytes,
                                         cudaStream_t stream) {
  using namespace nl::fa;
  if (dtype == NL_BF16) return nl_flash_attention_fwd(Q, K, V, O, L, n, s, d, stream);
  if (dtype != NL_F32) return NL_ERR_DTYPE;
  const size_t need = dt_workspace_bytes(kTargetFwd, n, s, d, dtype);
  if (need == 0) return NL_ERR_SHAPE;
  if (!workspace || ws_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) return NL_ERR_WORKSPACE;
  const long long elems = static_cast<long long>(n) * s * HD;
  const size_t t16 = ws_align(static_cast<size_t>(elems) * 2);
  char* w = static_cast<char*>(workspace);
  auto* qb = reinterpret_cast<__nv_bfloat16*>(w);
  auto* kb = reinterpret_cast<__nv_bfloat16*>(w + t16);
  auto* vb = reinterpret_cast<__nv_bfloat16*>(w + 2 * t16);
  auto* ob = reinterpret_cast<__nv_bfloat16*>(w + 3 * t16);
  int st;
  if ((st = cast_in(Q, qb, elems, stream)) || (st = cast_in(K, kb, elems, stream)) ||
      (st = cast_in(V, vb, elems, stream)))
    return st;
  if ((st = nl_flash_attention_fwd(qb, kb, vb, ob, L, n, s, d, stream))) return st;
  return widen_out(ob, nullptr, O, 1.f, elems, stream);
}

extern "C" int nl_flash_attention_bwd_dq_dt(const void* Q, const void* K, const void* V, const void* dO,
                                            const float* L, const float* D, void* dQ, int n, int s, int d, int dtype,
                                            void* workspace, size_t ws_bytes, cudaStream_t stream) {
  using namespace nl::fa;
  if (dtype != NL_F32 && dtype != NL_BF16) return NL_ERR_DTYPE;
  const size_t need = dt_workspace_bytes(kTargetBwdDq, n, s, d, dtype);
  if (need == 0 || !dQ) return NL_ERR_SHAPE;
  if (!workspace || ws_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) return NL_ERR_WORKSPACE;
  const long long elems = static_cast<long long>(n) * s * HD;
  const size_t t16 = ws_align(static_cast<size_t>(elems) * 2);
  char* w = static_cast<char*>(workspace);
  if (dtype == NL_BF16)
    return nl_flash_attention_bwd_dq(Q, K, V, dO, L, D, dQ, reinterpret_cast<float*>(w), n, s, d, stream);
  auto* qb = reinterpret_cast<__nv_bfloat16*>(w);
  auto* kb = reinterpret_cast<__nv_bfloat16*>(w + t16);
  auto* vb = reinterpret_cast<__nv_bfloat16*>(w + 2 * t16);
  auto* gb = reinterpret_cast<__nv_bfloat16*>(w + 3 * t16);
  auto* dqb = reinterpret_cast<__nv_bfloat16*>(w + 4 * t16);
  auto* acc = reinterpret_cast<float*>(w + 5 * t16);
  int st;
  if ((st = cast_in(Q, qb, elems, stream)) || (st = cast_in(K, kb, elems, stream)) ||
      (st = cast_in(V, vb, elems, stream)) || (st = cast_in(dO, gb, elems, stream)))
    return st;
  if ((st = nl_flash_attention_bwd_dq(qb, kb, vb, gb, L, D, dqb, acc, n, s, d, stream))) return st;
  // the accumulator holds sum_j dS_ij K_j unscaled; dQ = scale * acc in f32
  return widen_out(nullptr, acc, dQ, 1.f / sqrtf(static_cast<float>(HD)), elems, stream);
}

extern "C" int nl_flash_attention_bwd_dkdv_dt(const void* Q, const void* K, const void* V, const void* dO,
                                              const float* L, const float* D, void* dK, void* dV, int n, int s, int d,
                                              int dtype, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  using namespace nl::fa;
  if (dtype == NL_BF16) return nl_flash_attention_bwd_dkdv(Q, K, V, dO, L, D, dK, dV, n, s, d, stream);
  if (dtype != NL_F32) return NL_ERR_DTYPE;
  const size_t need = dt_workspace_bytes(kTargetBwdDkdv, n, s, d, dtype);
  if (need == 0 || !dK || !dV) return NL_ERR_SHAPE;
  if (!workspace || ws_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) return NL_ERR_WORKSPACE;
  const long long elems = static_cast<long long>(n) * s * HD;
  const size_t t16 = ws_align(static_cast<size_t>(elems) * 2);
  char* w = static_cast<char*>(workspace);
  __nv_bfloat16* b[6];
  for (int i = 0; i < 6; ++i) b[i] = reinterpret_cast<__nv_bfloat16*>(w + i * t16);
  int st;
  if ((st = cast_in(Q, b[0], elems, stream)) || (st = cast_in(K, b[1], elems, stream)) ||
      (st = cast_in(V, b[2], elems, stream)) || (st = cast_in(dO, b[3], elems, stream)))
    return st;
  if ((st = nl_flash_attention_bwd_dkdv(b[0], b[1], b[2], b[3], L, D, b[4], b[5], n, s, d, stream))) return st;
  if ((st = widen_out(b[4], nullptr, dK, 1.f, elems, stream))) return st;
  return widen_out(b[5], nullptr, dV, 1.f, elems, stream);
}
