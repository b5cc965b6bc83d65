// fa_fwd2.cuh — flash-attention forward with two ping-pong query tiles per
// CTA, bf16 in / fp32 softmax and accumulation / bf16 out, for sm_100a
// (tcgen05 + TMEM + TMA).
//
// Same result as fa_fwd.cuh (the reference's `attention_flash`,
// src/attention.py:210-291; oracle src/verifier.py:277-294, extended to bf16
// [B, H, S, D] tensors and a causal mask). What changes is the schedule.
//
// At head dim 128 one key tile costs the tensor core exactly as many cycles as
// the SM's exponential unit (MUFU ex2, 16 results per clock per SM) needs for
// its softmax, so the two can only both stay busy if the softmax of one tile
// always runs while the tensor core works on something else. Here a CTA owns
// two 128-row query tiles, A and B, of the same (batch, head) and walks the
// 64-key K/V tiles once for both (each K/V tile is loaded once and used by
// both query tiles). The single MMA-issuing thread interleaves the tiles:
//
//     S_A(j) = Q_A·K_j^T,  O_B += P_B(j-1)·V_{j-1},  S_B(j) = Q_B·K_j^T,  O_A += P_A(j)·V_j
//
// so while the softmax warps of tile A turn S_A(j) into P_A(j), the tensor
// core computes tile B's products, and the other way round. Each tile has its
// own softmax warpgroup (4 warps, one query row per thread, the whole 64-key
// row in registers: no cross-warp exchange for the row maximum).
//
// A commit on s_full_X(j) tracks every MMA issued before S_X(j), which
// includes O_X += P_X(j-1)·V_{j-1}; so when the softmax of tile X sees
// S_X(j), the previous P_X has been consumed and O_X is not being written:
// P_X needs one TMEM buffer and O_X can be rescaled there without a wait.
//
// Warps (512 threads): 0 TMA loads of Q_A, Q_B and the K ring; 1 TMEM
// allocation and the MMA-issuing lane; 2 TMA loads of the V ring; 3 idle;
// 4-7 softmax of tile A; 8-11 softmax of tile B; 12-15 epilogue (O / l in
// bf16 to global memory, tile A then tile B of every item).
// TMEM columns: S_A [0,64) S_B [64,128) P_A [128,160) P_B [160,192)
//               O_A [256,256+D) O_B [384,384+D) — 512 columns allocated.
// Softmax details as in fa_fwd.cuh: exponentials 2^(s·scale·log2e − m) on
// MUFU ex2, the running maximum raised (O and the row sum rescaled) only when
// it grows by more than 2^8, fp32 row sums, bf16 P. Every mbarrier wait is
// bounded; a timeout records DEV_MBAR_TIMEOUT and the CTA unwinds (loaders
// drain their copies, MMAs drain before TMEM is released).
#pragma once
#include "kt_common.cuh"
#include "sm100.cuh"

#ifndef KT_FA2_KSTAGES
#define KT_FA2_KSTAGES 4  // K ring depth (64-key tiles)
#endif
#ifndef KT_FA2_VSTAGES
#define KT_FA2_VSTAGES 4  // V ring depth
#endif
#ifndef KT_FA2_ORDER
#define KT_FA2_ORDER 0  // 0: ping-pong issue order (below); 1: in-phase order S_A(j), S_B(j), P_A(j-1)V, P_B(j-1)V
#endif
#ifndef KT_FA_EXP16
#define KT_FA_EXP16 0  // 1: exponentials as packed half-precision pairs (ex2.approx.f16x2); not offered
                       // by the tuner for this kernel: NaN on the first causal rows of heads whose
                       // scores reach ~300 (log2 units)
#endif
#ifndef KT_FA2_POLY
#define KT_FA2_POLY 0  // n > 0: every n-th pair of exponentials of a row is computed by a polynomial on the FMA pipe
#endif

namespace kt {
namespace fa2 {

constexpr int BM = 128;  // query rows per tile
constexpr int QT = 2;    // query tiles per CTA
constexpr int BN = 64;   // keys per K/V tile
constexpr int THREADS = 512;
constexpr int SOFTMAX_WARP0 = 4;
constexpr int EPI_WARP0 = 12;
constexpr int TILE_THREADS = 128;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kHeadGroup = 8;              // causal scheduling: heads whose K/V share L2

template <int D, int KST, int VST>
struct Cfg {
  static_assert(D == 64 || D == 128, "head dim");
  static constexpr int REGIONS = D / 64;      // 128-byte (64 bf16) column slabs
  static constexpr int Q_SLAB = BM * 128;     // one slab: 128 rows x 128 bytes
  static constexpr int KV_SLAB = BN * 128;    // 64 rows x 128 bytes
  static constexpr int Q_BYTES = REGIONS * Q_SLAB;
  static constexpr int KV_BYTES = REGIONS * KV_SLAB;
  static constexpr int Q_OFFSET = 0;
  static constexpr int K_OFFSET = Q_OFFSET + QT * Q_BYTES;
  static constexpr int V_OFFSET = K_OFFSET + KST * KV_BYTES;
  static constexpr int L_OFFSET = V_OFFSET + VST * KV_BYTES;  // row sums [QT][BM] fp32
  static constexpr int BAR_OFFSET = L_OFFSET + QT * BM * 4;
  // q_full[2] q_empty[2] k_full[KST] k_empty[KST] v_full[VST] v_empty[VST]
  // s_full[2] s_free[2] p_full[2] o_final[2] o_empty[2] l_full[2] l_empty[2] o_done[2] done
  static constexpr int NUM_BARS = 4 + 2 * KST + 2 * VST + 16 + 1;
  static constexpr int SMEM_BYTES = BAR_OFFSET + NUM_BARS * 8 + 16 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_P = 128, COL_O = 256;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA/ALU pipes (the same method as fa_fwd.cuh: x = n + f, n =
// round(x), 2^f by a least-squares cubic on [-1/2, 1/2], 2^n into the exponent
// field; max relative error 1.4e-4 on [-125, 8]).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -125.f);
  const float y = x + 12582912.0f;
  const float n = y - 12582912.0f;
  const float f = x - n;
  float p = fmaf(0.055029310286045074f, f, 0.2422567903995514f);
  p = fmaf(p, f, 0.6932530403137207f);
  p = fmaf(p, f, 0.9999513626098633f);
  const int ni = __float_as_int(y) - 0x4B400000;
  return __int_as_float(__float_as_int(p) + (ni << 23));
}

// 2^x0, 2^x1 from one packed half-precision MUFU operation (arguments rounded
// to fp16; results back in fp32), as fa_fwd.cuh's ex2_h2.
__device__ __forceinline__ void ex2_h2(float x0, float x1, float& p0, float& p1) {
  uint32_t h, e;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(x1), "f"(x0));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(e) : "r"(h));
  asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tcvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
      : "=f"(p0), "=f"(p1)
      : "r"(e));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// {lo, hi} fp32 pair in one 64-bit register and packed fp32x2 arithmetic
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  return ((uint64_t)__float_as_uint(hi) << 32) | (uint64_t)__float_as_uint(lo);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Work item w (two consecutive 128-row query tiles of one (b, h)) -> (qp, bh).
// Non-causal: the query pairs of one head are adjacent (its K/V stays in L2).
// Causal: heads in groups of kHeadGroup, inside a group the heaviest (latest)
// query pairs first.
template <bool CAUSAL>
__device__ __forceinline__ void item_coords(int w, int num_qp, int BH, int& qp, int& bh) {
  if (CAUSAL) {
    const int per_group = kHeadGroup * num_qp;
    const int group = w / per_group;
    const int r = w - group * per_group;
    const int gsize = min(kHeadGroup, BH - group * kHeadGroup);
    qp = num_qp - 1 - r / gsize;
    bh = group * kHeadGroup + r % gsize;
  } else {
    qp = w % num_qp;
    bh = w / num_qp;
  }
}

// K/V tiles that query tile x (0 = A, 1 = B) of query pair qp attends to.
template <bool CAUSAL>
__device__ __forceinline__ int kv_tiles(int qp, int x, int S) {
  const int all = (S + BN - 1) / BN;
  return CAUSAL ? min(all, (qp * 2 * BM + x * BM + BM + BN - 1) / BN) : all;
}

template <int D, int KST, int VST, bool CAUSAL, int ORDER>
__global__ void __launch_bounds__(THREADS, 1)
fa2_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, __nv_bfloat16* __restrict__ O, int S, int BH,
               float scale_log2) {
  using CF = Cfg<D, KST, VST>;
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  float* red_l = reinterpret_cast<float*>(base_ptr + CF::L_OFFSET);
  const uint32_t bar0 = base + CF::BAR_OFFSET;
  auto q_full = [&](int x) { return bar0 + 8u * x; };
  auto q_empty = [&](int x) { return bar0 + 8u * (2 + x); };
  auto k_full = [&](int s) { return bar0 + 8u * (4 + s); };
  auto k_empty = [&](int s) { return bar0 + 8u * (4 + KST + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (4 + 2 * KST + s); };
  auto v_empty = [&](int s) { return bar0 + 8u * (4 + 2 * KST + VST + s); };
  constexpr int R = 4 + 2 * KST + 2 * VST;
  auto s_full = [&](int x) { return bar0 + 8u * (R + x); };
  auto s_free = [&](int x) { return bar0 + 8u * (R + 2 + x); };
  auto p_full = [&](int x) { return bar0 + 8u * (R + 4 + x); };
  auto o_final = [&](int x) { return bar0 + 8u * (R + 6 + x); };
  auto o_empty = [&](int x) { return bar0 + 8u * (R + 8 + x); };
  auto l_full = [&](int x) { return bar0 + 8u * (R + 10 + x); };
  auto l_empty = [&](int x) { return bar0 + 8u * (R + 12 + x); };
  auto o_done = [&](int x) { return bar0 + 8u * (R + 14 + x); };  // in-phase order: one phase per P_x·V
  const uint32_t done_bar = bar0 + 8u * (R + 16);
  const uint32_t tmem_slot = bar0 + 8u * CF::NUM_BARS;
  const volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<const volatile uint32_t*>(base_ptr + CF::BAR_OFFSET + 8 * CF::NUM_BARS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_qp = (S + QT * BM - 1) / (QT * BM);
  const int num_items = BH * num_qp;

  if (threadIdx.x == 0) {
    for (int x = 0; x < 2; ++x) {
      mbar_init(q_full(x), 1);
      mbar_init(q_empty(x), 1);
      mbar_init(s_full(x), 1);
      mbar_init(s_free(x), TILE_THREADS);
      mbar_init(p_full(x), TILE_THREADS);
      mbar_init(o_final(x), 1);
      mbar_init(o_empty(x), TILE_THREADS);
      mbar_init(l_full(x), TILE_THREADS);
      mbar_init(l_empty(x), TILE_THREADS);
      mbar_init(o_done(x), 1);
    }
    for (int s = 0; s < KST; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, CF::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot_ptr;
  bool timed_out = false;

  if (warp == 0 || warp == 2) {
    if (lane == 0) {
      // warp 0: Q_A, Q_B of every item and the K ring; warp 2: the V ring.
      // Ring positions run on across items.
      const bool is_k = (warp == 0);
      constexpr int MAXS = KST > VST ? KST : VST;
      const int nst = is_k ? KST : VST;
      uint32_t last_ph[MAXS];
      bool pending[MAXS];
#pragma unroll
      for (int i = 0; i < MAXS; ++i) pending[i] = false;
      bool q_pending[2] = {false, false};
      uint32_t q_last_ph[2] = {0u, 0u};
      int pos = 0;
      int k = 0;
      for (int w = blockIdx.x; w < num_items && !timed_out; w += gridDim.x, ++k) {
        int qp, bh;
        item_coords<CAUSAL>(w, num_qp, BH, qp, bh);
        const int n_b = kv_tiles<CAUSAL>(qp, 1, S);
        if (is_k) {
          const uint32_t qph = (uint32_t)k & 1u;
          for (int x = 0; x < QT && !timed_out; ++x) {
            if (!mbar_wait(q_empty(x), qph ^ 1u)) {
              timed_out = true;
              break;
            }
            mbar_arrive_expect_tx(q_full(x), CF::Q_BYTES);
#pragma unroll
            for (int r = 0; r < CF::REGIONS; ++r)
              tma_load_3d(base + CF::Q_OFFSET + x * CF::Q_BYTES + r * CF::Q_SLAB, &tm_q, 64 * r,
                          (qp * QT + x) * BM, bh, q_full(x));
            q_pending[x] = true;
            q_last_ph[x] = qph;
          }
        }
        for (int j = 0; j < n_b && !timed_out; ++j, ++pos) {
          const int s = pos % nst;
          const uint32_t ph = (uint32_t)(pos / nst) & 1u;
          const uint32_t empty = is_k ? k_empty(s) : v_empty(s);
          const uint32_t full = is_k ? k_full(s) : v_full(s);
          if (!mbar_wait(empty, ph ^ 1u)) {
            timed_out = true;
            break;
          }
          const uint32_t dst = base + (is_k ? CF::K_OFFSET : CF::V_OFFSET) + s * CF::KV_BYTES;
          mbar_arrive_expect_tx(full, CF::KV_BYTES);
#pragma unroll
          for (int r = 0; r < CF::REGIONS; ++r)
            tma_load_3d(dst + r * CF::KV_SLAB, is_k ? &tm_k : &tm_v, 64 * r, j * BN, bh, full);
          last_ph[s] = ph;
          pending[s] = true;
        }
      }
      if (timed_out) {
        // let every copy still in flight land before the CTA exits
        for (int x = 0; x < 2; ++x)
          if (q_pending[x]) (void)mbar_wait(q_full(x), q_last_ph[x]);
        for (int i = 0; i < nst; ++i)
          if (pending[i]) (void)mbar_wait(is_k ? k_full(i) : v_full(i), last_ph[i]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f32acc(kFmtBF16, BM, BN, 0, 0);
      constexpr uint32_t idesc_o = idesc_f32acc(kFmtBF16, BM, D, 0, 1);
      // descriptors as (lo, hi) words: lo + byte offset / 16 addresses base + offset
      const uint64_t dk = desc_sw128(base, 16u, 1024u);                    // K-major operands (Q, K)
      const uint64_t dv = desc_sw128(base, (uint32_t)CF::KV_SLAB, 1024u);  // V, MN-major
      const uint32_t k_hi = (uint32_t)(dk >> 32), v_hi = (uint32_t)(dv >> 32);
      const uint32_t q_lo0 = (uint32_t)dk + (CF::Q_OFFSET >> 4);
      const uint32_t k_lo0 = (uint32_t)dk + (CF::K_OFFSET >> 4);
      const uint32_t v_lo0 = (uint32_t)dv + (CF::V_OFFSET >> 4);
      int kpos = 0, vpos0 = 0;           // K ring position, V ring position of this item's tile 0
      uint32_t s_cnt[2] = {0u, 0u};      // S tiles issued per query tile
      uint32_t p_cnt[2] = {0u, 0u};      // P tiles consumed per query tile
      bool ok = true;
      // S_x(j) = Q_x·K_j^T
      auto issue_s = [&](int x, int kslot) -> bool {
        if (s_cnt[x] > 0 && !mbar_wait(s_free(x), (s_cnt[x] - 1u) & 1u)) return false;
        tc_fence_after();
        const uint32_t q_lo = q_lo0 + (uint32_t)x * (CF::Q_BYTES >> 4);
        const uint32_t k_lo = k_lo0 + (uint32_t)kslot * (CF::KV_BYTES >> 4);
        const uint32_t d_tmem = tmem + CF::COL_S + (uint32_t)(x * BN);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qoff = (uint32_t)(((kk >> 2) * CF::Q_SLAB + (kk & 3) * 32) >> 4);
          const uint32_t koff = (uint32_t)(((kk >> 2) * CF::KV_SLAB + (kk & 3) * 32) >> 4);
          mma_f16_ss_w(d_tmem, q_lo + qoff, k_hi, k_lo + koff, k_hi, idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(s_full(x));
        ++s_cnt[x];
        return true;
      };
      // O_x (+)= P_x(j)·V_j; the first product of an item overwrites O_x once the
      // epilogue has read the previous item's O_x
      auto issue_pv = [&](int x, int j, int item, bool last_user, bool last_of_tile) -> bool {
        if (!mbar_wait(p_full(x), p_cnt[x] & 1u)) return false;
        ++p_cnt[x];
        const int vp = vpos0 + j;
        const int vslot = vp % VST;
        if (!mbar_wait(v_full(vslot), (uint32_t)(vp / VST) & 1u)) return false;
        if (j == 0 && !mbar_wait(o_empty(x), ((uint32_t)item & 1u) ^ 1u)) return false;
        tc_fence_after();
        const uint32_t v_lo = v_lo0 + (uint32_t)vslot * (CF::KV_BYTES >> 4);
        const uint32_t p_tmem = tmem + CF::COL_P + (uint32_t)(x * (BN / 2));
        const uint32_t o_tmem = tmem + CF::COL_O + (uint32_t)(x * 128);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_f16_ts_w(o_tmem, p_tmem + (uint32_t)(kk * 8), v_lo + (uint32_t)(kk * 16 * 128 / 16), v_hi, idesc_o,
                       (j > 0 || kk > 0) ? 1u : 0u);
        if (ORDER == 1) mma_commit(o_done(x));
        if (last_user) mma_commit(v_empty(vslot));
        if (last_of_tile) mma_commit(o_final(x));
        return true;
      };
      int k = 0;
      for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x, ++k) {
        int qp, bh;
        item_coords<CAUSAL>(w, num_qp, BH, qp, bh);
        const int n_a = kv_tiles<CAUSAL>(qp, 0, S), n_b = kv_tiles<CAUSAL>(qp, 1, S);
        const uint32_t qph = (uint32_t)k & 1u;
        if (!mbar_wait(q_full(0), qph) || !mbar_wait(q_full(1), qph)) {
          ok = false;
          break;
        }
        if constexpr (ORDER == 0) {
          for (int j = 0; j < n_b && ok; ++j, ++kpos) {
            const int kslot = kpos % KST;
            if (!mbar_wait(k_full(kslot), (uint32_t)(kpos / KST) & 1u)) {
              ok = false;
              break;
            }
            if (j < n_a) {
              if (!issue_s(0, kslot)) {
                ok = false;
                break;
              }
              if (j == n_a - 1) mma_commit(q_empty(0));
            }
            // tile B's product of the previous K/V tile; B is the last user of V_{j-1}
            if (j > 0 && !issue_pv(1, j - 1, k, true, false)) {
              ok = false;
              break;
            }
            if (!issue_s(1, kslot)) {
              ok = false;
              break;
            }
            mma_commit(k_empty(kslot));
            if (j == n_b - 1) mma_commit(q_empty(1));
            if (j < n_a && !issue_pv(0, j, k, false, j == n_a - 1)) {
              ok = false;
              break;
            }
          }
          if (ok && !issue_pv(1, n_b - 1, k, true, true)) ok = false;
        } else {
          // in phase: both scores of K_j, then both products of V_{j-1}
          for (int j = 0; j < n_b && ok; ++j, ++kpos) {
            const int kslot = kpos % KST;
            if (!mbar_wait(k_full(kslot), (uint32_t)(kpos / KST) & 1u)) {
              ok = false;
              break;
            }
            if (j < n_a) {
              if (!issue_s(0, kslot)) {
                ok = false;
                break;
              }
              if (j == n_a - 1) mma_commit(q_empty(0));
            }
            if (!issue_s(1, kslot)) {
              ok = false;
              break;
            }
            mma_commit(k_empty(kslot));
            if (j == n_b - 1) mma_commit(q_empty(1));
            if (j > 0) {
              if (j - 1 < n_a && !issue_pv(0, j - 1, k, false, j - 1 == n_a - 1)) {
                ok = false;
                break;
              }
              if (!issue_pv(1, j - 1, k, true, false)) {
                ok = false;
                break;
              }
            }
          }
          if (ok && n_b - 1 < n_a && !issue_pv(0, n_b - 1, k, false, true)) ok = false;
          if (ok && !issue_pv(1, n_b - 1, k, true, true)) ok = false;
        }
        vpos0 += n_b;
      }
      timed_out = !ok;
      mma_commit(done_bar);
    }
  } else if (warp >= SOFTMAX_WARP0 && warp < EPI_WARP0) {
    // softmax of tile x: TMEM lane quarter = warp % 4, one query row per thread
    const int x = (warp - SOFTMAX_WARP0) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + CF::COL_S + (uint32_t)(x * BN);
    const uint32_t p_addr = tmem + lane_off + CF::COL_P + (uint32_t)(x * (BN / 2));
    const uint32_t o_addr = tmem + lane_off + CF::COL_O + (uint32_t)(x * 128);
    const uint64_t c2 = f2(scale_log2, scale_log2);
    uint32_t cnt = 0;
    int k = 0;
    for (int w = blockIdx.x; w < num_items && !timed_out; w += gridDim.x, ++k) {
      int qp, bh;
      item_coords<CAUSAL>(w, num_qp, BH, qp, bh);
      const int n_x = kv_tiles<CAUSAL>(qp, x, S);
      const int r0 = (qp * QT + x) * BM;  // first query row of this tile
      const int qrow = r0 + row;
      float m_run = -INFINITY;  // running max of s·scale·log2e used by the exponentials
      float l_run = 0.f;
      for (int j = 0; j < n_x; ++j, ++cnt) {
        if (!__all_sync(0xffffffffu, mbar_wait(s_full(x), cnt & 1u))) {
          timed_out = true;
          break;
        }
        tc_fence_after();
        uint32_t sv[BN];
        tmem_ld32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld32(s_addr + 32u, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(s_free(x));  // S_x is in registers: the next S_x may overwrite it
        const int key0 = j * BN;
        if ((CAUSAL && key0 + BN - 1 > r0) || key0 + BN > S) {
#pragma unroll
          for (int c = 0; c < BN; ++c) {
            const int key = key0 + c;
            if (!(key < S && (!CAUSAL || key <= qrow))) sv[c] = __float_as_uint(-INFINITY);
          }
        }
        float m4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) m4[q] = __uint_as_float(sv[q]);
#pragma unroll
        for (int c = 4; c < BN; c += 8) {
#pragma unroll
          for (int q = 0; q < 4; ++q) m4[q] = max3(m4[q], __uint_as_float(sv[c + 2 * q]), __uint_as_float(sv[c + 2 * q + 1]));
        }
        const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        const float m_tile = mx * scale_log2;
        const bool raise = m_tile > m_run + kRescaleThreshold;
        float alpha = 1.f;
        if (raise) {
          alpha = (m_run == -INFINITY) ? 0.f : ex2(m_run - m_tile);
          m_run = m_tile;
          l_run *= alpha;
        }
        // in-phase order: P_x and O_x are free once the previous product into O_x is done
        if (ORDER == 1 && cnt > 0 && !__all_sync(0xffffffffu, mbar_wait(o_done(x), (cnt - 1u) & 1u))) {
          timed_out = true;
          break;
        }
        if (ORDER == 1) tc_fence_after();
        // p = 2^(s·c − m) (masked entries are −inf -> 0), row sum, bf16 P into TMEM
        const uint64_t nm2 = f2(-m_run, -m_run);
        uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int c = 0; c < BN; c += 32) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint64_t xx = fma2(f2(__uint_as_float(sv[c + 2 * i]), __uint_as_float(sv[c + 2 * i + 1])), c2, nm2);
            float p0, p1;
            if (KT_FA_EXP16) {
              ex2_h2(f2_lo(xx), f2_hi(xx), p0, p1);
            } else if (KT_FA2_POLY > 0 && ((c / 2 + i) % (KT_FA2_POLY > 0 ? KT_FA2_POLY : 1)) == (KT_FA2_POLY > 0 ? KT_FA2_POLY - 1 : 0)) {
              p0 = ex2_poly(f2_lo(xx));
              p1 = ex2_poly(f2_hi(xx));
            } else {
              p0 = ex2(f2_lo(xx));
              p1 = ex2(f2_hi(xx));
            }
            acc[i & 3] = add2(acc[i & 3], f2(p0, p1));
            pk[i] = pack_bf16(p0, p1);
          }
          tmem_st16(p_addr + (uint32_t)(c / 2), pk);
        }
        const uint64_t a01 = add2(acc[0], acc[1]), a23 = add2(acc[2], acc[3]);
        const uint64_t a = add2(a01, a23);
        l_run += f2_lo(a) + f2_hi(a);
        // O_x holds P_x(0..j-1)·V and no product into it is in flight until p_full(x)
        // (done after P, when the score registers are free)
        if (j > 0 && __any_sync(0xffffffffu, raise)) {
#pragma unroll 1
          for (int c = 0; c < D; c += 32) {
            uint32_t v[32];
            tmem_ld32(o_addr + (uint32_t)c, v);
            tmem_ld_wait();
            uint32_t w0[16], w1[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              w0[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
              w1[i] = __float_as_uint(__uint_as_float(v[16 + i]) * alpha);
            }
            tmem_st16(o_addr + (uint32_t)c, w0);
            tmem_st16(o_addr + (uint32_t)c + 16u, w1);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_full(x));
      }
      if (timed_out) break;
      // hand the row sum to the epilogue
      if (!__all_sync(0xffffffffu, mbar_wait(l_empty(x), ((uint32_t)k & 1u) ^ 1u))) {
        timed_out = true;
        break;
      }
      red_l[x * BM + row] = l_run;
      mbar_arrive(l_full(x));
    }
  } else if (warp >= EPI_WARP0) {
    // epilogue: O_x / l in bf16, one query row per thread; O_x is released to the
    // next item's first product as soon as it is in registers
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    int k = 0;
    for (int w = blockIdx.x; w < num_items && !timed_out; w += gridDim.x, ++k) {
      int qp, bh;
      item_coords<CAUSAL>(w, num_qp, BH, qp, bh);
      const uint32_t ph = (uint32_t)k & 1u;
      for (int x = 0; x < QT; ++x) {
        const int qrow = (qp * QT + x) * BM + row;
        if (!__all_sync(0xffffffffu, mbar_wait(o_final(x), ph)) ||
            !__all_sync(0xffffffffu, mbar_wait(l_full(x), ph))) {
          timed_out = true;
          break;
        }
        const float l = red_l[x * BM + row];
        mbar_arrive(l_empty(x));
        tc_fence_after();
        const float inv = 1.0f / l;
        const uint32_t o_addr = tmem + lane_off + CF::COL_O + (uint32_t)(x * 128);
        uint4* dst = reinterpret_cast<uint4*>(O + ((int64_t)bh * S + qrow) * D);
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          uint32_t v[32];
          tmem_ld32(o_addr + (uint32_t)c, v);
          tmem_ld_wait();
          if (c + 32 == D) {
            tc_fence_before();
            mbar_arrive(o_empty(x));  // all of O_x is in registers: the next item may overwrite it
          }
          if (qrow < S) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float* f = reinterpret_cast<const float*>(v) + 8 * i;
              dst[c / 8 + i] = make_uint4(pack_bf16(f[0] * inv, f[1] * inv), pack_bf16(f[2] * inv, f[3] * inv),
                                          pack_bf16(f[4] * inv, f[5] * inv), pack_bf16(f[6] * inv, f[7] * inv));
            }
          }
        }
      }
    }
  }
  if (timed_out) raise_device_error(DEV_MBAR_TIMEOUT);
  __syncthreads();
  if (warp == 1) {
    (void)__all_sync(0xffffffffu, mbar_wait(done_bar, 0));
    tc_fence_after();
    tmem_dealloc(tmem, CF::TMEM_COLS);
  }
}

// [B·H, S, D] bf16 viewed as a 3-D tensor (D, S, B·H); box 64 × rows × 1, 128-byte swizzle.
inline int make_tmap(CUtensorMap* map, const void* base, int64_t BH, int64_t S, int64_t D, uint32_t rows) {
  PFN_encodeTiled enc = get_encode_tiled();
  if (enc == nullptr) return fail(KT_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)S * D * 2};
  cuuint32_t box[3] = {64, rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KT_ERR_CUDA, "cuTensorMapEncodeTiled (attention) failed (%d)", (int)r);
  return KT_OK;
}

template <int D, bool CAUSAL>
inline int launch_t(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int64_t BH, int64_t S,
                    float scale, cudaStream_t st) {
  using CF = Cfg<D, KT_FA2_KSTAGES, KT_FA2_VSTAGES>;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap(&tq, Q, BH, S, D, BM);
  if (rc == KT_OK) rc = make_tmap(&tk, K, BH, S, D, BN);
  if (rc == KT_OK) rc = make_tmap(&tv, V, BH, S, D, BN);
  if (rc != KT_OK) return rc;
  auto kern = fa2_fwd_kernel<D, KT_FA2_KSTAGES, KT_FA2_VSTAGES, CAUSAL, KT_FA2_ORDER>;
  rc = ensure_smem((const void*)kern, CF::SMEM_BYTES, "attention: smem attribute");
  if (rc != KT_OK) return rc;
  const float scale_log2 = scale * 1.4426950408889634f;  // log2(e)
  // persistent: one CTA per SM (TMEM holds one CTA's 512 columns), items strided over the CTAs
  const int64_t items = BH * ((S + QT * BM - 1) / (QT * BM));
  const int64_t sms = sm_count();
  dim3 grid((unsigned)(items < sms ? items : sms));
  kern<<<grid, THREADS, CF::SMEM_BYTES, st>>>(tq, tk, tv, reinterpret_cast<__nv_bfloat16*>(O), (int)S, (int)BH,
                                              scale_log2);
  return check_launch("attention fwd (ping-pong)");
}

}  // namespace fa2
}  // namespace kt
