// fa_fwd.cuh — flash-attention forward, bf16 in / fp32 softmax and
// accumulation / bf16 out, for sm_100a (tcgen05 + TMEM + TMA).
//
// Computes O = softmax(scale·Q·K^T [+ causal mask]) · V per (batch, head) on
// [B, H, S, D] tensors — the reference's `attention_flash` /
// `attention_tiled` (src/attention.py:210-291, :75-176; oracle
// src/verifier.py:277-294), which are single-head fp32 SIMT kernels with one
// CTA per query row.
//
// CTA = one (b, h) and BM = 128 query rows; 352 threads:
//   warp 0     one lane: TMA loads of the Q tile (once) and of K tiles (BN = 128
//              keys) into a STAGES-slot ring; a K slot is released as soon as
//              S_j has read it (128-byte swizzle, 64-column boxes)
//   warp 10    one lane: TMA loads of V tiles into a VSTAGES-slot ring, released
//              after O += P_j·V_j. The two rings run ahead of the tensor core
//              independently, so load latency stays off its critical path.
//   warp 1     allocates 512 TMEM columns; one lane issues the MMAs:
//                S_j = Q·K_j^T  (kind::f16, M=128, N=128, A and B from smem)
//                O  += P_j·V_j   (kind::f16, M=128, N=D, A = P from TMEM, B = V MN-major)
//              S_{j+1} is issued before O += P_j·V_j so the tensor core works on
//              the next scores while the softmax warps process the current ones.
//   warps 2-9  softmax. TMEM lane = query row; warps w and w+4 share the 32
//              rows of lane quarter w%4 and split their 128 score columns in
//              halves. Per tile: the half-row maxima are exchanged through shared
//              memory (one mbarrier per warp pair, bounded wait), p =
//              2^(s·scale·log2e − m) for the own half (every 4th pair of values
//              by a polynomial on the FMA pipe, the rest by MUFU ex2), bf16 P back
//              to TMEM, partial row sum. The running max is only raised (O and
//              the sums rescaled) when it grows by more than 2^8, so O is rarely
//              touched. Final O / l in bf16.
// TMEM columns: S0 [0,128) S1 [128,256) O [256,256+D) P0 [384,448) P1 [448,512).
// Every mbarrier wait is bounded; a timeout records DEV_MBAR_TIMEOUT and the
// CTA unwinds (loader drains its copies, MMAs drain before TMEM is released).
#pragma once
#include "kt_common.cuh"
#include "sm100.cuh"

#ifndef KT_FA_STAGES
#define KT_FA_STAGES 2  // K ring depth (the V ring has KT_FA_VSTAGES slots)
#endif
#ifndef KT_FA_VSTAGES
#define KT_FA_VSTAGES 2
#endif
#ifndef KT_FA_BN
#define KT_FA_BN 128
#endif
#ifndef KT_FA_POLY
#define KT_FA_POLY 1  // share of exponentials on the FMA pipe: every 4th value pair when 1
#endif

namespace kt {
namespace fa {

constexpr int BM = 128;
constexpr int BN = 128;  // keys per tile (the S accumulator is 128 columns)
constexpr int SOFTMAX_WARPS = 8;
constexpr int V_LOADER_WARP = 2 + SOFTMAX_WARPS;
constexpr int THREADS = 96 + 32 * SOFTMAX_WARPS;
constexpr int SOFTMAX_THREADS = 32 * SOFTMAX_WARPS;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: O is rescaled only when the max grows by > 2^8
constexpr int kHeadGroup = 8;              // causal scheduling: heads whose K/V share L2

template <int D, int STAGES, int VSTAGES = KT_FA_VSTAGES>
struct Cfg {
  static_assert(D == 64 || D == 128, "head dim");
  static constexpr int REGIONS = D / 64;            // 128-byte (64 bf16) column slabs per row
  static constexpr int SLAB = 128 * 128;            // one slab of 128 rows × 128 bytes
  static constexpr int Q_BYTES = REGIONS * SLAB;    // 128 rows × D bf16
  static constexpr int K_BYTES = REGIONS * SLAB;    // BN keys × D
  static constexpr int V_BYTES = REGIONS * SLAB;
  static constexpr int Q_OFFSET = 0;
  static constexpr int K_OFFSET = Q_BYTES;
  static constexpr int V_OFFSET = K_OFFSET + STAGES * K_BYTES;
  // softmax exchange: [2 parity][2 half][128 rows] maxima + [2 half][128 rows] row sums
  static constexpr int RED_OFFSET = V_OFFSET + VSTAGES * V_BYTES;
  static constexpr int BAR_OFFSET = RED_OFFSET + 6 * 128 * 4;
  // q_full, k_full[S], k_empty[S], v_full[VS], v_empty[VS], s_full[2], s_free[2], p_full[2],
  // o_done, o_final, done, pair[4]
  static constexpr int NUM_BARS = 1 + 2 * STAGES + 2 * VSTAGES + 2 + 2 + 2 + 1 + 1 + 1 + 4;
  static constexpr int SMEM_BYTES = BAR_OFFSET + NUM_BARS * 8 + 16 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_O = 256, COL_P = 384;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA/ALU pipes: x = n + f with n = round(x) (|f| <= 1/2, via the
// 1.5·2^23 rounding constant), 2^f by a degree-3 polynomial least-squares fitted
// to 2^f on [-1/2, 1/2] (relative weight), 2^n inserted into the exponent field.
// x is clamped to >= -125 so the result stays a normal number. Max relative
// error 1.4e-4 on [-125, 8] (bf16 P keeps 8 mantissa bits).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -125.f);
  const float y = x + 12582912.0f;
  const float n = y - 12582912.0f;
  const float f = x - n;
  float p = fmaf(0.055029310286045074f, f, 0.2422567903995514f);
  p = fmaf(p, f, 0.6932530403137207f);
  p = fmaf(p, f, 0.9999513626098633f);
  const int ni = __float_as_int(y) - 0x4B400000;  // bits of 1.5·2^23
  return __int_as_float(__float_as_int(p) + (ni << 23));
}

// Pack two fp32 values into bf16x2 (round to nearest even); `lo` in the low half.
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <int D, int STAGES, bool CAUSAL>
__global__ void __launch_bounds__(THREADS, 1)
fa_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, __nv_bfloat16* __restrict__ O, int S, float scale_log2) {
  using CF = Cfg<D, STAGES>;
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  float* red = reinterpret_cast<float*>(base_ptr + CF::RED_OFFSET);
  const uint32_t bar0 = base + CF::BAR_OFFSET;
  constexpr int VSTAGES = KT_FA_VSTAGES;
  constexpr int R = 1 + 2 * STAGES + 2 * VSTAGES;  // first barrier after the load rings
  const uint32_t q_full = bar0;
  auto k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bar0 + 8u * (1 + STAGES + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (1 + 2 * STAGES + s); };
  auto v_empty = [&](int s) { return bar0 + 8u * (1 + 2 * STAGES + VSTAGES + s); };
  auto s_full = [&](int b) { return bar0 + 8u * (R + b); };
  auto s_free = [&](int b) { return bar0 + 8u * (R + 2 + b); };
  auto p_full = [&](int b) { return bar0 + 8u * (R + 4 + b); };
  const uint32_t o_done = bar0 + 8u * (R + 6);     // one phase per P·V product
  const uint32_t o_final = bar0 + 8u * (R + 7);    // single use: the last P·V product landed
  const uint32_t done_bar = bar0 + 8u * (R + 8);
  const uint32_t pair_bar0 = bar0 + 8u * (R + 9);  // 4 softmax warp-pair exchanges
  const uint32_t tmem_slot = bar0 + 8u * CF::NUM_BARS;
  const volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<const volatile uint32_t*>(base_ptr + CF::BAR_OFFSET + 8 * CF::NUM_BARS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_q_tiles = (S + BM - 1) / BM;
  // 1-D grid, blocks start in index order. Non-causal: the query tiles of one
  // head are adjacent, so the CTAs running together share that head's K/V in
  // L2. Causal: heads in groups of kHeadGroup (K/V of a group stays in L2),
  // inside a group the heaviest (latest) query tiles first.
  int qt, bh;
  if (CAUSAL) {
    const int per_group = kHeadGroup * num_q_tiles;
    const int group = (int)blockIdx.x / per_group;
    const int r = (int)blockIdx.x - group * per_group;
    const int gsize = min(kHeadGroup, (int)(gridDim.x / num_q_tiles) - group * kHeadGroup);
    qt = num_q_tiles - 1 - r / gsize;
    bh = group * kHeadGroup + r % gsize;
  } else {
    qt = (int)blockIdx.x % num_q_tiles;
    bh = (int)blockIdx.x / num_q_tiles;
  }
  const int q0 = qt * BM;
  const int num_kv_all = (S + BN - 1) / BN;
  const int n_kv = CAUSAL ? min(num_kv_all, (q0 + BM - 1) / BN + 1) : num_kv_all;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < VSTAGES; ++s) {
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(s_free(b), SOFTMAX_THREADS);
      mbar_init(p_full(b), SOFTMAX_THREADS);
    }
    mbar_init(o_done, 1);
    mbar_init(o_final, 1);
    mbar_init(done_bar, 1);
    for (int q = 0; q < 4; ++q) mbar_init(pair_bar0 + 8u * q, 64);
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

  if (warp == 0 || warp == V_LOADER_WARP) {
    if (lane == 0) {
      // warp 0: Q once, then K tiles; warp V_LOADER_WARP: V tiles
      const bool is_k = (warp == 0);
      const int nst = is_k ? STAGES : VSTAGES;
      if (is_k) {
        const uint32_t q_dst = base + CF::Q_OFFSET;
        mbar_arrive_expect_tx(q_full, CF::Q_BYTES);
#pragma unroll
        for (int r = 0; r < CF::REGIONS; ++r) tma_load_3d(q_dst + r * CF::SLAB, &tm_q, 64 * r, q0, bh, q_full);
      }
      int s = 0;
      uint32_t ph = 0;
      uint32_t last_ph[STAGES > VSTAGES ? STAGES : VSTAGES];
      bool pending[STAGES > VSTAGES ? STAGES : VSTAGES];
#pragma unroll
      for (int i = 0; i < (STAGES > VSTAGES ? STAGES : VSTAGES); ++i) pending[i] = false;
      for (int j = 0; j < n_kv; ++j) {
        const uint32_t empty = is_k ? k_empty(s) : v_empty(s);
        const uint32_t full = is_k ? k_full(s) : v_full(s);
        if (!mbar_wait(empty, ph ^ 1u)) {
          timed_out = true;
          break;
        }
        const uint32_t dst = base + (is_k ? CF::K_OFFSET + s * CF::K_BYTES : CF::V_OFFSET + s * CF::V_BYTES);
        mbar_arrive_expect_tx(full, CF::K_BYTES);
#pragma unroll
        for (int r = 0; r < CF::REGIONS; ++r)
          tma_load_3d(dst + r * CF::SLAB, is_k ? &tm_k : &tm_v, 64 * r, j * BN, bh, full);
        last_ph[s] = ph;
        pending[s] = true;
        if (++s == nst) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (timed_out) {
        if (is_k) (void)mbar_wait(q_full, 0);
        for (int i = 0; i < nst; ++i)
          if (pending[i]) (void)mbar_wait(is_k ? k_full(i) : v_full(i), last_ph[i]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f32acc(kFmtBF16, BM, BN, 0, 0);
      constexpr uint32_t idesc_o = idesc_f32acc(kFmtBF16, BM, D, 0, 1);
      const uint32_t q_src = base + CF::Q_OFFSET;
      auto issue_s = [&](int j, int stage) {
        const uint32_t k_src = base + CF::K_OFFSET + stage * CF::K_BYTES;
        const uint32_t d_tmem = tmem + CF::COL_S + (uint32_t)((j & 1) * BN);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * CF::SLAB + (kk & 3) * 32);
          mma_f16_ss(d_tmem, desc_sw128(q_src + off, 16u, 1024u), desc_sw128(k_src + off, 16u, 1024u), idesc_s,
                     kk > 0 ? 1u : 0u);
        }
        mma_commit(s_full(j & 1));
        mma_commit(k_empty(stage));  // the K slot is free once S_j has read it
      };
      auto issue_pv = [&](int j, int stage) {
        const uint32_t v_src = base + CF::V_OFFSET + stage * CF::V_BYTES;
        const uint32_t p_tmem = tmem + CF::COL_P + (uint32_t)((j & 1) * 64);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // 16 keys per MMA: rows 16kk..16kk+15 of every 64-column V slab; slabs CF::SLAB apart
          const uint64_t vd = desc_sw128(v_src + (uint32_t)(kk * 16 * 128), (uint32_t)CF::SLAB, 1024u);
          mma_f16_ts(tmem + CF::COL_O, p_tmem + (uint32_t)(kk * 8), vd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(o_done);
        mma_commit(v_empty(stage));
      };
      // P·V of tile j: needs P_j from the softmax and V_j from its ring
      auto pv_step = [&](int j) -> bool {
        if (!mbar_wait(p_full(j & 1), (uint32_t)(j >> 1) & 1u)) return false;
        if (!mbar_wait(v_full(j % VSTAGES), (uint32_t)(j / VSTAGES) & 1u)) return false;
        tc_fence_after();
        issue_pv(j, j % VSTAGES);
        return true;
      };
      if (!mbar_wait(q_full, 0)) timed_out = true;
      tc_fence_after();
      for (int j = 0; j < n_kv && !timed_out; ++j) {
        if (!mbar_wait(k_full(j % STAGES), (uint32_t)(j / STAGES) & 1u)) {
          timed_out = true;
          break;
        }
        // S buffer j&1 was last read by the softmax of tile j-2
        if (!mbar_wait(s_free(j & 1), ((uint32_t)(j >> 1) & 1u) ^ 1u)) {
          timed_out = true;
          break;
        }
        tc_fence_after();
        issue_s(j, j % STAGES);
        if (j > 0 && !pv_step(j - 1)) {
          timed_out = true;
          break;
        }
      }
      if (!timed_out && n_kv > 0) {
        if (pv_step(n_kv - 1)) mma_commit(o_final);
        else timed_out = true;
      }
      mma_commit(done_bar);
    }
  } else {
    // softmax: TMEM lane quarter = warp % 4, the two warps of a quarter split the columns
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int qrow = q0 + row;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t pair_mbar = pair_bar0 + 8u * (uint32_t)quarter;  // mbarrier of the two warps of this quarter
    uint32_t pair_uses = 0;                                        // completed exchanges (phase count)
    constexpr int HC = BN / 2;                         // score columns per thread
    constexpr int HD = D / 2;                          // O columns per thread
    float m_run = -INFINITY;  // running max of s·scale·log2e used by the exponentials (same in both halves)
    float l_part = 0.f;       // this half's share of the row sum
    for (int j = 0; j < n_kv; ++j) {
      const int b = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(s_full(b), (uint32_t)(j >> 1) & 1u))) {
        timed_out = true;
        break;
      }
      tc_fence_after();
      const uint32_t s_addr = tmem + lane_off + CF::COL_S + (uint32_t)(b * BN + half * HC);
      const int key0 = j * BN + half * HC;
      const bool mask_tile = (CAUSAL && j * BN + BN - 1 > q0) || (j * BN + BN > S);
      uint32_t sv[HC];
#pragma unroll
      for (int c = 0; c < HC; c += 32) tmem_ld32(s_addr + (uint32_t)c, *reinterpret_cast<uint32_t(*)[32]>(&sv[c]));
      tmem_ld_wait();
      if (mask_tile) {
#pragma unroll
        for (int t = 0; t < HC; ++t) {
          const int key = key0 + t;
          if (!(key < S && (!CAUSAL || key <= qrow))) sv[t] = __float_as_uint(-INFINITY);
        }
      }
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int t = 0; t < HC; ++t) m4[t & 3] = fmaxf(m4[t & 3], __uint_as_float(sv[t]));
      // exchange the half-row maxima (parity-double-buffered: the partner may
      // still read the previous tile's slot while this thread writes the next)
      float* red_max = red + (b * 2) * 128;
      red_max[half * 128 + row] = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      mbar_arrive(pair_mbar);  // release: the write above is visible to the partner after its wait
      if (!__all_sync(0xffffffffu, mbar_wait(pair_mbar, pair_uses & 1u))) {
        timed_out = true;
        break;
      }
      ++pair_uses;
      const float mx = fmaxf(red_max[row], red_max[128 + row]);
      const float m_tile = mx * scale_log2;
      const bool raise = m_tile > m_run + kRescaleThreshold;
      float alpha = 1.f;
      if (raise) {
        alpha = (m_run == -INFINITY) ? 0.f : ex2(m_run - m_tile);
        m_run = m_tile;
        l_part *= alpha;
      }
      // O holds P_0..P_{j-1}·V: rescale this half of it once the previous PV
      // product has landed. o_done is at phase j-1 or j here (s_full[j] was
      // committed after PV_{j-2} was issued, and PV_j needs this thread's P_j),
      // so a parity wait is exact.
      if (j > 0 && __any_sync(0xffffffffu, raise)) {
        if (!__all_sync(0xffffffffu, mbar_wait(o_done, (uint32_t)(j - 1) & 1u))) {
          timed_out = true;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          uint32_t v[32];
          const uint32_t oa = tmem + lane_off + CF::COL_O + (uint32_t)(half * HD + c);
          tmem_ld32(oa, v);
          tmem_ld_wait();
          uint32_t w0[16], w1[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            w0[t] = __float_as_uint(__uint_as_float(v[t]) * alpha);
            w1[t] = __float_as_uint(__uint_as_float(v[16 + t]) * alpha);
          }
          tmem_st16(oa, w0);
          tmem_st16(oa + 16u, w1);
        }
        tmem_st_wait();
      }
      // p = 2^(s·c − m) (masked entries are −inf -> 0), partial sum, bf16 P into TMEM
      const uint32_t p_addr = tmem + lane_off + CF::COL_P + (uint32_t)(b * 64 + half * (HC / 2));
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < HC; c += 32) {
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float x0 = fmaf(__uint_as_float(sv[c + 2 * t]), scale_log2, -m_run);
          const float x1 = fmaf(__uint_as_float(sv[c + 2 * t + 1]), scale_log2, -m_run);
          float p0, p1;
          if (KT_FA_POLY && !mask_tile && (t & 3) == 3) {
            p0 = ex2_poly(x0);
            p1 = ex2_poly(x1);
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          s4[t & 3] += p0 + p1;
          pk[t] = pack_bf16(p0, p1);
        }
        tmem_st16(p_addr + (uint32_t)(c / 2), pk);
      }
      l_part += (s4[0] + s4[1]) + (s4[2] + s4[3]);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(s_free(b));
      mbar_arrive(p_full(b));
    }
    // epilogue: O / l -> bf16 (each half writes its D/2 columns)
    if (!timed_out && n_kv > 0) {
      float* red_l = red + 4 * 128;  // own slot: no reader of the max slots can be overwritten
      red_l[half * 128 + row] = l_part;
      mbar_arrive(pair_mbar);
      const bool pair_ok = __all_sync(0xffffffffu, mbar_wait(pair_mbar, pair_uses & 1u));
      const float l_run = red_l[row] + red_l[128 + row];
      if (!pair_ok || !__all_sync(0xffffffffu, mbar_wait(o_final, 0))) {
        timed_out = true;
      } else {
        tc_fence_after();
        const float inv = 1.0f / l_run;
        __nv_bfloat16* orow = O + ((int64_t)bh * S + qrow) * D + half * HD;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + CF::COL_O + (uint32_t)(half * HD + c), v);
          tmem_ld_wait();
          if (qrow < S) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              uint4 w;
              w.x = pack_bf16(__uint_as_float(v[8 * t + 0]) * inv, __uint_as_float(v[8 * t + 1]) * inv);
              w.y = pack_bf16(__uint_as_float(v[8 * t + 2]) * inv, __uint_as_float(v[8 * t + 3]) * inv);
              w.z = pack_bf16(__uint_as_float(v[8 * t + 4]) * inv, __uint_as_float(v[8 * t + 5]) * inv);
              w.w = pack_bf16(__uint_as_float(v[8 * t + 6]) * inv, __uint_as_float(v[8 * t + 7]) * inv);
              dst[t] = w;
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

// [B·H, S, D] bf16 viewed as a 3-D tensor (D, S, B·H); box 64 × 128 × 1, 128-byte swizzle.
inline int make_tmap_bhsd(CUtensorMap* map, const void* base, int64_t BH, int64_t S, int64_t D) {
  PFN_encodeTiled enc = get_encode_tiled();
  if (enc == nullptr) return fail(KT_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)S * D * 2};
  cuuint32_t box[3] = {64, 128, 1};
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
  using CF = Cfg<D, KT_FA_STAGES, KT_FA_VSTAGES>;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_bhsd(&tq, Q, BH, S, D);
  if (rc == KT_OK) rc = make_tmap_bhsd(&tk, K, BH, S, D);
  if (rc == KT_OK) rc = make_tmap_bhsd(&tv, V, BH, S, D);
  if (rc != KT_OK) return rc;
  auto kern = fa_fwd_kernel<D, KT_FA_STAGES, CAUSAL>;
  static bool attr_set = false;
  if (!attr_set) {
    rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::SMEM_BYTES),
                     "attention: smem attribute");
    if (rc != KT_OK) return rc;
    attr_set = true;
  }
  const float scale_log2 = scale * 1.4426950408889634f;  // log2(e)
  const int64_t blocks = BH * ((S + BM - 1) / BM);
  dim3 grid((unsigned)blocks);
  kern<<<grid, THREADS, CF::SMEM_BYTES, st>>>(tq, tk, tv, reinterpret_cast<__nv_bfloat16*>(O), (int)S, scale_log2);
  return check_launch("attention fwd");
}

inline int launch(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int64_t B, int64_t H,
                  int64_t S, int64_t D, float scale, int causal, cudaStream_t st) {
  if (B < 0 || H < 0 || S < 0 || D < 0) return fail(KT_ERR_ARG, "attention: negative shape");
  if (B == 0 || H == 0 || S == 0) return KT_OK;
  if (!Q || !K || !V || !O) return fail(KT_ERR_ARG, "attention: null pointer");
  if (D != 64 && D != 128) return fail(KT_ERR_UNSUPPORTED, "attention: head dim %lld (64 or 128 supported)", (long long)D);
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O))
    return fail(KT_ERR_ARG, "attention: tensors must be 16-byte aligned");
  if (S > (int64_t)INT32_MAX / 2 || B * H * ((S + BM - 1) / BM) > (int64_t)INT32_MAX)
    return fail(KT_ERR_UNSUPPORTED, "attention: S or B*H too large");
  if (!(scale > 0.f) || !isfinite(scale)) return fail(KT_ERR_ARG, "attention: scale must be finite and > 0");
  const int64_t BH = B * H;
  if (D == 128) {
    return causal ? launch_t<128, true>(Q, K, V, O, BH, S, scale, st) : launch_t<128, false>(Q, K, V, O, BH, S, scale, st);
  }
  return causal ? launch_t<64, true>(Q, K, V, O, BH, S, scale, st) : launch_t<64, false>(Q, K, V, O, BH, S, scale, st);
}

}  // namespace fa
}  // namespace kt
