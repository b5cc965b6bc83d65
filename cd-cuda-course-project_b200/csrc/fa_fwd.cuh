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
//              2^(s·scale·log2e − m) for the own half (MUFU ex2; optionally every
//              4th pair by a polynomial on the FMA pipe), bf16 P back
//              to TMEM, partial row sum. The running max is only raised (O and
//              the sums rescaled) when it grows by more than 2^8, so O is rarely
//              touched. Final O / l in bf16.
// TMEM columns: S0 [0,128) S1 [128,256) O [256,256+D) P0 [384,448) P1 [448,512).
// Every mbarrier wait is bounded; a timeout records DEV_MBAR_TIMEOUT and the
// CTA unwinds (loader drains its copies, MMAs drain before TMEM is released).
#pragma once
#include <type_traits>
#include "kt_common.cuh"
#include "sm100.cuh"
#include "fa_fwd2.cuh"

#ifndef KT_FA_STAGES
#define KT_FA_STAGES 2  // K ring depth (the V ring has KT_FA_VSTAGES slots)
#endif
#ifndef KT_FA_VSTAGES
#define KT_FA_VSTAGES 2
#endif
#ifndef KT_FA_KIND
#define KT_FA_KIND 1  // 1: one query tile per CTA (this file); 2: two ping-pong query tiles per CTA (fa_fwd2.cuh)
#endif
#ifndef KT_FA_EXP16
#define KT_FA_EXP16 0  // 1: exponentials as packed half-precision pairs (ex2.approx.f16x2: two results per MUFU op)
#endif
#ifndef KT_FA_ISSUERS
#define KT_FA_ISSUERS 2  // 2: S = Q·K^T and O += P·V issued by two warps (one thread issues tcgen05.mma at ~73 clocks
                         // per instruction, above the 64-clock 128x128x16 MMA); 1: one issuing thread
#endif
#ifndef KT_FA_ALT
#define KT_FA_ALT 1  // 1: the two softmax warps of a TMEM lane quarter take alternate S tiles, whole 128-key
                     // rows (their latency phases overlap the other warp's exponentials); 0: column halves
#endif
#ifndef KT_FA_BN
#define KT_FA_BN 128  // keys per S tile: 128, or 96 (alternate-tile softmax; four S buffers fit TMEM)
#endif
#ifndef KT_FA_SBUF
// S accumulators in TMEM: 2 (P in its own columns), 3 or 4 (P written over its S tile; needs
// scores that are not reloaded after P is written)
#define KT_FA_SBUF (KT_FA_RELOAD ? 2 : (KT_FA_BN == 96 ? 4 : (KT_FA_ISSUERS == 2 ? 3 : 2)))
#endif
#ifndef KT_FA_X2
#define KT_FA_X2 1  // 1: the exponent arguments and row sums in packed fma.rn.f32x2 / add.rn.f32x2
#endif
#ifndef KT_FA_WARP_ARRIVE
#define KT_FA_WARP_ARRIVE 0  // 1: one arrival per warp (after __syncwarp) on the softmax / epilogue mbarriers
#endif
#ifndef KT_FA_PSPLIT
// alternate tiles: P_t·V issued in this many key ranges (1, 2 or 4), each once its P columns are stored
#define KT_FA_PSPLIT ((KT_FA_ALT && KT_FA_BN == 128) ? 2 : 1)
#endif
#ifndef KT_FA_FUSE
#define KT_FA_FUSE 0  // 1: alternate tiles, one speculative pass over the scores per tile (max checked per chunk)
#endif
#ifndef KT_FA_SPEC0
#define KT_FA_SPEC0 0  // 1: an item's first tile also speculates, on the previous item's final running max
#endif
#ifndef KT_FA_DEPHASE
#define KT_FA_DEPHASE 0  // clocks the second softmax warp of each lane quarter starts its first tile late
                         // (exponential phases of the two warps of a scheduler offset, not coinciding)
#endif
#ifndef KT_FA_SPEC
#define KT_FA_SPEC 1  // 1: exponentials start with the running max before the partner's half max is read
#endif
#ifndef KT_FA_RELOAD
#define KT_FA_RELOAD 0  // 1: the exponential pass reloads the scores from TMEM 32 columns at a time
#endif
#ifndef KT_FA_POLY
#define KT_FA_POLY 1  // n = 1..3: n of every 4 value pairs of exponentials on the FMA pipe (polynomial)
#endif

namespace kt {
namespace fa {

constexpr int BM = 128;
constexpr int BN = KT_FA_BN;  // keys per tile (the S accumulator is BN fp32 columns)
static_assert(BN == 128 || (BN == 96 && KT_FA_ALT), "96-key tiles: alternate-tile softmax only");
constexpr int SOFTMAX_WARPS = 8;
constexpr int V_LOADER_WARP = 2 + SOFTMAX_WARPS;
constexpr int EPI_THREADS = 128;  // warps 11-14: one query row per thread
constexpr int PV_WARP = V_LOADER_WARP + 1 + EPI_THREADS / 32;  // warp 15 (two issuers): issues O += P·V
constexpr int THREADS = 96 + 32 * SOFTMAX_WARPS + EPI_THREADS + (KT_FA_ISSUERS == 2 ? 32 : 0);
constexpr int SOFTMAX_THREADS = 32 * SOFTMAX_WARPS;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: O is rescaled only when the max grows by > 2^8
constexpr float kGuessSlack = 64.0f;       // log2 units: a first-tile guess may exceed the row max by this much
constexpr int kHeadGroup = 8;              // causal scheduling: heads whose K/V share L2

template <int D, int STAGES, int VSTAGES = KT_FA_VSTAGES>
struct Cfg {
  static_assert(D == 64 || D == 128, "head dim");
  static constexpr int REGIONS = D / 64;            // 128-byte (64 bf16) column slabs per row
  static constexpr int SLAB = 128 * 128;            // one slab of 128 rows × 128 bytes
  static constexpr int Q_BYTES = REGIONS * SLAB;    // 128 rows × D bf16
  static constexpr int K_BYTES = REGIONS * SLAB;    // slot of up to 128 keys × D (slabs SLAB apart)
  static constexpr int KV_TX = REGIONS * BN * 128;  // bytes one K or V tile of BN keys delivers
  static constexpr int V_BYTES = REGIONS * SLAB;
  static constexpr int Q_OFFSET = 0;                // two Q buffers: the next item's tile loads early
  static constexpr int K_OFFSET = 2 * Q_BYTES;
  static constexpr int V_OFFSET = K_OFFSET + STAGES * K_BYTES;
  // column halves: [2 tile parity][2 half][128 rows] softmax maxima + [2 item parity][2 half][128 rows] row sums;
  // alternate tiles: [2 item parity][128] running max, [2 item parity][2 parity][128] row-sum shares and
  // [2 item parity][2 parity][128] the maxima they are relative to
  static constexpr int RED_OFFSET = V_OFFSET + VSTAGES * V_BYTES;
  static constexpr int BAR_OFFSET = RED_OFFSET + 10 * 128 * 4;
  // q_full[2], q_empty[2], k_full[S], k_empty[S], v_full[VS], v_empty[VS], s_full[4], s_free[4],
  // p_full[4], l_full[2], l_empty[2], o_done[4], o_final, o_empty, done, pair[4], decision[4][2],
  // p_part[4][3]
  static constexpr int NUM_BARS = 4 + 2 * STAGES + 2 * VSTAGES + 35 + 12;
  static constexpr int SMEM_BYTES = BAR_OFFSET + NUM_BARS * 8 + 16 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static constexpr uint32_t TMEM_COLS = 512;
  // S buffers from column 0 (BN columns each), then O; with two S buffers P has its own
  // 2 x 64 columns, with three or four each P_t (bf16 pairs) is written over its S tile
  static constexpr int NB = KT_FA_SBUF;
  static_assert(NB == 2 || NB == 3 || NB == 4, "S buffers");
  static_assert(NB * BN + D <= 512 && (NB > 2 || BN == 128), "TMEM columns");
  static constexpr uint32_t COL_S = 0, COL_O = NB * BN, COL_P = 384;
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

// 2^x0, 2^x1 from one packed half-precision MUFU operation. The arguments are
// rounded to fp16 first (for |x| < 16 the rounding moves 2^x by at most 0.3 %,
// below the 0.4 % of the bf16 rounding that P gets anyway; values below 2^-24
// flush to 0, negligible against a row sum >= 1) and the results come back as
// fp32 for the row sum.
__device__ __forceinline__ void ex2_h2(float x0, float x1, float& p0, float& p1) {
  uint32_t h, e;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(x1), "f"(x0));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(e) : "r"(h));
  asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tcvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
      : "=f"(p0), "=f"(p1)
      : "r"(e));
}

// Pack two fp32 values into bf16x2 (round to nearest even); `lo` in the low half.
// (d0, d1) = (a0, a1) * (b, b) + (c, c) as one packed fp32 instruction
__device__ __forceinline__ void fma2_bc(float& d0, float& d1, float a0, float a1, float b, float c) {
  uint64_t d, a, bb, cc;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(bb) : "f"(b));
  asm("mov.b64 %0, {%1, %1};" : "=l"(cc) : "f"(c));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(bb), "l"(cc));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}
// (d0, d1) += (a0, a1) as one packed fp32 instruction
__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1) {
  uint64_t d, a;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(d0), "f"(d1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("add.rn.f32x2 %0, %0, %1;" : "+l"(d) : "l"(a));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}
// 2^x0, 2^x1 as ex2_poly with the floating-point steps on packed fp32 pairs (five
// instructions per pair instead of ten) and the exponent insertion as one shift-add
// per value: (bits(y) - bits(1.5·2^23)) << 23 equals bits(y) << 23 modulo 2^32.
__device__ __forceinline__ void ex2_poly_x2(float x0, float x1, float& p0, float& p1) {
  x0 = fmaxf(x0, -125.f);
  x1 = fmaxf(x1, -125.f);
  uint64_t x, y, n, f, p, c, nc, a3, a2, a1, a0;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(x0), "f"(x1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(c) : "f"(12582912.0f));
  asm("mov.b64 %0, {%1, %1};" : "=l"(nc) : "f"(-12582912.0f));
  asm("mov.b64 %0, {%1, %1};" : "=l"(a3) : "f"(0.055029310286045074f));
  asm("mov.b64 %0, {%1, %1};" : "=l"(a2) : "f"(0.2422567903995514f));
  asm("mov.b64 %0, {%1, %1};" : "=l"(a1) : "f"(0.6932530403137207f));
  asm("mov.b64 %0, {%1, %1};" : "=l"(a0) : "f"(0.9999513626098633f));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(y) : "l"(x), "l"(c));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(n) : "l"(y), "l"(nc));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(f) : "l"(x), "l"(n));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(p) : "l"(a3), "l"(f), "l"(a2));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(p) : "l"(p), "l"(f), "l"(a1));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(p) : "l"(p), "l"(f), "l"(a0));
  uint32_t pl, ph, yl, yh;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(pl), "=r"(ph) : "l"(p));
  asm("mov.b64 {%0, %1}, %2;" : "=r"(yl), "=r"(yh) : "l"(y));
  p0 = __uint_as_float(pl + (yl << 23));
  p1 = __uint_as_float(ph + (yh << 23));
}

// max of three fp32 values in one instruction
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Work item w (one 128-row query tile of one (b, h)) -> (qt, bh). Items are
// taken in index order by the persistent CTAs (item = CTA, CTA + grid, ...),
// so the items in flight together are adjacent. Non-causal: the query tiles
// of one head are adjacent (its K/V stays in L2). Causal: heads in groups of
// kHeadGroup, inside a group the heaviest (latest) query tiles first.
template <bool CAUSAL>
__device__ __forceinline__ void item_coords(int w, int num_q_tiles, int BH, int& qt, int& bh) {
  if (CAUSAL) {
    const int per_group = kHeadGroup * num_q_tiles;
    const int group = w / per_group;
    const int r = w - group * per_group;
    const int gsize = min(kHeadGroup, BH - group * kHeadGroup);
    qt = num_q_tiles - 1 - r / gsize;
    bh = group * kHeadGroup + r % gsize;
  } else {
    qt = w % num_q_tiles;
    bh = w / num_q_tiles;
  }
}

template <bool CAUSAL>
__device__ __forceinline__ int kv_tiles(int qt, int S) {
  const int all = (S + BN - 1) / BN;
  return CAUSAL ? min(all, (qt * BM + BM - 1) / BN + 1) : all;
}

template <int D, int STAGES, bool CAUSAL>
__global__ void __launch_bounds__(THREADS, 1)
fa_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, __nv_bfloat16* __restrict__ O, int S, int BH,
              float scale_log2) {
  using CF = Cfg<D, STAGES>;
  using namespace sm100;
  constexpr int VSTAGES = KT_FA_VSTAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  float* red = reinterpret_cast<float*>(base_ptr + CF::RED_OFFSET);
  const uint32_t bar0 = base + CF::BAR_OFFSET;
  // barrier map (8 bytes each)
  auto q_full = [&](int s) { return bar0 + 8u * s; };
  auto q_empty = [&](int s) { return bar0 + 8u * (2 + s); };
  auto k_full = [&](int s) { return bar0 + 8u * (4 + s); };
  auto k_empty = [&](int s) { return bar0 + 8u * (4 + STAGES + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (4 + 2 * STAGES + s); };
  auto v_empty = [&](int s) { return bar0 + 8u * (4 + 2 * STAGES + VSTAGES + s); };
  constexpr int R = 4 + 2 * STAGES + 2 * VSTAGES;
  constexpr int NB = CF::NB;
  static_assert(NB == 2 || !KT_FA_RELOAD, "P over S: scores not reloaded after P is written");
  // per-buffer P·V completion barriers (o_done_of): two issuers, or P over S
  constexpr bool PER_BUF = KT_FA_ISSUERS == 2 || NB > 2;
  // tile t uses S buffer sbuf(t); sph(t) is the phase parity of that buffer's barriers for tile t
  auto sbuf = [](int t) { return NB == 3 ? t % 3 : (t & (NB - 1)); };
  auto sph = [](int t) { return (uint32_t)((NB == 3 ? t / 3 : (t >> (NB == 4 ? 2 : 1))) & 1); };
  auto s_full = [&](int b) { return bar0 + 8u * (R + b); };
  auto s_free = [&](int b) { return bar0 + 8u * (R + 4 + b); };
  auto p_full = [&](int b) { return bar0 + 8u * (R + 8 + b); };
  auto l_full = [&](int b) { return bar0 + 8u * (R + 12 + b); };
  auto l_empty = [&](int b) { return bar0 + 8u * (R + 14 + b); };
  const uint32_t o_done = bar0 + 8u * (R + 16);  // one issuer: one phase per P·V product
  // two issuers: o_done_of(t) completes once per P_t·V of the tiles using S buffer sbuf(t)
  auto o_done_of = [&](int t) { return bar0 + 8u * (R + 16 + sbuf(t)); };
  const uint32_t o_final = bar0 + 8u * (R + 20);  // one phase per item: its last P·V product landed
  const uint32_t o_empty = bar0 + 8u * (R + 21);  // one phase per item: the epilogue has read O
  const uint32_t done_bar = bar0 + 8u * (R + 22);
  const uint32_t pair_bar0 = bar0 + 8u * (R + 23);  // 4 softmax warp-pair exchanges
  // alternate tiles: the running-max decision of tile parity p for lane quarter q
  auto dec_bar = [&](int q, int p) { return bar0 + 8u * (R + 27 + 2 * q + p); };
  // alternate tiles, P·V in KT_FA_PSPLIT key ranges: range i < KT_FA_PSPLIT-1 of buffer b is
  // stored (the last range is signalled by p_full)
  constexpr int PSPLIT = KT_FA_PSPLIT;
  static_assert(PSPLIT == 1 || (KT_FA_ALT && PSPLIT <= 4 && (BN / 32) % PSPLIT == 0),
                "P·V split: ranges of whole 32-key chunks, alternate tiles");
  auto p_part = [&](int b, int i) { return bar0 + 8u * (R + 35 + 3 * b + i); };
  const uint32_t tmem_slot = bar0 + 8u * CF::NUM_BARS;
  const volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<const volatile uint32_t*>(base_ptr + CF::BAR_OFFSET + 8 * CF::NUM_BARS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_q_tiles = (S + BM - 1) / BM;
  const int num_items = BH * num_q_tiles;

  // arrivals per warp on the barriers the softmax and epilogue warps signal: every
  // thread, or lane 0 after the warp has synchronised (its writes are ordered
  // before lane 0's release by __syncwarp)
  constexpr int AW = KT_FA_WARP_ARRIVE ? 1 : 32;
  auto warp_arrive = [&](uint32_t bar) {
    if (KT_FA_WARP_ARRIVE) {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar);
    } else {
      mbar_arrive(bar);
    }
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(q_full(s), 1);
      mbar_init(q_empty(s), 1);
      mbar_init(l_full(s), SOFTMAX_WARPS * AW);
      mbar_init(l_empty(s), EPI_THREADS / 32 * AW);
    }
    for (int s = 0; s < NB; ++s) {
      mbar_init(s_full(s), 1);
      // alternate tiles: only the four warps of the tile's parity use its S / P buffer
      mbar_init(s_free(s), (KT_FA_ALT ? SOFTMAX_WARPS / 2 : SOFTMAX_WARPS) * AW);
      mbar_init(p_full(s), (KT_FA_ALT ? SOFTMAX_WARPS / 2 : SOFTMAX_WARPS) * AW);
      mbar_init(o_done_of(s), 1);
      for (int i = 0; i + 1 < PSPLIT; ++i) mbar_init(p_part(s, i), SOFTMAX_WARPS / 2 * AW);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < VSTAGES; ++s) {
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    mbar_init(o_final, 1);
    mbar_init(o_empty, EPI_THREADS / 32 * AW);
    mbar_init(done_bar, KT_FA_ISSUERS);
    for (int q = 0; q < 4; ++q) mbar_init(pair_bar0 + 8u * q, 2 * AW);
    for (int q = 0; q < 4; ++q) {
      mbar_init(dec_bar(q, 0), AW);
      mbar_init(dec_bar(q, 1), AW);
    }
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
      // warp 0: Q of every item (2 buffers) and the K tiles; V_LOADER_WARP: the V tiles.
      // Ring positions run on across items.
      const bool is_k = (warp == 0);
      constexpr int MAXS = STAGES > VSTAGES ? STAGES : VSTAGES;
      const int nst = is_k ? STAGES : VSTAGES;
      uint32_t last_ph[MAXS];
      bool pending[MAXS];
      bool q_pending[2] = {false, false};
      uint32_t q_last_ph[2] = {0u, 0u};
#pragma unroll
      for (int i = 0; i < MAXS; ++i) pending[i] = false;
      int s = 0;
      uint32_t ph = 0;
      int k = 0;
      for (int w = blockIdx.x; w < num_items && !timed_out; w += gridDim.x, ++k) {
        int qt, bh;
        item_coords<CAUSAL>(w, num_q_tiles, BH, qt, bh);
        const int n_kv = kv_tiles<CAUSAL>(qt, S);
        if (is_k) {
          const int qb = k & 1;
          const uint32_t qph = (uint32_t)(k >> 1) & 1u;
          if (!mbar_wait(q_empty(qb), qph ^ 1u)) {
            timed_out = true;
            break;
          }
          mbar_arrive_expect_tx(q_full(qb), CF::Q_BYTES);
#pragma unroll
          for (int r = 0; r < CF::REGIONS; ++r)
            tma_load_3d(base + CF::Q_OFFSET + qb * CF::Q_BYTES + r * CF::SLAB, &tm_q, 64 * r, qt * BM, bh, q_full(qb));
          q_pending[qb] = true;
          q_last_ph[qb] = qph;
        }
        for (int j = 0; j < n_kv; ++j) {
          const uint32_t empty = is_k ? k_empty(s) : v_empty(s);
          const uint32_t full = is_k ? k_full(s) : v_full(s);
          if (!mbar_wait(empty, ph ^ 1u)) {
            timed_out = true;
            break;
          }
          const uint32_t dst = base + (is_k ? CF::K_OFFSET + s * CF::K_BYTES : CF::V_OFFSET + s * CF::V_BYTES);
          mbar_arrive_expect_tx(full, CF::KV_TX);
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
      }
      if (timed_out) {
        // let every copy still in flight land before the CTA exits
        for (int i = 0; i < 2; ++i)
          if (q_pending[i]) (void)mbar_wait(q_full(i), q_last_ph[i]);
        for (int i = 0; i < nst; ++i)
          if (pending[i]) (void)mbar_wait(is_k ? k_full(i) : v_full(i), last_ph[i]);
      }
    }
  } else if (warp == 1 || (KT_FA_ISSUERS == 2 && warp == PV_WARP)) {
    if (lane == 0) {
      const bool s_issuer = (warp == 1), pv_issuer = (KT_FA_ISSUERS == 1 || warp == PV_WARP);
      constexpr uint32_t idesc_s = idesc_f32acc(kFmtBF16, BM, BN, 0, 0);
      constexpr uint32_t idesc_o = idesc_f32acc(kFmtBF16, BM, D, 0, 1);
      int kc = 0, vc = 0;  // K / V ring positions
      // descriptors as (lo, hi) words: lo + byte offset / 16 addresses base + offset
      const uint64_t dk = desc_sw128(base, 16u, 1024u);                  // K-major operands (Q, K)
      const uint64_t dv = desc_sw128(base, (uint32_t)CF::SLAB, 1024u);   // V, MN-major
      const uint32_t k_hi = (uint32_t)(dk >> 32), v_hi = (uint32_t)(dv >> 32);
      const uint32_t q_lo0 = (uint32_t)dk + (CF::Q_OFFSET >> 4);
      const uint32_t k_lo0 = (uint32_t)dk + (CF::K_OFFSET >> 4);
      const uint32_t v_lo0 = (uint32_t)dv + (CF::V_OFFSET >> 4);
      // S_t = Q·K^T into S buffer t&1 from K slot kc
      auto issue_s = [&](int t, int qb) {
        const uint32_t q_lo = q_lo0 + (uint32_t)qb * (CF::Q_BYTES >> 4);
        const uint32_t k_lo = k_lo0 + (uint32_t)(kc % STAGES) * (CF::K_BYTES >> 4);
        const uint32_t d_tmem = tmem + CF::COL_S + (uint32_t)(sbuf(t) * BN);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(((kk >> 2) * CF::SLAB + (kk & 3) * 32) >> 4);
          mma_f16_ss_w(d_tmem, q_lo + off, k_hi, k_lo + off, k_hi, idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(s_full(sbuf(t)));
        mma_commit(k_empty(kc % STAGES));  // the K slot is free once S_t has read it
        ++kc;
      };
      // O += P_t·V (O = P_t·V for the first tile of an item); needs P_t and the V tile
      auto pv_step = [&](int t, int k, bool first, bool last) -> bool {
        if (!mbar_wait(PSPLIT > 1 ? p_part(sbuf(t), 0) : p_full(sbuf(t)), sph(t))) return false;
        if (!mbar_wait(v_full(vc % VSTAGES), (uint32_t)(vc / VSTAGES) & 1u)) return false;
        // the epilogue must have read the previous item's O before it is overwritten
        if (first && !mbar_wait(o_empty, ((uint32_t)k & 1u) ^ 1u)) return false;
        tc_fence_after();
        const uint32_t v_lo = v_lo0 + (uint32_t)(vc % VSTAGES) * (CF::V_BYTES >> 4);
        // P_t: 64 columns of its own (two S buffers) or over the S tile, keys 64h.. at column 64h
        const uint32_t p_tmem = NB == 2 ? tmem + CF::COL_P + (uint32_t)((t & 1) * 64)
                                        : tmem + CF::COL_S + (uint32_t)(sbuf(t) * BN);
        const uint32_t o_tmem = tmem + CF::COL_O;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // key range r = kk / (8 / PSPLIT) starts once its P columns are stored
          constexpr int PER = BN / 16 / PSPLIT;
          if (PSPLIT > 1 && kk > 0 && kk % PER == 0) {
            const int r = kk / PER;
            if (!mbar_wait(r + 1 < PSPLIT ? p_part(sbuf(t), r) : p_full(sbuf(t)), sph(t))) return false;
            tc_fence_after();
          }
          // 16 keys per MMA: rows 16kk..16kk+15 of every 64-column V slab; slabs CF::SLAB apart
          // P over S from column halves: keys 64h.. at column 64h; otherwise keys in order
          const uint32_t p_col =
              (NB == 2 || KT_FA_ALT) ? (uint32_t)(kk * 8) : (uint32_t)((kk >> 2) * 64 + (kk & 3) * 8);
          mma_f16_ts_w(o_tmem, p_tmem + p_col, v_lo + (uint32_t)(kk * 16 * 128 / 16), v_hi, idesc_o,
                       (!first || kk > 0) ? 1u : 0u);
        }
        mma_commit(PER_BUF ? o_done_of(t) : o_done);
        mma_commit(v_empty(vc % VSTAGES));
        if (last) mma_commit(o_final);
        ++vc;
        return true;
      };
      // Two issuers: warp 1 issues S_t as soon as its K tile and S buffer are free
      // and P_{t-NB}·V, the last reader of the P columns tile t reuses, is
      // complete (then the softmax's parity waits on o_done_of are exact: at tile
      // t at most P_{t-1}·V is outstanding); warp PV_WARP issues P_t·V as soon as
      // P_t is in TMEM. One issuer: the order below.
      if (KT_FA_ISSUERS == 2) {
        int t = 0, k = 0;
        for (int w = blockIdx.x; w < num_items && !timed_out; w += gridDim.x, ++k) {
          int qt, bh;
          item_coords<CAUSAL>(w, num_q_tiles, BH, qt, bh);
          const int n_kv = kv_tiles<CAUSAL>(qt, S);
          if (s_issuer && !mbar_wait(q_full(k & 1), (uint32_t)(k >> 1) & 1u)) {
            timed_out = true;
            break;
          }
          for (int j = 0; j < n_kv; ++j, ++t) {
            if (s_issuer) {
              if (!mbar_wait(k_full(kc % STAGES), (uint32_t)(kc / STAGES) & 1u) ||
                  !mbar_wait(s_free(sbuf(t)), sph(t) ^ 1u) ||
                  (t >= NB && !mbar_wait(o_done_of(t - NB), sph(t - NB)))) {
                timed_out = true;
                break;
              }
              tc_fence_after();
              issue_s(t, k & 1);
              if (j == n_kv - 1) mma_commit(q_empty(k & 1));
            }
            if (pv_issuer && !s_issuer && !pv_step(t, k, j == 0, j == n_kv - 1)) {
              timed_out = true;
              break;
            }
          }
        }
        mma_commit(done_bar);
      } else {
      // Issue order S_t, P_{t-1}·V: the tensor core computes the next scores while
      // the softmax warps work on the current ones, across item boundaries too.
      int t = 0, k = 0;
      bool have_prev = false, prev_first = false, prev_last = false;
      int prev_k = 0;
      for (int w = blockIdx.x; w < num_items && !timed_out; w += gridDim.x, ++k) {
        int qt, bh;
        item_coords<CAUSAL>(w, num_q_tiles, BH, qt, bh);
        const int n_kv = kv_tiles<CAUSAL>(qt, S);
        if (!mbar_wait(q_full(k & 1), (uint32_t)(k >> 1) & 1u)) {
          timed_out = true;
          break;
        }
        for (int j = 0; j < n_kv; ++j, ++t) {
          // K tile, and S buffer sbuf(t) last read by the softmax of tile t-NB (with P over
          // S also by P_{t-NB}·V, waited for explicitly)
          if (!mbar_wait(k_full(kc % STAGES), (uint32_t)(kc / STAGES) & 1u) ||
              !mbar_wait(s_free(sbuf(t)), sph(t) ^ 1u) ||
              (NB > 2 && t >= NB && !mbar_wait(o_done_of(t - NB), sph(t - NB)))) {
            timed_out = true;
            break;
          }
          tc_fence_after();
          issue_s(t, k & 1);
          if (j == n_kv - 1) mma_commit(q_empty(k & 1));
          if (have_prev && !pv_step(t - 1, prev_k, prev_first, prev_last)) {
            timed_out = true;
            break;
          }
          have_prev = true;
          prev_first = (j == 0);
          prev_last = (j == n_kv - 1);
          prev_k = k;
        }
      }
      if (!timed_out && have_prev && !pv_step(t - 1, prev_k, prev_first, prev_last)) timed_out = true;
      mma_commit(done_bar);
      }
      (void)s_issuer;
      (void)pv_issuer;
    }
  } else if (KT_FA_ALT && warp < V_LOADER_WARP) {
    // softmax, alternate tiles: the warp of lane quarter q = warp & 3 and parity h
    // takes the S tiles t with t % 2 == h, all 128 key columns of its 32 rows. The
    // running max a tile's exponentials use is decided right after the tile's row
    // maxima are known and published to the other parity's warp of the quarter,
    // which waits for that decision before its next tile: the exponentials of
    // consecutive tiles then overlap on the two warps of a scheduler instead of
    // running in lockstep. Each warp keeps its own row-sum share relative to the
    // last maximum it used; the epilogue brings both shares to the final maximum.
    const int quarter = warp & 3;
    const int h = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float* m_sh = red;              // [2 item parity][128]
    float* l_hand = red + 2 * 128;  // [2 item parity][2 parity][128]
    float* m_hand = red + 6 * 128;  // [2 item parity][2 parity][128]
    constexpr int HD4 = D;          // O columns this thread rescales (its whole row)
    int t = 0, k = 0;
    for (int w = blockIdx.x; w < num_items && !timed_out; w += gridDim.x, ++k) {
      int qt, bh;
      item_coords<CAUSAL>(w, num_q_tiles, BH, qt, bh);
      const int n_kv = kv_tiles<CAUSAL>(qt, S);
      const int q0 = qt * BM;
      const int qrow = q0 + row;
      float my_m = -INFINITY;    // the maximum l_part is relative to
      float my_dec = -INFINITY;  // this warp's decision for its previous tile of this item
      float l_part = 0.f;
      for (int j = 0; j < n_kv; ++j, ++t) {
        if ((t & 1) != h) continue;
        const uint32_t dec_prev = dec_bar(quarter, (t - 1) & 1);
        const uint32_t dec_prev_ph = (uint32_t)((t - 1) >> 1) & 1u;
        // Fused speculative pass (KT_FA_FUSE, from this warp's second tile of the item
        // on): one pass over the scores with the newest running max this warp knows,
        // checked against the exact decision of tile t-1 at the end. Otherwise two
        // passes: the row max first, then the exponentials with the decided max.
        const bool fuse = KT_FA_FUSE && j >= 2;
        bool known = true;
        if (!fuse) {
          // the decision of tile t-1 (made by the other parity's warp of this quarter)
          if (t > 0 && !__all_sync(0xffffffffu, mbar_wait(dec_prev, dec_prev_ph))) {
            timed_out = true;
            break;
          }
        } else {
          known = __all_sync(0xffffffffu, mbar_test_wait(dec_prev, dec_prev_ph));
        }
        float m_prev = (j == 0) ? -INFINITY : (known ? m_sh[(k & 1) * 128 + row] : my_dec);
        if (!__all_sync(0xffffffffu, mbar_wait(s_full(sbuf(t)), sph(t)))) {
          timed_out = true;
          break;
        }
        tc_fence_after();
        const uint32_t s_addr = tmem + lane_off + CF::COL_S + (uint32_t)(sbuf(t) * BN);
        const int key0 = j * BN;
        const bool mask_tile = (CAUSAL && j * BN + BN - 1 > q0) || (j * BN + BN > S);
        auto mask32 = [&](uint32_t (&v)[32], int c) {
          if (mask_tile) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int key = key0 + c + i;
              if (!(key < S && (!CAUSAL || key <= qrow))) v[i] = __float_as_uint(-INFINITY);
            }
          }
        };
        // P: 64 columns of its own, or over the scores (chunk c's P lands in columns c/2..c/2+15,
        // all of them already read)
        const uint32_t p_addr = NB == 2 ? tmem + lane_off + CF::COL_P + (uint32_t)(h * 64) : s_addr;
        // p = 2^(s·c − m) for one 32-key chunk into P (bf16); returns the chunk's sum
        auto exp_chunk = [&](const uint32_t (&sc)[32], int c, float m, auto poly_tag) -> float {
          constexpr bool POLY = decltype(poly_tag)::value;
          float s4[4] = {0.f, 0.f, 0.f, 0.f};
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float x0, x1;
            if (KT_FA_X2) {
              fma2_bc(x0, x1, __uint_as_float(sc[2 * i]), __uint_as_float(sc[2 * i + 1]), scale_log2, -m);
            } else {
              x0 = fmaf(__uint_as_float(sc[2 * i]), scale_log2, -m);
              x1 = fmaf(__uint_as_float(sc[2 * i + 1]), scale_log2, -m);
            }
            float p0, p1;
            if (KT_FA_EXP16) {
              ex2_h2(x0, x1, p0, p1);
            } else if (POLY && (i & 3) >= 4 - KT_FA_POLY) {
              if (KT_FA_X2) {
                ex2_poly_x2(x0, x1, p0, p1);
              } else {
                p0 = ex2_poly(x0);
                p1 = ex2_poly(x1);
              }
            } else {
              p0 = ex2(x0);
              p1 = ex2(x1);
            }
            if (KT_FA_X2) add2(s4[(i & 1) * 2], s4[(i & 1) * 2 + 1], p0, p1);
            else s4[i & 3] += p0 + p1;
            pk[i] = pack_bf16(p0, p1);
          }
          tmem_st16(p_addr + (uint32_t)(c / 2), pk);
          return (s4[0] + s4[1]) + (s4[2] + s4[3]);
        };
        // multiply the first `cols` columns of stored P (bf16 pairs) of this row by f
        auto rescale_p = [&](int cols, float f) {
          tmem_st_wait();
#pragma unroll 1
          for (int cc = 0; cc < cols; cc += 16) {
            uint32_t v[16];
            tmem_ld16(p_addr + (uint32_t)cc, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i)
              v[i] = pack_bf16(__uint_as_float(v[i] << 16) * f, __uint_as_float(v[i] & 0xffff0000u) * f);
            tmem_st16(p_addr + (uint32_t)cc, v);
          }
        };
        // O holds P_0..P_{j-1}·V of this item relative to m_from: rescale the raised rows
        auto rescale_o = [&](bool raise, float m_from, float m_to) -> bool {
          const float alpha = raise ? ((m_from == -INFINITY) ? 0.f : ex2(m_from - m_to)) : 1.f;
          const bool o_ready = PER_BUF ? mbar_wait(o_done_of(t - 1), sph(t - 1))
                                                  : mbar_wait(o_done, (uint32_t)(t - 1) & 1u);
          if (!__all_sync(0xffffffffu, o_ready)) return false;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < HD4; c += 32) {
            uint32_t v[32];
            const uint32_t oa = tmem + lane_off + CF::COL_O + (uint32_t)c;
            tmem_ld32(oa, v);
            tmem_ld_wait();
            uint32_t w0[16], w1[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              w0[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
              w1[i] = __float_as_uint(__uint_as_float(v[16 + i]) * alpha);
            }
            tmem_st16(oa, w0);
            tmem_st16(oa + 16u, w1);
          }
          tmem_st_wait();
          return true;
        };
        float m_new, tile_sum;
        if (!fuse) {
          // row maximum over the tile, two 32-column loads in flight at a time
          float mx = -INFINITY;
#pragma unroll
          for (int c = 0; c + 64 <= BN; c += 64) {
            uint32_t va[32], vb[32];
            tmem_ld32(s_addr + (uint32_t)c, va);
            tmem_ld32(s_addr + (uint32_t)(c + 32), vb);
            tmem_ld_wait();
            mask32(va, c);
            mask32(vb, c + 32);
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int i = 0; i < 32; ++i) m4[i & 3] = fmax3f(m4[i & 3], __uint_as_float(va[i]), __uint_as_float(vb[i]));
            mx = fmaxf(mx, fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])));
          }
          if constexpr (BN % 64 == 32) {  // the last 32 keys of a 96-key tile
            uint32_t va[32];
            tmem_ld32(s_addr + (uint32_t)(BN - 32), va);
            tmem_ld_wait();
            mask32(va, BN - 32);
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int i = 0; i < 32; i += 2)
              m4[(i >> 1) & 3] = fmax3f(m4[(i >> 1) & 3], __uint_as_float(va[i]), __uint_as_float(va[i + 1]));
            mx = fmaxf(mx, fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])));
          }
          const float m_tile = mx * scale_log2;
          const bool raise = m_tile > m_prev + kRescaleThreshold;
          m_new = raise ? m_tile : m_prev;
          m_sh[(k & 1) * 128 + row] = m_new;
          warp_arrive(dec_bar(quarter, t & 1));  // release: m_sh is visible to the waiting warp
          if (j > 0 && __any_sync(0xffffffffu, raise) && !rescale_o(raise, m_prev, m_new)) {
            timed_out = true;
            break;
          }
          // scores reloaded 32 columns at a time, P written as each chunk is done
          auto exp_row = [&](auto poly_tag) -> float {
            float sum = 0.f;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
              uint32_t sc[32];
              tmem_ld32(s_addr + (uint32_t)c, sc);
              tmem_ld_wait();
              mask32(sc, c);
              sum += exp_chunk(sc, c, m_new, poly_tag);
              // the P columns of a key range that is not the last: P·V may start on them
              constexpr int CPR = BN / 32 / PSPLIT;  // 32-key chunks per range
              if (PSPLIT > 1 && (c / 32 + 1) % CPR == 0 && c + 32 < BN) {
                tmem_st_wait();
                tc_fence_before();
                warp_arrive(p_part(sbuf(t), (c / 32 + 1) / CPR - 1));
              }
            }
            return sum;
          };
          tile_sum = (KT_FA_POLY && !mask_tile) ? exp_row(std::true_type{}) : exp_row(std::false_type{});
        } else {
          // one pass: each chunk's maximum is checked against the max in use; rows
          // whose scores pass it by more than the rescale threshold switch to the
          // tile's running max (their stored P and sum are scaled down to it)
          float m_use = m_prev, mt = -INFINITY, sum = 0.f;
          auto pass = [&](auto poly_tag) {
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
              uint32_t sc[32];
              tmem_ld32(s_addr + (uint32_t)c, sc);
              tmem_ld_wait();
              mask32(sc, c);
              float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
              for (int i = 0; i < 32; i += 2)
                m4[(i >> 1) & 3] = fmax3f(m4[(i >> 1) & 3], __uint_as_float(sc[i]), __uint_as_float(sc[i + 1]));
              const float cm = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * scale_log2;
              mt = fmaxf(mt, cm);
              const bool bad = cm > m_use + kRescaleThreshold;
              if (__any_sync(0xffffffffu, bad)) {
                const float f = bad ? ex2(m_use - mt) : 1.f;
                if (c > 0) rescale_p(c / 2, f);
                sum *= f;
                if (bad) m_use = mt;
              }
              sum += exp_chunk(sc, c, m_use, poly_tag);
            }
          };
          if (KT_FA_POLY && !mask_tile) pass(std::true_type{});
          else pass(std::false_type{});
          // the exact decision of tile t-1, then this tile's
          if (!known && !__all_sync(0xffffffffu, mbar_wait(dec_prev, dec_prev_ph))) {
            timed_out = true;
            break;
          }
          m_prev = m_sh[(k & 1) * 128 + row];
          const bool raise = mt > m_prev + kRescaleThreshold;
          m_new = raise ? mt : m_prev;
          m_sh[(k & 1) * 128 + row] = m_new;
          warp_arrive(dec_bar(quarter, t & 1));  // release: m_sh is visible to the waiting warp
          // P relative to the decided max (rare: a raise in the other warp's tile or a switch here)
          if (__any_sync(0xffffffffu, m_use != m_new)) {
            const float f = (m_use != m_new) ? ex2(m_use - m_new) : 1.f;
            rescale_p(BN / 2, f);
            sum *= f;
          }
          if (__any_sync(0xffffffffu, raise) && !rescale_o(raise, m_prev, m_new)) {
            timed_out = true;
            break;
          }
          tile_sum = sum;
        }
        // this warp's row-sum share follows the maximum
        if (my_m != m_new) {
          l_part = (my_m == -INFINITY) ? 0.f : l_part * ex2(my_m - m_new);
          my_m = m_new;
        }
        l_part += tile_sum;
        my_dec = m_new;
        tmem_st_wait();
        tc_fence_before();
        if (fuse) {
          // the split P·V ranges are signalled only now that P is final
          for (int i = 0; i + 1 < PSPLIT; ++i) warp_arrive(p_part(sbuf(t), i));
        }
        warp_arrive(s_free(sbuf(t)));
        warp_arrive(p_full(sbuf(t)));
      }
      if (timed_out) break;
      // hand this warp's share and its maximum to the epilogue (two slots, by item parity)
      const int lb = k & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(l_empty(lb), ((uint32_t)(k >> 1) & 1u) ^ 1u))) {
        timed_out = true;
        break;
      }
      l_hand[(lb * 2 + h) * 128 + row] = l_part;
      m_hand[(lb * 2 + h) * 128 + row] = my_m;
      warp_arrive(l_full(lb));
    }
  } else if (warp < V_LOADER_WARP) {
#if KT_FA_BN == 128  // the column-half split needs 64-key halves
    // softmax: TMEM lane quarter = warp % 4, the two warps of a quarter split the columns
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t pair_mbar = pair_bar0 + 8u * (uint32_t)quarter;  // mbarrier of the two warps of this quarter
    constexpr int HC = BN / 2;                                     // score columns per thread
    constexpr int HD = D / 2;                                      // O columns per thread (rescale)
    float m_guess = -INFINITY;  // the previous item's final running max (same in both halves)
    int t = 0, k = 0;
    for (int w = blockIdx.x; w < num_items && !timed_out; w += gridDim.x, ++k) {
      int qt, bh;
      item_coords<CAUSAL>(w, num_q_tiles, BH, qt, bh);
      const int n_kv = kv_tiles<CAUSAL>(qt, S);
      const int q0 = qt * BM;
      const int qrow = q0 + row;
      // running max of s·scale·log2e used by the exponentials (same in both halves); with
      // first-tile speculation it starts at the previous item's value until the exchange
      float m_run = KT_FA_SPEC0 ? m_guess : -INFINITY;
      float l_part = 0.f;  // this half's share of the row sum
      for (int j = 0; j < n_kv; ++j, ++t) {
        const int b = t & 1;       // tile parity: the max-exchange slots
        const int sb = sbuf(t);    // S (and P) buffer
        if (!__all_sync(0xffffffffu, mbar_wait(s_full(sb), sph(t)))) {
          timed_out = true;
          break;
        }
        tc_fence_after();
        if (KT_FA_DEPHASE > 0 && half == 1 && t == 0) {
          // once, after the first scores landed: the second warp of the pair starts late
          const long long c0 = clock64();
          while (clock64() - c0 < KT_FA_DEPHASE) {
          }
        }
        const uint32_t s_addr = tmem + lane_off + CF::COL_S + (uint32_t)(sb * BN + half * HC);
        const int key0 = j * BN + half * HC;
        const bool mask_tile = (CAUSAL && j * BN + BN - 1 > q0) || (j * BN + BN > S);
        uint32_t sv[HC];
#pragma unroll
        for (int c = 0; c < HC; c += 32) tmem_ld32(s_addr + (uint32_t)c, *reinterpret_cast<uint32_t(*)[32]>(&sv[c]));
        tmem_ld_wait();
        if (mask_tile) {
#pragma unroll
          for (int c = 0; c < HC; ++c) {
            const int key = key0 + c;
            if (!(key < S && (!CAUSAL || key <= qrow))) sv[c] = __float_as_uint(-INFINITY);
          }
        }
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < HC; ++c) m4[c & 3] = fmaxf(m4[c & 3], __uint_as_float(sv[c]));
        const float mh = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        // publish the half-row maximum to the partner warp (slots double-buffered by
        // tile parity: the partner may still read the previous tile's slot)
        float* red_max = red + (b * 2) * 128;
        red_max[half * 128 + row] = mh;
        warp_arrive(pair_mbar);  // release: the write above is visible to the partner after its wait
        const uint32_t p_addr = NB == 2 ? tmem + lane_off + CF::COL_P + (uint32_t)(b * 64 + half * (HC / 2))
                                        : s_addr;  // over this half's scores, which are in registers
        // p = 2^(s·c − m) (masked entries are −inf -> 0) into TMEM as bf16; returns this half's sum.
        // The polynomial share is chosen per tile (masked tiles use MUFU only).
        auto make_p = [&](float m, auto poly_tag) -> float {
          constexpr bool POLY = decltype(poly_tag)::value;
          float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int c = 0; c < HC; c += 32) {
            uint32_t pk[16];
            uint32_t sc[32];
            if (KT_FA_RELOAD) {
              // scores again from TMEM, 32 columns at a time: only this chunk is live
              tmem_ld32(s_addr + (uint32_t)c, sc);
              tmem_ld_wait();
              if (mask_tile) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                  const int key = key0 + c + i;
                  if (!(key < S && (!CAUSAL || key <= qrow))) sc[i] = __float_as_uint(-INFINITY);
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) sc[i] = sv[c + i];
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float x0, x1;
              if (KT_FA_X2) {
                fma2_bc(x0, x1, __uint_as_float(sc[2 * i]), __uint_as_float(sc[2 * i + 1]), scale_log2, -m);
              } else {
                x0 = fmaf(__uint_as_float(sc[2 * i]), scale_log2, -m);
                x1 = fmaf(__uint_as_float(sc[2 * i + 1]), scale_log2, -m);
              }
              float p0, p1;
              if (KT_FA_EXP16) {
                ex2_h2(x0, x1, p0, p1);
              } else if (POLY && (i & 3) >= 4 - KT_FA_POLY) {
                if (KT_FA_X2) {
                  ex2_poly_x2(x0, x1, p0, p1);
                } else {
                  p0 = ex2_poly(x0);
                  p1 = ex2_poly(x1);
                }
              } else {
                p0 = ex2(x0);
                p1 = ex2(x1);
              }
              if (KT_FA_X2) add2(s4[(i & 1) * 2], s4[(i & 1) * 2 + 1], p0, p1);
              else s4[i & 3] += p0 + p1;
              pk[i] = pack_bf16(p0, p1);
            }
            tmem_st16(p_addr + (uint32_t)(c / 2), pk);
          }
          return (s4[0] + s4[1]) + (s4[2] + s4[3]);
        };
        auto p_sum = [&](float m) -> float {
          if (KT_FA_POLY && !mask_tile) return make_p(m, std::true_type{});
          return make_p(m, std::false_type{});
        };
        // Speculation (j > 0): when no lane of this warp needs its running max raised
        // by its own half, P is computed with the current running max before the
        // partner's half maximum is read, so the exchange overlaps the exponentials.
        // Only if the partner's half then asks for a raise are P and the sum redone
        // below with the new maximum (the MMA reads P only after p_full).
        bool pair_seen = false, finished = false;
        // a first-tile guess must neither be exceeded by more than the threshold nor
        // exceed the row max by more than kGuessSlack (P would lose its range)
        auto guess_bad = [&](float mxs) {
          return mxs > m_run + kRescaleThreshold || (j == 0 && mxs < m_run - kGuessSlack);
        };
        if (KT_FA_SPEC && (j > 0 || (KT_FA_SPEC0 && __all_sync(0xffffffffu, m_run != -INFINITY))) &&
            !__any_sync(0xffffffffu, guess_bad(mh * scale_log2))) {
          const float spec_sum = p_sum(m_run);
          if (!__all_sync(0xffffffffu, mbar_wait(pair_mbar, (uint32_t)t & 1u))) {
            timed_out = true;
            break;
          }
          pair_seen = true;
          const float mx_s = fmaxf(red_max[row], red_max[128 + row]);
          if (!__any_sync(0xffffffffu, guess_bad(mx_s * scale_log2))) {
            l_part += spec_sum;
            finished = true;
          } else {
            tmem_st_wait();  // the speculative P is rewritten below
          }
        }
        if (!finished) {
          if (!pair_seen && !__all_sync(0xffffffffu, mbar_wait(pair_mbar, (uint32_t)t & 1u))) {
            timed_out = true;
            break;
          }
          const float mx = fmaxf(red_max[row], red_max[128 + row]);
          const float m_tile = mx * scale_log2;
          // a first-tile guess the row maxima reject (in either half: both see the same
          // maxima and take the same decision): start from the tile's max
          if (j == 0 && __any_sync(0xffffffffu, guess_bad(m_tile))) m_run = -INFINITY;
          const bool raise = m_tile > m_run + kRescaleThreshold;
          float alpha = 1.f;
          if (raise) {
            alpha = (m_run == -INFINITY) ? 0.f : ex2(m_run - m_tile);
            m_run = m_tile;
            l_part *= alpha;
          }
          // O holds P_0..P_{j-1}·V of this item: rescale this half of it once the
          // previous P·V product has landed. The o_done barrier of P_{t-1}·V has
          // completed P_{t-1-NB}·V (issued before P_{t-NB}·V, which S_t waited for)
          // and cannot complete P_{t-1+NB}·V (it needs this thread's P), so a
          // parity wait is exact.
          if (j > 0 && __any_sync(0xffffffffu, raise)) {
            const bool o_ready = PER_BUF ? mbar_wait(o_done_of(t - 1), sph(t - 1))
                                                    : mbar_wait(o_done, (uint32_t)(t - 1) & 1u);
            if (!__all_sync(0xffffffffu, o_ready)) {
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
              for (int i = 0; i < 16; ++i) {
                w0[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
                w1[i] = __float_as_uint(__uint_as_float(v[16 + i]) * alpha);
              }
              tmem_st16(oa, w0);
              tmem_st16(oa + 16u, w1);
            }
            tmem_st_wait();
          }
          l_part += p_sum(m_run);
        }
        tmem_st_wait();
        tc_fence_before();
        warp_arrive(s_free(sb));
        warp_arrive(p_full(sb));
      }
      if (timed_out) break;
      // hand this half's row sum to the epilogue warps (two slots, by item parity)
      const int lb = k & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(l_empty(lb), ((uint32_t)(k >> 1) & 1u) ^ 1u))) {
        timed_out = true;
        break;
      }
      red[(4 + 2 * lb + half) * 128 + row] = l_part;
      warp_arrive(l_full(lb));
      m_guess = m_run;
    }
#endif
  } else {
    // epilogue warps: O / l -> bf16, one query row per thread; O is released to the
    // next item's first P·V product as soon as it is in registers
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    int k = 0;
    for (int w = blockIdx.x; w < num_items; w += gridDim.x, ++k) {
      int qt, bh;
      item_coords<CAUSAL>(w, num_q_tiles, BH, qt, bh);
      const int qrow = qt * BM + row;
      const int lb = k & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(o_final, (uint32_t)k & 1u)) ||
          !__all_sync(0xffffffffu, mbar_wait(l_full(lb), (uint32_t)(k >> 1) & 1u))) {
        timed_out = true;
        break;
      }
      float l_run;
      if (KT_FA_ALT) {
        // both parities' shares, each relative to the last maximum its warp used, at the final maximum
        const float ma = red[(6 + lb * 2) * 128 + row], mb = red[(7 + lb * 2) * 128 + row];
        const float la = red[(2 + lb * 2) * 128 + row], lbs = red[(3 + lb * 2) * 128 + row];
        const float mf = fmaxf(ma, mb);
        l_run = (ma == -INFINITY ? 0.f : la * ex2(ma - mf)) + (mb == -INFINITY ? 0.f : lbs * ex2(mb - mf));
      } else {
        l_run = red[(4 + 2 * lb) * 128 + row] + red[(5 + 2 * lb) * 128 + row];
      }
      warp_arrive(l_empty(lb));
      tc_fence_after();
      const float inv = 1.0f / l_run;
      uint4* dst = reinterpret_cast<uint4*>(O + ((int64_t)bh * S + qrow) * D);
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + CF::COL_O + (uint32_t)c, v);
        tmem_ld_wait();
        if (c + 32 == D) {
          tc_fence_before();
          warp_arrive(o_empty);  // all of O is in registers: the next item may overwrite it
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
  if (timed_out) raise_device_error(DEV_MBAR_TIMEOUT);
  __syncthreads();
  if (warp == 1) {
    (void)__all_sync(0xffffffffu, mbar_wait(done_bar, 0));
    tc_fence_after();
    tmem_dealloc(tmem, CF::TMEM_COLS);
  }
}

// [B·H, S, D] bf16 viewed as a 3-D tensor (D, S, B·H); box 64 × rows × 1, 128-byte swizzle.
inline int make_tmap_bhsd(CUtensorMap* map, const void* base, int64_t BH, int64_t S, int64_t D, uint32_t rows = 128) {
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
  using CF = Cfg<D, KT_FA_STAGES, KT_FA_VSTAGES>;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_bhsd(&tq, Q, BH, S, D, BM);
  if (rc == KT_OK) rc = make_tmap_bhsd(&tk, K, BH, S, D, BN);  // K and V tiles of BN keys
  if (rc == KT_OK) rc = make_tmap_bhsd(&tv, V, BH, S, D, BN);
  if (rc != KT_OK) return rc;
  auto kern = fa_fwd_kernel<D, KT_FA_STAGES, CAUSAL>;
  rc = ensure_smem((const void*)kern, CF::SMEM_BYTES, "attention: smem attribute");
  if (rc != KT_OK) return rc;
  const float scale_log2 = scale * 1.4426950408889634f;  // log2(e)
  // persistent: one CTA per SM (TMEM holds one CTA's 512 columns), items strided over the CTAs
  const int64_t items = BH * ((S + BM - 1) / BM);
  const int64_t sms = sm_count();
  dim3 grid((unsigned)(items < sms ? items : sms));
  kern<<<grid, THREADS, CF::SMEM_BYTES, st>>>(tq, tk, tv, reinterpret_cast<__nv_bfloat16*>(O), (int)S, (int)BH,
                                              scale_log2);
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
  if (KT_FA_KIND == 2) {
    // two ping-pong query tiles per CTA (fa_fwd2.cuh)
    if (D == 128)
      return causal ? fa2::launch_t<128, true>(Q, K, V, O, BH, S, scale, st)
                    : fa2::launch_t<128, false>(Q, K, V, O, BH, S, scale, st);
    return causal ? fa2::launch_t<64, true>(Q, K, V, O, BH, S, scale, st)
                  : fa2::launch_t<64, false>(Q, K, V, O, BH, S, scale, st);
  }
  if (D == 128) {
    return causal ? launch_t<128, true>(Q, K, V, O, BH, S, scale, st) : launch_t<128, false>(Q, K, V, O, BH, S, scale, st);
  }
  return causal ? launch_t<64, true>(Q, K, V, O, BH, S, scale, st) : launch_t<64, false>(Q, K, V, O, BH, S, scale, st);
}

}  // namespace fa
}  // namespace kt
