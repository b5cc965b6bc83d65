// fa_fwd.cuh — flash-attention forward, bf16 in / fp32 softmax and
// accumulation / bf16 out, for sm_100a (tcgen05 + TMEM + TMA).
//
// Computes O = softmax(scale·Q·K^T [+ causal mask]) · V per (batch, head) on
// [B, H, S, D] tensors — the reference's `attention_flash` /
// `attention_tiled` (src/attention.py:210-291, :75-176; oracle
// src/verifier.py:277-294), which are single-head fp32 SIMT kernels with one
// CTA per query row.
//
// CTA = one (b, h) and BM = 128 query rows; 192 threads:
//   warp 0     one lane: TMA loads of the Q tile (once) and of K/V tiles
//              (BN = 128 keys) into a 2-slot ring (128-byte swizzle, 64-column boxes)
//   warp 1     allocates 512 TMEM columns; one lane issues the MMAs:
//                S_j = Q·K_j^T  (kind::f16, M=128, N=128, A and B from smem)
//                O  += P_j·V_j   (kind::f16, M=128, N=D, A = P from TMEM, B = V MN-major)
//              S_{j+1} is issued before O += P_j·V_j so the tensor core works on
//              the next scores while the softmax warps process the current ones.
//   warps 2-5  softmax, one query row per thread (TMEM lane = row): row max,
//              p = 2^(s·scale·log2e − m), row sum, bf16 P written back to TMEM;
//              the running max is only raised (and O, l rescaled) when it grows
//              by more than 2^8, so O is rarely touched; final O / l in bf16.
// TMEM columns: S0 [0,128) S1 [128,256) O [256,256+D) P0 [384,448) P1 [448,512).
// Every mbarrier wait is bounded; a timeout records DEV_MBAR_TIMEOUT and the
// CTA unwinds (loader drains its copies, MMAs drain before TMEM is released).
#pragma once
#include "kt_common.cuh"
#include "sm100.cuh"

#ifndef KT_FA_STAGES
#define KT_FA_STAGES 2
#endif
#ifndef KT_FA_BN
#define KT_FA_BN 128
#endif

namespace kt {
namespace fa {

constexpr int BM = 128;
constexpr int BN = 128;  // keys per tile (the S accumulator is 128 columns)
constexpr int THREADS = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: O is rescaled only when the max grows by > 2^8

template <int D, int STAGES>
struct Cfg {
  static_assert(D == 64 || D == 128, "head dim");
  static constexpr int REGIONS = D / 64;            // 128-byte (64 bf16) column slabs per row
  static constexpr int SLAB = 128 * 128;            // one slab of 128 rows × 128 bytes
  static constexpr int Q_BYTES = REGIONS * SLAB;    // 128 rows × D bf16
  static constexpr int K_BYTES = REGIONS * SLAB;    // BN keys × D
  static constexpr int V_BYTES = REGIONS * SLAB;
  static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
  static constexpr int Q_OFFSET = 0;
  static constexpr int KV_OFFSET = Q_BYTES;
  static constexpr int BAR_OFFSET = KV_OFFSET + STAGES * STAGE_BYTES;
  // q_full, kv_full[S], kv_empty[S], s_full[2], s_free[2], p_full[2], o_done, o_final, done
  static constexpr int NUM_BARS = 1 + 2 * STAGES + 2 + 2 + 2 + 1 + 1 + 1;
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
  const uint32_t bar0 = base + CF::BAR_OFFSET;
  const uint32_t q_full = bar0;
  auto kv_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto kv_empty = [&](int s) { return bar0 + 8u * (1 + STAGES + s); };
  auto s_full = [&](int b) { return bar0 + 8u * (1 + 2 * STAGES + b); };
  auto s_free = [&](int b) { return bar0 + 8u * (3 + 2 * STAGES + b); };
  auto p_full = [&](int b) { return bar0 + 8u * (5 + 2 * STAGES + b); };
  const uint32_t o_done = bar0 + 8u * (7 + 2 * STAGES);   // one phase per P·V product
  const uint32_t o_final = bar0 + 8u * (8 + 2 * STAGES);  // single use: the last P·V product landed
  const uint32_t done_bar = bar0 + 8u * (9 + 2 * STAGES);
  const uint32_t tmem_slot = bar0 + 8u * CF::NUM_BARS;
  const volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<const volatile uint32_t*>(base_ptr + CF::BAR_OFFSET + 8 * CF::NUM_BARS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_q_tiles = (S + BM - 1) / BM;
  // heaviest (latest) query tiles first when causal
  const int qt = CAUSAL ? (num_q_tiles - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int bh = blockIdx.y;
  const int q0 = qt * BM;
  const int num_kv_all = (S + BN - 1) / BN;
  const int n_kv = CAUSAL ? min(num_kv_all, (q0 + BM - 1) / BN + 1) : num_kv_all;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(s_free(b), 128);
      mbar_init(p_full(b), 128);
    }
    mbar_init(o_done, 1);
    mbar_init(o_final, 1);
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

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t q_dst = base + CF::Q_OFFSET;
      mbar_arrive_expect_tx(q_full, CF::Q_BYTES);
#pragma unroll
      for (int r = 0; r < CF::REGIONS; ++r) tma_load_3d(q_dst + r * CF::SLAB, &tm_q, 64 * r, q0, bh, q_full);
      int s = 0;
      uint32_t ph = 0;
      uint32_t last_ph[STAGES];
      bool pending[STAGES];
#pragma unroll
      for (int i = 0; i < STAGES; ++i) pending[i] = false;
      for (int j = 0; j < n_kv; ++j) {
        if (!mbar_wait(kv_empty(s), ph ^ 1u)) {
          timed_out = true;
          break;
        }
        const uint32_t k_dst = base + CF::KV_OFFSET + s * CF::STAGE_BYTES;
        const uint32_t v_dst = k_dst + CF::K_BYTES;
        mbar_arrive_expect_tx(kv_full(s), CF::STAGE_BYTES);
#pragma unroll
        for (int r = 0; r < CF::REGIONS; ++r) {
          tma_load_3d(k_dst + r * CF::SLAB, &tm_k, 64 * r, j * BN, bh, kv_full(s));
          tma_load_3d(v_dst + r * CF::SLAB, &tm_v, 64 * r, j * BN, bh, kv_full(s));
        }
        last_ph[s] = ph;
        pending[s] = true;
        if (++s == STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (timed_out) {
        (void)mbar_wait(q_full, 0);
        for (int i = 0; i < STAGES; ++i)
          if (pending[i]) (void)mbar_wait(kv_full(i), last_ph[i]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f32acc(kFmtBF16, BM, BN, 0, 0);
      constexpr uint32_t idesc_o = idesc_f32acc(kFmtBF16, BM, D, 0, 1);
      const uint32_t q_src = base + CF::Q_OFFSET;
      auto issue_s = [&](int j, int stage) {
        const uint32_t k_src = base + CF::KV_OFFSET + stage * CF::STAGE_BYTES;
        const uint32_t d_tmem = tmem + CF::COL_S + (uint32_t)((j & 1) * BN);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * CF::SLAB + (kk & 3) * 32);
          mma_f16_ss(d_tmem, desc_sw128(q_src + off, 16u, 1024u), desc_sw128(k_src + off, 16u, 1024u), idesc_s,
                     kk > 0 ? 1u : 0u);
        }
        mma_commit(s_full(j & 1));
      };
      auto issue_pv = [&](int j, int stage) {
        const uint32_t v_src = base + CF::KV_OFFSET + stage * CF::STAGE_BYTES + CF::K_BYTES;
        const uint32_t p_tmem = tmem + CF::COL_P + (uint32_t)((j & 1) * 64);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // 16 keys per MMA: rows 16kk..16kk+15 of every 64-column V slab; slabs CF::SLAB apart
          const uint64_t vd = desc_sw128(v_src + (uint32_t)(kk * 16 * 128), (uint32_t)CF::SLAB, 1024u);
          mma_f16_ts(tmem + CF::COL_O, p_tmem + (uint32_t)(kk * 8), vd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(o_done);
        mma_commit(kv_empty(stage));
      };
      if (!mbar_wait(q_full, 0)) timed_out = true;
      tc_fence_after();
      int s = 0;
      uint32_t ph = 0;
      int prev_stage = 0;
      for (int j = 0; j < n_kv && !timed_out; ++j) {
        if (!mbar_wait(kv_full(s), ph)) {
          timed_out = true;
          break;
        }
        // S buffer j&1 was last read by the softmax of tile j-2
        if (!mbar_wait(s_free(j & 1), ((uint32_t)(j >> 1) & 1u) ^ 1u)) {
          timed_out = true;
          break;
        }
        tc_fence_after();
        issue_s(j, s);
        if (j > 0) {
          if (!mbar_wait(p_full((j - 1) & 1), (uint32_t)((j - 1) >> 1) & 1u)) {
            timed_out = true;
            break;
          }
          tc_fence_after();
          issue_pv(j - 1, prev_stage);
        }
        prev_stage = s;
        if (++s == STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (!timed_out && n_kv > 0) {
        if (mbar_wait(p_full((n_kv - 1) & 1), (uint32_t)((n_kv - 1) >> 1) & 1u)) {
          tc_fence_after();
          issue_pv(n_kv - 1, prev_stage);
          mma_commit(o_final);
        } else {
          timed_out = true;
        }
      }
      mma_commit(done_bar);
    }
  } else {
    // softmax: thread <-> query row (TMEM lane)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qrow = q0 + row;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m_run = -INFINITY;  // running max of s·scale·log2e used by the exponentials
    float l_run = 0.f;
    for (int j = 0; j < n_kv; ++j) {
      const int b = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(s_full(b), (uint32_t)(j >> 1) & 1u))) {
        timed_out = true;
        break;
      }
      tc_fence_after();
      const uint32_t s_addr = tmem + lane_off + CF::COL_S + (uint32_t)(b * BN);
      const int key0 = j * BN;
      const bool mask_tile = (CAUSAL && key0 + BN - 1 > q0) || (key0 + BN > S);
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld32(s_addr + (uint32_t)c, v);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int key = key0 + c + t;
          const bool valid = !mask_tile || (key < S && (!CAUSAL || key <= qrow));
          if (valid) mx = fmaxf(mx, __uint_as_float(v[t]));
        }
      }
      const float m_tile = mx * scale_log2;
      bool raise = m_tile > m_run + kRescaleThreshold;
      float alpha = 1.f;
      if (raise) {
        alpha = (m_run == -INFINITY) ? 0.f : ex2(m_run - m_tile);
        m_run = m_tile;
        l_run *= alpha;
      }
      // O holds P_0..P_{j-1}·V: rescale it once the previous PV product has landed.
      // o_done is at phase j-1 or j here (s_full[j] was committed after PV_{j-2}
      // was issued, and PV_j needs this thread's P_j), so a parity wait is exact.
      if (j > 0 && __any_sync(0xffffffffu, raise)) {
        if (!__all_sync(0xffffffffu, mbar_wait(o_done, (uint32_t)(j - 1) & 1u))) {
          timed_out = true;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + CF::COL_O + (uint32_t)c, v);
          tmem_ld_wait();
          uint32_t w0[16], w1[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            w0[t] = __float_as_uint(__uint_as_float(v[t]) * alpha);
            w1[t] = __float_as_uint(__uint_as_float(v[16 + t]) * alpha);
          }
          tmem_st16(tmem + lane_off + CF::COL_O + (uint32_t)c, w0);
          tmem_st16(tmem + lane_off + CF::COL_O + (uint32_t)c + 16u, w1);
        }
        tmem_st_wait();
      }
      // pass 2: p = 2^(s·c − m), row sum, bf16 P into TMEM
      const uint32_t p_addr = tmem + lane_off + CF::COL_P + (uint32_t)(b * 64);
      float sum = 0.f;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld32(s_addr + (uint32_t)c, v);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          float p0 = ex2(fmaf(__uint_as_float(v[2 * t]), scale_log2, -m_run));
          float p1 = ex2(fmaf(__uint_as_float(v[2 * t + 1]), scale_log2, -m_run));
          if (mask_tile) {
            const int k0 = key0 + c + 2 * t;
            if (!(k0 < S && (!CAUSAL || k0 <= qrow))) p0 = 0.f;
            if (!(k0 + 1 < S && (!CAUSAL || k0 + 1 <= qrow))) p1 = 0.f;
          }
          sum += p0 + p1;
          pk[t] = pack_bf16(p0, p1);
        }
        tmem_st16(p_addr + (uint32_t)(c / 2), pk);
      }
      l_run += sum;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(s_free(b));
      mbar_arrive(p_full(b));
    }
    // epilogue: O / l -> bf16
    if (!timed_out && n_kv > 0) {
      if (!__all_sync(0xffffffffu, mbar_wait(o_final, 0))) {
        timed_out = true;
      } else {
        tc_fence_after();
        const float inv = 1.0f / l_run;
        __nv_bfloat16* orow = O + ((int64_t)bh * S + qrow) * D;
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + CF::COL_O + (uint32_t)c, v);
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
  using CF = Cfg<D, KT_FA_STAGES>;
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
  dim3 grid((unsigned)((S + BM - 1) / BM), (unsigned)BH);
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
  if (S > (int64_t)INT32_MAX / 2 || B * H > 65535) return fail(KT_ERR_UNSUPPORTED, "attention: S or B*H too large");
  if (!(scale > 0.f) || !isfinite(scale)) return fail(KT_ERR_ARG, "attention: scale must be finite and > 0");
  const int64_t BH = B * H;
  if (D == 128) {
    return causal ? launch_t<128, true>(Q, K, V, O, BH, S, scale, st) : launch_t<128, false>(Q, K, V, O, BH, S, scale, st);
  }
  return causal ? launch_t<64, true>(Q, K, V, O, BH, S, scale, st) : launch_t<64, false>(Q, K, V, O, BH, S, scale, st);
}

}  // namespace fa
}  // namespace kt
