// gemm_tf32.cuh — TF32 tensor-core GEMM for sm_100a: tcgen05.mma kind::tf32
// with the fp32 accumulator in TMEM, operands staged by TMA (128-byte swizzle),
// an mbarrier ring between the loader and the MMA issuer, and a double-
// buffered TMEM accumulator so the epilogue of one tile overlaps the main
// loop of the next.
//
// Computes the reference's `matmul_opt` product (src/generator.py:40-70):
// C = A·B with B row-major K×N, or, with transpose_b, C = A·Bt^T where B holds
// Bt row-major N×K (the layout the reference's transpose_b load reads,
// src/generator.py:286-293). Operands are fp32 in HBM; the tensor core reads
// them as tf32 (10-bit mantissa), products accumulate in fp32.
//
// CTA (192 threads, one per SM, persistent over output tiles):
//   warp 0   one lane issues TMA loads of A (BM×BK, K-major) and B (BN×BK:
//            K-major for Bt, MN-major 32-column slabs for B) into STAGES slots
//   warp 1   allocates TMEM (2·BN columns); one lane issues the MMAs
//            (M=128, N=BN, K=8 per instruction, 4 per 128-byte k-block) and
//            commits slot releases / accumulator hand-offs to mbarriers
//   warps 2-5  epilogue: tcgen05.ld of the accumulator (warp w owns TMEM lanes
//            32·(w%4)..+31 = tile rows), fp32 stores to C
// Every mbarrier wait is bounded (KT_WAIT_LIMIT_NS); a role that times out
// records DEV_MBAR_TIMEOUT in the device error word and unwinds, the loader
// waits for its own copies in flight, and TMEM is released after the MMAs drain.
#pragma once
#include "kt_common.cuh"
#include "sm100.cuh"
#include "gemm_ffma.cuh"

#ifndef KT_TC_BN
#define KT_TC_BN 256
#endif
#ifndef KT_TC_STAGES
#define KT_TC_STAGES 4
#endif

namespace kt {
namespace gemm_tf32 {

constexpr int BM = 128;
constexpr int BK = 32;       // fp32 elements per k-block: one 128-byte swizzle row
constexpr int THREADS = 192;
constexpr int GROUP_M = 16;  // rasterisation: GROUP_M m-tiles sweep the n-tiles together (L2 reuse of B)

template <int BN, int STAGES>
struct Cfg {
  // N of the accumulator tile: whole 32-column slabs, at most one 256-column MMA
  static_assert(BN % 32 == 0 && BN >= 128 && BN <= 256, "BN");
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // two accumulators; the allocation is a power of two of at least 2·BN columns
  static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static constexpr int NUM_BARS = 2 * STAGES + 4 + 1;
  static constexpr int BAR_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFFSET + NUM_BARS * 8 + 16 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mt, int& nt) {
  const int per_group = GROUP_M * num_n;
  const int group = t / per_group;
  const int first_m = group * GROUP_M;
  const int gsize = min(num_m - first_m, GROUP_M);
  const int r = t - group * per_group;
  mt = first_m + r % gsize;
  nt = r / gsize;
}

template <int BN, int STAGES, bool TB>
__global__ void __launch_bounds__(THREADS, 1)
gemm_tf32_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 float* __restrict__ C, int M, int N, int K) {
  using CF = Cfg<BN, STAGES>;
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // SW128 atoms need 1024-byte alignment
  uint8_t* base_ptr = smem_raw + (base - raw);
  const uint32_t bar0 = base + CF::BAR_OFFSET;
  const uint32_t done_bar = bar0 + 8u * (2 * STAGES + 4);
  const uint32_t tmem_slot = bar0 + 8u * CF::NUM_BARS;
  const volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<const volatile uint32_t*>(base_ptr + CF::BAR_OFFSET + 8 * CF::NUM_BARS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN, num_tiles = num_m * num_n;
  const int kblocks = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar0 + 8u * s, 1);             // full[s]: loader expect_tx + TMA bytes
      mbar_init(bar0 + 8u * (STAGES + s), 1);  // empty[s]: MMA commit
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar0 + 8u * (2 * STAGES + a), 1);      // tmem_full[a]: MMA commit
      mbar_init(bar0 + 8u * (2 * STAGES + 2 + a), 128);  // tmem_empty[a]: 128 epilogue threads
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, CF::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;
  bool timed_out = false;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t last_ph[STAGES];
      bool pending[STAGES];
#pragma unroll
      for (int i = 0; i < STAGES; ++i) pending[i] = false;
      for (int t = blockIdx.x; t < num_tiles && !timed_out; t += gridDim.x) {
        int mt, nt;
        tile_coords(t, num_m, num_n, mt, nt);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(bar0 + 8u * (STAGES + s), ph ^ 1u)) {
            timed_out = true;
            break;
          }
          const uint32_t full = bar0 + 8u * s;
          const uint32_t a_dst = base + s * CF::STAGE_BYTES;
          const uint32_t b_dst = a_dst + CF::A_BYTES;
          mbar_arrive_expect_tx(full, CF::STAGE_BYTES);
          tma_load_2d(a_dst, &tmap_a, kb * BK, mt * BM, full);
          if (TB) {
            tma_load_2d(b_dst, &tmap_b, kb * BK, nt * BN, full);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 32; ++j) tma_load_2d(b_dst + j * (BK * 128), &tmap_b, nt * BN + 32 * j, kb * BK, full);
          }
          last_ph[s] = ph;
          pending[s] = true;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (timed_out) {
        // let the copies this thread issued land before the CTA can exit
        for (int i = 0; i < STAGES; ++i)
          if (pending[i]) (void)mbar_wait(bar0 + 8u * i, last_ph[i]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f32acc(kFmtTF32, BM, BN, 0, TB ? 0 : 1);
      int s = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      for (int t = blockIdx.x; t < num_tiles && !timed_out; t += gridDim.x) {
        if (!mbar_wait(bar0 + 8u * (2 * STAGES + 2 + acc), aph ^ 1u)) {
          timed_out = true;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(bar0 + 8u * s, ph)) {
            timed_out = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_src = base + s * CF::STAGE_BYTES;
          const uint32_t b_src = a_src + CF::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            const uint64_t ad = desc_sw128(a_src + 32u * k, 16u, 1024u);
            // B: K-major rows (Bt) or MN-major 32-column slabs, 8 k-rows per MMA
            const uint64_t bd = TB ? desc_sw128(b_src + 32u * k, 16u, 1024u)
                                   : make_desc(b_src + 1024u * k, (uint32_t)(BK * 128), 512u, kLayoutSW128Base32B);
            mma_tf32(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit(bar0 + 8u * (STAGES + s));  // slot s is free once these MMAs have read it
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (timed_out) break;
        mma_commit(bar0 + 8u * (2 * STAGES + acc));  // accumulator ready for the epilogue
        acc ^= 1;
        if (acc == 0) aph ^= 1u;
      }
      mma_commit(done_bar);  // arrives when every MMA of this thread has completed
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int acc = 0;
    uint32_t aph = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int mt, nt;
      tile_coords(t, num_m, num_n, mt, nt);
      const bool ok = __all_sync(0xffffffffu, mbar_wait(bar0 + 8u * (2 * STAGES + acc), aph));
      if (!ok) {
        timed_out = true;
        break;
      }
      tc_fence_after();
      const int row = mt * BM + row_in_tile;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      float* crow = C + (int64_t)row * N;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld32(t_row + (uint32_t)c, v);
        tmem_ld_wait();
        const int col0 = nt * BN + c;
        if (row < M && col0 < N) {
          if (col0 + 32 <= N && (N & 3) == 0) {
            float4* dst = reinterpret_cast<float4*>(crow + col0);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                   __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < N) crow[col0 + j] = __uint_as_float(v[j]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(bar0 + 8u * (2 * STAGES + 2 + acc));
      acc ^= 1;
      if (acc == 0) aph ^= 1u;
    }
  }
  if (timed_out) raise_device_error(DEV_MBAR_TIMEOUT);
  __syncthreads();
  if (warp == 1) {
    (void)__all_sync(0xffffffffu, mbar_wait(done_bar, 0));  // MMAs drained before TMEM is released
    tc_fence_after();
    tmem_dealloc(tmem_base, CF::TMEM_COLS);
  }
}

// TFLOAT32 tensor maps make TMA round each fp32 element to tf32 (nearest) as
// it lands in shared memory; with FLOAT32 maps the tensor core truncates the
// low 13 mantissa bits instead, which biases every product toward zero
// (normwise error 6-7e-4 vs 2.4-3.0e-4 measured on B200 for U[-1,1] inputs).
#ifndef KT_TC_TMA_DTYPE
#define KT_TC_TMA_DTYPE CU_TENSOR_MAP_DATA_TYPE_TFLOAT32
#endif

template <int BN, int STAGES, bool TB>
inline int launch_t(const float* A, const float* B, float* C, int M, int N, int K, cudaStream_t st) {
  using CF = Cfg<BN, STAGES>;
  CUtensorMap ta, tb;
  const CUtensorMapDataType dt = KT_TC_TMA_DTYPE;
  int rc = make_tmap_2d(&ta, dt, 4, A, (uint64_t)M, (uint64_t)K, (uint64_t)K, BK, BM);
  if (rc != KT_OK) return rc;
  if (TB) rc = make_tmap_2d(&tb, dt, 4, B, (uint64_t)N, (uint64_t)K, (uint64_t)K, BK, BN);
  else rc = make_tmap_2d(&tb, dt, 4, B, (uint64_t)K, (uint64_t)N, (uint64_t)N, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  if (rc != KT_OK) return rc;
  auto kern = gemm_tf32_kernel<BN, STAGES, TB>;
  rc = ensure_smem((const void*)kern, CF::SMEM_BYTES, "gemm tf32: smem attribute");
  if (rc != KT_OK) return rc;
  const int64_t num_tiles = (((int64_t)M + BM - 1) / BM) * (((int64_t)N + BN - 1) / BN);
  const int grid = (int)(num_tiles < (int64_t)sm_count() ? num_tiles : (int64_t)sm_count());
  kern<<<grid, THREADS, CF::SMEM_BYTES, st>>>(ta, tb, C, M, N, K);
  return check_launch("gemm tf32");
}

// TMA needs 16-byte aligned bases and row pitches; other shapes run on the
// exact fp32 FFMA kernel instead.
inline bool tma_compatible(const float* A, const float* B, int64_t N, int64_t K, int tb) {
  return aligned16(A) && aligned16(B) && (K % 4 == 0) && (tb ? true : (N % 4 == 0));
}

inline int launch(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int tb, cudaStream_t st) {
  if (M < 0 || N < 0 || K < 0) return fail(KT_ERR_ARG, "gemm: negative shape");
  if (M == 0 || N == 0) return KT_OK;
  if (!C) return fail(KT_ERR_ARG, "gemm: null C");
  // with K == 0 nothing of A or B is read and C = 0
  if (K == 0) return cuda_status(cudaMemsetAsync(C, 0, sizeof(float) * (size_t)M * (size_t)N, st), "gemm: zero C");
  if (!A || !B) return fail(KT_ERR_ARG, "gemm: null pointer");
  // the kernel counts tiles and k-blocks in int: keep M+BM, N+BN, K+BK and the tile count below 2^31
  constexpr int64_t kDimMax = (int64_t)INT32_MAX - 1024;
  if (M > kDimMax || N > kDimMax || K > kDimMax) return fail(KT_ERR_UNSUPPORTED, "gemm tf32: dims >= 2^31 - 1024");
  if (((M + BM - 1) / BM) * ((N + 63) / 64) > (int64_t)INT32_MAX)
    return fail(KT_ERR_UNSUPPORTED, "gemm tf32: more than 2^31 output tiles");
  if (!tma_compatible(A, B, N, K, tb)) return gemm_ffma::launch(A, B, C, M, N, K, tb, st);
  if (tb) return launch_t<KT_TC_BN, KT_TC_STAGES, true>(A, B, C, (int)M, (int)N, (int)K, st);
  return launch_t<KT_TC_BN, KT_TC_STAGES, false>(A, B, C, (int)M, (int)N, (int)K, st);
}

}  // namespace gemm_tf32
}  // namespace kt
