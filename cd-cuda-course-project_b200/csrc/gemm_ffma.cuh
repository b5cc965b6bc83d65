// gemm_ffma.cuh — exact fp32 SIMT GEMM (FFMA), for sm_100a.
//
// C = A·B (B row-major K×N) or, with transpose_b, C = A·Bt^T (B holds Bt,
// row-major N×K). This is the reference `matmul_opt` template
// (src/generator.py:40-70, B loads at :286-299) restated as a
// register-blocked kernel: the reference computes one output per thread from
// T×T shared tiles (one FMA per two shared loads); here each of 256 threads
// owns an 8×8 block of a 128×128 CTA tile, so every k step does 64 FMAs for
// four 128-bit shared loads. Tiles are double-buffered through registers
// (one __syncthreads per k tile). Accumulation order per output is k-ascending
// fp32 FMA, like the reference's inner loop.
#pragma once
#include "kt_common.cuh"

// k tile of the wide kernel: the tuner's bk when a variant sets it, else 8 (measured
// 51.2 against 48.5 TFLOP/s with 16 at 8192^3)
#ifdef KT_FFMA_BK
#define KT_FFMA_WIDE_BK (KT_FFMA_BK >= 16 ? 16 : 8)
#else
#define KT_FFMA_WIDE_BK 8
#endif
#ifndef KT_FFMA_BK
#define KT_FFMA_BK 16
#endif
#ifndef KT_FFMA_MINB
#define KT_FFMA_MINB 2
#endif
#ifndef KT_FFMA_WIDE
#define KT_FFMA_WIDE 1  // 1: 128x256 CTA tile, 8x16 outputs per thread (sgemm_128x256); 0: 128x128, 8x8
#endif
#ifndef KT_FFMA_X2
#define KT_FFMA_X2 0  // 0: scalar FFMA (sgemm_128x128); 1: packed fma.rn.f32x2 kernel (sgemm_x2_128x128), measured slower
#endif

namespace kt {
namespace gemm_ffma {

constexpr int BM = 128, BN = 128, THREADS = 256;
constexpr int PAD = 4;  // row padding of the k-major shared tiles (bank spread)

// Load 4 consecutive elements along the contiguous dim of a row-major matrix
// (rows × cols, leading dim ld), zero outside. VEC: 16-byte aligned path.
template <bool VEC>
__device__ __forceinline__ float4 load4(const float* __restrict__ p, int64_t row, int64_t col, int64_t rows,
                                        int64_t cols, int64_t ld) {
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (row >= rows) return v;
  const float* q = p + row * ld + col;
  if (VEC) {
    if (col + 3 < cols) return __ldg(reinterpret_cast<const float4*>(q));
  }
  if (col + 0 < cols) v.x = __ldg(q + 0);
  if (col + 1 < cols) v.y = __ldg(q + 1);
  if (col + 2 < cols) v.z = __ldg(q + 2);
  if (col + 3 < cols) v.w = __ldg(q + 3);
  return v;
}

template <bool TB, bool VEC, int BK, int MINB>
__global__ void __launch_bounds__(THREADS, MINB)
sgemm_128x128(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int64_t M,
              int64_t N, int64_t K) {
  static_assert(BK == 8 || BK == 16 || BK == 32, "BK");
  // k-major tiles: As[k][m], Bs[k][n]
  __shared__ __align__(16) float As[2][BK][BM + PAD];
  __shared__ __align__(16) float Bs[2][BK][BN + PAD];
  constexpr int AV = BM * BK / 4 / THREADS;  // float4 per thread for a row-major-along-k tile
  constexpr int BV = BN * BK / 4 / THREADS;  // float4 per thread for a k-rows tile
  static_assert(AV >= 1 && BV >= 1, "tile/threads");
  constexpr int KQ = BK / 4;                  // float4 per tile row along k
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;

  float4 ra[AV], rb[BV];
  auto load_tile = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < AV; ++i) {
      const int e = tid + i * THREADS;
      const int r = e / KQ, kq = (e % KQ) * 4;
      ra[i] = load4<VEC>(A, m0 + r, k0 + kq, M, K, K);
    }
#pragma unroll
    for (int i = 0; i < BV; ++i) {
      const int e = tid + i * THREADS;
      if (TB) {
        const int r = e / KQ, kq = (e % KQ) * 4;
        rb[i] = load4<VEC>(B, n0 + r, k0 + kq, N, K, K);
      } else {
        const int kr = e / (BN / 4), nq = (e % (BN / 4)) * 4;
        rb[i] = load4<VEC>(B, k0 + kr, n0 + nq, K, N, N);
      }
    }
  };
  auto store_tile = [&](int buf) {
#pragma unroll
    for (int i = 0; i < AV; ++i) {
      const int e = tid + i * THREADS;
      const int r = e / KQ, kq = (e % KQ) * 4;
      As[buf][kq + 0][r] = ra[i].x;
      As[buf][kq + 1][r] = ra[i].y;
      As[buf][kq + 2][r] = ra[i].z;
      As[buf][kq + 3][r] = ra[i].w;
    }
#pragma unroll
    for (int i = 0; i < BV; ++i) {
      const int e = tid + i * THREADS;
      if (TB) {
        const int r = e / KQ, kq = (e % KQ) * 4;
        Bs[buf][kq + 0][r] = rb[i].x;
        Bs[buf][kq + 1][r] = rb[i].y;
        Bs[buf][kq + 2][r] = rb[i].z;
        Bs[buf][kq + 3][r] = rb[i].w;
      } else {
        const int kr = e / (BN / 4), nq = (e % (BN / 4)) * 4;
        *reinterpret_cast<float4*>(&Bs[buf][kr][nq]) = rb[i];
      }
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int64_t nk = (K + BK - 1) / BK;
  load_tile(0);
  store_tile(0);
  __syncthreads();
  for (int64_t t = 0; t < nk; ++t) {
    const int cur = (int)(t & 1);
    if (t + 1 < nk) load_tile((t + 1) * BK);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4 + 64]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4 + 64]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (t + 1 < nk) store_tile(cur ^ 1);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (row >= M) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t col = n0 + h * 64 + tx * 4;
      float* c = C + row * N + col;
      const float4 v = make_float4(acc[i][h * 4 + 0], acc[i][h * 4 + 1], acc[i][h * 4 + 2], acc[i][h * 4 + 3]);
      if (VEC && col + 3 < N) {
        *reinterpret_cast<float4*>(c) = v;
      } else {
        if (col + 0 < N) c[0] = v.x;
        if (col + 1 < N) c[1] = v.y;
        if (col + 2 < N) c[2] = v.z;
        if (col + 3 < N) c[3] = v.w;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Wide variant: a 128x256 CTA tile, 256 threads, 8x16 outputs per thread
// (rows ty*4+{0..3} and 64+ty*4+{0..3}, columns tx*4+{0..3} + {0, 64, 128, 192}).
// Every k step is 128 FMAs for six 128-bit shared loads (64 for four in the
// 128x128 kernel): a larger share of the issue slots goes to the FMA pipe. One
// CTA per SM (about 170 registers per thread); k-major shared tiles
// double-buffered through registers, as in sgemm_128x128. Results are
// bit-identical to sgemm_128x128 (one fp32 fma per k, k ascending).
// ---------------------------------------------------------------------------
constexpr int WBN = 256;

template <int BK>
constexpr size_t wide_smem_bytes() {
  return sizeof(float) * 2 * (size_t)BK * ((BM + PAD) + (WBN + PAD));
}

template <bool TB, bool VEC, int BK>
__global__ void __launch_bounds__(THREADS, 1)
sgemm_128x256(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int64_t M, int64_t N,
              int64_t K) {
  static_assert(BK == 8 || BK == 16, "BK");
  // dynamic shared memory: [2][BK][BM + PAD] A tiles, then [2][BK][WBN + PAD] B tiles
  extern __shared__ __align__(16) float wide_smem[];
  auto As = reinterpret_cast<float(*)[BK][BM + PAD]>(wide_smem);
  auto Bs = reinterpret_cast<float(*)[BK][WBN + PAD]>(wide_smem + 2 * BK * (BM + PAD));
  constexpr int AV = BM * BK / 4 / THREADS;
  constexpr int BV = WBN * BK / 4 / THREADS;
  static_assert(AV >= 1 && BV >= 1, "tile/threads");
  constexpr int KQ = BK / 4;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * WBN;

  float4 ra[AV], rb[BV];
  auto load_tile = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < AV; ++i) {
      const int e = tid + i * THREADS;
      const int r = e / KQ, kq = (e % KQ) * 4;
      ra[i] = load4<VEC>(A, m0 + r, k0 + kq, M, K, K);
    }
#pragma unroll
    for (int i = 0; i < BV; ++i) {
      const int e = tid + i * THREADS;
      if (TB) {
        const int r = e / KQ, kq = (e % KQ) * 4;
        rb[i] = load4<VEC>(B, n0 + r, k0 + kq, N, K, K);
      } else {
        const int kr = e / (WBN / 4), nq = (e % (WBN / 4)) * 4;
        rb[i] = load4<VEC>(B, k0 + kr, n0 + nq, K, N, N);
      }
    }
  };
  auto store_tile = [&](int buf) {
#pragma unroll
    for (int i = 0; i < AV; ++i) {
      const int e = tid + i * THREADS;
      const int r = e / KQ, kq = (e % KQ) * 4;
      As[buf][kq + 0][r] = ra[i].x;
      As[buf][kq + 1][r] = ra[i].y;
      As[buf][kq + 2][r] = ra[i].z;
      As[buf][kq + 3][r] = ra[i].w;
    }
#pragma unroll
    for (int i = 0; i < BV; ++i) {
      const int e = tid + i * THREADS;
      if (TB) {
        const int r = e / KQ, kq = (e % KQ) * 4;
        Bs[buf][kq + 0][r] = rb[i].x;
        Bs[buf][kq + 1][r] = rb[i].y;
        Bs[buf][kq + 2][r] = rb[i].z;
        Bs[buf][kq + 3][r] = rb[i].w;
      } else {
        const int kr = e / (WBN / 4), nq = (e % (WBN / 4)) * 4;
        *reinterpret_cast<float4*>(&Bs[buf][kr][nq]) = rb[i];
      }
    }
  };

  float acc[8][16];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[i][j] = 0.f;

  const int64_t nk = (K + BK - 1) / BK;
  load_tile(0);
  store_tile(0);
  __syncthreads();
  for (int64_t t = 0; t < nk; ++t) {
    const int cur = (int)(t & 1);
    if (t + 1 < nk) load_tile((t + 1) * BK);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4 + 64]);
      float b[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 bq = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4 + 64 * q]);
        b[4 * q + 0] = bq.x;
        b[4 * q + 1] = bq.y;
        b[4 * q + 2] = bq.z;
        b[4 * q + 3] = bq.w;
      }
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (t + 1 < nk) store_tile(cur ^ 1);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (row >= M) continue;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int64_t col = n0 + q * 64 + tx * 4;
      float* c = C + row * N + col;
      const float4 v = make_float4(acc[i][4 * q + 0], acc[i][4 * q + 1], acc[i][4 * q + 2], acc[i][4 * q + 3]);
      if (VEC && col + 3 < N) {
        *reinterpret_cast<float4*>(c) = v;
      } else {
        if (col + 0 < N) c[0] = v.x;
        if (col + 1 < N) c[1] = v.y;
        if (col + 2 < N) c[2] = v.z;
        if (col + 3 < N) c[3] = v.w;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Packed variant: the same 128x128 CTA tile and 8x8 outputs per thread, with
// the FMAs issued as fma.rn.f32x2 (two fp32 FMAs per lane per instruction, a
// Blackwell instruction). Each packed FMA updates two outputs of one row:
//   {c[i][j], c[i][j+1]} += {a[i], a[i]} * {b[j], b[j+1]}
// so A is kept in shared memory with every value stored twice ({a, a} pairs)
// and both operands come out of 128-bit shared loads ready to use. One k step
// is 32 packed FMAs and 6 shared loads per thread, against 64 FMAs and 4 loads
// in sgemm_128x128: half the issue slots for the same FMA-pipe work. Every
// output is still one fp32 fma.rn per k in k-ascending order, so results are
// bit-identical to sgemm_128x128.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fma2(unsigned long long& c, unsigned long long a, unsigned long long b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c) : "l"(a), "l"(b));
}

template <int BK>
struct X2Smem {
  static constexpr int A_ROW = 2 * BM + 4;  // floats per k row of the duplicated A tile (16-byte multiple)
  static constexpr int B_ROW = BN + 4;
  static constexpr int A_FLOATS = 2 * BK * A_ROW;  // two buffers
  static constexpr int B_FLOATS = 2 * BK * B_ROW;
  static constexpr size_t BYTES = sizeof(float) * (size_t)(A_FLOATS + B_FLOATS);
};

template <bool TB, bool VEC, int BK, int MINB>
__global__ void __launch_bounds__(THREADS, MINB)
sgemm_x2_128x128(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int64_t M,
                 int64_t N, int64_t K) {
  static_assert(BK == 8 || BK == 16 || BK == 32, "BK");
  using SM = X2Smem<BK>;
  extern __shared__ __align__(16) float x2_smem[];
  float* As = x2_smem;                  // [2][BK][A_ROW]: {a, a} pairs, k-major
  float* Bs = x2_smem + SM::A_FLOATS;   // [2][BK][B_ROW], k-major
  constexpr int AV = BM * BK / 4 / THREADS;
  constexpr int BV = BN * BK / 4 / THREADS;
  static_assert(AV >= 1 && BV >= 1, "tile/threads");
  constexpr int KQ = BK / 4;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;

  float4 ra[AV], rb[BV];
  auto load_tile = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < AV; ++i) {
      const int e = tid + i * THREADS;
      const int r = e / KQ, kq = (e % KQ) * 4;
      ra[i] = load4<VEC>(A, m0 + r, k0 + kq, M, K, K);
    }
#pragma unroll
    for (int i = 0; i < BV; ++i) {
      const int e = tid + i * THREADS;
      if (TB) {
        const int r = e / KQ, kq = (e % KQ) * 4;
        rb[i] = load4<VEC>(B, n0 + r, k0 + kq, N, K, K);
      } else {
        const int kr = e / (BN / 4), nq = (e % (BN / 4)) * 4;
        rb[i] = load4<VEC>(B, k0 + kr, n0 + nq, K, N, N);
      }
    }
  };
  auto store_tile = [&](int buf) {
    float* as = As + buf * BK * SM::A_ROW;
    float* bs = Bs + buf * BK * SM::B_ROW;
#pragma unroll
    for (int i = 0; i < AV; ++i) {
      const int e = tid + i * THREADS;
      const int r = e / KQ, kq = (e % KQ) * 4;
      *reinterpret_cast<float2*>(&as[(kq + 0) * SM::A_ROW + 2 * r]) = make_float2(ra[i].x, ra[i].x);
      *reinterpret_cast<float2*>(&as[(kq + 1) * SM::A_ROW + 2 * r]) = make_float2(ra[i].y, ra[i].y);
      *reinterpret_cast<float2*>(&as[(kq + 2) * SM::A_ROW + 2 * r]) = make_float2(ra[i].z, ra[i].z);
      *reinterpret_cast<float2*>(&as[(kq + 3) * SM::A_ROW + 2 * r]) = make_float2(ra[i].w, ra[i].w);
    }
#pragma unroll
    for (int i = 0; i < BV; ++i) {
      const int e = tid + i * THREADS;
      if (TB) {
        const int r = e / KQ, kq = (e % KQ) * 4;
        bs[(kq + 0) * SM::B_ROW + r] = rb[i].x;
        bs[(kq + 1) * SM::B_ROW + r] = rb[i].y;
        bs[(kq + 2) * SM::B_ROW + r] = rb[i].z;
        bs[(kq + 3) * SM::B_ROW + r] = rb[i].w;
      } else {
        const int kr = e / (BN / 4), nq = (e % (BN / 4)) * 4;
        *reinterpret_cast<float4*>(&bs[kr * SM::B_ROW + nq]) = rb[i];
      }
    }
  };

  // acc[i][p] = {c[row i][col 2p], c[row i][col 2p+1]} over this thread's 8 rows x 8 columns
  unsigned long long acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int p = 0; p < 4; ++p) acc[i][p] = 0ull;

  const int64_t nk = (K + BK - 1) / BK;
  load_tile(0);
  store_tile(0);
  __syncthreads();
  for (int64_t t = 0; t < nk; ++t) {
    const int cur = (int)(t & 1);
    if (t + 1 < nk) load_tile((t + 1) * BK);
    const float* as = As + cur * BK * SM::A_ROW;
    const float* bs = Bs + cur * BK * SM::B_ROW;
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      const ulonglong2 a0 = *reinterpret_cast<const ulonglong2*>(&as[k * SM::A_ROW + 2 * (ty * 4)]);
      const ulonglong2 a1 = *reinterpret_cast<const ulonglong2*>(&as[k * SM::A_ROW + 2 * (ty * 4) + 4]);
      const ulonglong2 a2 = *reinterpret_cast<const ulonglong2*>(&as[k * SM::A_ROW + 2 * (64 + ty * 4)]);
      const ulonglong2 a3 = *reinterpret_cast<const ulonglong2*>(&as[k * SM::A_ROW + 2 * (64 + ty * 4) + 4]);
      const ulonglong2 b0 = *reinterpret_cast<const ulonglong2*>(&bs[k * SM::B_ROW + tx * 4]);
      const ulonglong2 b1 = *reinterpret_cast<const ulonglong2*>(&bs[k * SM::B_ROW + 64 + tx * 4]);
      const unsigned long long a[8] = {a0.x, a0.y, a1.x, a1.y, a2.x, a2.y, a3.x, a3.y};
      const unsigned long long b[4] = {b0.x, b0.y, b1.x, b1.y};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int p = 0; p < 4; ++p) fma2(acc[i][p], a[i], b[p]);
    }
    if (t + 1 < nk) store_tile(cur ^ 1);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (row >= M) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t col = n0 + h * 64 + tx * 4;
      float* c = C + row * N + col;
      const float2 lo = *reinterpret_cast<const float2*>(&acc[i][2 * h]);
      const float2 hi = *reinterpret_cast<const float2*>(&acc[i][2 * h + 1]);
      const float4 v = make_float4(lo.x, lo.y, hi.x, hi.y);
      if (VEC && col + 3 < N) {
        *reinterpret_cast<float4*>(c) = v;
      } else {
        if (col + 0 < N) c[0] = v.x;
        if (col + 1 < N) c[1] = v.y;
        if (col + 2 < N) c[2] = v.z;
        if (col + 3 < N) c[3] = v.w;
      }
    }
  }
}

template <bool TB, bool VEC>
inline int launch_t(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, cudaStream_t st) {
  dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM));
  if constexpr (KT_FFMA_WIDE != 0) {
    dim3 wgrid((unsigned)((N + WBN - 1) / WBN), (unsigned)((M + BM - 1) / BM));
    constexpr int WBK = KT_FFMA_WIDE_BK;
    auto kern = sgemm_128x256<TB, VEC, WBK>;
    constexpr size_t smem = wide_smem_bytes<WBK>();
    int rc = ensure_smem((const void*)kern, smem, "gemm ffma: smem attribute");
    if (rc != KT_OK) return rc;
    kern<<<wgrid, THREADS, smem, st>>>(A, B, C, M, N, K);
  } else if constexpr (KT_FFMA_X2 != 0) {
    auto kern = sgemm_x2_128x128<TB, VEC, KT_FFMA_BK, KT_FFMA_MINB>;
    constexpr size_t smem = X2Smem<KT_FFMA_BK>::BYTES;
    int rc = ensure_smem((const void*)kern, smem, "gemm ffma: smem attribute");
    if (rc != KT_OK) return rc;
    kern<<<grid, THREADS, smem, st>>>(A, B, C, M, N, K);
  } else {
    sgemm_128x128<TB, VEC, KT_FFMA_BK, KT_FFMA_MINB><<<grid, THREADS, 0, st>>>(A, B, C, M, N, K);
  }
  return KT_OK;
}

inline int launch(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int tb,
                  cudaStream_t st) {
  if (M < 0 || N < 0 || K < 0) return fail(KT_ERR_ARG, "gemm: negative shape");
  if (M == 0 || N == 0) return KT_OK;
  if (!C) return fail(KT_ERR_ARG, "gemm: null C");
  // with K == 0 nothing of A or B is read and C = 0
  if (K == 0) return cuda_status(cudaMemsetAsync(C, 0, sizeof(float) * (size_t)M * (size_t)N, st), "gemm: zero C");
  if (!A || !B) return fail(KT_ERR_ARG, "gemm: null pointer");
  if ((M + BM - 1) / BM > 65535) return fail(KT_ERR_UNSUPPORTED, "gemm: M too large for the grid");
  const bool vec = aligned16(A) && aligned16(B) && aligned16(C) && (K % 4 == 0) && (tb ? true : (N % 4 == 0)) &&
                   (N % 4 == 0);
  int rc;
  if (tb) rc = vec ? launch_t<true, true>(A, B, C, M, N, K, st) : launch_t<true, false>(A, B, C, M, N, K, st);
  else rc = vec ? launch_t<false, true>(A, B, C, M, N, K, st) : launch_t<false, false>(A, B, C, M, N, K, st);
  if (rc != KT_OK) return rc;
  return check_launch("gemm ffma");
}

}  // namespace gemm_ffma
}  // namespace kt
