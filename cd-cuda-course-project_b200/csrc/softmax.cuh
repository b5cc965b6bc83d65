// softmax.cuh — numerically stable row softmax, fp32, for sm_100a.
//
// Computes y[r,:] = exp(x[r,:] - max_r) / sum_r, the formula of the
// reference's oracle `_ref_softmax` (src/verifier.py:245-250) and kernels
// `softmax_opt` (src/generator.py:110-153) / `softmax_naive`
// (src/kernels/baseline_kernels.cu:52-77).
//
// Design (HBM-bound: algorithmic traffic 2·rows·cols·4 bytes):
//   * rows_vec   — one CTA per row; the whole row stays in registers
//                  (BLOCK threads × VPT float4 each), so x is read once and y
//                  written once with 128-bit streaming accesses. The reference
//                  template makes 3 global passes (5·R·C·4 bytes).
//   * rows_scalar— same, for rows whose start is not 16-byte aligned.
//   * rows_warp  — one warp per row for short rows (cols <= 512).
//   * clustered  — rows_cluster.cuh: each row split across a thread-block
//                  cluster (DSMEM exchange of partial max / sum), one read + one
//                  write for rows up to 8x the register capacity; also a tuner
//                  option (cluster_size) for rows that one CTA could hold.
//   * rows_stream— rows longer than that, or not 16-byte aligned: one online
//                  (max, sum) pass, then one normalising pass (2 reads + 1 write).
// expf is CUDA's accurate expf (no fast-math); the result is scaled by the
// reciprocal of the row sum.
#pragma once
#include "kt_common.cuh"
#include "rows_staged.cuh"
#include "rows_cluster.cuh"

#ifndef KT_SOFTMAX_BLOCK
#define KT_SOFTMAX_BLOCK 256
#endif
#ifndef KT_SOFTMAX_VPT
#define KT_SOFTMAX_VPT 4
#endif
#ifndef KT_SOFTMAX_MINB
#define KT_SOFTMAX_MINB 1
#endif
#ifndef KT_SOFTMAX_CLUSTER
#define KT_SOFTMAX_CLUSTER 1  // > 1: every row split across a cluster of this many CTAs (rows_cluster.cuh)
#endif
#ifndef KT_SOFTMAX_STAGES
#define KT_SOFTMAX_STAGES 2  // rows in flight per CTA through the TMA bulk-copy ring (0: register kernel)
#endif

namespace kt {
namespace softmax {

template <int BLOCK, int VPT, int MINB>
__global__ void __launch_bounds__(BLOCK, MINB)
rows_vec(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int cols) {
  __shared__ float red_max[32];
  __shared__ float red_sum[32];
  const int nvec = cols >> 2;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * (int64_t)cols);
    float4* yr = reinterpret_cast<float4*>(y + row * (int64_t)cols);
    float4 v[VPT];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < nvec) {
        v[i] = ld_stream4(xr + idx);
        m = fmaxf(m, max4(v[i]));
      }
    }
    m = block_max<BLOCK>(m, red_max);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < nvec) {
        v[i].x = expf(v[i].x - m);
        v[i].y = expf(v[i].y - m);
        v[i].z = expf(v[i].z - m);
        v[i].w = expf(v[i].w - m);
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      }
    }
    s = block_sum<BLOCK>(s, red_sum);
    const float inv = 1.0f / s;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < nvec) {
        st_stream4(yr + idx, make_float4(v[i].x * inv, v[i].y * inv, v[i].z * inv, v[i].w * inv));
      }
    }
  }
}

template <int BLOCK, int EPT>
__global__ void __launch_bounds__(BLOCK)
rows_scalar(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int cols) {
  __shared__ float red_max[32];
  __shared__ float red_sum[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * (int64_t)cols;
    float* yr = y + row * (int64_t)cols;
    float v[EPT];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < cols) {
        v[i] = ld_stream1(xr + idx);
        m = fmaxf(m, v[i]);
      }
    }
    m = block_max<BLOCK>(m, red_max);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < cols) {
        v[i] = expf(v[i] - m);
        s += v[i];
      }
    }
    s = block_sum<BLOCK>(s, red_sum);
    const float inv = 1.0f / s;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < cols) st_stream1(yr + idx, v[i] * inv);
    }
  }
}

// One warp per row; WPB warps per CTA; EPT elements per lane (cols <= 32*EPT).
template <int WPB, int EPT>
__global__ void __launch_bounds__(WPB * 32)
rows_warp(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int cols) {
  const int lane = threadIdx.x & 31;
  const int64_t first = (int64_t)blockIdx.x * WPB + (threadIdx.x >> 5);
  for (int64_t row = first; row < rows; row += (int64_t)gridDim.x * WPB) {
    const float* xr = x + row * (int64_t)cols;
    float* yr = y + row * (int64_t)cols;
    float v[EPT];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = lane + i * 32;
      if (idx < cols) {
        v[i] = xr[idx];
        m = fmaxf(m, v[i]);
      }
    }
    m = warp_max(m);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = lane + i * 32;
      if (idx < cols) {
        v[i] = expf(v[i] - m);
        s += v[i];
      }
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = lane + i * 32;
      if (idx < cols) yr[idx] = v[i] * inv;
    }
  }
}

// Rows too long for registers: online (max, sum) in one read, then write.
template <int BLOCK>
__global__ void __launch_bounds__(BLOCK)
rows_stream(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int64_t cols) {
  __shared__ float red_max[32];
  __shared__ float red_sum[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * cols;
    float* yr = y + row * cols;
    float m = -INFINITY, s = 0.f;
    for (int64_t i = threadIdx.x; i < cols; i += BLOCK) {
      const float v = xr[i];
      if (v > m) {
        s = s * expf(m - v) + 1.0f;
        m = v;
      } else {
        s += expf(v - m);
      }
    }
    const float gm = block_max<BLOCK>(m, red_max);
    const float scaled = (m == -INFINITY) ? 0.f : s * expf(m - gm);
    const float total = block_sum<BLOCK>(scaled, red_sum);
    const float inv = 1.0f / total;
    for (int64_t i = threadIdx.x; i < cols; i += BLOCK) yr[i] = expf(xr[i] - gm) * inv;
    __syncthreads();
  }
}

// Host-side dispatcher. Grid: one CTA (or warp) per row, capped; the kernels
// stride over the remaining rows.
inline int launch(const float* x, float* y, int64_t rows, int64_t cols, cudaStream_t st) {
  if (rows < 0 || cols < 0) return fail(KT_ERR_ARG, "softmax: negative shape rows=%lld cols=%lld",
                                        (long long)rows, (long long)cols);
  if (rows == 0 || cols == 0) return KT_OK;
  if (x == nullptr || y == nullptr) return fail(KT_ERR_ARG, "softmax: null pointer");
  if (cols > (int64_t)INT32_MAX) return fail(KT_ERR_UNSUPPORTED, "softmax: cols > 2^31-1");
  const int c = (int)cols;
  const int64_t max_grid = 1 << 30;
  if (c <= 512) {
    constexpr int WPB = 4;
    const int64_t g64 = (rows + WPB - 1) / WPB;
    const unsigned g = (unsigned)(g64 < max_grid ? g64 : max_grid);
    if (c <= 32) rows_warp<WPB, 1><<<g, WPB * 32, 0, st>>>(x, y, rows, c);
    else if (c <= 64) rows_warp<WPB, 2><<<g, WPB * 32, 0, st>>>(x, y, rows, c);
    else if (c <= 128) rows_warp<WPB, 4><<<g, WPB * 32, 0, st>>>(x, y, rows, c);
    else if (c <= 256) rows_warp<WPB, 8><<<g, WPB * 32, 0, st>>>(x, y, rows, c);
    else rows_warp<WPB, 16><<<g, WPB * 32, 0, st>>>(x, y, rows, c);
    return check_launch("softmax rows_warp");
  }
  constexpr int BLOCK = KT_SOFTMAX_BLOCK;
  constexpr int VPT = KT_SOFTMAX_VPT;
  constexpr int CAP = BLOCK * VPT * 4;
  constexpr int CST = KT_SOFTMAX_STAGES > 0 ? KT_SOFTMAX_STAGES : 2;  // chunk ring depth of the cluster kernel
  const unsigned g = (unsigned)(rows < max_grid ? rows : max_grid);
  const bool al = (c & 3) == 0 && aligned16(x) && aligned16(y);
  if (KT_SOFTMAX_CLUSTER > 1 && al && clustered::fits<BLOCK, VPT, CST>(KT_SOFTMAX_CLUSTER, c))
    return clustered::launch<BLOCK, VPT, CST, 0>(KT_SOFTMAX_CLUSTER, x, nullptr, nullptr, y, rows, c, 0.f,
                                                 KT_ROWS_BOX, st);
  if (c <= CAP) {
    if ((c & 3) == 0 && aligned16(x) && aligned16(y)) {
      if (KT_SOFTMAX_STAGES > 0 && staged::smem_bytes<(KT_SOFTMAX_STAGES > 0 ? KT_SOFTMAX_STAGES : 1)>(c) <= 200 * 1024) {
        constexpr int ST = KT_SOFTMAX_STAGES > 0 ? KT_SOFTMAX_STAGES : 1;
        auto kern = staged::softmax_rows<BLOCK, VPT, ST>;
        const size_t smem = staged::smem_bytes<ST>(c);
        int grid = 0;
        int rc = staged::launch_grid(kern, BLOCK, smem, rows, &grid);
        if (rc != KT_OK) return rc;
        kern<<<grid, BLOCK, smem, st>>>(x, y, rows, c);
        return check_launch("softmax staged rows");
      }
      rows_vec<BLOCK, VPT, KT_SOFTMAX_MINB><<<g, BLOCK, 0, st>>>(x, y, rows, c);
      return check_launch("softmax rows_vec");
    }
    rows_scalar<BLOCK, VPT * 4><<<g, BLOCK, 0, st>>>(x, y, rows, c);
    return check_launch("softmax rows_scalar");
  }
  // wider than one CTA holds: split each row across a cluster when the chunks fit
  if (al) {
    const int C = clustered::smallest_fit<BLOCK, VPT, CST>(c);
    if (C > 0) return clustered::launch<BLOCK, VPT, CST, 0>(C, x, nullptr, nullptr, y, rows, c, 0.f, KT_ROWS_BOX, st);
  }
  rows_stream<BLOCK><<<g, BLOCK, 0, st>>>(x, y, rows, cols);
  return check_launch("softmax rows_stream");
}

}  // namespace softmax
}  // namespace kt
