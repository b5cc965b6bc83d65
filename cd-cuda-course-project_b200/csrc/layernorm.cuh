// layernorm.cuh — LayerNorm over the last dimension, fp32, for sm_100a.
//
// y = gamma * (x - mean) / sqrt(var + eps) + beta with the biased variance,
// following the reference oracle `_ref_layernorm` (src/verifier.py:267-274)
// and kernels `layernorm_opt` (src/generator.py:166-213) / `layernorm_naive`
// (src/kernels/baseline_kernels.cu:110-142).
//
// Design (HBM-bound: 2·rows·cols·4 + 2·cols·4 bytes): the row is read once
// into registers with 128-bit streaming loads; mean and variance are two
// block reductions over the register copy (variance from the centred values,
// so no E[x²]-E[x]² cancellation); gamma/beta are small and L2-resident.
// The reference template reads x three times (src/generator.py:182-212).
#pragma once
#include "kt_common.cuh"
#include "rows_staged.cuh"
#include "rows_cluster.cuh"

#ifndef KT_LN_BLOCK
#define KT_LN_BLOCK 256
#endif
#ifndef KT_LN_VPT
#define KT_LN_VPT 4
#endif
#ifndef KT_LN_MINB
#define KT_LN_MINB 1
#endif
#ifndef KT_LN_CLUSTER
#define KT_LN_CLUSTER 1  // > 1: every row split across a cluster of this many CTAs (rows_cluster.cuh)
#endif
#ifndef KT_LN_STAGES
#define KT_LN_STAGES 2  // rows in flight per CTA through the TMA bulk-copy ring (0: register kernel)
#endif

namespace kt {
namespace layernorm {

template <int BLOCK, int VPT, int MINB>
__global__ void __launch_bounds__(BLOCK, MINB)
rows_vec(const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
         float* __restrict__ y, int64_t rows, int cols, float eps) {
  __shared__ float red_a[32];
  __shared__ float red_b[32];
  const int nvec = cols >> 2;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  const float fcols = (float)cols;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * (int64_t)cols);
    float4* yr = reinterpret_cast<float4*>(y + row * (int64_t)cols);
    float4 v[VPT];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < nvec) {
        v[i] = ld_stream4(xr + idx);
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      }
    }
    const float mean = block_sum<BLOCK>(s, red_a) / fcols;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < nvec) {
        v[i].x -= mean; v[i].y -= mean; v[i].z -= mean; v[i].w -= mean;
        q += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
      }
    }
    const float var = block_sum<BLOCK>(q, red_b) / fcols;
    const float rstd = rsqrtf(var + eps);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < nvec) {
        const float4 g = __ldg(g4 + idx);
        const float4 b = __ldg(b4 + idx);
        float4 o;
        o.x = fmaf(v[i].x * rstd, g.x, b.x);
        o.y = fmaf(v[i].y * rstd, g.y, b.y);
        o.z = fmaf(v[i].z * rstd, g.z, b.z);
        o.w = fmaf(v[i].w * rstd, g.w, b.w);
        st_stream4(yr + idx, o);
      }
    }
  }
}

template <int BLOCK, int EPT>
__global__ void __launch_bounds__(BLOCK)
rows_scalar(const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
            float* __restrict__ y, int64_t rows, int cols, float eps) {
  __shared__ float red_a[32];
  __shared__ float red_b[32];
  const float fcols = (float)cols;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * (int64_t)cols;
    float* yr = y + row * (int64_t)cols;
    float v[EPT];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < cols) {
        v[i] = ld_stream1(xr + idx);
        s += v[i];
      }
    }
    const float mean = block_sum<BLOCK>(s, red_a) / fcols;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < cols) {
        v[i] -= mean;
        q += v[i] * v[i];
      }
    }
    const float var = block_sum<BLOCK>(q, red_b) / fcols;
    const float rstd = rsqrtf(var + eps);
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < cols) st_stream1(yr + idx, fmaf(v[i] * rstd, __ldg(gamma + idx), __ldg(beta + idx)));
    }
  }
}

template <int WPB, int EPT>
__global__ void __launch_bounds__(WPB * 32)
rows_warp(const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
          float* __restrict__ y, int64_t rows, int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const float fcols = (float)cols;
  const int64_t first = (int64_t)blockIdx.x * WPB + (threadIdx.x >> 5);
  for (int64_t row = first; row < rows; row += (int64_t)gridDim.x * WPB) {
    const float* xr = x + row * (int64_t)cols;
    float* yr = y + row * (int64_t)cols;
    float v[EPT];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = lane + i * 32;
      if (idx < cols) {
        v[i] = xr[idx];
        s += v[i];
      }
    }
    const float mean = warp_sum(s) / fcols;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = lane + i * 32;
      if (idx < cols) {
        v[i] -= mean;
        q += v[i] * v[i];
      }
    }
    const float rstd = rsqrtf(warp_sum(q) / fcols + eps);
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int idx = lane + i * 32;
      if (idx < cols) yr[idx] = fmaf(v[i] * rstd, gamma[idx], beta[idx]);
    }
  }
}

// Rows longer than the register capacity: Welford-free two-pass over global
// memory (mean pass, centred-variance pass, write pass).
template <int BLOCK>
__global__ void __launch_bounds__(BLOCK)
rows_stream(const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
            float* __restrict__ y, int64_t rows, int64_t cols, float eps) {
  __shared__ double red_a[32];
  __shared__ double red_b[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * cols;
    float* yr = y + row * cols;
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < cols; i += BLOCK) s += (double)xr[i];
    const float mean = (float)(block_sum<BLOCK>(s, red_a) / (double)cols);
    double q = 0.0;
    for (int64_t i = threadIdx.x; i < cols; i += BLOCK) {
      const float d = xr[i] - mean;
      q += (double)(d * d);
    }
    const float rstd = rsqrtf((float)(block_sum<BLOCK>(q, red_b) / (double)cols) + eps);
    for (int64_t i = threadIdx.x; i < cols; i += BLOCK) yr[i] = fmaf((xr[i] - mean) * rstd, gamma[i], beta[i]);
    __syncthreads();
  }
}

inline int launch(const float* x, const float* gamma, const float* beta, float* y, int64_t rows,
                  int64_t cols, float eps, cudaStream_t st) {
  if (rows < 0 || cols < 0) return fail(KT_ERR_ARG, "layernorm: negative shape rows=%lld cols=%lld",
                                        (long long)rows, (long long)cols);
  if (rows == 0 || cols == 0) return KT_OK;
  if (!x || !gamma || !beta || !y) return fail(KT_ERR_ARG, "layernorm: null pointer");
  if (!(eps >= 0.f)) return fail(KT_ERR_ARG, "layernorm: eps must be >= 0");
  if (cols > (int64_t)INT32_MAX) return fail(KT_ERR_UNSUPPORTED, "layernorm: cols > 2^31-1");
  const int c = (int)cols;
  const int64_t max_grid = 1 << 30;
  if (c <= 512) {
    constexpr int WPB = 4;
    const int64_t g64 = (rows + WPB - 1) / WPB;
    const unsigned g = (unsigned)(g64 < max_grid ? g64 : max_grid);
    if (c <= 32) rows_warp<WPB, 1><<<g, WPB * 32, 0, st>>>(x, gamma, beta, y, rows, c, eps);
    else if (c <= 64) rows_warp<WPB, 2><<<g, WPB * 32, 0, st>>>(x, gamma, beta, y, rows, c, eps);
    else if (c <= 128) rows_warp<WPB, 4><<<g, WPB * 32, 0, st>>>(x, gamma, beta, y, rows, c, eps);
    else if (c <= 256) rows_warp<WPB, 8><<<g, WPB * 32, 0, st>>>(x, gamma, beta, y, rows, c, eps);
    else rows_warp<WPB, 16><<<g, WPB * 32, 0, st>>>(x, gamma, beta, y, rows, c, eps);
    return check_launch("layernorm rows_warp");
  }
  constexpr int BLOCK = KT_LN_BLOCK;
  constexpr int VPT = KT_LN_VPT;
  constexpr int CAP = BLOCK * VPT * 4;
  constexpr int CST = KT_LN_STAGES > 0 ? KT_LN_STAGES : 2;  // chunk ring depth of the cluster kernel
  const unsigned g = (unsigned)(rows < max_grid ? rows : max_grid);
  const bool al = (c & 3) == 0 && aligned16(x) && aligned16(y) && aligned16(gamma) && aligned16(beta);
  if (KT_LN_CLUSTER > 1 && al && clustered::fits<BLOCK, VPT, CST>(KT_LN_CLUSTER, c))
    return clustered::launch<BLOCK, VPT, CST, 1>(KT_LN_CLUSTER, x, gamma, beta, y, rows, c, eps, KT_ROWS_BOX, st);
  if (c <= CAP) {
    if ((c & 3) == 0 && aligned16(x) && aligned16(y) && aligned16(gamma) && aligned16(beta)) {
      if (KT_LN_STAGES > 0 && staged::smem_bytes<(KT_LN_STAGES > 0 ? KT_LN_STAGES : 1)>(c) <= 200 * 1024) {
        constexpr int ST = KT_LN_STAGES > 0 ? KT_LN_STAGES : 1;
        auto kern = staged::layernorm_rows<BLOCK, VPT, ST>;
        const size_t smem = staged::smem_bytes<ST>(c);
        int grid = 0;
        int rc = staged::launch_grid(kern, BLOCK, smem, rows, &grid);
        if (rc != KT_OK) return rc;
        kern<<<grid, BLOCK, smem, st>>>(x, gamma, beta, y, rows, c, eps);
        return check_launch("layernorm staged rows");
      }
      rows_vec<BLOCK, VPT, KT_LN_MINB><<<g, BLOCK, 0, st>>>(x, gamma, beta, y, rows, c, eps);
      return check_launch("layernorm rows_vec");
    }
    rows_scalar<BLOCK, VPT * 4><<<g, BLOCK, 0, st>>>(x, gamma, beta, y, rows, c, eps);
    return check_launch("layernorm rows_scalar");
  }
  // wider than one CTA holds: split each row across a cluster when the chunks fit
  if (al) {
    const int C = clustered::smallest_fit<BLOCK, VPT, CST>(c);
    if (C > 0) return clustered::launch<BLOCK, VPT, CST, 1>(C, x, gamma, beta, y, rows, c, eps, KT_ROWS_BOX, st);
  }
  rows_stream<BLOCK><<<g, BLOCK, 0, st>>>(x, gamma, beta, y, rows, cols, eps);
  return check_launch("layernorm rows_stream");
}

}  // namespace layernorm
}  // namespace kt
