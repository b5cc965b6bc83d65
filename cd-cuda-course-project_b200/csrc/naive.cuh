// naive.cuh — deliberately naive GPU baselines for the Welch-t comparison.
//
// These restate the algorithms of the reference's naive kernels
// (src/kernels/baseline_kernels.cu:32-181; timed by
// src/kernels/benchmark_runner.cu:74-104 with the launch shapes of :179-208):
// one thread per output row or element, serial loops over global memory,
// no tiling and no vector loads. They exist only as the "before" point of the
// tuner's speed-up statistics, never as a fallback for the tuned ops.
#pragma once
#include "kt_common.cuh"

namespace kt {
namespace naive {

// One thread per row, launched as <<<rows, 1>>> like the reference
// (src/kernels/benchmark_runner.cu:186-189): max pass, exp+sum pass, divide pass.
__global__ void softmax_rows(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int64_t cols) {
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    if (threadIdx.x != 0) continue;
    const float* xr = x + row * cols;
    float* yr = y + row * cols;
    float m = xr[0];
    for (int64_t i = 1; i < cols; ++i) m = fmaxf(m, xr[i]);
    float s = 0.f;
    for (int64_t i = 0; i < cols; ++i) {
      yr[i] = expf(xr[i] - m);
      s += yr[i];
    }
    for (int64_t i = 0; i < cols; ++i) yr[i] /= s;
  }
}

__global__ void layernorm_rows(const float* __restrict__ x, const float* __restrict__ gamma,
                               const float* __restrict__ beta, float* __restrict__ y, int64_t rows,
                               int64_t cols, float eps) {
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    if (threadIdx.x != 0) continue;
    const float* xr = x + row * cols;
    float* yr = y + row * cols;
    float mean = 0.f;
    for (int64_t i = 0; i < cols; ++i) mean += xr[i];
    mean /= (float)cols;
    float var = 0.f;
    for (int64_t i = 0; i < cols; ++i) {
      const float d = xr[i] - mean;
      var += d * d;
    }
    var /= (float)cols;
    const float inv_std = rsqrtf(var + eps);
    for (int64_t i = 0; i < cols; ++i) yr[i] = gamma[i] * (xr[i] - mean) * inv_std + beta[i];
  }
}

// Interleaved-addressing shared-memory tree with the divergent modulo test,
// one partial per 256-thread block; a single thread then adds the partials.
__global__ void reduce_partials(const float* __restrict__ x, int64_t n, float* __restrict__ partials) {
  extern __shared__ float sdata[];
  const int tid = threadIdx.x;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + tid;
  sdata[tid] = gid < n ? x[gid] : 0.f;
  __syncthreads();
  for (int stride = 1; stride < (int)blockDim.x; stride *= 2) {
    if (tid % (2 * stride) == 0) sdata[tid] += sdata[tid + stride];
    __syncthreads();
  }
  if (tid == 0) partials[blockIdx.x] = sdata[0];
}

__global__ void reduce_final(const float* __restrict__ partials, int64_t count, double* out64, float* out32) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double s = 0.0;
  for (int64_t i = 0; i < count; ++i) s += (double)partials[i];
  *out64 = s;
  if (out32) *out32 = (float)s;
}

// One thread per C element (16×16 blocks), B read down a column.
__global__ void gemm_elem(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C,
                          int64_t M, int64_t N, int64_t K, int transpose_b) {
  const int64_t row = (int64_t)blockIdx.y * blockDim.y + threadIdx.y;
  const int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= M || col >= N) return;
  float s = 0.f;
  if (transpose_b) {
    for (int64_t k = 0; k < K; ++k) s += A[row * K + k] * B[col * K + k];
  } else {
    for (int64_t k = 0; k < K; ++k) s += A[row * K + k] * B[k * N + col];
  }
  C[row * N + col] = s;
}

// One thread per query row, the full score row kept in dynamic shared memory
// (S floats), as the reference's attention_naive (<<<S,1,S*4>>>).
__global__ void attention_rows(const __nv_bfloat16* __restrict__ Q, const __nv_bfloat16* __restrict__ K,
                               const __nv_bfloat16* __restrict__ V, __nv_bfloat16* __restrict__ O,
                               int64_t BH, int64_t S, int64_t D, float scale, int causal) {
  extern __shared__ float scores[];
  if (threadIdx.x != 0) return;
  for (int64_t r = blockIdx.x; r < BH * S; r += gridDim.x) {
    const int64_t bh = r / S, i = r % S;
    const __nv_bfloat16* q = Q + r * D;
    const __nv_bfloat16* k = K + bh * S * D;
    const __nv_bfloat16* v = V + bh * S * D;
    const int64_t jmax = causal ? i + 1 : S;
    for (int64_t j = 0; j < jmax; ++j) {
      float dot = 0.f;
      for (int64_t d = 0; d < D; ++d) dot += __bfloat162float(q[d]) * __bfloat162float(k[j * D + d]);
      scores[j] = dot * scale;
    }
    float m = scores[0];
    for (int64_t j = 1; j < jmax; ++j) m = fmaxf(m, scores[j]);
    float s = 0.f;
    for (int64_t j = 0; j < jmax; ++j) {
      scores[j] = expf(scores[j] - m);
      s += scores[j];
    }
    for (int64_t d = 0; d < D; ++d) {
      float acc = 0.f;
      for (int64_t j = 0; j < jmax; ++j) acc += scores[j] * __bfloat162float(v[j * D + d]);
      O[r * D + d] = __float2bfloat16_rn(acc / s);
    }
  }
}

inline unsigned capped_grid(int64_t want) {
  const int64_t cap = 1 << 30;
  if (want < 1) want = 1;
  return (unsigned)(want < cap ? want : cap);
}

inline int softmax(const float* x, float* y, int64_t rows, int64_t cols, cudaStream_t st) {
  if (rows < 0 || cols < 0) return fail(KT_ERR_ARG, "naive softmax: negative shape");
  if (rows == 0 || cols == 0) return KT_OK;
  if (!x || !y) return fail(KT_ERR_ARG, "naive softmax: null pointer");
  softmax_rows<<<capped_grid(rows), 1, 0, st>>>(x, y, rows, cols);
  return check_launch("naive softmax");
}

inline int layernorm(const float* x, const float* g, const float* b, float* y, int64_t rows, int64_t cols,
                     float eps, cudaStream_t st) {
  if (rows < 0 || cols < 0) return fail(KT_ERR_ARG, "naive layernorm: negative shape");
  if (rows == 0 || cols == 0) return KT_OK;
  if (!x || !g || !b || !y) return fail(KT_ERR_ARG, "naive layernorm: null pointer");
  layernorm_rows<<<capped_grid(rows), 1, 0, st>>>(x, g, b, y, rows, cols, eps);
  return check_launch("naive layernorm");
}

constexpr int kNaiveReduceBlock = 256;

inline size_t reduce_workspace_bytes(int64_t n) {
  const int64_t blocks = (n + kNaiveReduceBlock - 1) / kNaiveReduceBlock;
  return sizeof(float) * (size_t)(blocks > 0 ? blocks : 1);
}

inline int reduce(const float* x, int64_t n, double* out64, float* out32, void* ws, size_t ws_bytes,
                  cudaStream_t st) {
  if (n < 0 || out64 == nullptr) return fail(KT_ERR_ARG, "naive reduce: bad arguments");
  const int64_t blocks = (n + kNaiveReduceBlock - 1) / kNaiveReduceBlock;
  if (blocks > (int64_t)INT32_MAX) return fail(KT_ERR_UNSUPPORTED, "naive reduce: n too large");
  if (ws == nullptr || ws_bytes < reduce_workspace_bytes(n))
    return fail(KT_ERR_ARG, "naive reduce: workspace too small (%zu < %zu)", ws_bytes, reduce_workspace_bytes(n));
  float* partials = static_cast<float*>(ws);
  if (blocks > 0) {
    reduce_partials<<<(unsigned)blocks, kNaiveReduceBlock, kNaiveReduceBlock * sizeof(float), st>>>(x, n, partials);
    int rc = check_launch("naive reduce partials");
    if (rc != KT_OK) return rc;
  }
  reduce_final<<<1, 32, 0, st>>>(partials, blocks, out64, out32);
  return check_launch("naive reduce final");
}

inline int gemm(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int tb,
                cudaStream_t st) {
  if (M < 0 || N < 0 || K < 0) return fail(KT_ERR_ARG, "naive gemm: negative shape");
  if (M == 0 || N == 0) return KT_OK;
  if (!A || !B || !C) return fail(KT_ERR_ARG, "naive gemm: null pointer");
  if ((N + 15) / 16 > 0x7fffffff || (M + 15) / 16 > 65535) return fail(KT_ERR_UNSUPPORTED, "naive gemm: shape too large");
  dim3 block(16, 16), grid((unsigned)((N + 15) / 16), (unsigned)((M + 15) / 16));
  gemm_elem<<<grid, block, 0, st>>>(A, B, C, M, N, K, tb);
  return check_launch("naive gemm");
}

inline int attention(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int64_t B, int64_t H,
                     int64_t S, int64_t D, float scale, int causal, cudaStream_t st) {
  if (B < 0 || H < 0 || S < 0 || D < 0) return fail(KT_ERR_ARG, "naive attention: negative shape");
  if (B == 0 || H == 0 || S == 0 || D == 0) return KT_OK;
  if (!Q || !K || !V || !O) return fail(KT_ERR_ARG, "naive attention: null pointer");
  const size_t smem = sizeof(float) * (size_t)S;
  if (smem > 227 * 1024) return fail(KT_ERR_UNSUPPORTED, "naive attention: S too long for the score row");
  int rc = ensure_smem((const void*)attention_rows, smem, "naive attention: smem attribute");
  if (rc != KT_OK) return rc;
  attention_rows<<<capped_grid(B * H * S), 1, smem, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(Q), reinterpret_cast<const __nv_bfloat16*>(K),
      reinterpret_cast<const __nv_bfloat16*>(V), reinterpret_cast<__nv_bfloat16*>(O), B * H, S, D, scale, causal);
  return check_launch("naive attention");
}

}  // namespace naive
}  // namespace kt
