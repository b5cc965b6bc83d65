// reduce.cuh — full fp32 sum reduction with fp64 accumulation, for sm_100a.
//
// The reference kernel `reduction_opt` (src/generator.py:82-98 with the body
// at :302-324) only writes one fp32 partial per block; its verifier compares
// those partials (src/verifier.py:253-264). The required result here is the
// whole sum, checked against `x.sum(dtype=float64)`.
//
// Design (HBM-bound: n·4 bytes read):
//   * a persistent grid of BLOCKS_PER_SM CTAs per SM; every thread keeps
//     UNROLL independent 16-byte streaming loads in flight per iteration;
//   * each group of UNROLL·4 values is summed in fp32 (16-ish terms, error far
//     below the 1e-4 budget) and added to a per-thread fp64 accumulator, so the
//     long accumulation chain is fp64 (2^28 U[-1,1] terms have |sum| ~ 1e4
//     against sum|x| ~ 1.3e8; fp32 chains lose too much there);
//   * CTA partials are combined by warp shuffles in fp64 and written to the
//     caller's workspace; the last CTA to finish (atomic ticket) sums the
//     partials in a fixed order, so the result is deterministic for a grid.
// Workspace layout: [0,4) ticket (zeroed by the launcher), [16, 16+8·grid) partials.
#pragma once
#include "kt_common.cuh"

#ifndef KT_REDUCE_BLOCK
#define KT_REDUCE_BLOCK 512
#endif
#ifndef KT_REDUCE_UNROLL
#define KT_REDUCE_UNROLL 4
#endif
#ifndef KT_REDUCE_BPSM
#define KT_REDUCE_BPSM 4
#endif

namespace kt {
namespace reduce {

constexpr size_t kPartialsOffset = 16;

template <int BLOCK, int UNROLL>
__global__ void __launch_bounds__(BLOCK)
sum_f32(const float* __restrict__ x, int64_t n, int head, double* __restrict__ partials,
        unsigned int* __restrict__ ticket, double* __restrict__ out64, float* __restrict__ out32) {
  __shared__ double red[32];
  __shared__ int is_last;
  const float4* xv = reinterpret_cast<const float4*>(x + head);
  const int64_t nvec = (n - head) >> 2;
  const int64_t stride = (int64_t)gridDim.x * BLOCK;
  int64_t i = (int64_t)blockIdx.x * BLOCK + threadIdx.x;
  double acc = 0.0;
  for (; i + (int64_t)(UNROLL - 1) * stride < nvec; i += (int64_t)UNROLL * stride) {
    float4 v[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) v[u] = ld_stream4(xv + i + (int64_t)u * stride);
    float s = 0.f;
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) s += (v[u].x + v[u].y) + (v[u].z + v[u].w);
    acc += (double)s;
  }
  for (; i < nvec; i += stride) {
    const float4 v = ld_stream4(xv + i);
    acc += (double)((v.x + v.y) + (v.z + v.w));
  }
  if (blockIdx.x == 0 && threadIdx.x < 4) {
    // up to 3 unaligned head values and up to 3 tail values
    const int t = threadIdx.x;
    if (t < head) acc += (double)x[t];
    const int64_t tail = (int64_t)head + nvec * 4 + t;
    if (t < 3 && tail < n) acc += (double)x[tail];
  }
  acc = block_sum<BLOCK>(acc, red);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = acc;
    __threadfence();
    const unsigned int t = atomicAdd(ticket, 1u);
    is_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (is_last) {
    __threadfence();
    double s = 0.0;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += BLOCK) s += __ldcg(partials + b);
    s = block_sum<BLOCK>(s, red);
    if (threadIdx.x == 0) {
      *out64 = s;
      if (out32 != nullptr) *out32 = (float)s;
      *ticket = 0u;
    }
  }
}

inline int grid_for(int64_t n) {
  const int64_t nvec = n > 0 ? (n >> 2) : 0;
  int64_t g = (int64_t)sm_count() * KT_REDUCE_BPSM;
  const int64_t need = (nvec + KT_REDUCE_BLOCK - 1) / KT_REDUCE_BLOCK;
  if (need < g) g = need;
  if (g < 1) g = 1;
  return (int)g;
}

inline size_t workspace_bytes(int64_t n) {
  return kPartialsOffset + sizeof(double) * (size_t)grid_for(n);
}

// Launches on caller scratch `ws` whose ticket word must be zero on entry
// (the kernel leaves it zero again).
inline int launch_on(const float* x, int64_t n, double* out64, float* out32, void* ws, int grid,
                     cudaStream_t st) {
  const uintptr_t addr = reinterpret_cast<uintptr_t>(x);
  int head = (int)(((16 - (addr & 15)) & 15) >> 2);
  if ((int64_t)head > n) head = (int)n;
  unsigned int* ticket = reinterpret_cast<unsigned int*>(ws);
  double* partials = reinterpret_cast<double*>(static_cast<char*>(ws) + kPartialsOffset);
  sum_f32<KT_REDUCE_BLOCK, KT_REDUCE_UNROLL><<<grid, KT_REDUCE_BLOCK, 0, st>>>(
      x, n, head, partials, ticket, out64, out32);
  return check_launch("reduce sum_f32");
}

inline int launch(const float* x, int64_t n, double* out64, float* out32, void* ws, size_t ws_bytes,
                  cudaStream_t st) {
  if (n < 0) return fail(KT_ERR_ARG, "reduce: negative n=%lld", (long long)n);
  if (out64 == nullptr) return fail(KT_ERR_ARG, "reduce: out64 is null");
  if (n > 0 && x == nullptr) return fail(KT_ERR_ARG, "reduce: x is null");
  if ((reinterpret_cast<uintptr_t>(x) & 3u) != 0) return fail(KT_ERR_ARG, "reduce: x not 4-byte aligned");
  const int grid = grid_for(n);
  const size_t need = kPartialsOffset + sizeof(double) * (size_t)grid;
  if (ws == nullptr || ws_bytes < need)
    return fail(KT_ERR_ARG, "reduce: workspace %zu bytes < required %zu", ws_bytes, need);
  if ((reinterpret_cast<uintptr_t>(ws) & 15u) != 0) return fail(KT_ERR_ARG, "reduce: workspace not 16-byte aligned");
  int rc = cuda_status(cudaMemsetAsync(ws, 0, sizeof(unsigned int), st), "reduce: ticket reset");
  if (rc != KT_OK) return rc;
  return launch_on(x, n, out64, out32, ws, grid, st);
}

}  // namespace reduce
}  // namespace kt
