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

// This CTA's share of the sum of x[0, n) (x + head 16-byte aligned), in fp64,
// returned to every thread of the CTA. `red` holds >= 32 doubles.
template <int BLOCK, int UNROLL>
__device__ __forceinline__ double cta_sum(const float* __restrict__ x, int64_t n, int head, double* red) {
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
  return block_sum<BLOCK>(acc, red);
}

// Publishes this CTA's partial and tells whether it is the last CTA to do so
// (atomic ticket); the last CTA returns the whole-grid fp64 sum in *total
// (same value in every thread, fixed summation order) and re-zeroes the ticket.
template <int BLOCK>
__device__ __forceinline__ bool last_cta_total(double cta, double* __restrict__ partials,
                                               unsigned int* __restrict__ ticket, double* red, double* total) {
  __shared__ int is_last;
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = cta;
    __threadfence();
    const unsigned int t = atomicAdd(ticket, 1u);
    is_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return false;
  __threadfence();
  double s = 0.0;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += BLOCK) s += __ldcg(partials + b);
  s = block_sum<BLOCK>(s, red);
  if (threadIdx.x == 0) *ticket = 0u;
  *total = s;
  return true;
}

template <int BLOCK, int UNROLL>
__global__ void __launch_bounds__(BLOCK)
sum_f32(const float* __restrict__ x, int64_t n, int head, double* __restrict__ partials,
        unsigned int* __restrict__ ticket, double* __restrict__ out64, float* __restrict__ out32) {
  __shared__ double red[32];
  const double cta = cta_sum<BLOCK, UNROLL>(x, n, head, red);
  double total;
  if (last_cta_total<BLOCK>(cta, partials, ticket, red, &total) && threadIdx.x == 0) {
    *out64 = total;
    if (out32 != nullptr) *out32 = (float)total;
  }
}

// ---------------------------------------------------------------------------
// Whole-job sum over `world` GPUs (one process per GPU) without a collective
// library: the last CTA of every rank stores its fp64 shard sum into a slot of
// every rank's exchange buffer over NVLink (plain peer stores, value then a
// release store of the call's epoch), then waits for the `world` slots of its
// own buffer to carry the epoch (acquire loads, bounded in time) and adds
// them in rank order, so every rank gets the same bits.
//
// Exchange buffer (KT_XRANK_EXCHANGE_BYTES per rank): 2 phases x KT_XRANK_MAX
// slots of {double value; uint64 epoch}. A call uses phase epoch & 1. A rank
// writes phase p of call e+2 only after it saw every rank's call e+1 slot,
// which each rank writes only after finishing call e (stream order), so no
// rank overwrites a slot its owner has not read yet.
// ---------------------------------------------------------------------------
struct XrankSlot {
  double value;
  unsigned long long epoch;
};
static_assert(sizeof(XrankSlot) == 16, "slot layout");
static_assert(KT_XRANK_EXCHANGE_BYTES == 2 * KT_XRANK_MAX * 16, "exchange size");

struct XrankPeers {
  XrankSlot* p[KT_XRANK_MAX];  // every rank's exchange buffer as mapped in this process
};

constexpr unsigned long long kXrankWaitNs = 2000000000ull;  // 2 s: a rank that never arrives is an error

__device__ __forceinline__ void st_relaxed_sys_f64(double* p, double v) {
  asm volatile("st.relaxed.sys.global.f64 [%0], %1;" ::"l"(p), "d"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ double ld_relaxed_sys_f64(const double* p) {
  double v;
  asm volatile("ld.relaxed.sys.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long gtimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

template <int BLOCK, int UNROLL>
__global__ void __launch_bounds__(BLOCK)
sum_f32_xrank(const float* __restrict__ x, int64_t n, int head, double* __restrict__ partials,
              unsigned int* __restrict__ ticket, double* __restrict__ out64, float* __restrict__ out32,
              const __grid_constant__ XrankPeers peers, int rank, int world, unsigned long long epoch) {
  __shared__ double red[32];
  __shared__ double vals[KT_XRANK_MAX];
  __shared__ int timed_out;
  const double cta = cta_sum<BLOCK, UNROLL>(x, n, head, red);
  double local;
  if (!last_cta_total<BLOCK>(cta, partials, ticket, red, &local)) return;
  if (threadIdx.x == 0) timed_out = 0;
  const int phase = (int)(epoch & 1ull);
  __syncthreads();
  // peers is a __grid_constant__ parameter read with compile-time indices, so
  // no thread copies the pointer table to local memory (a by-value parameter
  // indexed at run time was copied by every thread of every CTA)
  XrankSlot* to_peer = nullptr;
  XrankSlot* own = nullptr;
#pragma unroll
  for (int r = 0; r < KT_XRANK_MAX; ++r) {
    if ((int)threadIdx.x == r) to_peer = peers.p[r];
    if (rank == r) own = peers.p[r];
  }
  if (world > 1 && threadIdx.x < world) {
    XrankSlot* dst = to_peer + phase * KT_XRANK_MAX + rank;
    st_relaxed_sys_f64(&dst->value, local);
    st_release_sys_u64(&dst->epoch, epoch);
  }
  if (world > 1 && threadIdx.x < world) {
    const XrankSlot* src = own + phase * KT_XRANK_MAX + threadIdx.x;
    const unsigned long long t0 = gtimer_ns();
    bool ok = false;
    for (unsigned int it = 0; it < (1u << 26); ++it) {
      if (ld_acquire_sys_u64(&src->epoch) == epoch) {
        ok = true;
        break;
      }
      if ((it & 63u) == 63u && gtimer_ns() - t0 > kXrankWaitNs) break;
      __nanosleep(32);
    }
    if (ok) vals[threadIdx.x] = ld_relaxed_sys_f64(&src->value);
    else atomicExch(&timed_out, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double total = local;
    if (world > 1) {
      total = 0.0;
      for (int r = 0; r < world; ++r) total += vals[r];
    }
    if (timed_out) {
      raise_device_error(DEV_XRANK_TIMEOUT);
      total = __longlong_as_double(0x7ff8000000000000ll);  // NaN: no whole-job sum
    }
    *out64 = total;
    if (out32 != nullptr) *out32 = (float)total;
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

// Whole-job sum across ranks (see sum_f32_xrank). The ticket word of `ws`
// must be zero before the first call on that workspace (the kernel leaves it
// zero), so no per-call reset is issued.
inline int launch_xrank(const float* x, int64_t n, double* out64, float* out32, void* ws, size_t ws_bytes,
                        void* const* exchange, int rank, int world, unsigned long long epoch, cudaStream_t st) {
  if (n < 0) return fail(KT_ERR_ARG, "reduce xrank: negative n=%lld", (long long)n);
  if (out64 == nullptr) return fail(KT_ERR_ARG, "reduce xrank: out64 is null");
  if (n > 0 && x == nullptr) return fail(KT_ERR_ARG, "reduce xrank: x is null");
  if ((reinterpret_cast<uintptr_t>(x) & 3u) != 0) return fail(KT_ERR_ARG, "reduce xrank: x not 4-byte aligned");
  if (world < 1 || world > KT_XRANK_MAX) return fail(KT_ERR_ARG, "reduce xrank: world %d not in [1, %d]", world, KT_XRANK_MAX);
  if (rank < 0 || rank >= world) return fail(KT_ERR_ARG, "reduce xrank: rank %d not in [0, %d)", rank, world);
  if (epoch == 0) return fail(KT_ERR_ARG, "reduce xrank: epoch must be >= 1 (exchange buffers start zeroed)");
  XrankPeers peers{};
  if (world > 1) {
    if (exchange == nullptr) return fail(KT_ERR_ARG, "reduce xrank: exchange pointer array is null");
    for (int r = 0; r < world; ++r) {
      if (exchange[r] == nullptr || !aligned16(exchange[r]))
        return fail(KT_ERR_ARG, "reduce xrank: exchange[%d] null or not 16-byte aligned", r);
      peers.p[r] = static_cast<XrankSlot*>(exchange[r]);
    }
  }
  const int grid = grid_for(n);
  const size_t need = kPartialsOffset + sizeof(double) * (size_t)grid;
  if (ws == nullptr || ws_bytes < need)
    return fail(KT_ERR_ARG, "reduce xrank: workspace %zu bytes < required %zu", ws_bytes, need);
  if (!aligned16(ws)) return fail(KT_ERR_ARG, "reduce xrank: workspace not 16-byte aligned");
  const uintptr_t addr = reinterpret_cast<uintptr_t>(x);
  int head = (int)(((16 - (addr & 15)) & 15) >> 2);
  if ((int64_t)head > n) head = (int)n;
  sum_f32_xrank<KT_REDUCE_BLOCK, KT_REDUCE_UNROLL><<<grid, KT_REDUCE_BLOCK, 0, st>>>(
      x, n, head, reinterpret_cast<double*>(static_cast<char*>(ws) + kPartialsOffset),
      reinterpret_cast<unsigned int*>(ws), out64, out32, peers, rank, world, epoch);
  return check_launch("reduce sum_f32_xrank");
}

}  // namespace reduce
}  // namespace kt
