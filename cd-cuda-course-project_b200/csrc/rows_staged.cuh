// rows_staged.cuh — persistent row kernels fed by TMA bulk copies (sm_100a).
//
// Each CTA owns rows blockIdx.x, blockIdx.x + gridDim.x, ... One thread keeps
// STAGES whole rows in flight: it streams each row into a shared-memory slot
// with a 1-D cp.async.bulk (completion counted on the slot's mbarrier); all
// threads copy their 128-bit pieces of the landed row into registers, the slot
// is refilled with the row STAGES ahead, and the row is finished from
// registers (block reductions, then 128-bit streaming stores). With several
// CTAs per SM this keeps ~100-200 KB of reads in flight per SM without
// depending on how many CTAs happen to be in their load phase — the limit of
// the one-row-per-CTA register kernels.
//
// Waits are bounded; the timeout decision is made block-uniform with
// __syncthreads_or before anyone leaves the loop, the issuing thread then
// drains its outstanding copies, and the device error word records it.
#pragma once
#include "kt_common.cuh"
#include "sm100.cuh"

#ifndef KT_ROWS_BOX
#define KT_ROWS_BOX 0  // bytes per bulk copy of a row (a multiple of 16); 0: the whole row in one copy
#endif
static_assert(KT_ROWS_BOX % 16 == 0, "bulk copies move multiples of 16 bytes");

namespace kt {
namespace staged {

// Copy one row into a slot as bulk copies of at most KT_ROWS_BOX bytes each
// (0: one copy), all completing on the slot's mbarrier.
__device__ __forceinline__ void load_row(uint32_t dst, const float* src, uint32_t bytes, uint32_t bar) {
  using namespace sm100;
  mbar_arrive_expect_tx(bar, bytes);
  const uint32_t piece = KT_ROWS_BOX == 0 ? bytes : (uint32_t)KT_ROWS_BOX;
  for (uint32_t off = 0; off < bytes; off += piece) {
    const uint32_t n = bytes - off < piece ? bytes - off : piece;
    bulk_load(dst + off, reinterpret_cast<const uint8_t*>(src) + off, n, bar);
  }
}

// Shared-memory layout: STAGES row slots of `cols` floats (16-byte aligned),
// then STAGES mbarriers.
template <int STAGES>
__host__ __device__ constexpr size_t smem_bytes(int cols) {
  return (size_t)STAGES * (size_t)cols * 4 + STAGES * 8 + 16;
}

// Iterates this CTA's rows with the bulk-copy ring; `body(v, row)` receives
// the thread's VPT float4 pieces (index tid + i·BLOCK; entries beyond the row
// are left untouched) and finishes the row. Returns false on a timeout.
template <int BLOCK, int VPT, int STAGES, class Body>
__device__ __forceinline__ bool for_each_row(const float* __restrict__ x, int64_t rows, int cols, Body body) {
  using namespace sm100;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  float4* slots = reinterpret_cast<float4*>(smem_raw);
  const uint32_t slot0 = smem_u32(smem_raw);
  const uint32_t row_bytes = (uint32_t)cols * 4u;
  const uint32_t bar0 = slot0 + STAGES * row_bytes;
  const int nvec = cols >> 2;
  const int64_t count = rows > (int64_t)blockIdx.x ? (rows - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(bar0 + 8u * s, 1);
    fence_mbar_init();
    for (int s = 0; s < STAGES && s < count; ++s) {
      const int64_t row = blockIdx.x + (int64_t)s * gridDim.x;
      load_row(slot0 + s * row_bytes, x + row * cols, row_bytes, bar0 + 8u * s);
    }
  }
  __syncthreads();
  bool ok = true;
  int64_t k = 0;
  for (; k < count; ++k) {
    const int s = (int)(k % STAGES);
    const uint32_t parity = (uint32_t)((k / STAGES) & 1);
    const bool landed = mbar_wait(bar0 + 8u * s, parity);
    if (__syncthreads_or(!landed)) {
      ok = false;
      break;
    }
    float4 v[VPT];
    const float4* slot = slots + (size_t)s * nvec;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < nvec) v[i] = slot[idx];
    }
    __syncthreads();  // every thread holds its pieces: the slot can be refilled
    if (threadIdx.x == 0 && k + STAGES < count) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic reads before the async write
      const int64_t row = blockIdx.x + (k + STAGES) * gridDim.x;
      load_row(slot0 + s * row_bytes, x + row * cols, row_bytes, bar0 + 8u * s);
    }
    body(v, blockIdx.x + k * gridDim.x);
  }
  if (!ok) {
    raise_device_error(DEV_MBAR_TIMEOUT);
    if (threadIdx.x == 0) {
      // copies issued for rows k .. k+STAGES-1 may still be landing
      for (int64_t r = k; r < count && r < k + STAGES; ++r)
        (void)mbar_wait(bar0 + 8u * (uint32_t)(r % STAGES), (uint32_t)((r / STAGES) & 1));
    }
  }
  return ok;
}

template <int BLOCK, int VPT, int STAGES>
__global__ void __launch_bounds__(BLOCK)
softmax_rows(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int cols) {
  __shared__ float red_max[32];
  __shared__ float red_sum[32];
  const int nvec = cols >> 2;
  for_each_row<BLOCK, VPT, STAGES>(x, rows, cols, [&](float4 (&v)[VPT], int64_t row) {
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
      if (threadIdx.x + i * BLOCK < nvec) m = fmaxf(m, max4(v[i]));
    m = block_max<BLOCK>(m, red_max);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      if (threadIdx.x + i * BLOCK < nvec) {
        v[i].x = expf(v[i].x - m);
        v[i].y = expf(v[i].y - m);
        v[i].z = expf(v[i].z - m);
        v[i].w = expf(v[i].w - m);
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      }
    }
    s = block_sum<BLOCK>(s, red_sum);
    const float inv = 1.0f / s;
    float4* yr = reinterpret_cast<float4*>(y + row * (int64_t)cols);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < nvec) st_stream4(yr + idx, make_float4(v[i].x * inv, v[i].y * inv, v[i].z * inv, v[i].w * inv));
    }
  });
}

template <int BLOCK, int VPT, int STAGES>
__global__ void __launch_bounds__(BLOCK)
layernorm_rows(const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
               float* __restrict__ y, int64_t rows, int cols, float eps) {
  __shared__ float red_a[32];
  __shared__ float red_b[32];
  const int nvec = cols >> 2;
  const float fcols = (float)cols;
  // gamma/beta pieces of this thread, the same for every row
  float4 g[VPT], bt[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * BLOCK;
    if (idx < nvec) {
      g[i] = __ldg(reinterpret_cast<const float4*>(gamma) + idx);
      bt[i] = __ldg(reinterpret_cast<const float4*>(beta) + idx);
    }
  }
  for_each_row<BLOCK, VPT, STAGES>(x, rows, cols, [&](float4 (&v)[VPT], int64_t row) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
      if (threadIdx.x + i * BLOCK < nvec) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    const float mean = block_sum<BLOCK>(s, red_a) / fcols;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      if (threadIdx.x + i * BLOCK < nvec) {
        v[i].x -= mean; v[i].y -= mean; v[i].z -= mean; v[i].w -= mean;
        q += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
      }
    }
    const float rstd = rsqrtf(block_sum<BLOCK>(q, red_b) / fcols + eps);
    float4* yr = reinterpret_cast<float4*>(y + row * (int64_t)cols);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < nvec) {
        float4 o;
        o.x = fmaf(v[i].x * rstd, g[i].x, bt[i].x);
        o.y = fmaf(v[i].y * rstd, g[i].y, bt[i].y);
        o.z = fmaf(v[i].z * rstd, g[i].z, bt[i].z);
        o.w = fmaf(v[i].w * rstd, g[i].w, bt[i].w);
        st_stream4(yr + idx, o);
      }
    }
  });
}

// Grid: as many CTAs as fit (CTAS_PER_SM per SM by shared memory), at most one per row.
// The shared-memory opt-in and the occupancy query are made once per
// (kernel, launch shape, device) (kt_common.cuh: resident_ctas).
template <class K>
inline int launch_grid(K kern, int block, size_t smem, int64_t rows, int* grid_out) {
  int per_sm = 0;
  int rc = resident_ctas((const void*)kern, block, smem, &per_sm, "staged rows: launch shape");
  if (rc != KT_OK) return rc;
  if (per_sm < 1) return fail(KT_ERR_UNSUPPORTED, "staged rows: no CTA fits (smem %zu)", smem);
  const int64_t g = (int64_t)sm_count() * per_sm;
  *grid_out = (int)(rows < g ? rows : g);
  return KT_OK;
}

}  // namespace staged
}  // namespace kt
