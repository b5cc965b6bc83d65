// rows_cluster.cuh — row softmax / LayerNorm with each row split across a
// thread-block cluster (sm_100a: clusters + distributed shared memory).
//
// A cluster of C CTAs (C = 2, 4 or 8) owns rows clusterid, clusterid +
// nclusters, ...; CTA r of the cluster owns columns [r·cols/C, (r+1)·cols/C)
// of every such row. Each CTA streams its column chunk of STAGES rows ahead
// into shared memory with 1-D bulk copies (as rows_staged.cuh does for whole
// rows), keeps the chunk in registers, reduces it to two partial statistics,
// and stores them into every CTA of the cluster (st.shared::cluster through
// mapa addresses). One cluster barrier later every CTA merges the C partials
// in rank order (the same bits in every CTA) and finishes its chunk:
//   softmax:   partial (m_r = max, s_r = sum exp(x - m_r)); M = max m_r,
//              S = sum s_r·exp(m_r - M); y = exp(x - m_r)·exp(m_r - M)/S
//   LayerNorm: partial (mean_r, M2_r = sum (x - mean_r)^2) over equal chunks;
//              mean = avg mean_r, M2 = sum M2_r + n_r·(mean_r - mean)^2
//              (the pairwise-merge of Chan et al.), var = M2 / cols.
// Every element is read once and written once, for rows up to C times wider
// than one CTA can hold (beyond that rows_stream reads x twice), and a batch
// with fewer rows than resident CTAs spreads over C times as many SMs.
//
// Partials are double-buffered by row parity: a CTA writes row k+1's partials
// only after the barrier of row k, which every CTA reaches after reading row
// k-1's. A copy that times out is not a reason to leave the loop alone (the
// other CTAs would wait at the next cluster barrier): the flag travels with
// the partials and the whole cluster leaves at the same row. A cluster
// barrier at entry (all CTAs running before any remote store) and one at exit
// (no CTA leaves while another may still store into its shared memory) close
// the kernel.
#pragma once
#include "kt_common.cuh"
#include "sm100.cuh"

namespace kt {
namespace clustered {

constexpr int kMaxCluster = 8;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t num_clusters() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store v at the shared-memory address `local` (this CTA's layout) of CTA `rank` of the cluster.
__device__ __forceinline__ void st_cluster(uint32_t local, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// Shared memory: STAGES chunk slots (chunk floats each), STAGES mbarriers.
template <int STAGES>
__host__ __device__ constexpr size_t smem_bytes(int chunk) {
  return (size_t)STAGES * (size_t)chunk * 4 + STAGES * 8 + 16;
}

// Issue the copy of one chunk in pieces of at most `box` bytes (0: one piece),
// all completing on the same mbarrier.
__device__ __forceinline__ void load_chunk(uint32_t dst, const float* src, uint32_t bytes, uint32_t box, uint32_t bar) {
  using namespace sm100;
  mbar_arrive_expect_tx(bar, bytes);
  const uint32_t piece = box == 0 ? bytes : box;
  for (uint32_t off = 0; off < bytes; off += piece) {
    const uint32_t n = bytes - off < piece ? bytes - off : piece;
    bulk_load(dst + off, reinterpret_cast<const uint8_t*>(src) + off, n, bar);
  }
}

// KIND 0: softmax; KIND 1: LayerNorm. cols % (4·C) == 0, chunk = cols / C
// <= BLOCK·VPT·4, x / y / gamma / beta 16-byte aligned (checked by the launcher).
template <int BLOCK, int VPT, int STAGES, int KIND>
__global__ void __launch_bounds__(BLOCK)
rows_kernel(const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
            float* __restrict__ y, int64_t rows, int cols, float eps, uint32_t box) {
  using namespace sm100;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ float red_a[32];
  __shared__ float red_b[32];
  __shared__ float xch[2][kMaxCluster][4];  // [row parity][source rank] {a, b, flag, -}
  const uint32_t rank = cluster_rank(), C = cluster_size();
  const int chunk = cols / (int)C;
  const int col0 = (int)rank * chunk;
  const int nvec = chunk >> 2;
  const uint32_t chunk_bytes = (uint32_t)chunk * 4u;
  float4* slots = reinterpret_cast<float4*>(smem_raw);
  const uint32_t slot0 = smem_u32(smem_raw);
  const uint32_t bar0 = slot0 + STAGES * chunk_bytes;
  const int64_t cid = cluster_id(), ncl = num_clusters();
  const int64_t count = rows > cid ? (rows - 1 - cid) / ncl + 1 : 0;

  float4 g[VPT], bt[VPT];
  if (KIND == 1) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * BLOCK;
      if (idx < nvec) {
        g[i] = __ldg(reinterpret_cast<const float4*>(gamma + col0) + idx);
        bt[i] = __ldg(reinterpret_cast<const float4*>(beta + col0) + idx);
      }
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(bar0 + 8u * s, 1);
    fence_mbar_init();
    for (int s = 0; s < STAGES && s < count; ++s) {
      const int64_t row = cid + (int64_t)s * ncl;
      load_chunk(slot0 + s * chunk_bytes, x + row * cols + col0, chunk_bytes, box, bar0 + 8u * s);
    }
  }
  __syncthreads();
  cluster_sync();  // every CTA of the cluster runs before any partial is stored remotely

  bool failed = false;
  int64_t k = 0;
  for (; k < count; ++k) {
    const int s = (int)(k % STAGES);
    const uint32_t parity = (uint32_t)((k / STAGES) & 1);
    const bool bad = __syncthreads_or(!mbar_wait(bar0 + 8u * s, parity)) != 0;
    float4 v[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!bad) {
      const float4* slot = slots + (size_t)s * nvec;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int idx = threadIdx.x + i * BLOCK;
        if (idx < nvec) v[i] = slot[idx];
      }
    }
    __syncthreads();  // the slot is read: it can be refilled
    if (threadIdx.x == 0 && !bad && k + STAGES < count) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      const int64_t row = cid + (k + STAGES) * ncl;
      load_chunk(slot0 + s * chunk_bytes, x + row * cols + col0, chunk_bytes, box, bar0 + 8u * s);
    }
    // partial statistics of this chunk
    float pa, pb;
    if (KIND == 0) {
      float m = -INFINITY;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (threadIdx.x + i * BLOCK < nvec) m = fmaxf(m, max4(v[i]));
      m = block_max<BLOCK>(m, red_a);
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        if (threadIdx.x + i * BLOCK < nvec) {
          v[i].x = expf(v[i].x - m);
          v[i].y = expf(v[i].y - m);
          v[i].z = expf(v[i].z - m);
          v[i].w = expf(v[i].w - m);
          sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        }
      }
      pa = m;
      pb = block_sum<BLOCK>(sum, red_b);
    } else {
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (threadIdx.x + i * BLOCK < nvec) sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      const float mean_r = block_sum<BLOCK>(sum, red_a) / (float)chunk;
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        if (threadIdx.x + i * BLOCK < nvec) {
          v[i].x -= mean_r; v[i].y -= mean_r; v[i].z -= mean_r; v[i].w -= mean_r;
          q += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
        }
      }
      pa = mean_r;
      pb = block_sum<BLOCK>(q, red_b);
    }
    // exchange: this CTA's partials into slot [k&1][rank] of every CTA of the cluster
    const int buf = (int)(k & 1);
    if (threadIdx.x < C) {
      const uint32_t dst = smem_u32(&xch[buf][rank][0]);
      st_cluster(dst, threadIdx.x, pa);
      st_cluster(dst + 4u, threadIdx.x, pb);
      st_cluster(dst + 8u, threadIdx.x, bad ? 1.f : 0.f);
    }
    cluster_sync();
    bool any_bad = false;
    float a_all[kMaxCluster], b_all[kMaxCluster];
#pragma unroll
    for (int r = 0; r < kMaxCluster; ++r) {
      if (r < (int)C) {
        a_all[r] = xch[buf][r][0];
        b_all[r] = xch[buf][r][1];
        any_bad |= xch[buf][r][2] != 0.f;
      }
    }
    if (any_bad) {
      failed = true;
      break;  // the whole cluster leaves at this row
    }
    const int64_t row = cid + k * ncl;
    float4* yr = reinterpret_cast<float4*>(y + row * (int64_t)cols + col0);
    if (KIND == 0) {
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < kMaxCluster; ++r)
        if (r < (int)C) M = fmaxf(M, a_all[r]);
      float S = 0.f;
#pragma unroll
      for (int r = 0; r < kMaxCluster; ++r)
        if (r < (int)C) S += b_all[r] * expf(a_all[r] - M);
      const float f = expf(pa - M) / S;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int idx = threadIdx.x + i * BLOCK;
        if (idx < nvec) st_stream4(yr + idx, make_float4(v[i].x * f, v[i].y * f, v[i].z * f, v[i].w * f));
      }
    } else {
      float mean = 0.f;
#pragma unroll
      for (int r = 0; r < kMaxCluster; ++r)
        if (r < (int)C) mean += a_all[r];
      mean /= (float)C;
      float m2 = 0.f;
#pragma unroll
      for (int r = 0; r < kMaxCluster; ++r) {
        if (r < (int)C) {
          const float d = a_all[r] - mean;
          m2 += b_all[r] + (float)chunk * d * d;
        }
      }
      const float rstd = rsqrtf(m2 / (float)cols + eps);
      const float shift = pa - mean;  // v holds x - mean_r
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int idx = threadIdx.x + i * BLOCK;
        if (idx < nvec) {
          float4 o;
          o.x = fmaf((v[i].x + shift) * rstd, g[i].x, bt[i].x);
          o.y = fmaf((v[i].y + shift) * rstd, g[i].y, bt[i].y);
          o.z = fmaf((v[i].z + shift) * rstd, g[i].z, bt[i].z);
          o.w = fmaf((v[i].w + shift) * rstd, g[i].w, bt[i].w);
          st_stream4(yr + idx, o);
        }
      }
    }
  }
  if (failed) {
    raise_device_error(DEV_MBAR_TIMEOUT);
    if (threadIdx.x == 0) {
      // copies issued for rows k .. k+STAGES-1 may still be landing
      for (int64_t r = k; r < count && r < k + STAGES; ++r)
        (void)mbar_wait(bar0 + 8u * (uint32_t)(r % STAGES), (uint32_t)((r / STAGES) & 1));
    }
    __syncthreads();
  }
  cluster_sync();  // no CTA leaves while another may still store into its shared memory
}

// Launch with a cluster of C CTAs along x. Grid: as many clusters as fit at once
// (cudaOccupancyMaxActiveClusters), at most one per row.
template <int BLOCK, int VPT, int STAGES, int KIND>
inline int launch(int C, const float* x, const float* gamma, const float* beta, float* y, int64_t rows, int cols,
                  float eps, uint32_t box, cudaStream_t st) {
  auto kern = rows_kernel<BLOCK, VPT, STAGES, KIND>;
  const int chunk = cols / C;
  const size_t smem = smem_bytes<STAGES>(chunk);
  int rc = ensure_smem((const void*)kern, smem, "cluster rows: smem attribute");
  if (rc != KT_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(BLOCK);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.gridDim = dim3((unsigned)(C * sm_count()));
  int max_clusters = 0;
  rc = cuda_status(cudaOccupancyMaxActiveClusters(&max_clusters, (const void*)kern, &cfg), "cluster rows: occupancy");
  if (rc != KT_OK) return rc;
  if (max_clusters < 1) return fail(KT_ERR_UNSUPPORTED, "cluster rows: no cluster of %d CTAs fits (smem %zu)", C, smem);
  const int64_t n_cl = rows < (int64_t)max_clusters ? rows : (int64_t)max_clusters;
  cfg.gridDim = dim3((unsigned)(n_cl * C));
  rc = cuda_status(cudaLaunchKernelEx(&cfg, kern, x, gamma, beta, y, rows, cols, eps, box), "cluster rows: launch");
  if (rc != KT_OK) return rc;
  return check_launch("cluster rows");
}

// Whether a cluster of C CTAs can take rows of `cols` floats: equal 16-byte
// chunks that one CTA holds in registers and STAGES of which fit in shared memory.
template <int BLOCK, int VPT, int STAGES>
inline bool fits(int C, int64_t cols) {
  if (C < 2 || C > kMaxCluster || cols % (4 * C) != 0) return false;
  const int64_t chunk = cols / C;
  return chunk <= (int64_t)BLOCK * VPT * 4 && smem_bytes<STAGES>((int)chunk) <= 200 * 1024;
}

// Smallest cluster (2, 4, 8) that fits, or 0.
template <int BLOCK, int VPT, int STAGES>
inline int smallest_fit(int64_t cols) {
  for (int C = 2; C <= kMaxCluster; C *= 2)
    if (fits<BLOCK, VPT, STAGES>(C, cols)) return C;
  return 0;
}

}  // namespace clustered
}  // namespace kt
