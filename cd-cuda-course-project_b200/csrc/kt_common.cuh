// kt_common.cuh — shared host/device helpers for the sm_100a kernel library.
//
// Status handling: every exported entry point returns a KT_* status and
// records a thread-local message (kt_last_error). Device code never traps; a
// kernel that has to give up (a bounded wait that ran out) writes a code to
// the device error word `g_kt_device_error` and returns.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <string.h>
#include <math.h>

#include <mutex>

#include "kt_abi.h"

#define KT_ABI_VERSION 1

namespace kt {

// ----------------------------------------------------------------------------
// Host: last-error text and status helpers
// ----------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_error("%s", buf);
  return code;
}

inline int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return KT_OK;
  return fail(KT_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// Check the launch that was just issued.
inline int check_launch(const char* what) {
  return cuda_status(cudaGetLastError(), what);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

// Per-(kernel, device) launch facts that cost a driver call to establish.
//  * The dynamic shared-memory opt-in (cudaFuncAttributeMaxDynamicSharedMemorySize)
//    is a property of the function in each device's context, so it is set on
//    every device the kernel runs on. It only ever grows: lowering it while
//    another host thread launches the same kernel with more would fail that
//    launch.
//  * The resident-CTA count for a (block, smem) launch shape.
// Lookups and inserts are serialised by one mutex; a full table only repeats
// the driver calls.
namespace detail {
struct FactsTable {
  struct Smem {
    const void* fn;
    int dev;
    size_t bytes;
  };
  struct Occ {
    const void* fn;
    int dev;
    int block;
    size_t smem;
    int per_sm;
  };
  std::mutex mu;
  Smem smem[64];
  int n_smem = 0;
  Occ occ[64];
  int n_occ = 0;
};
inline FactsTable& facts() {
  static FactsTable t;
  return t;
}
// Caller holds facts().mu.
inline int ensure_smem_locked(FactsTable& t, const void* fn, int dev, size_t bytes, const char* what) {
  if (bytes <= 48 * 1024) return KT_OK;
  for (int i = 0; i < t.n_smem; ++i)
    if (t.smem[i].fn == fn && t.smem[i].dev == dev) {
      if (t.smem[i].bytes >= bytes) return KT_OK;
      int rc = cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes), what);
      if (rc == KT_OK) t.smem[i].bytes = bytes;
      return rc;
    }
  int rc = cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes), what);
  if (rc == KT_OK && t.n_smem < 64) t.smem[t.n_smem++] = FactsTable::Smem{fn, dev, bytes};
  return rc;
}
}  // namespace detail

// Opt `fn` into `bytes` of dynamic shared memory on the current device.
inline int ensure_smem(const void* fn, size_t bytes, const char* what) {
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev), what);
  if (rc != KT_OK) return rc;
  detail::FactsTable& t = detail::facts();
  std::lock_guard<std::mutex> lock(t.mu);
  return detail::ensure_smem_locked(t, fn, dev, bytes, what);
}

// ensure_smem, then the number of CTAs of (block, smem) resident per SM.
inline int resident_ctas(const void* fn, int block, size_t smem, int* per_sm, const char* what) {
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev), what);
  if (rc != KT_OK) return rc;
  detail::FactsTable& t = detail::facts();
  std::lock_guard<std::mutex> lock(t.mu);
  rc = detail::ensure_smem_locked(t, fn, dev, smem, what);
  if (rc != KT_OK) return rc;
  for (int i = 0; i < t.n_occ; ++i) {
    const auto& e = t.occ[i];
    if (e.fn == fn && e.dev == dev && e.block == block && e.smem == smem) {
      *per_sm = e.per_sm;
      return KT_OK;
    }
  }
  int n = 0;
  rc = cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, block, smem), what);
  if (rc != KT_OK) return rc;
  if (t.n_occ < 64) t.occ[t.n_occ++] = detail::FactsTable::Occ{fn, dev, block, smem, n};
  *per_sm = n;
  return KT_OK;
}

// ----------------------------------------------------------------------------
// Device: error word, loads/stores, reductions
// ----------------------------------------------------------------------------
enum DeviceErr : int {
  DEV_OK = 0,
  DEV_MBAR_TIMEOUT = 1,   // an mbarrier wait exceeded its iteration bound
  DEV_BAD_SHAPE = 2,      // a kernel-side bounds check refused an index
  DEV_XRANK_TIMEOUT = 3   // a cross-GPU exchange wait ran out (a rank never arrived)
};

}  // namespace kt

// Device error word of this library (one translation unit per library, so one
// word per library and device). Kernels name it directly; host code reads it
// with cudaMemcpyFromSymbol (kt_device_error).
static __device__ int g_kt_device_error = 0;

namespace kt {

// First error wins; later ones are dropped.
__device__ __forceinline__ void raise_device_error(int code) { atomicCAS(&g_kt_device_error, 0, code); }

// Streaming 128-bit read that does not allocate in L1 (data read once).
__device__ __forceinline__ float4 ld_stream4(const float4* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float ld_stream1(const float* p) {
  float v;
  asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

// Streaming (evict-first) 128-bit store.
__device__ __forceinline__ void st_stream4(float4* p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}

__device__ __forceinline__ void st_stream1(float* p, float v) {
  asm volatile("st.global.cs.f32 [%0], %1;" :: "l"(p), "f"(v) : "memory");
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; every thread receives the result. `scratch` holds >= 32
// entries and must not be reused by the caller before the next __syncthreads.
template <int BLOCK, typename T>
__device__ __forceinline__ T block_sum(T v, T* scratch) {
  static_assert(BLOCK % 32 == 0 && BLOCK <= 1024, "block size");
  constexpr int NW = BLOCK / 32;
  v = warp_sum(v);
  if constexpr (NW == 1) {
    return v;
  } else {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    T t = lane < NW ? scratch[lane] : T(0);
    return warp_sum(t);
  }
}

template <int BLOCK>
__device__ __forceinline__ float block_max(float v, float* scratch) {
  static_assert(BLOCK % 32 == 0 && BLOCK <= 1024, "block size");
  constexpr int NW = BLOCK / 32;
  v = warp_max(v);
  if constexpr (NW == 1) {
    return v;
  } else {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    float t = lane < NW ? scratch[lane] : -INFINITY;
    return warp_max(t);
  }
}

__device__ __forceinline__ float max4(float4 v) {
  return fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
}

}  // namespace kt
