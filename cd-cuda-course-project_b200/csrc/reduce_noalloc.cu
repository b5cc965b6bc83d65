// reduce_noalloc.cu — the sum reduction for callers that cannot allocate.
//
// kt_reduce_sum_f32 needs a few KB of device scratch (per-CTA partials and
// a completion ticket) that the caller passes in. Some callers have no way to
// provide it: code running inside a host callback or a real-time loop where
// cudaMalloc would block or synchronize the device, embedders that own a
// fixed memory budget and forbid runtime allocations, and foreign-language
// bindings (cgo, JNI) whose callers hold only the input/output buffers.
// kt_reduce_sum_f32_noalloc serves them: the scratch is a fixed array in the
// library's own device memory, so nothing is allocated per call.
//
// The array lives for as long as the library is loaded, on every device the
// library is used on. Every call looks its device address up on the host with
// cudaGetSymbolAddress, with the caller's device current (a host-side lookup
// once the library's device code is loaded; no address is cached, so a
// cudaDeviceReset or a switch of context cannot leave a stale one). The first
// call on a device loads that code there, so make the first call outside any
// stream capture. The ticket word is cleared before each launch; the partials
// are overwritten.
// All calls on one device share this one array: two calls whose kernels may
// overlap on the GPU (different streams, no ordering between them) race and
// give wrong sums. Serialize such calls on one stream.
//
// This translation unit is included once by kt_entry.cuh, so every built
// library exports the entry point.
#pragma once

#include "kt_common.cuh"
#include "reduce.cuh"

// KT_NOALLOC_SCRATCH_BYTES (kt_abi.h) = 16 KiB: the 16-byte ticket header plus
// 2046 fp64 partials — room for a grid of up to 2046 CTAs (this kernel uses
// KT_REDUCE_BPSM CTAs per SM: 592 on a B200).
static_assert(KT_NOALLOC_SCRATCH_BYTES % 256 == 0 && KT_NOALLOC_SCRATCH_BYTES >= 4096, "scratch size");

static __device__ __align__(256) unsigned char g_kt_noalloc_scratch[KT_NOALLOC_SCRATCH_BYTES];

namespace kt {
namespace noalloc {

// Device address of g_kt_noalloc_scratch on the current device. The name
// g_kt_noalloc_scratch in host code is only a host-side stand-in; a kernel
// must be given this address instead.
inline int scratch_for_current_device(void** out) {
  void* p = nullptr;
  int rc = cuda_status(cudaGetSymbolAddress(&p, g_kt_noalloc_scratch), "reduce noalloc: cudaGetSymbolAddress");
  if (rc != KT_OK) return rc;
  if (p == nullptr) return fail(KT_ERR_CUDA, "reduce noalloc: scratch address is null");
  *out = p;
  return KT_OK;
}

}  // namespace noalloc
}  // namespace kt

extern "C" int kt_reduce_sum_f32_noalloc(const float* x, int64_t n, double* out64, float* out32,
                                         kt_stream_t stream) {
  kt::clear_error();
  if (n < 0) return kt::fail(KT_ERR_ARG, "reduce noalloc: negative n=%lld", (long long)n);
  if (out64 == nullptr) return kt::fail(KT_ERR_ARG, "reduce noalloc: out64 is null");
  if (n > 0 && x == nullptr) return kt::fail(KT_ERR_ARG, "reduce noalloc: x is null");
  if ((reinterpret_cast<uintptr_t>(x) & 3u) != 0) return kt::fail(KT_ERR_ARG, "reduce noalloc: x not 4-byte aligned");
  const int grid = kt::reduce::grid_for(n);
  const size_t need = kt::reduce::kPartialsOffset + sizeof(double) * (size_t)grid;
  if (need > (size_t)KT_NOALLOC_SCRATCH_BYTES)
    return kt::fail(KT_ERR_UNSUPPORTED,
                    "reduce noalloc: this launch needs %zu bytes of scratch (%d CTAs), more than the fixed %d bytes",
                    need, grid, KT_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  int rc = kt::noalloc::scratch_for_current_device(&scratch);
  if (rc != KT_OK) return rc;
  // the completion ticket must start at zero; partials are fully overwritten
  rc = kt::cuda_status(cudaMemsetAsync(scratch, 0, sizeof(unsigned int), stream), "reduce noalloc: ticket reset");
  if (rc != KT_OK) return rc;
  return kt::reduce::launch_on(x, n, out64, out32, scratch, grid, stream);
}
