// fa_fwd.cuh — flash-attention forward, bf16, tcgen05, for sm_100a.
#pragma once
#include "kt_common.cuh"

namespace kt {
namespace fa {

inline int launch(const uint16_t*, const uint16_t*, const uint16_t*, uint16_t*, int64_t, int64_t, int64_t, int64_t,
                  float, int, cudaStream_t) {
  return fail(KT_ERR_UNSUPPORTED, "flash-attention forward: not implemented yet");
}

}  // namespace fa
}  // namespace kt
