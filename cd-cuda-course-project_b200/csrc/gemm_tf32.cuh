// gemm_tf32.cuh — TF32 tensor-core GEMM (tcgen05.mma kind::tf32), for sm_100a.
#pragma once
#include "kt_common.cuh"

namespace kt {
namespace gemm_tf32 {

inline int launch(const float*, const float*, float*, int64_t, int64_t, int64_t, int, int*, cudaStream_t) {
  return fail(KT_ERR_UNSUPPORTED, "gemm tf32: not implemented yet");
}

}  // namespace gemm_tf32
}  // namespace kt
