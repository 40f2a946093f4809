// tcgen05 (5th-generation tensor core) GEMMs for sm_100a: placeholder until the kernels land.
#pragma once

#include "common.cuh"

namespace lng {

inline int tc_gemm_bf16(const __nv_bfloat16*, int64_t, const __nv_bfloat16*, int64_t, void*, int32_t, int64_t, int64_t,
                        int64_t, int64_t, const float*, cudaStream_t) {
  return LNG_ERR_UNSUPPORTED;
}
inline int tc_router_codes(const __nv_bfloat16*, int64_t, int64_t, int64_t, const float*, int64_t, int32_t, uint8_t*,
                           cudaStream_t) {
  return LNG_ERR_UNSUPPORTED;
}

}  // namespace lng
