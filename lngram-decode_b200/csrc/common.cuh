// Shared helpers of the lngram_b200 CUDA library: status/error plumbing, dtype conversion,
// warp reductions and bounded mbarrier waits.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "../../include/lngram_b200.h"

namespace lng {

// ------------------------------------------------------------------ errors
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int cuda_status(cudaError_t e, const char* what);

#define LNG_REQUIRE(cond, msg)                                      \
  do {                                                              \
    if (!(cond)) return ::lng::fail(LNG_ERR_ARGUMENT, (msg));       \
  } while (0)

#define LNG_CUDA(call)                                              \
  do {                                                              \
    cudaError_t _e = (call);                                        \
    if (_e != cudaSuccess) return ::lng::cuda_status(_e, #call);    \
  } while (0)

#define LNG_LAUNCHED(what)                                          \
  do {                                                              \
    cudaError_t _e = cudaGetLastError();                            \
    if (_e != cudaSuccess) return ::lng::cuda_status(_e, what);     \
  } while (0)

// A device-side error word: kernels that detect a bad index or an expired bounded wait write a
// nonzero code here instead of trapping; the host checks it when it synchronises anyway.
unsigned int* device_error_word();
int check_device_error(cudaStream_t stream);

inline int dtype_size(int dt) {
  switch (dt) {
    case LNG_F32: case LNG_I32: return 4;
    case LNG_BF16: case LNG_F16: return 2;
    case LNG_U8: case LNG_BOOL: return 1;
    case LNG_I64: return 8;
    default: return 0;
  }
}
inline bool is_float_dtype(int dt) { return dt == LNG_F32 || dt == LNG_BF16 || dt == LNG_F16; }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

int num_sms();

// ------------------------------------------------------------------ device conversions
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// SiLU with the fast exponential and divide (a few ulp, far inside the fp32 / bf16 output bars);
// for x -> -inf the divisor overflows and the quotient is 0, the function's limit.
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// ------------------------------------------------------------------ mbarrier / bulk copies (sm_90+)
// Round a byte count up to a multiple of 256 (sub-buffer alignment inside one allocation).
inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `limit` polls (each try_wait itself suspends for a bounded
// hardware time slice), records `code` in the device error word and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned int* err,
                                                  unsigned int code, uint32_t limit = (1u << 22)) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  if (err) atomicCAS(err, 0u, code);
  return false;
}
// 16-byte global->shared copy through the load/store path (cp.async, L2 only); src_bytes < 16
// zero-fills the rest (0: no global read at all).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// The mbarrier's current phase also waits for this thread's earlier cp.async copies: .noinc counts
// the arrival against the expected count; without it the arrival is net zero (the pending count
// is raised first).
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// One bulk global->shared copy (TMA engine, no tensor map): 16-byte aligned addresses, size % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace lng
