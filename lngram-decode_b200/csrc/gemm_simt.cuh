// CUDA-core GEMM C[M, N] = rowscale[m] * (A[M, K] . B[N, K]^T) (+ C) with fp32 accumulation, for
// the fp32 (parity) path and odd shapes.  64 x 64 tiles, 256 threads, 4 x 4 outputs per thread.
#pragma once

#include "common.cuh"

namespace lng {

constexpr int GS_TILE = 64, GS_K = 16;

template <typename AT, typename BT, typename CT>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const AT* __restrict__ A, int64_t lda, const BT* __restrict__ B,
                                                        int64_t ldb, CT* __restrict__ C, int64_t ldc, int64_t M,
                                                        int64_t N, int64_t K, const float* __restrict__ rowscale,
                                                        int accumulate) {
  __shared__ float As[GS_K][GS_TILE + 4];
  __shared__ float Bs[GS_K][GS_TILE + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t m0 = int64_t(blockIdx.y) * GS_TILE, n0 = int64_t(blockIdx.x) * GS_TILE;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += GS_K) {
    for (int e = threadIdx.x; e < GS_TILE * GS_K; e += 256) {
      const int r = e / GS_K, k = e % GS_K;
      const int64_t gk = k0 + k;
      As[k][r] = (m0 + r < M && gk < K) ? to_f32(A[(m0 + r) * lda + gk]) : 0.f;
      Bs[k][r] = (n0 + r < N && gk < K) ? to_f32(B[(n0 + r) * ldb + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < GS_K; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[k][ty * 4 + i];
        b[i] = Bs[k][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= M) continue;
    const float s = rowscale ? rowscale[m] : 1.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v = acc[i][j] * s;
      if (accumulate) v += to_f32(C[m * ldc + n]);
      C[m * ldc + n] = from_f32<CT>(v);
    }
  }
}

}  // namespace lng
