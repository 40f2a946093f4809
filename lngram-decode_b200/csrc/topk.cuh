// Draft logits h . E^T with a fused top-k (never materialising the [n, V] logits unless asked):
// ffnmem/memory/draft.py:88-91 (logits against the tied embedding), drafting/cpu/drafter.cpp:537-556
// (full-vocabulary scoring, top-k by (logit desc, id asc)).
#pragma once

#include "address.cuh"

namespace lng {

constexpr int TK_ROWS = 8;     // draft rows per CTA
constexpr int TK_VC = 256;     // vocabulary entries per CTA
constexpr int TK_MAXK = 8;

__device__ __forceinline__ bool tk_better(float v, int64_t id, float bv, int64_t bid) {
  return v > bv || (v == bv && id < bid);
}

// Pass 1: logits of TK_ROWS rows x TK_VC vocab entries, then each row's top-k of the chunk into
// scratch [n, nchunks, k] (value, id).
template <typename ET>
__global__ void __launch_bounds__(256) logits_chunk_topk_kernel(const float* __restrict__ h, int64_t n, int64_t d,
                                                                const ET* __restrict__ E, int64_t V, int k,
                                                                float* __restrict__ cand_v, int64_t* __restrict__ cand_i,
                                                                float* __restrict__ logits) {
  extern __shared__ float tk_sm[];
  float* hs = tk_sm;                    // [TK_ROWS, d]
  float* ls = hs + TK_ROWS * d;         // [TK_ROWS, TK_VC]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int64_t r0 = int64_t(blockIdx.y) * TK_ROWS;
  const int64_t v0 = int64_t(blockIdx.x) * TK_VC;
  const int64_t nchunks = gridDim.x;
  for (int64_t e = threadIdx.x; e < TK_ROWS * d; e += blockDim.x) {
    const int64_t r = e / d;
    hs[e] = (r0 + r < n) ? h[(r0 + r) * d + e % d] : 0.f;
  }
  __syncthreads();
  for (int vl = warp; vl < TK_VC; vl += nw) {
    const int64_t v = v0 + vl;
    float acc[TK_ROWS];
#pragma unroll
    for (int r = 0; r < TK_ROWS; ++r) acc[r] = 0.f;
    if (v < V) {
      const ET* er = E + v * d;
      for (int64_t j = lane; j < d; j += 32) {
        const float ev = to_f32(er[j]);
#pragma unroll
        for (int r = 0; r < TK_ROWS; ++r) acc[r] = fmaf(ev, hs[r * d + j], acc[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < TK_ROWS; ++r) {
      const float s = warp_sum(acc[r]);
      if (lane == 0) {
        ls[r * TK_VC + vl] = v < V ? s : -INFINITY;
        if (logits && v < V && r0 + r < n) logits[(r0 + r) * V + v] = s;
      }
    }
  }
  __syncthreads();
  for (int r = warp; r < TK_ROWS; r += nw) {
    if (r0 + r >= n) continue;
    const float* lr = ls + r * TK_VC;
    float prev_v = INFINITY;
    int64_t prev_i = -1;
    for (int kk = 0; kk < k; ++kk) {
      float bv = -INFINITY;
      int64_t bi = INT64_MAX;
      for (int vl = lane; vl < TK_VC; vl += 32) {
        const int64_t id = v0 + vl;
        const float v = lr[vl];
        // strictly after the previous pick in (value desc, id asc) order
        const bool after = v < prev_v || (v == prev_v && id > prev_i);
        if (id < V && after && tk_better(v, id, bv, bi)) {
          bv = v;
          bi = id;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (tk_better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      const int64_t slot = ((r0 + r) * nchunks + blockIdx.x) * k + kk;
      if (lane == 0) {
        cand_v[slot] = bv;
        cand_i[slot] = bi == INT64_MAX ? -1 : bi;
      }
      prev_v = bv;
      prev_i = bi;
    }
  }
}

// Pass 2: merge each row's chunk candidates into the final top-k (one warp per row).
__global__ void topk_merge_kernel(const float* __restrict__ cand_v, const int64_t* __restrict__ cand_i, int64_t n,
                                  int64_t nchunks, int k, int64_t* __restrict__ ids, float* __restrict__ vals) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5;
  if (row >= n) return;
  const int64_t nc = nchunks * k;
  const float* cv = cand_v + row * nc;
  const int64_t* ci = cand_i + row * nc;
  float prev_v = INFINITY;
  int64_t prev_i = -1;
  for (int kk = 0; kk < k; ++kk) {
    float bv = -INFINITY;
    int64_t bi = INT64_MAX;
    for (int64_t c = lane; c < nc; c += 32) {
      const float v = cv[c];
      const int64_t id = ci[c];
      if (id < 0) continue;
      // strictly after the previous pick in (value desc, id asc) order
      const bool after = v < prev_v || (v == prev_v && id > prev_i);
      if (after && tk_better(v, id, bv, bi)) {
        bv = v;
        bi = id;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (tk_better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      ids[row * k + kk] = bi == INT64_MAX ? -1 : bi;
      vals[row * k + kk] = bi == INT64_MAX ? -INFINITY : bv;
    }
    prev_v = bv;
    prev_i = bi;
  }
}

}  // namespace lng
