// Materialised route tokens: _lookup_route_chunk (ffnmem/memory/lngram_v2.py:1047-1113) and the
// windowed lookup of lookup_rows_at / tree_route_tokens (ffnmem/memory/draft.py:26-47,
// drafting/tree.py:130-136).  One warp per (item, route): the warp's lanes copy the order rows
// (or zeros) of one route token with 16-byte vector accesses where the row width allows.
#pragma once

#include "address.cuh"

namespace lng {

template <typename CodeT, typename TabT, typename OutT>
__global__ void lookup_kernel(TableSet ts, CodeSource src, int64_t M, int64_t route_start, int64_t route_end,
                              OutT* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t nr = route_end - route_start;
  const int64_t total = M * nr;
  const int64_t Dt = int64_t(ts.n_orders) * ts.mem_dim;
  for (int64_t w = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; w < total;
       w += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    const int64_t item = w / nr;
    const int64_t r = route_start + w % nr;
    OutT* dst = out + w * Dt;
    for (int o = 0; o < ts.n_orders; ++o) {
      const int64_t row = ngram_row<CodeT>(src, item, r, ts.order[o], ts.bits);
      const TabT* s = static_cast<const TabT*>(ts.tab[o]) + (row < 0 ? 0 : row) * ts.mem_dim;
      OutT* d = dst + o * ts.mem_dim;
      for (int64_t j = lane; j < ts.mem_dim; j += 32) {
        d[j] = row < 0 ? from_f32<OutT>(0.f) : from_f32<OutT>(to_f32(s[j]));
      }
    }
  }
}

// Same-dtype copy with 16-byte vectors when a row is a whole number of vectors.
template <typename CodeT>
__global__ void lookup_vec_kernel(TableSet ts, CodeSource src, int64_t M, int64_t route_start, int64_t route_end,
                                  int elem_bytes, uint4* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t nr = route_end - route_start;
  const int64_t total = M * nr;
  const int64_t vecs = ts.mem_dim * elem_bytes / 16;  // per order row
  for (int64_t w = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; w < total;
       w += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    const int64_t item = w / nr;
    const int64_t r = route_start + w % nr;
    uint4* dst = out + w * vecs * ts.n_orders;
    for (int o = 0; o < ts.n_orders; ++o) {
      const int64_t row = ngram_row<CodeT>(src, item, r, ts.order[o], ts.bits);
      const uint4* s = reinterpret_cast<const uint4*>(ts.tab[o]) + (row < 0 ? 0 : row) * vecs;
      for (int64_t j = lane; j < vecs; j += 32) {
        dst[o * vecs + j] = row < 0 ? make_uint4(0, 0, 0, 0) : __ldg(s + j);
      }
    }
  }
}

}  // namespace lng
