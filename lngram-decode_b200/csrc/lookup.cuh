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

// Route tokens from tables the device reaches over PCIe (pinned host memory mapped into the device
// address space): the same per-(item, route) warp walk with plain 16-byte loads -- no read-only-cache
// or bulk-copy path -- so each row crosses PCIe once, straight into the output.
template <typename CodeT>
__global__ void lookup_host_kernel(TableSet ts, CodeSource src, int64_t M, int64_t route_start, int64_t route_end,
                                   int elem_bytes, uint4* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t nr = route_end - route_start;
  const int64_t total = M * nr;
  const int64_t vecs = ts.mem_dim * elem_bytes / 16;
  for (int64_t w = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; w < total;
       w += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    const int64_t item = w / nr;
    const int64_t r = route_start + w % nr;
    uint4* dst = out + w * vecs * ts.n_orders;
    for (int o = 0; o < ts.n_orders; ++o) {
      const int64_t row = ngram_row<CodeT>(src, item, r, ts.order[o], ts.bits);
      const uint4* s = reinterpret_cast<const uint4*>(ts.tab[o]) + (row < 0 ? 0 : row) * vecs;
      for (int64_t j = lane; j < vecs; j += 32) dst[o * vecs + j] = row < 0 ? make_uint4(0, 0, 0, 0) : s[j];
    }
  }
}

// The serving-layout copy of one order's table (serving/layout.py:26-43): within every route's block of
// A^n rows, row j of dst is row reverse_digits(j) of src (the n base-A digits in reverse order).
// One warp per destination row, 16-byte vectors.
__global__ void serving_permute_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t rows,
                                       int order, int bits, int64_t vecs) {
  const int lane = threadIdx.x & 31;
  const int64_t block = int64_t(1) << (bits * order);
  const int64_t amask = (int64_t(1) << bits) - 1;
  for (int64_t row = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; row < rows;
       row += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    const int64_t r = row / block, j = row % block;
    int64_t rev = 0;
    for (int k = 0; k < order; ++k) rev |= ((j >> (k * bits)) & amask) << ((order - 1 - k) * bits);
    const uint4* s = src + (r * block + rev) * vecs;
    uint4* d = dst + row * vecs;
    for (int64_t v = lane; v < vecs; v += 32) d[v] = s[v];
  }
}

// The packed n-gram suffix of the incremental readout (lngram_v2.py:1714-1760): packed[b, r] holds the
// codes of the last maxn positions, the newest in digit maxn - 1 (digits `bits` wide).  advance == 0
// packs the last min(T, maxn) positions of codes [B, T, R] (_pack_suffix); advance == 1 shifts
// packed_in down one digit and puts codes [B, 1, R] in the top digit (_advance_packed).  The digits are
// also written unpacked as window codes [B, maxn, R] (slot j = digit j) for the window-mode readout.
template <typename CodeT>
__global__ void packed_suffix_kernel(const CodeT* __restrict__ codes, int64_t B, int64_t T, int64_t R, int bits,
                                     int maxn, const int32_t* __restrict__ packed_in, int advance,
                                     int32_t* __restrict__ packed_out, uint8_t* __restrict__ window) {
  const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= B * R) return;
  const int64_t b = i / R, r = i % R;
  const uint32_t amask = (1u << bits) - 1;
  uint32_t v = 0;
  if (advance) {
    const uint32_t c = uint32_t(codes[b * R + r]) & amask;
    v = (uint32_t(packed_in[i]) >> bits) | (c << ((maxn - 1) * bits));
  } else {
    const int64_t keep = T < maxn ? T : maxn;
    const int first = int(maxn - keep);
    for (int64_t k = 0; k < keep; ++k) {
      const uint32_t c = uint32_t(codes[(b * T + T - keep + k) * R + r]) & amask;
      v |= c << ((first + int(k)) * bits);
    }
  }
  packed_out[i] = int32_t(v);
  if (window)
    for (int j = 0; j < maxn; ++j) window[(b * maxn + j) * R + r] = uint8_t((v >> (j * bits)) & amask);
}

// A tree's node windows: ctx[b, i, w, r] = gok[i, w] ? (gidx[i, w] < h0 ? the cached code at L - h0 + gidx
// : the new code of node gidx - h0) : 0; and the nodes' new codes stored in the cache at L .. L+n-1 (slots
// disjoint from the history read here, so one launch does both).
__global__ void tree_windows_kernel(const uint8_t* __restrict__ codes_new, uint8_t* cache_codes, int64_t B, int64_t n,
                                    int64_t W, int64_t R, int64_t L, int64_t h0, int64_t max_len,
                                    const int64_t* __restrict__ gidx, const uint8_t* __restrict__ gok,
                                    uint8_t* __restrict__ ctx) {
  const int64_t nctx = B * n * W * R, nnew = B * n * R;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < nctx + nnew;
       e += int64_t(gridDim.x) * blockDim.x) {
    if (e < nctx) {
      const int64_t r = e % R, w = (e / R) % W, i = (e / (R * W)) % n, b = e / (R * W * n);
      uint8_t v = 0;
      if (gok[i * W + w]) {
        const int64_t g = gidx[i * W + w];
        v = g < h0 ? cache_codes[(b * max_len + L - h0 + g) * R + r] : codes_new[(b * n + g - h0) * R + r];
      }
      ctx[e] = v;
    } else {
      const int64_t f = e - nctx, r = f % R, i = (f / R) % n, b = f / (R * n);
      cache_codes[(b * max_len + L + i) * R + r] = codes_new[f];
    }
  }
}

}  // namespace lng

