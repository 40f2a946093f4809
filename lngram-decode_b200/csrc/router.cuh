// Router: fp32 GEMM x . W^T with the sign-pack epilogue, and the pack of given logits.
//
// Reference: ffnmem/memory/wrapper.py:98-101 (fp32 linear router, autocast off),
// ffnmem/memory/lngram_v2.py:74-89, :1012-1017 (bit j of route r = logit[r*bits + j] > 0).
#pragma once

#include <cooperative_groups.h>

#include "address.cuh"

namespace lng {

namespace cg = cooperative_groups;

template <typename CodeOutT>
__global__ void quantize_logits_kernel(const float* __restrict__ logits, int64_t n, int64_t routes, int bits,
                                       CodeOutT* __restrict__ codes) {
  const int64_t total = n * routes;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const float* l = logits + i * bits;
    int v = 0;
    for (int j = 0; j < bits; ++j) v |= (l[j] > 0.0f ? 1 : 0) << j;
    codes[i] = static_cast<CodeOutT>(v);
  }
}

// CUDA-core fp32 router: a CTA computes 64 rows x 16 routes (all `bits` logits of each route),
// thread (ty, tx) owns rows 4*ty..4*ty+3 of route tx, so the pack needs no exchange.
// Exact fp32 FMAs in ascending k; used for fp32 router inputs and small batches.
constexpr int RT_ROWS = 64, RT_ROUTES = 16, RT_K = 32, RT_MAXBITS = 8;

template <typename XT, typename CodeOutT>
__global__ void __launch_bounds__(256) router_simt_kernel(const XT* __restrict__ x, int64_t n, int64_t in_dim,
                                                          int64_t x_stride, const float* __restrict__ w,
                                                          int64_t routes, int bits, CodeOutT* __restrict__ codes,
                                                          float* __restrict__ logits) {
  __shared__ float As[RT_K][RT_ROWS + 1];
  __shared__ float Bs[RT_K][RT_ROUTES * RT_MAXBITS + 1];
  const int tx = threadIdx.x % RT_ROUTES;  // route within the tile
  const int ty = threadIdx.x / RT_ROUTES;  // row group (4 rows)
  const int64_t row0 = int64_t(blockIdx.x) * RT_ROWS;
  const int64_t route0 = int64_t(blockIdx.y) * RT_ROUTES;
  const int ncol = RT_ROUTES * bits;       // logits columns in the tile
  const int64_t C = routes * bits;
  float acc[4][RT_MAXBITS];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < RT_MAXBITS; ++j) acc[i][j] = 0.f;

  for (int64_t k0 = 0; k0 < in_dim; k0 += RT_K) {
    for (int e = threadIdx.x; e < RT_ROWS * RT_K; e += blockDim.x) {
      const int r = e / RT_K, k = e % RT_K;
      const int64_t gr = row0 + r, gk = k0 + k;
      As[k][r] = (gr < n && gk < in_dim) ? to_f32(x[gr * x_stride + gk]) : 0.f;
    }
    for (int e = threadIdx.x; e < ncol * RT_K; e += blockDim.x) {
      const int c = e / RT_K, k = e % RT_K;
      const int64_t gc = route0 * bits + c, gk = k0 + k;
      Bs[k][c] = (gc < C && gk < in_dim) ? w[gc * in_dim + gk] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int k = 0; k < RT_K; ++k) {
      float a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < RT_MAXBITS; ++j) {
        if (j < bits) {
          const float b = Bs[k][tx * bits + j];
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[i][j] = fmaf(a[i], b, acc[i][j]);
        }
      }
    }
    __syncthreads();
  }
  const int64_t r = route0 + tx;
  if (r >= routes) return;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gr = row0 + ty * 4 + i;
    if (gr >= n) continue;
    int v = 0;
#pragma unroll
    for (int j = 0; j < RT_MAXBITS; ++j) {
      if (j < bits) {
        v |= (acc[i][j] > 0.f ? 1 : 0) << j;
        if (logits) logits[gr * C + r * bits + j] = acc[i][j];
      }
    }
    codes[gr * routes + r] = static_cast<CodeOutT>(v);
  }
}

// Small-batch CUDA-core router: a cluster of RS_SPLIT CTAs shares one block of RS_RPC routes (all
// `bits` logits of each), each CTA summing 1/RS_SPLIT of the input features for RS_ROWS rows; rank 0
// adds the partial logits of the ranks in rank order through distributed shared memory
// (deterministic) and packs the codes.  For row counts that leave router_simt_kernel's row tiles
// too few CTAs to fill the GPU (drafting: one row per sequence).
constexpr int RS_SPLIT = 8, RS_RPC = 4, RS_ROWS = 64, RS_KC = 64;

template <typename XT, typename CodeOutT>
__global__ void __cluster_dims__(RS_SPLIT, 1, 1) __launch_bounds__(256)
    router_small_kernel(const XT* __restrict__ x, int64_t n, int64_t in_dim, int64_t x_stride,
                        const float* __restrict__ w, int64_t routes, int bits, CodeOutT* __restrict__ codes,
                        float* __restrict__ logits) {
  __shared__ float xs[RS_ROWS][RS_KC + 1];
  __shared__ float ws[RS_RPC * RT_MAXBITS][RS_KC + 1];
  __shared__ float part[RS_ROWS * RS_RPC * RT_MAXBITS];
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank();
  const int r = threadIdx.x >> 2, g = threadIdx.x & 3;  // row within the tile, route within the block
  const int64_t rb = blockIdx.x / RS_SPLIT;              // route block
  const int64_t row0 = int64_t(blockIdx.y) * RS_ROWS;
  const int ncol = RS_RPC * bits;
  const int64_t col0 = rb * RS_RPC * bits;               // first logit column of the block
  const int64_t C = routes * bits;
  const int64_t ks = (in_dim + RS_SPLIT - 1) / RS_SPLIT;
  const int64_t kbeg = int64_t(rank) * ks, kend = kbeg + ks < in_dim ? kbeg + ks : in_dim;
  float acc[RT_MAXBITS];
#pragma unroll
  for (int j = 0; j < RT_MAXBITS; ++j) acc[j] = 0.f;
  // the next chunk's x and w are loaded into registers (all loads in flight together) while the
  // current chunk is multiplied out of shared memory
  constexpr int XPT = RS_ROWS * RS_KC / 256, WPT = RS_RPC * RT_MAXBITS * RS_KC / 256;
  float xr[XPT], wr[WPT];
  auto fetch = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < XPT; ++i) {
      const int e = threadIdx.x + i * 256, rr = e / RS_KC, kk = e % RS_KC;
      const int64_t gr = row0 + rr, gk = k0 + kk;
      xr[i] = (gr < n && gk < kend) ? to_f32(x[gr * x_stride + gk]) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < WPT; ++i) {
      const int e = threadIdx.x + i * 256, c = e / RS_KC, kk = e % RS_KC;
      const int64_t gc = col0 + c, gk = k0 + kk;
      wr[i] = (c < ncol && gc < C && gk < kend) ? w[gc * in_dim + gk] : 0.f;
    }
  };
  if (kbeg < kend) fetch(kbeg);
  for (int64_t k0 = kbeg; k0 < kend; k0 += RS_KC) {
    __syncthreads();  // the previous chunk's products are done with the tiles
#pragma unroll
    for (int i = 0; i < XPT; ++i) {
      const int e = threadIdx.x + i * 256;
      xs[e / RS_KC][e % RS_KC] = xr[i];
    }
#pragma unroll
    for (int i = 0; i < WPT; ++i) {
      const int e = threadIdx.x + i * 256;
      ws[e / RS_KC][e % RS_KC] = wr[i];
    }
    __syncthreads();
    if (k0 + RS_KC < kend) fetch(k0 + RS_KC);
#pragma unroll 4
    for (int kk = 0; kk < RS_KC; ++kk) {
      const float a = xs[r][kk];
#pragma unroll
      for (int j = 0; j < RT_MAXBITS; ++j)
        if (j < bits) acc[j] = fmaf(a, ws[g * bits + j][kk], acc[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < RT_MAXBITS; ++j)
    if (j < bits) part[(r * RS_RPC + g) * RT_MAXBITS + j] = acc[j];
  cluster.sync();
  if (rank == 0) {
    float sum[RT_MAXBITS];
#pragma unroll
    for (int j = 0; j < RT_MAXBITS; ++j) sum[j] = 0.f;
    for (unsigned q = 0; q < RS_SPLIT; ++q) {
      const float* pq = cluster.map_shared_rank(part, q);
#pragma unroll
      for (int j = 0; j < RT_MAXBITS; ++j)
        if (j < bits) sum[j] += pq[(r * RS_RPC + g) * RT_MAXBITS + j];
    }
    const int64_t gr = row0 + r, route = rb * RS_RPC + g;
    if (gr < n && route < routes) {
      int v = 0;
#pragma unroll
      for (int j = 0; j < RT_MAXBITS; ++j) {
        if (j < bits) {
          v |= (sum[j] > 0.f ? 1 : 0) << j;
          if (logits) logits[gr * C + route * bits + j] = sum[j];
        }
      }
      codes[gr * routes + route] = static_cast<CodeOutT>(v);
    }
  }
  cluster.sync();  // the other ranks' partials stay resident until rank 0 has read them
}

// embed2 router features (ffnmem/memory/router.py:50-69): one 128-thread CTA per item, the
// previous and current token rows each RMS-normalised with their own weight, written to the first
// 2d columns of the item's output row (row stride out_stride >= 2d); with `split`, also the row's three
// bf16 parts [3 x split_width] (split_width = the router's input width) for the tensor-core router.
template <typename ET>
__global__ void __launch_bounds__(128) embed2_features_kernel(const int64_t* __restrict__ cur,
                                                              const int64_t* __restrict__ prev, int64_t n,
                                                              const ET* __restrict__ E, int64_t vocab, int64_t d,
                                                              const float* __restrict__ prev_w,
                                                              const float* __restrict__ cur_w,
                                                              const float* __restrict__ start, float eps,
                                                              float* __restrict__ out, int64_t out_stride,
                                                              __nv_bfloat16* __restrict__ split = nullptr,
                                                              int64_t split_width = 0) {
  __shared__ float red[2][4];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t item = blockIdx.x; item < n; item += gridDim.x) {
    const int64_t tc = cur[item];
    const int64_t tp = prev ? prev[item] : -1;
    if (tc < 0 || tc >= vocab || tp >= vocab) {
      if (threadIdx.x == 0) atomicCAS(&g_error_word, 0u, (unsigned int)DEV_ERR_TOKEN_RANGE);
      continue;
    }
    float* o = out + item * out_stride;
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      const int64_t tok = part == 0 ? tp : tc;
#pragma unroll 8
      for (int64_t j = threadIdx.x; j < d; j += blockDim.x) {
        const float v = tok >= 0 ? to_f32(E[tok * d + j]) : start[j];
        ss[part] += v * v;
      }
      ss[part] = warp_sum(ss[part]);
      if (lane == 0) red[part][warp] = ss[part];
    }
    __syncthreads();
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      const float tot = red[part][0] + red[part][1] + red[part][2] + red[part][3];
      const float rs = rsqrtf(tot / float(d) + eps);
      const float* wv = part == 0 ? prev_w : cur_w;
      const int64_t tok = part == 0 ? tp : tc;
#pragma unroll 8
      for (int64_t j = threadIdx.x; j < d; j += blockDim.x) {
        const float v = tok >= 0 ? to_f32(E[tok * d + j]) : start[j];
        const float y = v * rs * wv[j];
        o[part * d + j] = y;
        if (split) {  // the row's three bf16 parts (split_rows_bf16x3_kernel's arithmetic), for the router
          const __nv_bfloat16 a = __float2bfloat16_rn(y);
          const float r1 = y - __bfloat162float(a);
          const __nv_bfloat16 b = __float2bfloat16_rn(r1);
          __nv_bfloat16* xs = split + item * 3 * split_width + part * d + j;
          xs[0] = a;
          xs[split_width] = b;
          xs[2 * split_width] = __float2bfloat16_rn(r1 - __bfloat162float(b));
        }
      }
    }
    __syncthreads();
  }
}

}  // namespace lng
