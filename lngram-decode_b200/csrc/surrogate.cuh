// Backward of the training-mode lookup (ffnmem/memory/lngram_v2.py:1047-1113): the rows' gradient into
// the order tables (the nn.Embedding backward of the gathered rows) and the route-code gradient of the
// surrogate (_LngramSurrogate.backward, :359-447).
//
// Surrogate, for the window of order n ending at t (row idx = r A^n + sum_k c[t-n+1+k] A^k) and the
// gradient g of its row:
//   approximate -- digit k, bit j: flip that address bit, s = (E[idx ^ 2^(k bits + j)] - E[idx]) . g, with
//                  the sign - when the bit is set; summed into dq[t-n+1+k, j], then multiplied by
//                  scale T p (1 - p), p = sigmoid(T q);
//   exact       -- digit k, every code c: dq[t-n+1+k] += scale T P(c) (bit(c) - p) (E[row(c)] . g), P(c) the
//                  probability of code c under independent bits p.
// One warp per (b, position, route) gathers over the windows whose digit sits at that position (in
// digit order, as the reference adds them), so every value is written once: no atomics, deterministic.
// Masked windows (before the start, across segments, invalid tokens) have a zero gradient and are
// skipped, as the reference's grad * mask makes them.
#pragma once

#include "address.cuh"

namespace lng {

constexpr int SG_MAXE = 8;     // row elements per lane: mem_dim <= 256
constexpr int SG_MAXBITS = 8;

struct LookupGradParams {
  TableSet ts;
  int table_dtype;
  CodeSource src;         // sequence mode over codes [B, T, R] (segment / valid-token masks included)
  int64_t B, T;
  int64_t route_start, Rc;  // the chunk's routes [route_start, route_start + Rc)
  const void* grad;       // [B, T, Rc, Dt] gradient of the route tokens
  int grad_dtype;
  const float* q;         // [B, T, Rq, bits] route logits (the chunk's routes at route_start ..)
  int64_t Rq;
  float temperature, scale;
  int exact;
  float* grad_q;          // [B, T, Rc, bits]
  float* gtab[LNG_MAX_ORDERS];  // fp32 [rows, mem_dim] per order (accumulated), or null
};

__device__ __forceinline__ float load_any(const void* p, int dtype, int64_t i) {
  if (dtype == LNG_F32) return static_cast<const float*>(p)[i];
  if (dtype == LNG_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

template <typename CodeT>
__global__ void surrogate_grad_kernel(LookupGradParams p) {
  const int lane = threadIdx.x & 31;
  const int bits = p.ts.bits;
  const int64_t md = p.ts.mem_dim;
  const int64_t Dt = int64_t(p.ts.n_orders) * md;
  const float st = p.scale * p.temperature;
  const int64_t total = p.B * p.T * p.Rc;
  for (int64_t w = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; w < total;
       w += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    const int64_t rl = w % p.Rc;
    const int64_t bt = w / p.Rc;
    const int64_t b = bt / p.T, pos = bt % p.T;
    const int64_t r = p.route_start + rl;
    float pr[SG_MAXBITS], acc[SG_MAXBITS];
#pragma unroll
    for (int j = 0; j < SG_MAXBITS; ++j) {
      acc[j] = 0.f;
      pr[j] = j < bits ? sigmoid_f(p.temperature * p.q[(bt * p.Rq + r) * bits + j]) : 0.f;
    }
    const int64_t src_code = read_code<CodeT>(p.src, bt, r);
    for (int o = 0; o < p.ts.n_orders; ++o) {
      const int n = p.ts.order[o];
      const void* tab = p.ts.tab[o];
      for (int k = 0; k < n; ++k) {  // this position is digit k of the window ending at t_end
        const int64_t t_end = pos - k + n - 1;
        if (pos - k < 0 || t_end >= p.T) continue;
        const int64_t idx = ngram_row<CodeT>(p.src, b * p.T + t_end, r, n, bits);
        if (idx < 0) continue;
        float g[SG_MAXE];
        const int64_t gbase = ((b * p.T + t_end) * p.Rc + rl) * Dt + int64_t(o) * md;
#pragma unroll
        for (int e = 0; e < SG_MAXE; ++e) {
          const int64_t j = lane + 32 * e;
          g[e] = j < md ? load_any(p.grad, p.grad_dtype, gbase + j) : 0.f;
        }
        auto dot = [&](int64_t row) {
          float s = 0.f;
#pragma unroll
          for (int e = 0; e < SG_MAXE; ++e) {
            const int64_t j = lane + 32 * e;
            if (j < md) s = fmaf(load_any(tab, p.table_dtype, row * md + j), g[e], s);
          }
          return warp_sum(s);
        };
        const int64_t digit = int64_t(1) << (int64_t(k) * bits);
        if (!p.exact) {
          const float cur = dot(idx);
          for (int j = 0; j < bits; ++j) {
            const int64_t mask = digit << j;
            const float flipped = dot(idx ^ mask);
            const float sign = (idx & mask) ? -1.f : 1.f;
            acc[j] += (flipped - cur) * sign;
          }
        } else {
          const int64_t base = idx - src_code * digit;
          for (int64_t c = 0; c < (int64_t(1) << bits); ++c) {
            const float d = dot(base + c * digit);
            float cp = 1.f;
            for (int j = 0; j < bits; ++j) cp *= ((c >> j) & 1) ? pr[j] : 1.f - pr[j];
            for (int j = 0; j < bits; ++j) acc[j] += cp * (float((c >> j) & 1) - pr[j]) * d * st;
          }
        }
      }
    }
    if (lane == 0) {
      float* out = p.grad_q + (bt * p.Rc + rl) * bits;
      for (int j = 0; j < bits; ++j) out[j] = p.exact ? acc[j] : acc[j] * (st * pr[j] * (1.f - pr[j]));
    }
  }
}

// The rows' gradient: grad_table[o][row of (b, t, r)] += grad[b, t, r, order o's columns] for every
// valid window (one warp per (b, t, route, order); fp32 atomics, as several windows may read one row).
template <typename CodeT>
__global__ void table_grad_kernel(LookupGradParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t md = p.ts.mem_dim;
  const int64_t Dt = int64_t(p.ts.n_orders) * md;
  const int64_t total = p.B * p.T * p.Rc * p.ts.n_orders;
  for (int64_t w = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; w < total;
       w += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    const int o = int(w % p.ts.n_orders);
    const int64_t wr = w / p.ts.n_orders;
    const int64_t rl = wr % p.Rc;
    const int64_t bt = wr / p.Rc;
    if (!p.gtab[o]) continue;
    const int64_t idx = ngram_row<CodeT>(p.src, bt, p.route_start + rl, p.ts.order[o], p.ts.bits);
    if (idx < 0) continue;
    const int64_t gbase = (bt * p.Rc + rl) * Dt + int64_t(o) * md;
    for (int64_t j = lane; j < md; j += 32) atomicAdd(p.gtab[o] + idx * md + j, load_any(p.grad, p.grad_dtype, gbase + j));
  }
}

}  // namespace lng
