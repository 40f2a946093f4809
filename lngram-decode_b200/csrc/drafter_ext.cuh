// Drafter features beyond the embed2 router with full-vocabulary scoring:
//
// * the SD-C diagonal SSM over token embeddings (ffnmem/memory/ssm.py:1-11, :49-55; the C++ drafter's
//   advance, drafting/cpu/drafter.cpp:396-403): u[t] = W_in RMSNorm(E[x[t]]), s[t] = a s[t-1] + (1-a) u[t]
//   with s[-1] = 0, whose state joins the router features (router_kind "embed2_ssm", drafter.cpp:412) and
//   the draft query (query_ssm: q += W_sq s, drafter.cpp:505-508);
// * the sketch shortlist (drafter.cpp:438-474, drafting/cpu_drafter.py:191-217): per position, every
//   valid (order, route) row's K (token id, count) sketch entries are summed per token id, the ids are
//   ordered by (count desc, id asc) and cut at `cap`, then padded from the bundle's fallback list with ids
//   not already taken; the draft logits are E[id] . h over that list only, the top-k by (logit desc,
//   list position asc) (drafter.cpp:547-556).
#pragma once

#include "address.cuh"

namespace lng {

// ------------------------------------------------------------------ SSM recurrence
// One thread per (sequence, channel): s = a s + (1 - a) u along the sequence's L positions, starting
// from s0 (or zero), written as states[seq, t - out_from, :] for t >= out_from.  The products and the
// sum are rounded separately (no fused multiply-add), as the fp32 reference evaluates them.
__global__ void ssm_scan_kernel(const float* __restrict__ u, int64_t nseq, int64_t L, int64_t N,
                                const float* __restrict__ a, const float* __restrict__ s0, int64_t out_from,
                                float* __restrict__ states) {
  const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i >= nseq * N) return;
  const int64_t seq = i / N, ch = i % N;
  const float ac = a[ch], bc = __fsub_rn(1.f, ac);
  float s = s0 ? s0[seq * N + ch] : 0.f;
  const float* up = u + seq * L * N + ch;
  float* op = states + seq * (L - out_from) * N + ch;
  for (int64_t t = 0; t < L; ++t) {
    s = __fadd_rn(__fmul_rn(ac, s), __fmul_rn(bc, up[t * N]));
    if (t >= out_from) op[(t - out_from) * N] = s;
  }
}

// Rows of `src` [n, N] copied into columns [col, col + N) of `dst` [n, dst_stride] (the SSM state
// appended to the embed2 router features).
__global__ void copy_cols_kernel(const float* __restrict__ src, int64_t n, int64_t N, float* __restrict__ dst,
                                 int64_t dst_stride, int64_t col) {
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n * N; e += int64_t(gridDim.x) * blockDim.x)
    dst[(e / N) * dst_stride + col + e % N] = src[e];
}

// ------------------------------------------------------------------ sketch shortlist
struct ShortlistParams {
  CodeSource src;
  int orders[LNG_MAX_ORDERS];
  int n_orders;
  int bits;
  int64_t R;
  const int32_t* sk_ids[LNG_MAX_ORDERS];  // [R * 2^(bits*n), K] token ids
  const int32_t* sk_cnt[LNG_MAX_ORDERS];  // [R * 2^(bits*n), K] counts (<= 0: empty slot)
  int K;
  const int32_t* fallback;                // [n_fallback]
  int n_fallback;
  int cap;
  int64_t V, d;
  const void* E;
  int e_dtype;
  const float* hn;                        // [M, d] draft hidden states
  int64_t M;
  int ht;                                 // hash-table slots (power of two >= 2 x candidates)
  // draft mode (topk > 0): top-k of the shortlist -> ids / vals [M, topk]
  int topk;
  int64_t* ids;
  float* vals;
  // trace mode (topk == 0): the shortlist and its logits in list order -> [M, S]
  int64_t S;
  int64_t* list_ids;
  float* list_lg;
};

constexpr int SL_THREADS = 256;
constexpr int SL_MAX_SLOTS = 16384;     // hash slots per item (128 KB of shared memory)
constexpr uint64_t SL_ID_BITS = 20;     // token ids < 2^20 - 1
constexpr uint64_t SL_CNT_BITS = 44;    // per-id count sums (<= 8192 entries x (2^31 - 1) < 2^44)
constexpr uint64_t SL_CNT_MASK = (1ull << SL_CNT_BITS) - 1;

__device__ __forceinline__ float dot_row(const void* E, int e_dtype, int64_t row, int64_t d, const float* h, int lane) {
  float acc = 0.f;
  if (e_dtype == LNG_F32) {
    const float* e = static_cast<const float*>(E) + row * d;
    for (int64_t j = lane; j < d; j += 32) acc = fmaf(e[j], h[j], acc);
  } else if (e_dtype == LNG_BF16) {
    const __nv_bfloat16* e = static_cast<const __nv_bfloat16*>(E) + row * d;
    for (int64_t j = lane; j < d; j += 32) acc = fmaf(__bfloat162float(e[j]), h[j], acc);
  } else {
    const __half* e = static_cast<const __half*>(E) + row * d;
    for (int64_t j = lane; j < d; j += 32) acc = fmaf(__half2float(e[j]), h[j], acc);
  }
  return warp_sum(acc);
}

// one lane's dot product of a whole row (the rare full-vocabulary case of an empty list)
__device__ __forceinline__ float dot_row_serial(const void* E, int e_dtype, int64_t row, int64_t d, const float* h) {
  float acc = 0.f;
  for (int64_t j = 0; j < d; ++j) {
    const float e = e_dtype == LNG_F32    ? static_cast<const float*>(E)[row * d + j]
                    : e_dtype == LNG_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(E)[row * d + j])
                                          : __half2float(static_cast<const __half*>(E)[row * d + j]);
    acc = fmaf(e, h[j], acc);
  }
  return acc;
}

// (logit desc, position asc) order of two candidates
__device__ __forceinline__ bool better(float va, int64_t pa, float vb, int64_t pb) {
  return va > vb || (va == vb && pa < pb);
}

// Insert (v, i) into a lane's sorted top-k list (k <= TK_MAXK).
__device__ __forceinline__ void topk_insert(float (&bv)[TK_MAXK], int64_t (&bp)[TK_MAXK], int k, float v, int64_t i) {
#pragma unroll
  for (int j = TK_MAXK - 1; j >= 0; --j) {
    if (j < k && better(v, i, bv[j], bp[j])) {
      if (j + 1 < TK_MAXK) {
        bv[j + 1] = bv[j];
        bp[j + 1] = bp[j];
      }
      bv[j] = v;
      bp[j] = i;
    }
  }
}

// One CTA per item.  Shared memory: the hash slots u64[ht] (tag = id + 1 in the top 20 bits, the id's
// count sum in the low 44), reused in place as the sort keys; the hidden state float[d]; the list
// int32[cap] and its logits float[cap].
template <typename CodeT>
__global__ void __launch_bounds__(SL_THREADS) shortlist_kernel(ShortlistParams p) {
  extern __shared__ __align__(16) unsigned char sl_smem[];
  unsigned long long* slot = reinterpret_cast<unsigned long long*>(sl_smem);
  float* hs = reinterpret_cast<float*>(slot + p.ht);
  int32_t* list = reinterpret_cast<int32_t*>(hs + p.d);
  float* lg = reinterpret_cast<float*>(list + p.cap);
  __shared__ int n_list;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = SL_THREADS / 32;
  const uint32_t mask = uint32_t(p.ht - 1);
  const uint64_t idmask = (1ull << SL_ID_BITS) - 1;

  for (int64_t item = blockIdx.x; item < p.M; item += gridDim.x) {
    for (int i = tid; i < p.ht; i += SL_THREADS) slot[i] = 0ull;
    for (int64_t j = tid; j < p.d; j += SL_THREADS) hs[j] = p.hn[item * p.d + j];
    __syncthreads();
    // 1. count sums per token id over every valid row's sketch entries (open addressing; the table
    //    has at least twice as many slots as entries, so every probe sequence ends)
    const int64_t pairs = int64_t(p.n_orders) * p.R * p.K;
    for (int64_t e = tid; e < pairs; e += SL_THREADS) {
      const int o = int(e / (p.R * p.K));
      const int64_t r = (e / p.K) % p.R;
      const int k = int(e % p.K);
      const int64_t row = ngram_row<CodeT>(p.src, item, r, p.orders[o], p.bits);
      if (row < 0) continue;
      const int32_t c = p.sk_cnt[o][row * p.K + k];
      const int32_t id = p.sk_ids[o][row * p.K + k];
      if (c <= 0 || id < 0 || int64_t(id) >= p.V) continue;
      const unsigned long long tag = (unsigned long long)(id + 1) << SL_CNT_BITS;
      uint32_t at = (uint32_t(id) * 2654435761u) & mask;
      for (int probe = 0; probe < p.ht; ++probe) {
        const unsigned long long prev = atomicCAS(&slot[at], 0ull, tag);
        if (prev == 0ull || (prev & ~SL_CNT_MASK) == tag) {
          atomicAdd(&slot[at], (unsigned long long)c);
          break;
        }
        at = (at + 1) & mask;
      }
    }
    __syncthreads();
    // 2. slots -> sort keys (count desc, id asc); empty slots are 0 and sort last
    for (int i = tid; i < p.ht; i += SL_THREADS) {
      const unsigned long long v = slot[i];
      if (v) {
        const uint64_t id = (v >> SL_CNT_BITS) - 1;
        slot[i] = ((v & SL_CNT_MASK) << SL_ID_BITS) | (idmask - id);
      }
    }
    __syncthreads();
    for (int kk = 2; kk <= p.ht; kk <<= 1) {       // bitonic sort, descending
      for (int jj = kk >> 1; jj > 0; jj >>= 1) {
        for (int i = tid; i < p.ht; i += SL_THREADS) {
          const int l = i ^ jj;
          if (l > i) {
            const unsigned long long a = slot[i], b = slot[l];
            if (((i & kk) == 0) ? (a < b) : (a > b)) {
              slot[i] = b;
              slot[l] = a;
            }
          }
        }
        __syncthreads();
      }
    }
    // 3. the list: the first `cap` ids, then fallback ids not already taken
    // (the keys are sorted, so the nonzero ones among the first `cap` are a prefix)
    int taken = 0;
    const int lim = p.cap < p.ht ? p.cap : p.ht;
    for (int base = 0; base < lim; base += SL_THREADS) {
      const int i = base + tid;
      taken += __syncthreads_count(i < lim && slot[i] != 0ull);
    }
    for (int i = tid; i < taken; i += SL_THREADS) list[i] = int32_t(idmask - (slot[i] & idmask));
    __syncthreads();
    if (warp == 0) {
      int n = taken;
      for (int f = 0; f < p.n_fallback && n < p.cap; ++f) {
        const int32_t id = p.fallback[f];
        if (id < 0 || int64_t(id) >= p.V) continue;
        bool have = false;
        for (int i = lane; i < n; i += 32) have = have || list[i] == id;
        if (__any_sync(0xffffffffu, have)) continue;
        if (lane == 0) list[n] = id;
        __syncwarp();
        ++n;
      }
      if (lane == 0) n_list = n;
    }
    __syncthreads();
    const int nl = n_list;
    // 4. logits over the list (an empty list means the whole vocabulary, drafter.cpp:539-542)
    for (int i = warp; i < nl; i += nwarps) {
      const float v = dot_row(p.E, p.e_dtype, list[i], p.d, hs, lane);
      if (lane == 0) lg[i] = v;
    }
    __syncthreads();
    if (p.topk > 0) {
      // 5a. top-k by (logit desc, list position asc)
      if (warp == 0) {
        float bv[TK_MAXK];
        int64_t bp[TK_MAXK];
#pragma unroll
        for (int j = 0; j < TK_MAXK; ++j) {
          bv[j] = -INFINITY;
          bp[j] = INT64_MAX;
        }
        if (nl > 0) {
          for (int i = lane; i < nl; i += 32) topk_insert(bv, bp, p.topk, lg[i], i);
        } else {
          for (int64_t i = lane; i < p.V; i += 32) topk_insert(bv, bp, p.topk, dot_row_serial(p.E, p.e_dtype, i, p.d, hs), i);
        }
        // merge the lanes' sorted lists: one warp arg-best per output; positions are distinct across
        // lanes, so exactly one lane wins each round and drops its head
        for (int j = 0; j < p.topk; ++j) {
          float wv = bv[0];
          int64_t wp = bp[0];
          for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, wv, off);
            const int64_t op = __shfl_xor_sync(0xffffffffu, wp, off);
            if (better(ov, op, wv, wp)) {
              wv = ov;
              wp = op;
            }
          }
          if (lane == 0) {
            const bool ok = wp != INT64_MAX;
            p.ids[item * p.topk + j] = ok ? (nl > 0 ? int64_t(list[wp]) : wp) : -1;
            p.vals[item * p.topk + j] = ok ? wv : -INFINITY;
          }
          if (bp[0] == wp && wp != INT64_MAX) {
#pragma unroll
            for (int q = 0; q + 1 < TK_MAXK; ++q) {
              bv[q] = bv[q + 1];
              bp[q] = bp[q + 1];
            }
            bv[TK_MAXK - 1] = -INFINITY;
            bp[TK_MAXK - 1] = INT64_MAX;
          }
        }
      }
    } else {
      // 5b. trace: the list in order with its logits; an empty list reads ids 0 .. S-1 of the vocabulary
      for (int64_t i = tid; i < p.S; i += SL_THREADS) {
        int64_t id = -1;
        float v = -INFINITY;
        if (nl > 0) {
          if (i < nl) {
            id = list[i];
            v = lg[i];
          }
        } else if (i < p.V) {
          id = i;
          v = dot_row_serial(p.E, p.e_dtype, i, p.d, hs);
        }
        p.list_ids[item * p.S + i] = id;
        p.list_lg[item * p.S + i] = v;
      }
    }
    __syncthreads();
  }
}

}  // namespace lng
