// Row-wise kernels of the readout: RMS statistics, RMSNorm, the short causal conv finish
// (ffnmem/memory/lngram_v2.py:207-286, :1354-1359), its window form for the decode / tree seams
// (ffnmem/infer.py:176-182, drafting/tree.py:186-195), the readout fold, and the shard combine.
#pragma once

#include <type_traits>

#include "address.cuh"

namespace lng {

// Sixteen bytes of a row as floats (8 bf16 / f16 or 4 f32), from a 16-byte aligned address.
template <typename XT>
struct Vec16 {
  static constexpr int N = 16 / int(sizeof(XT));
  __device__ __forceinline__ static void load(const XT* p, float (&v)[N]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const XT* e = reinterpret_cast<const XT*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = to_f32(e[i]);
  }
};

// Sum of squares of one row (warp-cooperative); 16-byte loads when `vec`.
template <typename XT>
__device__ __forceinline__ float row_sumsq(const XT* xr, int64_t d, bool vec, int lane) {
  float ss = 0.f;
  if (vec) {
    constexpr int N = Vec16<XT>::N;
#pragma unroll 4
    for (int64_t j = int64_t(lane) * N; j < d; j += 32 * N) {
      float v[N];
      Vec16<XT>::load(xr + j, v);
#pragma unroll
      for (int i = 0; i < N; ++i) ss = fmaf(v[i], v[i], ss);
    }
  } else {
#pragma unroll 8
    for (int64_t j = lane; j < d; j += 32) {
      const float v = to_f32(xr[j]);
      ss = fmaf(v, v, ss);
    }
  }
  return warp_sum(ss);
}

// One warp per row: rs[row] = 1 / sqrt(mean(x^2) + eps) (or the plain sum of squares with SUMSQ).
template <typename XT, bool SUMSQ = false>
__global__ void rms_rows_kernel(const XT* __restrict__ x, int64_t n, int64_t d, float eps, float* __restrict__ rs) {
  const int lane = threadIdx.x & 31;
  const bool vec = d % Vec16<XT>::N == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  for (int64_t row = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; row < n;
       row += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    const float ss = row_sumsq(x + row * d, d, vec, lane);
    if (lane == 0) rs[row] = SUMSQ ? ss : rsqrtf(ss / float(d) + eps);
  }
}

template <typename XT, typename YT>
__global__ void rms_norm_kernel(const XT* x, int64_t n, int64_t d, const float* __restrict__ w, float eps, YT* y) {
  const int lane = threadIdx.x & 31;
  const bool vec = d % Vec16<XT>::N == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  for (int64_t row = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; row < n;
       row += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    const XT* xr = x + row * d;
    const float r = rsqrtf(row_sumsq(xr, d, vec, lane) / float(d) + eps);
    __syncwarp();
#pragma unroll 8
    for (int64_t j = lane; j < d; j += 32) {
      const float v = to_f32(xr[j]) * r;
      y[row * d + j] = from_f32<YT>(w ? v * w[j] : v);
    }
  }
}

// RMSNorm of rows short enough to stay in registers (d = 32 lanes x nv vectors x 16 bytes,
// nv <= RN_NV): one warp per row reads the row once, reduces, and writes the scaled row.
constexpr int RN_NV = 16;
template <typename XT, typename YT>
__global__ void __launch_bounds__(256) rms_norm_reg_kernel(const XT* __restrict__ x, int64_t n, int64_t d, int nv,
                                                           const float* __restrict__ w, float eps, YT* __restrict__ y) {
  constexpr int N = Vec16<XT>::N;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= n) return;
  const XT* xr = x + row * d;
  float v[RN_NV][N];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < RN_NV; ++i) {
    if (i < nv) {
      Vec16<XT>::load(xr + (int64_t(i) * 32 + lane) * N, v[i]);
#pragma unroll
      for (int k = 0; k < N; ++k) ss = fmaf(v[i][k], v[i][k], ss);
    }
  }
  const float r = rsqrtf(warp_sum(ss) / float(d) + eps);
  YT* yr = y + row * d;
#pragma unroll
  for (int i = 0; i < RN_NV; ++i) {
    if (i < nv) {
      const int64_t j0 = (int64_t(i) * 32 + lane) * N;
#pragma unroll
      for (int k = 0; k < N; ++k) yr[j0 + k] = from_f32<YT>(w ? v[i][k] * r * w[j0 + k] : v[i][k] * r);
    }
  }
}

// RMSNorm with the rounding order of the model's block norm (ffnmem/model.py:39-48):
//   y = cast_y( cast_x(x * rsqrt(mean(x^2) + eps)) * w )
// i.e. the normalised row is rounded to x's own dtype first and only then multiplied by the
// weight (w fp32 or bf16, or none); one warp per row, the row kept in registers when it fits
// (nv > 0, 16-byte vectors) and re-read from global memory otherwise.
template <typename XT>
__device__ __forceinline__ float round_to(float v) {
  return to_f32(from_f32<XT>(v));
}

template <typename XT>
__global__ void __launch_bounds__(256) rms_norm_model_kernel(const XT* __restrict__ x, int64_t n, int64_t d, int nv,
                                                             const void* __restrict__ w, int w_bf16, float eps,
                                                             void* __restrict__ y, int y_dtype) {
  constexpr int N = Vec16<XT>::N;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= n) return;
  const XT* xr = x + row * d;
  auto weight = [&](int64_t j) -> float {
    if (!w) return 1.f;
    return w_bf16 ? to_f32(static_cast<const __nv_bfloat16*>(w)[j]) : static_cast<const float*>(w)[j];
  };
  auto store = [&](int64_t j, float v) {
    if (y_dtype == LNG_F32) static_cast<float*>(y)[row * d + j] = v;
    else if (y_dtype == LNG_BF16) static_cast<__nv_bfloat16*>(y)[row * d + j] = __float2bfloat16_rn(v);
    else static_cast<__half*>(y)[row * d + j] = __float2half_rn(v);
  };
  if (nv > 0) {
    float v[RN_NV][N];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < RN_NV; ++i) {
      if (i < nv) {
        Vec16<XT>::load(xr + (int64_t(i) * 32 + lane) * N, v[i]);
#pragma unroll
        for (int k = 0; k < N; ++k) ss = fmaf(v[i][k], v[i][k], ss);
      }
    }
    const float r = rsqrtf(warp_sum(ss) / float(d) + eps);
#pragma unroll
    for (int i = 0; i < RN_NV; ++i) {
      if (i < nv) {
        const int64_t j0 = (int64_t(i) * 32 + lane) * N;
#pragma unroll
        for (int k = 0; k < N; ++k) store(j0 + k, round_to<XT>(v[i][k] * r) * weight(j0 + k));
      }
    }
  } else {
    const float r = rsqrtf(row_sumsq(xr, d, false, lane) / float(d) + eps);
    for (int64_t j = lane; j < d; j += 32) store(j, round_to<XT>(to_f32(xr[j]) * r) * weight(j));
  }
}

struct ConvParams {
  int64_t d;
  int k, dil;
  const float* norm_w;
  const float* weight;  // [d, k]
  const float* bias;    // [d] or null
};

// Sequence-mode conv finish as position streams (the form used for whole batches): a thread owns
// 16 bytes of channels and one stream of positions p0 + res + j * dil (j < CS_RUN) of its CTA's run,
// so the k taps of every output are the stream's own last k inputs, held in registers.  Every input
// row is read once (plus a (k-1)-row halo per stream) with 16-byte loads straight from global
// memory (a warp reads 512 contiguous bytes of one position), CS_PF rows ahead of their use; the
// arithmetic runs on channel pairs with the packed fp32 instructions (f32x2) and no shared memory.
// Semantics as conv_seq_kernel below (zero left padding, segment mask, valid mask).  For bf16
// activations SiLU(x) = h + h tanh(h), h = x / 2 (one hardware tanh, relative error about 2^-11,
// below the bf16 output's resolution); fp32 activations use x / (1 + e^-x).
constexpr int CS_RUN = 32;  // positions per stream
constexpr int CS_PF = 4;    // rows loaded ahead

__device__ __forceinline__ uint64_t f2_bits(float2 a) { return *reinterpret_cast<uint64_t*>(&a); }
__device__ __forceinline__ float2 f2_from(uint64_t b) { return *reinterpret_cast<float2*>(&b); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {  // a * b + c, two lanes of fp32
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return f2_from(d);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_from(d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_from(d);
}
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ uint4 ld_nc16(const T* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
// 16 bytes of activations as channel pairs
template <typename T>
__device__ __forceinline__ void unpack_pairs(const uint4& w, float2 (&v)[8 / sizeof(T)]) {
  if constexpr (std::is_same<T, float>::value) {
    v[0] = make_float2(__uint_as_float(w.x), __uint_as_float(w.y));
    v[1] = make_float2(__uint_as_float(w.z), __uint_as_float(w.w));
  } else {
    const uint32_t w4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = make_float2(__uint_as_float(w4[i] << 16), __uint_as_float(w4[i] & 0xffff0000u));
  }
}
template <typename T>
__device__ __forceinline__ uint4 pack_pairs(const float2 (&v)[8 / sizeof(T)]) {
  if constexpr (std::is_same<T, float>::value) {
    return make_uint4(__float_as_uint(v[0].x), __float_as_uint(v[0].y), __float_as_uint(v[1].x),
                      __float_as_uint(v[1].y));
  } else {
    uint32_t w4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(v[i].x, v[i].y);
      w4[i] = *reinterpret_cast<uint32_t*>(&b2);
    }
    return make_uint4(w4[0], w4[1], w4[2], w4[3]);
  }
}

template <typename T, int K>
__global__ void __launch_bounds__(128) conv_stream_kernel(ConvParams cp, const T* __restrict__ mixed,
                                                          const float* __restrict__ rs, int M, int T_,
                                                          const int64_t* __restrict__ seg,
                                                          const uint8_t* __restrict__ valid, T* __restrict__ out,
                                                          T* __restrict__ conv_in) {
  constexpr int NP = 8 / int(sizeof(T));  // channel pairs per 16 bytes
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  const int chunks = int(cp.d / (2 * NP));
  const int c = int(blockIdx.z) * 128 + int(threadIdx.x);
  if (c >= chunks) return;
  const int dil = cp.dil;
  const int p_first = int(blockIdx.x) * CS_RUN * dil + int(blockIdx.y);
  const int64_t cc = int64_t(c) * 2 * NP;
  const int64_t step = int64_t(dil) * cp.d;  // elements between consecutive positions of the stream
  // per-channel parameters, with the norm weight folded into the taps
  float2 gw[NP], wt[K][NP], bias[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    gw[i] = make_float2(__ldg(cp.norm_w + cc + 2 * i), __ldg(cp.norm_w + cc + 2 * i + 1));
    bias[i] = cp.bias ? make_float2(__ldg(cp.bias + cc + 2 * i), __ldg(cp.bias + cc + 2 * i + 1)) : make_float2(0.f, 0.f);
#pragma unroll
    for (int tap = 0; tap < K; ++tap)
      wt[tap][i] = make_float2(__ldg(cp.weight + (cc + 2 * i) * K + tap) * gw[i].x,
                               __ldg(cp.weight + (cc + 2 * i + 1) * K + tap) * gw[i].y);
  }
  // the stream's previous K-1 normalised inputs (oldest first); rows before position 0 are zero
  float2 win[K - 1][NP];
#pragma unroll
  for (int h = 0; h < K - 1; ++h) {
    const int q = p_first - (K - 1 - h) * dil;
    float2 v[NP];
    unpack_pairs<T>(q >= 0 ? ld_nc16(mixed + int64_t(q) * cp.d + cc) : make_uint4(0, 0, 0, 0), v);
    const float rq = q >= 0 ? __ldg(rs + q) : 0.f;
#pragma unroll
    for (int i = 0; i < NP; ++i) win[h][i] = fmul2(v[i], make_float2(rq, rq));
  }
  const T* src = mixed + int64_t(p_first) * cp.d + cc;  // row of position p_first
  uint4 ring[CS_PF];
  float rring[CS_PF];
#pragma unroll
  for (int i = 0; i < CS_PF; ++i) {
    const int q = p_first + i * dil;
    ring[i] = q < M ? ld_nc16(src + i * step) : make_uint4(0, 0, 0, 0);
    rring[i] = q < M ? __ldg(rs + q) : 0.f;
  }
  T* dst = out + int64_t(p_first) * cp.d + cc;
  int t = p_first % T_;
#pragma unroll
  for (int j = 0; j < CS_RUN; ++j) {
    const int pos = p_first + j * dil;
    if (pos >= M) break;
    float2 v[NP];
    unpack_pairs<T>(ring[j % CS_PF], v);
    const float rq = rring[j % CS_PF];
    if (j + CS_PF < CS_RUN) {
      const int q = pos + CS_PF * dil;
      ring[j % CS_PF] = q < M ? ld_nc16(src + (j + CS_PF) * step) : make_uint4(0, 0, 0, 0);
      rring[j % CS_PF] = q < M ? __ldg(rs + q) : 0.f;
    }
    float2 y[NP], acc[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) y[i] = fmul2(v[i], make_float2(rq, rq));
    if (!seg && t >= (K - 1) * dil) {  // every tap inside the sequence (uniform across the CTA)
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        acc[i] = bias[i];
#pragma unroll
        for (int tap = 0; tap < K - 1; ++tap) acc[i] = ffma2(wt[tap][i], win[tap][i], acc[i]);
        acc[i] = ffma2(wt[K - 1][i], y[i], acc[i]);
      }
    } else {
      const int64_t sp = seg ? seg[pos] : 0;
#pragma unroll
      for (int i = 0; i < NP; ++i) acc[i] = bias[i];
#pragma unroll
      for (int tap = 0; tap < K; ++tap) {
        const int lag = (K - 1 - tap) * dil;
        if (t - lag >= 0 && (!seg || seg[pos - lag] == sp)) {
#pragma unroll
          for (int i = 0; i < NP; ++i) acc[i] = ffma2(wt[tap][i], tap == K - 1 ? y[i] : win[tap][i], acc[i]);
        }
      }
    }
    float2 o[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      if constexpr (BF) {
        const float2 h = fmul2(acc[i], make_float2(0.5f, 0.5f));
        o[i] = fadd2(v[i], ffma2(h, make_float2(tanh_approx(h.x), tanh_approx(h.y)), h));
      } else {
        o[i] = make_float2(v[i].x + silu_f(acc[i].x), v[i].y + silu_f(acc[i].y));
      }
    }
    if (valid && !valid[pos]) {
#pragma unroll
      for (int i = 0; i < NP; ++i) o[i] = make_float2(0.f, 0.f);
    }
    *reinterpret_cast<uint4*>(dst + j * step) = pack_pairs<T>(o);
    if (conv_in) {
#pragma unroll
      for (int i = 0; i < NP; ++i) o[i] = fmul2(y[i], gw[i]);
      *reinterpret_cast<uint4*>(conv_in + int64_t(pos) * cp.d + cc) = pack_pairs<T>(o);
    }
#pragma unroll
    for (int h = 0; h + 1 < K - 1; ++h)
#pragma unroll
      for (int i = 0; i < NP; ++i) win[h][i] = win[h + 1][i];
#pragma unroll
    for (int i = 0; i < NP; ++i) win[K - 2][i] = y[i];
    t += dil;
    while (t >= T_) t -= T_;
  }
}

// Sequence-mode conv finish: out[p, c] = mixed[p, c] + SiLU(bias + sum_tap w[c, tap] y[p - lag, c] ok),
// y = mixed * rs * g (rs precomputed per position), zero left padding, segment mask, valid mask.
template <typename T>
__global__ void conv_seq_kernel(ConvParams cp, const T* __restrict__ mixed, const float* __restrict__ rs, int64_t B,
                                int64_t T_, const int64_t* __restrict__ seg, const uint8_t* __restrict__ valid,
                                T* __restrict__ out, T* __restrict__ conv_in) {
  const int64_t total = B * T_ * cp.d;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t c = e % cp.d;
    const int64_t pos = e / cp.d;
    const int64_t t = pos % T_;
    const float g = cp.norm_w[c];
    float acc = cp.bias ? cp.bias[c] : 0.f;
    for (int tap = 0; tap < cp.k; ++tap) {
      const int64_t lag = int64_t(cp.k - 1 - tap) * cp.dil;
      if (t - lag < 0) continue;
      const int64_t q = pos - lag;
      if (seg && seg[q] != seg[pos]) continue;
      const float y = to_f32(mixed[q * cp.d + c]) * rs[q] * g;
      acc = fmaf(cp.weight[c * cp.k + tap], y, acc);
    }
    const float m = to_f32(mixed[e]);
    float o = m + silu_f(acc);
    if (valid && !valid[pos]) o = 0.f;
    out[e] = from_f32<T>(o);
    if (conv_in) conv_in[e] = from_f32<T>(m * rs[pos] * g);
  }
}

// Vectorised sequence-mode conv finish: a thread owns 8 channels (16-byte bf16 / 2 x 16-byte fp32
// accesses) and walks POS positions; the channel's norm weight, taps and bias stay in registers.
// Requires d % 8 == 0, k <= 8 and M < 2^31 (checked by the host).
template <typename T, int KMAX>
__global__ void __launch_bounds__(256) conv_seq_vec_kernel(ConvParams cp, const T* __restrict__ mixed,
                                                           const float* __restrict__ rs, int M, int T_,
                                                           const int64_t* __restrict__ seg,
                                                           const uint8_t* __restrict__ valid, T* __restrict__ out,
                                                           T* __restrict__ conv_in, int pos_per_block) {
  const int groups = int(cp.d / 8);
  const int grp = threadIdx.x % groups;
  const int prow = threadIdx.x / groups;
  const int prows = blockDim.x / groups;
  const int c0 = grp * 8;
  float gw[8], wt[KMAX][8], bias[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    gw[i] = cp.norm_w[c0 + i];
    bias[i] = cp.bias ? cp.bias[c0 + i] : 0.f;
#pragma unroll
    for (int tap = 0; tap < KMAX; ++tap) wt[tap][i] = tap < cp.k ? cp.weight[(c0 + i) * cp.k + tap] : 0.f;
  }
  const int p_end = min(M, (int(blockIdx.x) + 1) * pos_per_block);
  for (int pos = int(blockIdx.x) * pos_per_block + prow; pos < p_end; pos += prows) {
    const int t = pos % T_;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = bias[i];
    float self[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int tap = 0; tap < KMAX; ++tap) {
      if (tap >= cp.k) break;
      const int lag = (cp.k - 1 - tap) * cp.dil;
      if (t - lag < 0) continue;
      const int q = pos - lag;
      if (seg && seg[q] != seg[pos]) continue;
      float v[8];
      if constexpr (std::is_same<T, float>::value) {
        const float4 a = *reinterpret_cast<const float4*>(mixed + int64_t(q) * cp.d + c0);
        const float4 b = *reinterpret_cast<const float4*>(mixed + int64_t(q) * cp.d + c0 + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
        const uint4 a = *reinterpret_cast<const uint4*>(mixed + int64_t(q) * cp.d + c0);
        const uint32_t w4[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[2 * i] = __uint_as_float(w4[i] << 16);
          v[2 * i + 1] = __uint_as_float(w4[i] & 0xffff0000u);
        }
      }
      if (lag == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) self[i] = v[i];
      }
      const float r = rs[q];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(wt[tap][i], v[i] * r * gw[i], acc[i]);
    }
    const bool keep = !valid || valid[pos];
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = keep ? self[i] + silu_f(acc[i]) : 0.f;
    if constexpr (std::is_same<T, float>::value) {
      *reinterpret_cast<float4*>(out + int64_t(pos) * cp.d + c0) = make_float4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<float4*>(out + int64_t(pos) * cp.d + c0 + 4) = make_float4(o[4], o[5], o[6], o[7]);
      if (conv_in) {
        const float r = rs[pos];
        *reinterpret_cast<float4*>(conv_in + int64_t(pos) * cp.d + c0) =
            make_float4(self[0] * r * gw[0], self[1] * r * gw[1], self[2] * r * gw[2], self[3] * r * gw[3]);
        *reinterpret_cast<float4*>(conv_in + int64_t(pos) * cp.d + c0 + 4) =
            make_float4(self[4] * r * gw[4], self[5] * r * gw[5], self[6] * r * gw[6], self[7] * r * gw[7]);
      }
    } else {
      uint32_t w4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 b2 = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
        w4[i] = *reinterpret_cast<uint32_t*>(&b2);
      }
      *reinterpret_cast<uint4*>(out + int64_t(pos) * cp.d + c0) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      if (conv_in) {
        const float r = rs[pos];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          __nv_bfloat162 b2 = __floats2bfloat162_rn(self[2 * i] * r * gw[2 * i], self[2 * i + 1] * r * gw[2 * i + 1]);
          w4[i] = *reinterpret_cast<uint32_t*>(&b2);
        }
        *reinterpret_cast<uint4*>(conv_in + int64_t(pos) * cp.d + c0) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
    }
  }
}

// Window form, step 1: cache[new_slot[i]] = RMSNorm(mixed[i]) (rs precomputed).
template <typename T>
__global__ void conv_cache_write_kernel(ConvParams cp, const T* __restrict__ mixed, const float* __restrict__ rs,
                                        int64_t n, const int64_t* __restrict__ new_slot, T* __restrict__ cache) {
  const int64_t total = n * cp.d;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = e / cp.d, c = e % cp.d;
    cache[new_slot[i] * cp.d + c] = from_f32<T>(to_f32(mixed[e]) * rs[i] * cp.norm_w[c]);
  }
}

// Window form, step 2: out[i] = mixed[i] + SiLU(bias + sum_tap w[:, tap] cache[slot[i, tap]]).
template <typename T>
__global__ void conv_window_kernel(ConvParams cp, const T* __restrict__ mixed, int64_t n, const T* __restrict__ cache,
                                   const int64_t* __restrict__ slot, T* __restrict__ out) {
  const int64_t total = n * cp.d;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = e / cp.d, c = e % cp.d;
    float acc = cp.bias ? cp.bias[c] : 0.f;
    for (int tap = 0; tap < cp.k; ++tap) {
      const int64_t s = slot[i * cp.k + tap];
      if (s < 0) continue;
      acc = fmaf(cp.weight[c * cp.k + tap], to_f32(cache[s * cp.d + c]), acc);
    }
    out[e] = from_f32<T>(to_f32(mixed[e]) + silu_f(acc));
  }
}

// Readout fold (see lng_readout in the public header): one thread per output element.
template <typename OT>
__global__ void fold_qk_kernel(int64_t d, int64_t Dt, int QH, int G, int HD, float scale, const float* __restrict__ q_norm,
                               const float* __restrict__ q_proj, const float* __restrict__ mem_norm,
                               const float* __restrict__ kv_proj, OT* __restrict__ w_qk) {
  const int64_t total = int64_t(QH) * Dt * d;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = e % d;
    const int64_t k = (e / d) % Dt;
    const int hg = int(e / (d * Dt));
    const int h = hg / G;
    float acc = 0.f;
    for (int j = 0; j < HD; ++j) acc = fmaf(kv_proj[(int64_t(h) * HD + j) * Dt + k], q_proj[(int64_t(hg) * HD + j) * d + i], acc);
    w_qk[e] = from_f32<OT>(acc * scale * mem_norm[k] * q_norm[i]);
  }
}

template <typename OT>
__global__ void fold_vo_kernel(int64_t d, int64_t Dt, int QH, int G, int HD, int KV, const float* __restrict__ mem_norm,
                               const float* __restrict__ kv_proj, const float* __restrict__ o_proj, OT* __restrict__ w_vo) {
  const int64_t total = d * QH * Dt;
  const int64_t vbase = int64_t(KV) * HD;  // value rows follow the key rows in kv_proj
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t col = e % (int64_t(QH) * Dt);
    const int64_t o = e / (int64_t(QH) * Dt);
    const int hg = int(col / Dt);
    const int64_t k = col % Dt;
    const int h = hg / G;
    float acc = 0.f;
    for (int j = 0; j < HD; ++j)
      acc = fmaf(o_proj[o * QH * HD + int64_t(hg) * HD + j], kv_proj[(vbase + int64_t(h) * HD + j) * Dt + k], acc);
    w_vo[e] = from_f32<OT>(acc * mem_norm[k]);
  }
}

// Shard combine: l *= exp(m - m_glob), u *= exp(m - m_glob).
__global__ void attend_rescale_kernel(const float* __restrict__ m, const float* __restrict__ mg, float* __restrict__ l,
                                      float* __restrict__ u, int64_t MQ, int64_t Dt) {
  const int64_t total = MQ * Dt;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t iq = e / Dt;
    const float s = expf(m[iq] - mg[iq]);
    u[e] *= s;
    if (e % Dt == 0) l[iq] *= s;
  }
}

// Route-shard combine in head space: pack[i, q, :HD] = o[i, q, :] * s, pack[i, q, HD] = l[i, q] * s
// with s = exp(m_local - m_glob) (the streaming update of lngram_v2.py:1922-1942 across shards).
template <typename PT>
__global__ void attend_pack_kernel(const float* __restrict__ m, const float* __restrict__ mg,
                                   const float* __restrict__ l, const float* __restrict__ o, int64_t MQ, int HD,
                                   PT* __restrict__ pack) {
  const int64_t total = MQ * (HD + 1);
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t iq = e / (HD + 1);
    const int j = int(e % (HD + 1));
    const float s = expf(m[iq] - mg[iq]);
    pack[e] = from_f32<PT>((j < HD ? o[iq * HD + j] : l[iq]) * s);
  }
}

// pack[i, q, :] *= exp(m_local - m_glob) where the two differ (shards share the offset b0 unless a
// score exceeded it by a margin, so usually no row is touched).
template <typename PT>
__global__ void attend_pack_rescale_kernel(const float* __restrict__ m, const float* __restrict__ mg, int64_t MQ,
                                           int HD, PT* __restrict__ pack) {
  for (int64_t iq = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; iq < MQ; iq += int64_t(gridDim.x) * blockDim.x) {
    const float a = m[iq], b = mg[iq];
    if (a == b) continue;
    const float sc = expf(a - b);
    PT* row = pack + iq * (HD + 1);
    for (int j = 0; j <= HD; ++j) row[j] = from_f32<PT>(to_f32(row[j]) * sc);
  }
}

// head[i, q, :] = pack[i, q, :HD] / pack[i, q, HD]  (the final division of lngram_v2.py:2066-2070)
template <typename PT, typename OT>
__global__ void attend_unpack_kernel(const PT* __restrict__ pack, int64_t MQ, int HD, OT* __restrict__ head) {
  const int64_t total = MQ * HD;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t iq = e / HD;
    const int j = int(e % HD);
    head[e] = from_f32<OT>(to_f32(pack[iq * (HD + 1) + j]) / fmaxf(to_f32(pack[iq * (HD + 1) + HD]), 1.17549435e-38f));
  }
}

template <typename UT>
__global__ void attend_normalize_kernel(const float* __restrict__ l, const float* __restrict__ u, int64_t MQ, int64_t Dt,
                                        UT* __restrict__ out) {
  const int64_t total = MQ * Dt;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    out[e] = from_f32<UT>(u[e] / fmaxf(l[e / Dt], 1.17549435e-38f));
  }
}

// Sink attention with explicit K / V (the reference's _manual_gqa, ffnmem/memory/lngram_v2.py:1899-1920):
// one CTA per (item, kv head); q [M, KV*G, HD], k/v [M, KV, R, HD], out [M, KV*G, HD].
template <typename T>
__global__ void sink_gqa_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, int64_t M,
                                int KV, int G, int R, int HD, float scale, float sink, T* __restrict__ out) {
  extern __shared__ float gq_sm[];
  float* ks = gq_sm;              // [R, HD]
  float* vs = ks + R * HD;        // [R, HD]
  float* qs = vs + R * HD;        // [G, HD]
  float* sc = qs + G * HD;        // [G, R]
  const int64_t item = blockIdx.x / KV;
  const int h = blockIdx.x % KV;
  if (item >= M) return;
  const T* kb = k + (item * KV + h) * int64_t(R) * HD;
  const T* vb = v + (item * KV + h) * int64_t(R) * HD;
  const T* qb = q + (item * KV * G + int64_t(h) * G) * HD;
  for (int e = threadIdx.x; e < R * HD; e += blockDim.x) {
    ks[e] = to_f32(kb[e]);
    vs[e] = to_f32(vb[e]);
  }
  for (int e = threadIdx.x; e < G * HD; e += blockDim.x) qs[e] = to_f32(qb[e]);
  __syncthreads();
  for (int e = threadIdx.x; e < G * R; e += blockDim.x) {
    const int g = e / R, r = e % R;
    float acc = 0.f;
    for (int j = 0; j < HD; ++j) acc = fmaf(qs[g * HD + j], ks[r * HD + j], acc);
    sc[e] = acc * scale;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int g = warp; g < G; g += nw) {
    float mx = sink;
    for (int r = lane; r < R; r += 32) mx = fmaxf(mx, sc[g * R + r]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int r = lane; r < R; r += 32) {
      const float e = expf(sc[g * R + r] - mx);
      sc[g * R + r] = e;
      sum += e;
    }
    sum = warp_sum(sum) + expf(sink - mx);
    __syncwarp();
    for (int r = lane; r < R; r += 32) sc[g * R + r] /= sum;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * HD; e += blockDim.x) {
    const int g = e / HD, j = e % HD;
    float acc = 0.f;
    for (int r = 0; r < R; ++r) acc = fmaf(sc[g * R + r], vs[r * HD + j], acc);
    out[(item * KV * G + int64_t(h) * G + g) * HD + j] = from_f32<T>(acc);
  }
}

}  // namespace lng
