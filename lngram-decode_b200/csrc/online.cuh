// The acceptance harness's in-context online-count mixer (drafting/drafters.py:117-143): the verified
// pairs of one record vote for their next token with the number of (order, route) n-gram rows they
// share with each query window, and the votes' distribution is mixed into the drafter's p.
//
// Four launches: the pairs' keys [n_orders, T-1, R], the queries' rows [n_orders, N, R]; one thread per
// (query, pair) counting shared rows (integer-valued fp32, so the atomic sums into tot[j] and into the
// vote scratch sc[j, v] are exact in any order); one thread per (query, token) mixing in the reference's
// fp32 order (explicit _rn operations: no contraction into fused multiply-adds).
#pragma once

#include "address.cuh"

namespace lng {

constexpr int OC_MAX_ORDERS = 8;

struct OnlineParams {
  const int64_t* codes;  // [T, R]
  int64_t T, R;
  int orders[OC_MAX_ORDERS];
  int n_orders, bits;
  const int64_t* x;      // [T]
  const int64_t* win;    // [N, W, R]
  const uint8_t* real;   // [N, W]
  int64_t N, W;
  const int64_t* deadline;
  int64_t V;
};

// keys[o][t][r] (t < T-1) = row of the order-n n-gram ending at t (oldest code least significant), or -1
__global__ void online_keys_kernel(OnlineParams p, int64_t* __restrict__ keys) {
  const int64_t T1 = p.T - 1, per = T1 * p.R;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < per * p.n_orders;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int o = int(e / per);
    const int64_t rem = e - int64_t(o) * per, t = rem / p.R, r = rem - t * p.R;
    const int n = p.orders[o];
    int64_t row = -1;
    if (t >= n - 1) {
      int64_t addr = 0;
      for (int k = 0; k < n; ++k) addr |= p.codes[(t - n + 1 + k) * p.R + r] << (k * p.bits);
      row = r * (int64_t(1) << (p.bits * n)) + addr;
    }
    keys[e] = row;
  }
}

// q[o][j][r] = row of the order-n n-gram ending at window j's last slot, or -1 unless those n slots are real
__global__ void online_queries_kernel(OnlineParams p, int64_t* __restrict__ q) {
  const int64_t per = p.N * p.R;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < per * p.n_orders;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int o = int(e / per);
    const int64_t rem = e - int64_t(o) * per, j = rem / p.R, r = rem - j * p.R;
    const int n = p.orders[o];
    bool ok = true;
    int64_t addr = 0;
    for (int k = 0; k < n; ++k) {
      const int64_t slot = p.W - n + k;
      ok = ok && p.real[j * p.W + slot] != 0;
      addr |= p.win[(j * p.W + slot) * p.R + r] << (k * p.bits);
    }
    q[e] = ok ? r * (int64_t(1) << (p.bits * n)) + addr : -1;
  }
}

// One thread per (query j, pair t): its vote weight (shared rows, 0 past the deadline), added to tot[j]
// and to sc[j, x[t+1]].
__global__ void online_votes_kernel(OnlineParams p, const int64_t* __restrict__ keys, const int64_t* __restrict__ q,
                                    float* __restrict__ tot, float* __restrict__ sc) {
  const int64_t T1 = p.T - 1;
  const int64_t j = blockIdx.y;
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < T1; t += int64_t(gridDim.x) * blockDim.x) {
    if (t > p.deadline[j]) continue;
    int cnt = 0;
    for (int o = 0; o < p.n_orders; ++o) {
      const int64_t* kr = keys + (int64_t(o) * T1 + t) * p.R;
      const int64_t* qr = q + (int64_t(o) * p.N + j) * p.R;
      for (int64_t r = 0; r < p.R; ++r) cnt += (kr[r] == qr[r] && qr[r] >= 0) ? 1 : 0;
    }
    if (cnt == 0) continue;
    const int64_t v = p.x[t + 1];
    if (v < 0 || v >= p.V) {
      atomicCAS(&g_error_word, 0u, (unsigned int)DEV_ERR_TOKEN_RANGE);
      continue;
    }
    atomicAdd(tot + j, float(cnt));
    atomicAdd(sc + j * p.V + v, float(cnt));
  }
}

// out[j, v] = (1 - lam) p + (lam sc) / max(tot, 1e-9): sc arrives in `out` (the vote scratch), in place
__global__ void online_mix_kernel(const float* __restrict__ pin, const float* __restrict__ tot, int64_t N, int64_t V,
                                  float routes_orders, float kappa, float* out) {
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < N * V; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t j = e / V;
    const float tj = tot[j];
    const float n_eff = __fdiv_rn(tj, routes_orders);
    const float lam = __fdiv_rn(n_eff, __fadd_rn(n_eff, kappa));
    const float a = __fmul_rn(__fsub_rn(1.f, lam), pin[e]);
    const float b = __fdiv_rn(__fmul_rn(lam, out[e]), fmaxf(tj, 1e-9f));
    out[e] = __fadd_rn(a, b);
  }
}

}  // namespace lng
