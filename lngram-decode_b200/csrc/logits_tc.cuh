// Draft-head logits + fused top-k on the tcgen05 tensor cores (bf16 vocabulary matrix):
// ffnmem/memory/draft.py:88-91 (logits against the tied embedding) with the candidate order of
// drafting/cpu/drafter.cpp:537-556 ((logit desc, id asc)).
//
// One CTA owns 256 vocabulary rows (two 128-lane TMEM accumulators, M side) and BN draft rows
// (N side; for BN <= 64 the three parts of the draft rows form one N = 3 BN operand).  The fp32 draft rows are split once (split_rows_bf16x3_kernel) into three bf16 parts
// h = h1 + h2 + h3 (exact to ~2^-24 relative); the vocabulary tile and the three parts of each
// 64-element k block arrive by TMA (128-byte swizzle, K-major),
// so logits = E . h1 + E . h2 + E . h3 accumulate in fp32 with every bf16 x bf16 product exact:
// fp32-accurate logits while the bf16 vocabulary is read from HBM once.  The epilogue reads the
// accumulators back (tcgen05.ld), takes each draft row's top-k over the tile's 256 entries (warp
// shuffles, then a merge of the four warps in shared memory) and writes the per-tile candidates
// that topk_merge_kernel reduces over tiles -- the [n, V] logits reach memory only when asked.
#pragma once

#include <climits>

#include "gemm_tc.cuh"
#include "topk.cuh"

namespace lng {

constexpr int LT_BM = 256;  // vocabulary rows per CTA (= TK_VC: the candidate layout is shared)
static_assert(LT_BM == TK_VC, "per-tile candidates must use the top-k scratch layout");

template <int BN>
struct LtCfg {
  static constexpr uint32_t A_BYTES = LT_BM * TC_BK * 2;   // 32 KB vocabulary tile per k block
  static constexpr uint32_t B_PART = BN * TC_BK * 2;       // one bf16 part of the draft rows
  static constexpr uint32_t STAGE_BYTES = A_BYTES + 3 * B_PART;
  static constexpr int STAGES = (224 * 1024) / STAGE_BYTES > 6 ? 6 : (224 * 1024) / STAGE_BYTES;
  // The three parts sit back to back in a stage (3 BN rows of 128 bytes), so while 3 BN <= 256 one
  // MMA of N = 3 BN multiplies the vocabulary tile by all of them, each part into its own column
  // block, summed in the epilogue: a third of the MMA instructions, each three times as wide.
  static constexpr bool STACKED = 3 * BN <= 256;
  static constexpr uint32_t ACC_COLS = STACKED ? 3 * BN : BN;  // accumulator columns per vocabulary half
  static constexpr uint32_t TMEM_COLS = 2 * ACC_COLS <= 32 ? 32 : 2 * ACC_COLS <= 64 ? 64 : 2 * ACC_COLS <= 128 ? 128
                                        : 2 * ACC_COLS <= 256 ? 256 : 512;
  static constexpr size_t SMEM = size_t(STAGES) * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(STAGES >= 2, "pipeline needs two stages");
  static_assert(B_PART % 1024 == 0 && A_BYTES % 1024 == 0, "swizzle atoms must stay 1024-byte aligned");
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

// (v, id) strictly after (pv, pid) in (value desc, id asc) order
__device__ __forceinline__ bool lt_after(float v, int id, float pv, int pid) {
  return v < pv || (v == pv && id > pid);
}
__device__ __forceinline__ bool lt_better(float v, int id, float bv, int bid) {
  return v > bv || (v == bv && id < bid);
}

// h [n, d] fp32 -> [n, 3d] bf16 rows (h1 | h2 | h3) with h = h1 + h2 + h3: h1 = bf16(h),
// h2 = bf16(h - h1), h3 = bf16(h - h1 - h2); both differences are exact in fp32.
__global__ void split_rows_bf16x3_kernel(const float* __restrict__ h, int64_t n, int64_t d,
                                         __nv_bfloat16* __restrict__ out) {
  const int64_t total = n * d;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / d, k = e - r * d;
    const float x = h[e];
    const __nv_bfloat16 a = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(a);
    const __nv_bfloat16 b = __float2bfloat16_rn(r1);
    const float r2 = r1 - __bfloat162float(b);
    __nv_bfloat16* o = out + r * 3 * d;
    o[k] = a;
    o[d + k] = b;
    o[2 * d + k] = __float2bfloat16_rn(r2);
  }
}

template <int BN>
__global__ void __launch_bounds__(128, 1)
    logits_tc_topk_kernel(const __grid_constant__ CUtensorMap tma_e, const __grid_constant__ CUtensorMap tma_h,
                          int64_t n, int64_t d, int64_t V, int k, float* __restrict__ cand_v,
                          int64_t* __restrict__ cand_i, float* __restrict__ logits) {
  using Cfg = LtCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t lt_smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(lt_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + size_t(STAGES) * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_bar = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t v0 = int64_t(blockIdx.y) * LT_BM, r0 = int64_t(blockIdx.x) * BN;
  const int KB = int(d / TC_BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // TMA: vocabulary tile + the three parts of the draft rows
      mbar_init(&empty[s], 1);  // MMA commit
    }
    mbar_init(acc_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tma_e);
    tma_prefetch_desc(&tma_h);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(Cfg::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      // The vocabulary tiles do not depend on the kernel before this one (launched as a programmatic
      // dependent, this kernel may start while that one still writes the draft rows' parts): the
      // first stages' tiles are requested before waiting for it, the parts after.
      const int pre = KB < STAGES ? KB : STAGES;
      for (int kb = 0; kb < pre; ++kb) {
        mbar_arrive_expect_tx(&full[kb], Cfg::STAGE_BYTES);
        tma_load_2d(base + size_t(kb) * Cfg::STAGE_BYTES, &tma_e, int32_t(kb * TC_BK), int32_t(v0), &full[kb]);
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");  // no-op unless launched as a dependent
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % STAGES;
        uint8_t* st = base + size_t(s) * Cfg::STAGE_BYTES;
        if (kb >= pre) {
          if (!mbar_wait_bounded(&empty[s], uint32_t(((kb / STAGES) - 1) & 1), &g_error_word, DEV_ERR_WAIT_TIMEOUT))
            break;
          mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
          tma_load_2d(st, &tma_e, int32_t(kb * TC_BK), int32_t(v0), &full[s]);
        }
#pragma unroll
        for (int part = 0; part < 3; ++part)
          tma_load_2d(st + Cfg::A_BYTES + part * Cfg::B_PART, &tma_h, int32_t(part * d + kb * TC_BK), int32_t(r0),
                      &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer: 4 k steps x (1 stacked or 3) parts x 2 vocabulary halves per stage
      constexpr uint32_t idesc = umma_idesc_bf16(128, int(Cfg::STACKED ? 3 * BN : BN));
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % STAGES;
        if (!mbar_wait_bounded(&full[s], uint32_t((kb / STAGES) & 1), &g_error_word, DEV_ERR_WAIT_TIMEOUT)) break;
        tc_fence_after();
        const uint8_t* st = base + size_t(s) * Cfg::STAGE_BYTES;
        const uint64_t da0 = umma_desc_sw128(st), da1 = umma_desc_sw128(st + Cfg::A_BYTES / 2);
#pragma unroll
        for (int kk = 0; kk < TC_BK / 16; ++kk) {
#pragma unroll
          for (int part = 0; part < (Cfg::STACKED ? 1 : 3); ++part) {
            const uint64_t db = umma_desc_sw128(st + Cfg::A_BYTES + part * Cfg::B_PART);
            const uint32_t acc = (kb | kk | part) != 0 ? 1u : 0u;
            umma_bf16(tmem, da0 + uint64_t(2 * kk), db + uint64_t(2 * kk), idesc, acc);
            umma_bf16(tmem + Cfg::ACC_COLS, da1 + uint64_t(2 * kk), db + uint64_t(2 * kk), idesc, acc);
          }
        }
        umma_commit(&empty[s]);
      }
      umma_commit(acc_bar);
    }
  }
  __syncwarp();

  // epilogue: warp w reads TMEM lanes 32w..32w+31 of both accumulators (vocabulary rows
  // v0 + 32w + lane and v0 + 128 + 32w + lane); per draft row, the warp's top-k -> shared memory
  const bool acc_ok = __all_sync(0xffffffffu, mbar_wait_bounded(acc_bar, 0u, &g_error_word, DEV_ERR_WAIT_TIMEOUT));
  tc_fence_after();
  float* cv_s = reinterpret_cast<float*>(base);   // [BN][4][k] (pipeline stages are drained)
  int* ci_s = reinterpret_cast<int*>(cv_s + BN * 4 * k);
  const int64_t va = v0 + warp * 32 + lane, vb = va + 128;
  const bool oka = va < V, okb = vb < V;
  const uint32_t tl = tmem + (uint32_t(warp * 32) << 16);
#pragma unroll 1
  for (int c = 0; c < BN; c += 16) {
    float xa[16] = {}, xb[16] = {};
    if (acc_ok) {
      tmem_ld16(tl + uint32_t(c), xa);
      tmem_ld16(tl + Cfg::ACC_COLS + uint32_t(c), xb);
      if (Cfg::STACKED) {  // logits = part 1 + (part 2 + part 3): the small corrections first
        float ya[16], yb[16], za[16], zb[16];
        tmem_ld16(tl + uint32_t(BN + c), ya);
        tmem_ld16(tl + Cfg::ACC_COLS + uint32_t(BN + c), yb);
        tmem_ld16(tl + uint32_t(2 * BN + c), za);
        tmem_ld16(tl + Cfg::ACC_COLS + uint32_t(2 * BN + c), zb);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          xa[i] += ya[i] + za[i];
          xb[i] += yb[i] + zb[i];
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int col = c + i;
      const int64_t hr = r0 + col;
      if (hr >= n) continue;  // uniform over the warp
      const float a = xa[i], b = xb[i];
      if (logits && acc_ok) {
        if (oka) logits[hr * V + va] = a;
        if (okb) logits[hr * V + vb] = b;
      }
      float pv = INFINITY;
      int pid = -1;
      for (int kk = 0; kk < k; ++kk) {
        float bv = -INFINITY;
        int bid = INT_MAX;
        if (acc_ok) {
          if (oka && lt_after(a, int(va), pv, pid) && lt_better(a, int(va), bv, bid)) {
            bv = a;
            bid = int(va);
          }
          if (okb && lt_after(b, int(vb), pv, pid) && lt_better(b, int(vb), bv, bid)) {
            bv = b;
            bid = int(vb);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oid = __shfl_xor_sync(0xffffffffu, bid, o);
          if (lt_better(ov, oid, bv, bid)) {
            bv = ov;
            bid = oid;
          }
        }
        if (lane == 0) {
          cv_s[(col * 4 + warp) * k + kk] = bv;
          ci_s[(col * 4 + warp) * k + kk] = bid;
        }
        pv = bv;
        pid = bid;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::TMEM_COLS) : "memory");
  }
  // merge the four warps' candidates of each draft row -> this tile's k candidates
  const int64_t nch = gridDim.y;
  for (int col = threadIdx.x; col < BN; col += blockDim.x) {
    const int64_t hr = r0 + col;
    if (hr >= n) continue;
    const float* cv = cv_s + col * 4 * k;
    const int* ci = ci_s + col * 4 * k;
    float pv = INFINITY;
    int pid = -1;
    for (int kk = 0; kk < k; ++kk) {
      float bv = -INFINITY;
      int bid = INT_MAX;
      for (int e = 0; e < 4 * k; ++e) {
        const int id = ci[e];
        if (id == INT_MAX) continue;
        if (lt_after(cv[e], id, pv, pid) && lt_better(cv[e], id, bv, bid)) {
          bv = cv[e];
          bid = id;
        }
      }
      const int64_t slot = (hr * nch + blockIdx.y) * k + kk;
      cand_v[slot] = bv;
      cand_i[slot] = bid == INT_MAX ? -1 : int64_t(bid);
      pv = bv;
      pid = bid;
    }
  }
}

}  // namespace lng
