// Draft-head logits + fused top-k on the tcgen05 tensor cores (bf16 vocabulary matrix):
// ffnmem/memory/draft.py:88-91 (logits against the tied embedding) with the candidate order of
// drafting/cpu/drafter.cpp:537-556 ((logit desc, id asc)).
//
// One CTA owns 256 vocabulary rows (two 128-lane TMEM accumulators, M side) and BN draft rows
// (N side).  The vocabulary tile (128-byte swizzle, K-major, 64-element k blocks) and the fp32
// draft rows of each k block arrive by TMA; two converter warps split the rows into three bf16
// parts h = h1 + h2 + h3 (each rounding exact to ~2^-24 relative) in the same swizzled layout,
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
  static constexpr uint32_t H_BYTES = BN * TC_BK * 4;      // fp32 draft rows of the k block (TMA)
  static constexpr uint32_t B_PART = BN * TC_BK * 2;       // one bf16 part of the draft rows
  static constexpr uint32_t STAGE_BYTES = A_BYTES + H_BYTES + 3 * B_PART;
  static constexpr int STAGES = (224 * 1024) / STAGE_BYTES > 6 ? 6 : (224 * 1024) / STAGE_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr size_t SMEM = size_t(STAGES) * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(STAGES >= 2, "pipeline needs two stages");
  static_assert(B_PART % 1024 == 0 && A_BYTES % 1024 == 0 && H_BYTES % 1024 == 0,
                "swizzle atoms must stay 1024-byte aligned");
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// (v, id) strictly after (pv, pid) in (value desc, id asc) order
__device__ __forceinline__ bool lt_after(float v, int id, float pv, int pid) {
  return v < pv || (v == pv && id > pid);
}
__device__ __forceinline__ bool lt_better(float v, int id, float bv, int bid) {
  return v > bv || (v == bv && id < bid);
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
  uint64_t* loaded = reinterpret_cast<uint64_t*>(base + size_t(STAGES) * Cfg::STAGE_BYTES);
  uint64_t* full = loaded + STAGES;
  uint64_t* empty = full + STAGES;
  uint64_t* acc_bar = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t v0 = int64_t(blockIdx.y) * LT_BM, r0 = int64_t(blockIdx.x) * BN;
  const int KB = int(d / TC_BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&loaded[s], 1);  // TMA: vocabulary tile + fp32 draft rows
      mbar_init(&full[s], 2);    // one arrive per converter warp
      mbar_init(&empty[s], 1);   // MMA commit
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
    if (lane == 0) {  // TMA producer: the vocabulary tile and the draft rows of each k block
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % STAGES;
        if (kb >= STAGES &&
            !mbar_wait_bounded(&empty[s], uint32_t(((kb / STAGES) - 1) & 1), &g_error_word, DEV_ERR_WAIT_TIMEOUT))
          break;
        uint8_t* st = base + size_t(s) * Cfg::STAGE_BYTES;
        mbar_arrive_expect_tx(&loaded[s], Cfg::A_BYTES + Cfg::H_BYTES);
        tma_load_2d(st, &tma_e, int32_t(kb * TC_BK), int32_t(v0), &loaded[s]);
        tma_load_2d(st + Cfg::A_BYTES, &tma_h, int32_t(kb * TC_BK), int32_t(r0), &loaded[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer: 4 k steps x 3 parts x 2 vocabulary halves per stage
      constexpr uint32_t idesc = umma_idesc_bf16(128, BN);
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % STAGES;
        if (!mbar_wait_bounded(&full[s], uint32_t((kb / STAGES) & 1), &g_error_word, DEV_ERR_WAIT_TIMEOUT)) break;
        tc_fence_after();
        const uint8_t* st = base + size_t(s) * Cfg::STAGE_BYTES;
        const uint64_t da0 = umma_desc_sw128(st), da1 = umma_desc_sw128(st + Cfg::A_BYTES / 2);
#pragma unroll
        for (int kk = 0; kk < TC_BK / 16; ++kk) {
#pragma unroll
          for (int part = 0; part < 3; ++part) {
            const uint64_t db = umma_desc_sw128(st + Cfg::A_BYTES + Cfg::H_BYTES + part * Cfg::B_PART);
            const uint32_t acc = (kb | kk | part) != 0 ? 1u : 0u;
            umma_bf16(tmem, da0 + uint64_t(2 * kk), db + uint64_t(2 * kk), idesc, acc);
            umma_bf16(tmem + uint32_t(BN), da1 + uint64_t(2 * kk), db + uint64_t(2 * kk), idesc, acc);
          }
        }
        umma_commit(&empty[s]);
      }
      umma_commit(acc_bar);
    }
  } else {
    // converters (warps 2, 3): the k block's fp32 draft rows (TMA-staged [BN][64], rows past n are
    // zero-filled) split into three bf16 parts in the 128-byte-swizzled K-major layout (row r at
    // r*128 bytes, 16-byte chunk c stored at c ^ (r & 7))
    const int t = threadIdx.x - 64;
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % STAGES;
      const bool ok = mbar_wait_bounded(&loaded[s], uint32_t((kb / STAGES) & 1), &g_error_word, DEV_ERR_WAIT_TIMEOUT);
      if (!__all_sync(0xffffffffu, ok)) break;
      uint8_t* st = base + size_t(s) * Cfg::STAGE_BYTES;
      const float* hs = reinterpret_cast<const float*>(st + Cfg::A_BYTES);
      uint8_t* bt = st + Cfg::A_BYTES + Cfg::H_BYTES;
#pragma unroll 4
      for (int q = t; q < BN * 8; q += 64) {
        const int r = q >> 3, c = q & 7;
        const float4 a = *reinterpret_cast<const float4*>(hs + r * TC_BK + c * 8);
        const float4 b = *reinterpret_cast<const float4*>(hs + r * TC_BK + c * 8 + 4);
        const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        uint32_t p1[4], p2[4], p3[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float a1 = __bfloat162float(__float2bfloat16_rn(x[2 * i]));
          const float b1 = __bfloat162float(__float2bfloat16_rn(x[2 * i + 1]));
          const float ra = x[2 * i] - a1, rb = x[2 * i + 1] - b1;
          const float a2 = __bfloat162float(__float2bfloat16_rn(ra)), b2 = __bfloat162float(__float2bfloat16_rn(rb));
          p1[i] = pack_bf16x2(a1, b1);
          p2[i] = pack_bf16x2(a2, b2);
          p3[i] = pack_bf16x2(ra - a2, rb - b2);
        }
        const uint32_t off = uint32_t(r) * 128u + (uint32_t(c ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(bt + off) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
        *reinterpret_cast<uint4*>(bt + Cfg::B_PART + off) = make_uint4(p2[0], p2[1], p2[2], p2[3]);
        *reinterpret_cast<uint4*>(bt + 2 * Cfg::B_PART + off) = make_uint4(p3[0], p3[1], p3[2], p3[3]);
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor cores' async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
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
      tmem_ld16(tl + uint32_t(BN + c), xb);
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

// 2D fp32 tensor map over a row-major [rows, cols] matrix (row stride ld elements), box
// TC_BK x box_rows, no swizzle; rows past the end read as zeros.
inline int make_tmap_f32(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(LNG_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (driver entry point)");
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * 4};
  const cuuint32_t box[2] = {uint32_t(TC_BK), uint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LNG_ERR_CUDA, "cuTensorMapEncodeTiled (f32) failed: " + std::to_string(int(r)));
  return LNG_OK;
}

}  // namespace lng
