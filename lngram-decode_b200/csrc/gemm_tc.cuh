// tcgen05 GEMMs for sm_100a: C[M, N] = A[M, K] . B[N, K]^T with bf16 operands staged by TMA
// (128-byte swizzle) into a shared-memory ring, one elected thread issuing tcgen05.mma into a
// TMEM fp32 accumulator (128 lanes x BN columns), and all four warps reading it back with
// tcgen05.ld for the epilogue.
//
// Two epilogues: MODE 0 stores C (f32 or bf16, optional per-row scale); MODE 1 is the router:
// logits of 32 routes x `bits` per tile are sign-packed into uint8 codes in registers
// (ffnmem/memory/lngram_v2.py:74-89), so the fp32 logits never reach memory.  For the router the
// fp32 weight is split once into three bf16 parts W = W1 + W2 + W3 stored side by side along K
// and A's k coordinate wraps (a_kperiod): x . W^T = x . W1^T + x . W2^T + x . W3^T with every
// bf16 x bf16 product exact and fp32 accumulation -- fp32-accurate logits from the tensor cores.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "address.cuh"

namespace lng {

constexpr int TC_BM = 128, TC_BK = 64;

struct TcGemmParams {
  int64_t M, N, K;       // K = total reduction length seen by B (A wraps with a_kperiod)
  int64_t a_kperiod;
  void* C;
  int64_t ldc;
  int c_dtype;           // LNG_F32 / LNG_BF16 (MODE 0)
  const float* rowscale; // MODE 0, may be null
  int bits;              // MODE 1
  int64_t routes;        // MODE 1
  uint8_t* codes;        // MODE 1, [M, routes]
  // Operand parts (npairs > 0): the reduction runs over npairs products A_part . B_part^T, each
  // part_k long; k block kb reads A at x = a_part[kb / pkb] * part_k + (kb % pkb) * 64 and B at
  // b_part[..] likewise (pkb = part_k / 64).  K is then npairs * part_k.
  int npairs;
  int a_part[8], b_part[8];
  int64_t part_k;
  // Split-K (splits > 1, MODE 0): the k blocks are divided into `splits` ranges and range s writes
  // its partial product to C + s * split_stride (fp32).
  int splits;
  int64_t split_stride;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// K-major operand tile written by TMA with 128-byte swizzle: 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* tile) {
  const uint64_t addr = smem_addr(tile);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;        // start address
  d |= uint64_t(1) << 16;              // leading byte offset (unused for swizzled K-major)
  d |= uint64_t(1024 >> 4) << 32;      // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1) << 46;              // descriptor version (sm_100)
  d |= uint64_t(2) << 61;              // SWIZZLE_128B
  return d;
}
// kind::f16 instruction descriptor: bf16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4)                     // D format f32
         | (1u << 7)                   // A format bf16
         | (1u << 10)                  // B format bf16
         | (uint32_t(N >> 3) << 17)    // N / 8
         | (uint32_t(M >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN>
struct TcCfg {
  static constexpr uint32_t A_BYTES = TC_BM * TC_BK * 2;
  static constexpr uint32_t B_BYTES = BN * TC_BK * 2;
  // two k blocks per stage ([A0 | A1 | B0 | B1], half the stage handshakes) whenever three such stages
  // fit; one otherwise (BN = 256)
  static constexpr int KPS = (200 * 1024) / (2 * (A_BYTES + B_BYTES)) >= 3 ? 2 : 1;
  static constexpr uint32_t STAGE_BYTES = KPS * (A_BYTES + B_BYTES);
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 8 ? 8 : (200 * 1024) / STAGE_BYTES;
  // two accumulators (tile i and tile i + 1) of BN columns each, allocated as a power of two
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
  static constexpr size_t SMEM = size_t(STAGES) * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

// Persistent GEMM: one CTA per SM walks the output tiles (m-major, so neighbouring CTAs share A
// rows in L2).  Warp 0 issues the TMA loads, warp 1 the MMAs into one of two TMEM accumulators,
// warps 2-5 (one per TMEM lane quadrant) run the epilogue of tile i while the MMAs of tile i + 1
// proceed.  All waits are bounded; an expired wait records DEV_ERR_WAIT_TIMEOUT and every role
// leaves its loop.
template <int BN, int MODE, int BITS = 1>
__global__ void __launch_bounds__(192, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, TcGemmParams p) {
  using Cfg = TcCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t tc_smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + size_t(STAGES) * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2] MMA commit: accumulator ready
  uint64_t* acc_empty = acc_full + 2;    // [2] 128 epilogue arrivals: accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_tiles = (p.N + BN - 1) / BN, m_tiles = (p.M + TC_BM - 1) / TC_BM;
  const int splits = p.splits > 1 ? p.splits : 1;
  const int64_t mn_tiles = n_tiles * m_tiles, tiles = mn_tiles * splits;
  const int KB = int((p.K + TC_BK - 1) / TC_BK);
  const int pkb = p.npairs > 0 ? int(p.part_k / TC_BK) : 1;
  // tile t -> (split, m, n) and its k-block range
  auto tile_of = [&](int64_t t, int64_t& m0, int64_t& n0, int& kb0, int& kb1, int& sp) {
    sp = int(t / mn_tiles);
    const int64_t r = t - int64_t(sp) * mn_tiles;
    m0 = (r / n_tiles) * TC_BM;
    n0 = (r % n_tiles) * BN;
    kb0 = int(int64_t(KB) * sp / splits);
    kb1 = int(int64_t(KB) * (sp + 1) / splits);
  };
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait_bounded(bar, parity, &g_error_word, DEV_ERR_WAIT_TIMEOUT)) return true;
    *abort_flag = 1u;
    return false;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    *abort_flag = 0u;
    fence_mbar_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
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
    if (lane == 0) {  // TMA producer over all tiles of this CTA
      uint32_t it = 0;
      for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        int64_t m0, n0;
        int kb0, kb1, sp;
        tile_of(t, m0, n0, kb0, kb1, sp);
        bool ok = true;
        for (int kb = kb0; kb < kb1; kb += Cfg::KPS, ++it) {
          const int s = int(it % STAGES);
          if (it >= uint32_t(STAGES) && !wait(&empty[s], ((it / STAGES) - 1) & 1)) {
            ok = false;
            break;
          }
          const int nk = kb1 - kb < Cfg::KPS ? kb1 - kb : Cfg::KPS;  // k blocks in this stage
          mbar_arrive_expect_tx(&full[s], uint32_t(nk) * (Cfg::A_BYTES + Cfg::B_BYTES));
          uint8_t* st = base + size_t(s) * Cfg::STAGE_BYTES;
          for (int j = 0; j < nk; ++j) {
            int32_t ka, kbx;
            if (p.npairs > 0) {
              const int pr = (kb + j) / pkb, kk = (kb + j - pr * pkb) * TC_BK;
              ka = int32_t(p.a_part[pr] * p.part_k + kk);
              kbx = int32_t(p.b_part[pr] * p.part_k + kk);
            } else {
              ka = int32_t((int64_t(kb + j) * TC_BK) % p.a_kperiod);
              kbx = int32_t((kb + j) * TC_BK);
            }
            tma_load_2d(st + j * Cfg::A_BYTES, &tma_a, ka, int32_t(m0), &full[s]);
            tma_load_2d(st + Cfg::KPS * Cfg::A_BYTES + j * Cfg::B_BYTES, &tma_b, kbx, int32_t(n0), &full[s]);
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = umma_idesc_bf16(TC_BM, BN);
      uint32_t it = 0, ti = 0;
      for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++ti) {
        const uint32_t ab = ti & 1;
        int64_t m0, n0;
        int kb0, kb1, sp;
        tile_of(t, m0, n0, kb0, kb1, sp);
        if (ti >= 2 && !wait(&acc_empty[ab], ((ti >> 1) - 1) & 1)) break;
        tc_fence_after();
        const uint32_t d = tmem + ab * uint32_t(BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; kb += Cfg::KPS, ++it) {
          const int s = int(it % STAGES);
          if (!wait(&full[s], (it / STAGES) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = base + size_t(s) * Cfg::STAGE_BYTES;
          const int nk = kb1 - kb < Cfg::KPS ? kb1 - kb : Cfg::KPS;
          for (int j = 0; j < nk; ++j) {
            const uint64_t da = umma_desc_sw128(st + j * Cfg::A_BYTES),
                           db = umma_desc_sw128(st + Cfg::KPS * Cfg::A_BYTES + j * Cfg::B_BYTES);
#pragma unroll
            for (int k = 0; k < TC_BK / 16; ++k)
              // advance 16 bf16 = 32 bytes along K inside the swizzle atom (+2 in 16-byte units)
              umma_bf16(d, da + uint64_t(2 * k), db + uint64_t(2 * k), idesc, (kb + j != kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[ab]);
      }
    }
  } else {
    // epilogue warps 2-5: warp w drains TMEM lanes 32 (w % 4) .. +31 = tile rows
    const int q = warp & 3;
    uint32_t ti = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++ti) {
      const uint32_t ab = ti & 1;
      int64_t m0, n0;
      int kb0, kb1, sp;
      tile_of(t, m0, n0, kb0, kb1, sp);
      const bool acc_ok = wait(&acc_full[ab], (ti >> 1) & 1);
      __syncwarp();
      tc_fence_after();
      const int64_t row = m0 + q * 32 + lane;
      const uint32_t tbase = tmem + (uint32_t(q * 32) << 16) + ab * uint32_t(BN);
      if (__all_sync(0xffffffffu, acc_ok)) {
        if constexpr (MODE == 0) {
          const float sc = (p.rowscale && row < p.M) ? p.rowscale[row] : 1.f;
#pragma unroll 1
          for (int c = 0; c < BN; c += 16) {
            float v[16];
            tmem_ld16(tbase + uint32_t(c), v);
            const int64_t col = n0 + c;
            if (row >= p.M || col >= p.N) continue;
            if (p.c_dtype == LNG_F32) {
              float* dst = static_cast<float*>(p.C) + int64_t(sp) * p.split_stride + row * p.ldc + col;
              if (col + 16 <= p.N) {
#pragma unroll
                for (int i = 0; i < 16; i += 4)
                  *reinterpret_cast<float4*>(dst + i) =
                      make_float4(v[i] * sc, v[i + 1] * sc, v[i + 2] * sc, v[i + 3] * sc);
              } else {
                for (int i = 0; i < 16 && col + i < p.N; ++i) dst[i] = v[i] * sc;
              }
            } else {
              __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.C) + row * p.ldc + col;
              if (col + 16 <= p.N) {
                uint32_t w[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * i] * sc, v[2 * i + 1] * sc);
                  w[i] = *reinterpret_cast<uint32_t*>(&b2);
                }
                *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
                *reinterpret_cast<uint4*>(dst + 8) = make_uint4(w[4], w[5], w[6], w[7]);
              } else {
                for (int i = 0; i < 16 && col + i < p.N; ++i) dst[i] = __float2bfloat16_rn(v[i] * sc);
              }
            }
          }
        } else {
          // router: this tile holds routes r0 .. r0+RPT-1 (RPT * BITS logits per row); every index is
          // static, so the codes are assembled in registers
          constexpr int RPT = BN / BITS;
          const int64_t r0 = n0 / BITS;
          uint32_t packed[(RPT + 3) / 4];
#pragma unroll
          for (int i = 0; i < (RPT + 3) / 4; ++i) packed[i] = 0u;
#pragma unroll
          for (int c = 0; c < BN; c += 16) {
            float v[16];
            tmem_ld16(tbase + uint32_t(c), v);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int col = c + i, qq = col / BITS, bit = col % BITS;
              packed[qq >> 2] |= uint32_t(v[i] > 0.f ? 1u : 0u) << ((qq & 3) * 8 + bit);
            }
          }
          if (row < p.M) {
            uint8_t* dst = p.codes + row * p.routes + r0;
            const int64_t left = p.routes - r0;
            const int nr = int(left < RPT ? left : RPT);
            if (nr == RPT && RPT % 4 == 0 && (p.routes & 3) == 0 && (r0 & 3) == 0) {
#pragma unroll
              for (int i = 0; i < RPT / 4; ++i) reinterpret_cast<uint32_t*>(dst)[i] = packed[i];
            } else {
#pragma unroll
              for (int i = 0; i < RPT; ++i)
                if (i < nr) dst[i] = uint8_t(packed[i >> 2] >> ((i & 3) * 8));
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------------ two-SM form (cta_group::2)
// A cluster of two CTAs on two SMs computes 256 x BN output tiles with M = 256 MMAs issued by the
// first CTA of the pair (the leader): each CTA stages its own 128 rows of A and half of the BN rows
// of B (TMA, 128-byte swizzle), so every SM loads 2/3 of the operand bytes the one-CTA form loads
// per FLOP (the one-CTA GEMM is bounded by L2->SM operand traffic at these shapes).  Each CTA's TMEM
// holds its 128 rows x BN fp32 accumulator, twice (tile i and tile i + 1).
//   * both CTAs' TMA loads complete on the leader's full[s] barrier (.cta_group::2 loads), whose
//     expected bytes the leader's producer posts for the pair;
//   * the leader's MMA commits free a stage in both CTAs (tcgen05.commit multicast to empty[s]) and
//     mark an accumulator ready in both (acc_full);
//   * all 256 epilogue threads of the pair arrive on the leader's acc_empty before the accumulator is
//     reused (the second CTA's threads remotely).
// Waits are bounded as in the one-CTA form; both CTAs meet at cluster barriers after set-up and
// before the TMEM is released.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of this CTA's shared variable `p` as seen in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_addr(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {  // every thread of both CTAs (warps converged)
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
// arrive (once the MMAs issued so far complete) on the barrier at this offset in both CTAs
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_addr(bar))
      : "memory");
}

template <int BN>
struct Tc2Cfg {
  static constexpr int BM = 256;  // rows per pair tile (128 per CTA)
  static constexpr uint32_t A_BYTES = TC_BM * TC_BK * 2;
  static constexpr uint32_t B_BYTES = (BN / 2) * TC_BK * 2;
  // two 64-element k blocks per stage, [A0 | A1 | B0 | B1]: half the stage handshakes per FLOP (measured
  // at the SB shapes: 12-13 % less time than one k block per stage with the same shared memory)
  static constexpr int KPS = 2;
  static constexpr uint32_t STAGE_BYTES = KPS * (A_BYTES + B_BYTES);
  // eight epilogue warps: two per TMEM lane quadrant, each draining half of the tile's columns
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  // epilogue staging: one 32-row x 128-byte buffer per epilogue warp (swizzled 16-byte chunks)
  static constexpr uint32_t EPI_BYTES = EPI_WARPS * 4096;
  static constexpr int FIT = int((227 * 1024 - EPI_BYTES - 1024 - 256) / STAGE_BYTES);
  static constexpr int STAGES = FIT > 8 ? 8 : FIT;
  static constexpr uint32_t TMEM_COLS = TcCfg<BN>::TMEM_COLS;
  static constexpr size_t SMEM = size_t(STAGES) * STAGE_BYTES + EPI_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert((BN / 2) % 16 == 0 && BN <= 256, "pair tile width (each epilogue half whole 16-column loads)");
  static_assert(STAGES >= 3, "pair pipeline depth");
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
};

// 32 TMEM columns of this warp's 32 lanes; tmem_wait32 makes the registers valid (it names them as
// operands, so no use can be scheduled above it).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait32(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                 "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

template <int BN, int MODE, int BITS = 1>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Tc2Cfg<BN>::THREADS, 1)
    tc_gemm2_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                    TcGemmParams p) {
  using Cfg = Tc2Cfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t tc_smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi = base + size_t(STAGES) * Cfg::STAGE_BYTES;  // epilogue staging buffers
  uint64_t* full = reinterpret_cast<uint64_t*>(epi + Cfg::EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2] (both CTAs) leader's MMA commit: accumulator ready
  uint64_t* acc_empty = acc_full + 2;   // [2] (leader) 256 epilogue arrivals: accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int64_t pair = blockIdx.x >> 1, npair = gridDim.x >> 1;
  const int64_t n_tiles = (p.N + BN - 1) / BN, m_tiles = (p.M + Cfg::BM - 1) / Cfg::BM;
  const int64_t tiles = n_tiles * m_tiles;
  const int KB = int((p.K + TC_BK - 1) / TC_BK);
  auto tile_of = [&](int64_t t, int64_t& m0, int64_t& n0) {
    m0 = (t / n_tiles) * Cfg::BM;
    n0 = (t % n_tiles) * BN;
  };
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait_bounded(bar, parity, &g_error_word, DEV_ERR_WAIT_TIMEOUT)) return true;
    *abort_flag = 1u;
    return false;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 2 * 32 * Cfg::EPI_WARPS);
    }
    *abort_flag = 0u;
    fence_mbar_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(Cfg::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer: this CTA's A rows and B half, completing on the leader's barrier
      uint32_t it = 0;
      const uint32_t full_l0 = mapa_shared(&full[0], 0);
      for (int64_t t = pair; t < tiles; t += npair) {
        int64_t m0, n0;
        tile_of(t, m0, n0);
        bool ok = true;
        for (int kb = 0; kb < KB; kb += Cfg::KPS, ++it) {
          const int s = int(it % STAGES);
          if (it >= uint32_t(STAGES) && !wait(&empty[s], ((it / STAGES) - 1) & 1)) {
            ok = false;
            break;
          }
          const int nk = KB - kb < Cfg::KPS ? KB - kb : Cfg::KPS;  // k blocks in this stage
          if (leader) mbar_arrive_expect_tx(&full[s], 2u * uint32_t(nk) * (Cfg::A_BYTES + Cfg::B_BYTES));
          uint8_t* st = base + size_t(s) * Cfg::STAGE_BYTES;
          const uint32_t fb = full_l0 + uint32_t(s) * 8u;
          for (int j = 0; j < nk; ++j) {
            const int32_t ka = int32_t((int64_t(kb + j) * TC_BK) % p.a_kperiod), kbx = int32_t((kb + j) * TC_BK);
            tma_load_2d_pair(st + j * Cfg::A_BYTES, &tma_a, ka, int32_t(m0 + int64_t(rank) * TC_BM), fb);
            tma_load_2d_pair(st + Cfg::KPS * Cfg::A_BYTES + j * Cfg::B_BYTES, &tma_b, kbx,
                             int32_t(n0 + int64_t(rank) * (BN / 2)), fb);
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // MMA issuer for the pair
      constexpr uint32_t idesc = umma_idesc_bf16(Cfg::BM, BN);
      uint32_t it = 0, ti = 0;
      for (int64_t t = pair; t < tiles; t += npair, ++ti) {
        const uint32_t ab = ti & 1;
        if (ti >= 2 && !wait(&acc_empty[ab], ((ti >> 1) - 1) & 1)) break;
        tc_fence_after();
        const uint32_t d = tmem + ab * uint32_t(BN);
        bool ok = true;
        for (int kb = 0; kb < KB; kb += Cfg::KPS, ++it) {
          const int s = int(it % STAGES);
          if (!wait(&full[s], (it / STAGES) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = base + size_t(s) * Cfg::STAGE_BYTES;
          const int nk = KB - kb < Cfg::KPS ? KB - kb : Cfg::KPS;
          for (int j = 0; j < nk; ++j) {
            const uint64_t da = umma_desc_sw128(st + j * Cfg::A_BYTES),
                           db = umma_desc_sw128(st + Cfg::KPS * Cfg::A_BYTES + j * Cfg::B_BYTES);
#pragma unroll
            for (int k = 0; k < TC_BK / 16; ++k)
              umma_bf16_pair(d, da + uint64_t(2 * k), db + uint64_t(2 * k), idesc, (kb + j != 0 || k != 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty[s]);
        }
        if (!ok) break;
        umma_commit_pair(&acc_full[ab]);
      }
    }
  } else {
    // epilogue warps 2-9 of each CTA: TMEM lanes 32 (w % 4) .. +31 = this CTA's tile rows, warps 2-5
    // the tile's first half of the columns, warps 6-9 the second
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    constexpr int HB = BN / 2;  // columns per epilogue warp
    const uint32_t acc_empty_l0 = mapa_shared(&acc_empty[0], 0);
    uint32_t ti = 0;
    for (int64_t t = pair; t < tiles; t += npair, ++ti) {
      const uint32_t ab = ti & 1;
      int64_t m0, n0;
      tile_of(t, m0, n0);
      const bool acc_ok = wait(&acc_full[ab], (ti >> 1) & 1);
      __syncwarp();
      tc_fence_after();
      const int64_t row = m0 + int64_t(rank) * TC_BM + q * 32 + lane;
      const uint32_t tbase = tmem + (uint32_t(q * 32) << 16) + ab * uint32_t(BN);
      if (__all_sync(0xffffffffu, acc_ok)) {
        if constexpr (MODE == 0) {
          // 128-byte column chunks (64 bf16 / 32 f32) of this warp's 32 rows: TMEM -> registers (row
          // per lane) -> this warp's staging buffer (16-byte pieces swizzled by row) -> read back four
          // rows per instruction, so each global store writes whole 128-byte row segments
          const float sc = (p.rowscale && row < p.M) ? p.rowscale[row] : 1.f;
          const bool f32 = p.c_dtype == LNG_F32;
          const int CW = f32 ? 32 : 64;
          const int esz = f32 ? 4 : 2;
          const int64_t y0 = m0 + int64_t(rank) * TC_BM + q * 32;
          uint8_t* buf = epi + (warp - 2) * 4096;
#pragma unroll 1
          for (int c = half * HB; c < (half + 1) * HB; c += CW) {
            uint32_t r0[32], r1[32];
            tmem_ld32(tbase + uint32_t(c), r0);
            if (!f32) tmem_ld32(tbase + uint32_t(c) + 32u, r1);
            tmem_wait32(r0);
            if (!f32) tmem_wait32(r1);
            uint4* rowp = reinterpret_cast<uint4*>(buf + lane * 128);
            if (f32) {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                rowp[j ^ (lane & 7)] = make_uint4(__float_as_uint(__uint_as_float(r0[4 * j]) * sc),
                                                  __float_as_uint(__uint_as_float(r0[4 * j + 1]) * sc),
                                                  __float_as_uint(__uint_as_float(r0[4 * j + 2]) * sc),
                                                  __float_as_uint(__uint_as_float(r0[4 * j + 3]) * sc));
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const uint32_t(&rr)[32] = j < 4 ? r0 : r1;
                const int b = (j & 3) * 8;
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(rr[b + 2 * i]) * sc,
                                                            __uint_as_float(rr[b + 2 * i + 1]) * sc);
                  w[i] = *reinterpret_cast<uint32_t*>(&b2);
                }
                rowp[j ^ (lane & 7)] = make_uint4(w[0], w[1], w[2], w[3]);
              }
            }
            __syncwarp();
            const int j = lane & 7;                  // this lane's 16-byte piece of a row
            const int64_t col = n0 + c + j * (16 / esz);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int rr = i * 4 + (lane >> 3);      // row within the warp's 32
              const int64_t grow = y0 + rr;
              const uint4 v = *reinterpret_cast<const uint4*>(buf + rr * 128 + ((j ^ (rr & 7)) * 16));
              if (grow >= p.M || col >= p.N) continue;
              uint8_t* dst = static_cast<uint8_t*>(p.C) + (grow * p.ldc + col) * esz;
              if (col + 16 / esz <= p.N) {
                *reinterpret_cast<uint4*>(dst) = v;
              } else {  // ragged last columns
                const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
                for (int e = 0; e < 16 / esz && col + e < p.N; ++e) {
                  if (f32) reinterpret_cast<uint32_t*>(dst)[e] = vv[e];
                  else reinterpret_cast<uint16_t*>(dst)[e] = uint16_t(vv[e >> 1] >> ((e & 1) * 16));
                }
              }
            }
            __syncwarp();
          }
        } else {
          constexpr int RPT = HB / BITS;  // routes of this warp's half of the tile
          const int64_t r0 = n0 / BITS + half * RPT;
          uint32_t packed[(RPT + 3) / 4];
#pragma unroll
          for (int i = 0; i < (RPT + 3) / 4; ++i) packed[i] = 0u;
#pragma unroll
          for (int c = 0; c < HB; c += 16) {
            float v[16];
            tmem_ld16(tbase + uint32_t(half * HB + c), v);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int col = c + i, qq = col / BITS, bit = col % BITS;
              packed[qq >> 2] |= uint32_t(v[i] > 0.f ? 1u : 0u) << ((qq & 3) * 8 + bit);
            }
          }
          if (row < p.M && r0 < p.routes) {
            uint8_t* dst = p.codes + row * p.routes + r0;
            const int64_t left = p.routes - r0;
            const int nr = int(left < RPT ? left : RPT);
            if (nr == RPT && RPT % 4 == 0 && (p.routes & 3) == 0 && (r0 & 3) == 0) {
#pragma unroll
              for (int i = 0; i < RPT / 4; ++i) reinterpret_cast<uint32_t*>(dst)[i] = packed[i];
            } else {
#pragma unroll
              for (int i = 0; i < RPT; ++i)
                if (i < nr) dst[i] = uint8_t(packed[i >> 2] >> ((i & 3) * 8));
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(acc_empty_l0 + ab * 8u);
    }
  }
  tc_fence_before();
  cluster_sync_all();  // every MMA of the pair retired and read before the TMEM is released
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::TMEM_COLS) : "memory");
  }
}

// fp32 weight -> [rows, 3*in_dim] bf16 (W1 | W2 | W3) with W = W1 + W2 + W3.
__global__ void split_bf16x3_kernel(const float* __restrict__ w, int64_t rows, int64_t in_dim,
                                    __nv_bfloat16* __restrict__ out) {
  const int64_t total = rows * in_dim;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / in_dim, k = e % in_dim;
    const float x = w[e];
    const __nv_bfloat16 a = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(a);
    const __nv_bfloat16 b = __float2bfloat16_rn(r1);
    const float r2 = r1 - __bfloat162float(b);
    const __nv_bfloat16 c = __float2bfloat16_rn(r2);
    __nv_bfloat16* o = out + r * 3 * in_dim;
    o[k] = a;
    o[in_dim + k] = b;
    o[2 * in_dim + k] = c;
  }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// 2D bf16 tensor map over a row-major [rows, cols] matrix with row stride ld (elements); box 64 x box_rows.
inline int make_tmap_bf16(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(LNG_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (driver entry point)");
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  const cuuint32_t box[2] = {uint32_t(TC_BK), uint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LNG_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return LNG_OK;
}

template <int BN, int MODE, int BITS = 1>
inline int launch_tc_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const TcGemmParams& p, cudaStream_t stream) {
  // the MODE 0 epilogue stores 16-byte vectors: rows and split slices must keep that alignment
  if (MODE == 0 && ((reinterpret_cast<uintptr_t>(p.C) & 15) || p.ldc % (p.c_dtype == LNG_F32 ? 4 : 8) ||
                    p.split_stride % (p.c_dtype == LNG_F32 ? 4 : 8)))
    return fail(LNG_ERR_ARGUMENT, "tc_gemm: output base / row stride not 16-byte aligned");
  auto kern = tc_gemm_kernel<BN, MODE, BITS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(TcCfg<BN>::SMEM));
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(tc_gemm_kernel)");
  const int64_t tiles = ((p.N + BN - 1) / BN) * ((p.M + TC_BM - 1) / TC_BM) * (p.splits > 1 ? p.splits : 1);
  const int grid = int(tiles < num_sms() ? tiles : num_sms());
  kern<<<grid, 192, TcCfg<BN>::SMEM, stream>>>(ta, tb, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "tc_gemm_kernel launch");
  return LNG_OK;
}

// The two-SM form for large row counts (at least one 256-row tile per SM pair); npairs / splits
// are not supported by it.
template <int BN, int MODE, int BITS = 1>
inline int launch_tc_gemm2(const CUtensorMap& ta, const CUtensorMap& tb, const TcGemmParams& p, cudaStream_t stream) {
  if (MODE == 0 && ((reinterpret_cast<uintptr_t>(p.C) & 15) || p.ldc % (p.c_dtype == LNG_F32 ? 4 : 8)))
    return fail(LNG_ERR_ARGUMENT, "tc_gemm: output base / row stride not 16-byte aligned");
  auto kern = tc_gemm2_kernel<BN, MODE, BITS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Tc2Cfg<BN>::SMEM));
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(tc_gemm2_kernel)");
  const int64_t tiles = ((p.N + BN - 1) / BN) * ((p.M + Tc2Cfg<BN>::BM - 1) / Tc2Cfg<BN>::BM);
  const int64_t pairs = tiles < num_sms() / 2 ? tiles : num_sms() / 2;
  kern<<<int(2 * pairs), Tc2Cfg<BN>::THREADS, Tc2Cfg<BN>::SMEM, stream>>>(ta, tb, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "tc_gemm2_kernel launch");
  return LNG_OK;
}
#ifndef TC_PAIR_MIN_M
#define TC_PAIR_MIN_M 8192
#endif
constexpr int64_t TC2_MIN_M = TC_PAIR_MIN_M;  // rows from which the two-SM form is used

inline bool tc_aligned(const void* p, int64_t ld) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && (ld % 8) == 0;
}

// Few rows (a draft step's 64): the (row tile, column tile) grid alone would leave most SMs idle with
// each CTA streaming all of K, so K is split over `splits` CTAs per tile as well, each writing an fp32
// partial product [M, N] (rowscale applied) at partials + s * M * N; splitk_reduce_kernel sums them.
// Returns the split count to use (1: the plain GEMM is better).
inline int tc_gemm_small_m_splits(int64_t M, int64_t N, int64_t K) {
  constexpr int BN = 128;
  const int64_t tiles = ((M + TC_BM - 1) / TC_BM) * ((N + BN - 1) / BN);
  const int64_t kb = (K + TC_BK - 1) / TC_BK;
  if (M > TC_BM || 2 * tiles > num_sms() || kb < 4) return 1;
  return int(std::min<int64_t>(kb / 2, num_sms() / tiles));
}

inline int tc_gemm_bf16_splitk(const __nv_bfloat16* A, int64_t lda, const __nv_bfloat16* B, int64_t ldb,
                               float* partials, int splits, int64_t M, int64_t N, int64_t K, const float* rowscale,
                               cudaStream_t stream) {
  if (!tc_aligned(A, lda) || !tc_aligned(B, ldb) || K < 16 || N < 16 || M < 1 || (N % 4))
    return LNG_ERR_UNSUPPORTED;
  CUtensorMap ta, tb;
  int st = make_tmap_bf16(&ta, A, M, K, lda, TC_BM);
  if (st) return st;
  st = make_tmap_bf16(&tb, B, N, K, ldb, 128);
  if (st) return st;
  TcGemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_kperiod = (K + TC_BK - 1) / TC_BK * TC_BK;  // no wrap
  p.C = partials;
  p.ldc = N;
  p.c_dtype = LNG_F32;
  p.rowscale = rowscale;
  p.splits = splits;
  p.split_stride = M * N;
  return launch_tc_gemm<128, 0>(ta, tb, p, stream);
}

// C[M, N] (+ ldc) = sum over s of partials[s] (fp32, [M, N] each), in split order.
template <typename CT>
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int64_t M, int64_t N,
                                     CT* __restrict__ C, int64_t ldc) {
  const int64_t n4 = N / 4, total = M * n4, stride = M * N;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / n4, c = (e - r * n4) * 4;
    float4 a = *reinterpret_cast<const float4*>(part + r * N + c);
    for (int s = 1; s < splits; ++s) {
      const float4 b = *reinterpret_cast<const float4*>(part + s * stride + r * N + c);
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    CT* o = C + r * ldc + c;
    o[0] = from_f32<CT>(a.x);
    o[1] = from_f32<CT>(a.y);
    o[2] = from_f32<CT>(a.z);
    o[3] = from_f32<CT>(a.w);
  }
}

// Plain bf16 GEMM on the tensor cores; LNG_ERR_UNSUPPORTED when the operands do not meet TMA rules.
inline int tc_gemm_bf16(const __nv_bfloat16* A, int64_t lda, const __nv_bfloat16* B, int64_t ldb, void* C,
                        int32_t c_dtype, int64_t ldc, int64_t M, int64_t N, int64_t K, const float* rowscale,
                        cudaStream_t stream) {
  if (c_dtype != LNG_F32 && c_dtype != LNG_BF16) return LNG_ERR_UNSUPPORTED;
  if (!tc_aligned(A, lda) || !tc_aligned(B, ldb) || (reinterpret_cast<uintptr_t>(C) & 15) || (ldc % 8) || K < 16 ||
      N < 16 || M < 1)
    return LNG_ERR_UNSUPPORTED;
  // 256-column tiles (twice the tensor-pipe efficiency of 128 measured here) unless N <= 128; 128 for
  // few rows was also measured and was slower (each CTA still streams all of K)
  const int BN = N > 128 ? 256 : 128;
  const bool pair = M >= TC2_MIN_M;
  CUtensorMap ta, tb;
  int st = make_tmap_bf16(&ta, A, M, K, lda, TC_BM);
  if (st) return st;
  st = make_tmap_bf16(&tb, B, N, K, ldb, pair ? BN / 2 : BN);
  if (st) return st;
  TcGemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_kperiod = (K + TC_BK - 1) / TC_BK * TC_BK;  // no wrap
  p.C = C;
  p.ldc = ldc;
  p.c_dtype = c_dtype;
  p.rowscale = rowscale;
  if (pair) return BN == 256 ? launch_tc_gemm2<256, 0>(ta, tb, p, stream) : launch_tc_gemm2<128, 0>(ta, tb, p, stream);
  return BN == 256 ? launch_tc_gemm<256, 0>(ta, tb, p, stream) : launch_tc_gemm<128, 0>(ta, tb, p, stream);
}

// Router codes on the tensor cores from bf16 inputs and the split weight [routes*bits, 3*in_dim].
inline int tc_router_split(const __nv_bfloat16* x, int64_t n, int64_t in_dim, int64_t x_stride,
                           const __nv_bfloat16* w_split, int64_t routes, int32_t bits, uint8_t* codes,
                           cudaStream_t stream) {
  if (bits < 1 || bits > 6 || in_dim % TC_BK != 0 || !tc_aligned(x, x_stride) || !tc_aligned(w_split, 3 * in_dim))
    return LNG_ERR_UNSUPPORTED;
  const bool pair = n >= TC2_MIN_M;
  // 64 routes per tile up to 4 bits, else 32; 16 when the row tiles are so few that wider tiles
  // would leave most SMs idle (measured 2-3 % faster on the 1,024-node tree step)
  int BN = bits <= 4 ? 64 * bits : 32 * bits;
  const bool narrow = !pair && ((n + TC_BM - 1) / TC_BM) * ((routes * bits + BN - 1) / BN) < num_sms() / 2;
  if (narrow) BN = 16 * bits;
  CUtensorMap ta, tb;
  int st = make_tmap_bf16(&ta, x, n, in_dim, x_stride, TC_BM);
  if (st) return st;
  st = make_tmap_bf16(&tb, w_split, routes * bits, 3 * in_dim, 3 * in_dim, pair ? BN / 2 : BN);
  if (st) return st;
  TcGemmParams p{};
  p.M = n;
  p.N = routes * bits;
  p.K = 3 * in_dim;
  p.a_kperiod = in_dim;
  p.bits = bits;
  p.routes = routes;
  p.codes = codes;
  if (pair) {
    switch (bits) {
      case 1: return launch_tc_gemm2<64, 1, 1>(ta, tb, p, stream);
      case 2: return launch_tc_gemm2<128, 1, 2>(ta, tb, p, stream);
      case 3: return launch_tc_gemm2<192, 1, 3>(ta, tb, p, stream);
      case 4: return launch_tc_gemm2<256, 1, 4>(ta, tb, p, stream);
      case 5: return launch_tc_gemm2<160, 1, 5>(ta, tb, p, stream);
      default: return launch_tc_gemm2<192, 1, 6>(ta, tb, p, stream);
    }
  }
  if (narrow) {
    switch (bits) {
      case 1: return launch_tc_gemm<16, 1, 1>(ta, tb, p, stream);
      case 2: return launch_tc_gemm<32, 1, 2>(ta, tb, p, stream);
      case 3: return launch_tc_gemm<48, 1, 3>(ta, tb, p, stream);
      case 4: return launch_tc_gemm<64, 1, 4>(ta, tb, p, stream);
      case 5: return launch_tc_gemm<80, 1, 5>(ta, tb, p, stream);
      default: return launch_tc_gemm<96, 1, 6>(ta, tb, p, stream);
    }
  }
  switch (bits) {
    case 1: return launch_tc_gemm<64, 1, 1>(ta, tb, p, stream);
    case 2: return launch_tc_gemm<128, 1, 2>(ta, tb, p, stream);
    case 3: return launch_tc_gemm<192, 1, 3>(ta, tb, p, stream);
    case 4: return launch_tc_gemm<256, 1, 4>(ta, tb, p, stream);
    case 5: return launch_tc_gemm<160, 1, 5>(ta, tb, p, stream);
    default: return launch_tc_gemm<192, 1, 6>(ta, tb, p, stream);
  }
}

// Without a prepared split weight the router stays on the CUDA cores.
inline int tc_router_codes(const __nv_bfloat16*, int64_t, int64_t, int64_t, const float*, int64_t, int32_t, uint8_t*,
                           cudaStream_t) {
  return LNG_ERR_UNSUPPORTED;
}

}  // namespace lng
