// Fused gather + sink attention over routes (folded readout core).
//
// Reference math (ffnmem/memory/lngram_v2.py): route tokens of _lookup_route_chunk (:1047-1113),
// RMSNorm + kv_proj of _project_memory (:1120-1131), grouped scores * HD^-1/2 and the sink
// probabilities of _real_route_probabilities / _manual_gqa (:1877-1920), in the online (route
// chunk) form of _streaming_gqa (:1944-2070): the running state starts at (max = b0, sum = 1,
// value = 0), i.e. the zero-value sink, and each chunk of routes updates it.
//
// Folded form: with qa = the folded query of the item (w_qk . h, see lng_fold_readout) the score of
// route r is qscale * rms(tok_r)^-1 * (qa . tok_r) and the output is u = sum_r p_r rms(tok_r)^-1 tok_r,
// so the tokens are read once, straight from the tables, and never projected.  A route whose
// n-gram window is invalid has a zero token and still takes part with score 0, exactly as the
// reference's zero rows do.
#pragma once

#include <type_traits>

#include "address.cuh"

namespace lng {

struct AttendParams {
  TableSet ts;
  CodeSource src;
  int64_t M;
  int64_t route_start, route_end;
  int qh;          // query heads
  float eps;
  float sink;      // b0
  const void* qa;  // [M, qh, Dt]
  const float* qscale;
  void* u;         // [M, qh, Dt]
  int partial;
  float* m_out;
  float* l_out;
  int rows32;      // every table row index fits int32 (the tensor-core gather's cooperative copies)
  int64_t route_split;  // the tensor-core kernel's SPLIT form (partial mode 1): block row y takes routes
                        // [route_start + y split, + split) and writes state y of [gridDim.y, M, ...];
                        // only y = 0 seeds the sink
};

// ------------------------------------------------------------------ generic CUDA-core version
// One CTA per item (grid-stride), chunks of ATT_C routes.  Any Dt / heads / table dtype.
constexpr int ATT_C = 32;

template <typename CodeT, typename TabT, typename QT, typename UT>
__global__ void __launch_bounds__(128) attend_simt_kernel(AttendParams p) {
  extern __shared__ float sm[];
  const int Dt = p.ts.n_orders * int(p.ts.mem_dim);
  const int QH = p.qh;
  float* qa = sm;                       // [QH, Dt]
  float* U = qa + QH * Dt;              // [QH, Dt]
  float* tok = U + QH * Dt;             // [C, Dt]
  float* rx = tok + ATT_C * Dt;         // [C]
  float* sc = rx + ATT_C;               // [QH, C]
  float* mrow = sc + QH * ATT_C;        // [QH]
  float* lrow = mrow + QH;              // [QH]
  float* alpha = lrow + QH;             // [QH]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const bool sink_in = p.partial != 2;  // partial == 2: a route shard whose state leaves the sink to another

  for (int64_t item = blockIdx.x; item < p.M; item += gridDim.x) {
    const float qs = p.qscale ? p.qscale[item] : 1.f;
    const QT* qg = static_cast<const QT*>(p.qa) + item * QH * Dt;
    for (int e = threadIdx.x; e < QH * Dt; e += blockDim.x) {
      qa[e] = to_f32(qg[e]);
      U[e] = 0.f;
    }
    for (int q = threadIdx.x; q < QH; q += blockDim.x) {
      mrow[q] = sink_in ? p.sink : -INFINITY;
      lrow[q] = sink_in ? 1.f : 0.f;
    }
    __syncthreads();
    for (int64_t c0 = p.route_start; c0 < p.route_end; c0 += ATT_C) {
      // gather the chunk's tokens (fp32) and their inverse RMS
      for (int rl = warp; rl < ATT_C; rl += nwarps) {
        const int64_t r = c0 + rl;
        float ss = 0.f;
        for (int o = 0; o < p.ts.n_orders; ++o) {
          int64_t row = -1;
          if (r < p.route_end) row = ngram_row<CodeT>(p.src, item, r, p.ts.order[o], p.ts.bits);
          const TabT* s = static_cast<const TabT*>(p.ts.tab[o]) + (row < 0 ? 0 : row) * p.ts.mem_dim;
          for (int j = lane; j < p.ts.mem_dim; j += 32) {
            const float v = row < 0 ? 0.f : to_f32(s[j]);
            tok[rl * Dt + o * p.ts.mem_dim + j] = v;
            ss += v * v;
          }
        }
        ss = warp_sum(ss);
        if (lane == 0) rx[rl] = rsqrtf(ss / float(Dt) + p.eps);
      }
      __syncthreads();
      for (int e = threadIdx.x; e < QH * ATT_C; e += blockDim.x) {
        const int q = e / ATT_C, rl = e % ATT_C;
        float s = -INFINITY;
        if (c0 + rl < p.route_end) {
          float acc = 0.f;
          for (int k = 0; k < Dt; ++k) acc = fmaf(qa[q * Dt + k], tok[rl * Dt + k], acc);
          s = acc * qs * rx[rl];
        }
        sc[e] = s;
      }
      __syncthreads();
      for (int q = threadIdx.x; q < QH; q += blockDim.x) {
        float mx = mrow[q];
        for (int rl = 0; rl < ATT_C; ++rl) mx = fmaxf(mx, sc[q * ATT_C + rl]);
        const float a = expf(mrow[q] - mx);
        float sum = 0.f;
        for (int rl = 0; rl < ATT_C; ++rl) {
          const float e = expf(sc[q * ATT_C + rl] - mx);
          sc[q * ATT_C + rl] = e * rx[rl];
          sum += e;
        }
        lrow[q] = lrow[q] * a + sum;
        mrow[q] = mx;
        alpha[q] = a;
      }
      __syncthreads();
      for (int e = threadIdx.x; e < QH * Dt; e += blockDim.x) {
        const int q = e / Dt, k = e % Dt;
        float acc = U[e] * alpha[q];
        for (int rl = 0; rl < ATT_C; ++rl) acc = fmaf(sc[q * ATT_C + rl], tok[rl * Dt + k], acc);
        U[e] = acc;
      }
      __syncthreads();
    }
    if (p.partial) {
      float* uo = static_cast<float*>(p.u) + item * QH * Dt;
      for (int e = threadIdx.x; e < QH * Dt; e += blockDim.x) uo[e] = U[e];
      for (int q = threadIdx.x; q < QH; q += blockDim.x) {
        p.m_out[item * QH + q] = mrow[q];
        p.l_out[item * QH + q] = lrow[q];
      }
    } else {
      UT* uo = static_cast<UT*>(p.u) + item * QH * Dt;
      for (int e = threadIdx.x; e < QH * Dt; e += blockDim.x) {
        const int q = e / Dt;
        uo[e] = from_f32<UT>(U[e] / fmaxf(lrow[q], 1.17549435e-38f));
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ tensor-core version (bf16 / f16)
// One warp per item; routes in chunks of 32 streamed through a per-warp ring of two shared-memory
// stages: the rows of a single-order table by the warp's own 16-byte cp.async copies, multi-order
// tokens by one bulk (TMA-engine) copy per (route, order) row; the item's folded query arrives by
// one bulk copy with its first chunk.  Scores
// (16 x 32 per chunk) and the weighted row sum (16 x Dt) are mma.sync m16n8k16 products with fp32
// accumulation: the per-item products are 16 x 32 x Dt, below the 64-row minimum of a tcgen05 MMA,
// and every item has its own B operand, so the warp-level MMA is the fitting unit here.
template <typename T>
struct MmaType;
template <>
struct MmaType<__nv_bfloat16> {
  static constexpr const char* name = "bf16";
};
template <>
struct MmaType<__half> {
  static constexpr const char* name = "f16";
};

__device__ __forceinline__ uint32_t pack2(float lo, float hi, __nv_bfloat16*) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi, __half*) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {  // 2^x (PTX ex2.approx.ftz.f32)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int DT>
struct AttendMmaCfg {
  static constexpr int C = 32;                   // routes per chunk (= lanes: one route per lane)
  static constexpr int KT = (DT + 15) / 16;      // k16 steps of the score product
  static constexpr int NTU = DT / 8;             // n8 tiles of the weighted row sum
  static constexpr int ROWB = DT * 2;            // bytes per token row in shared memory
  static constexpr int SS_OFF = C * ROWB + 32;   // zero pad read by the last k-step, then the rows' sums of squares
  static constexpr int QS_OFF = SS_OFF + C * 4;  // the item's query scale (stages holding an item's first chunk)
  static constexpr int QA_OFF = QS_OFF + 16;     // the item's folded query [16 heads][DT] (same stages)
  static constexpr int STAGES = 2;
  static constexpr int STAGE_BYTES = QA_OFF + 16 * ROWB;
  // warps per CTA: as many as 227 KB of shared memory holds, at most 8 (register file: ~250 per thread)
  static constexpr int FIT = (227 * 1024) / (STAGES * (STAGE_BYTES + 8));
  static constexpr int WARPS = FIT < 8 ? FIT : 8;
  static_assert(FIT >= 1, "route token too wide for the tensor-core gather");
};

template <typename CodeT, typename T, int DT, int WARPS, int STAGES, bool SPLIT = false>
__global__ void __launch_bounds__(WARPS * 32) attend_mma_kernel(AttendParams p) {
  using Cfg = AttendMmaCfg<DT>;
  constexpr int C = Cfg::C, KT = Cfg::KT, NTU = Cfg::NTU, ROWB = Cfg::ROWB, SB = Cfg::STAGE_BYTES;
  static_assert(DT % 8 == 0, "route token width must be a multiple of 8");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned char* stage_base = smem_raw + size_t(warp) * STAGES * SB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + size_t(WARPS) * STAGES * SB) + warp * STAGES;

  // this block's routes (a route split gives every block row y its own slice and state)
  // (the unsplit form reads the bounds straight from the parameters, as before the split existed)
  const int64_t split_lo = SPLIT ? p.route_start + int64_t(blockIdx.y) * p.route_split : 0;
  const int64_t split_hi = SPLIT ? min(split_lo + p.route_split, p.route_end) : 0;
#define LNG_RLO (SPLIT ? split_lo : p.route_start)
#define LNG_RHI (SPLIT ? split_hi : p.route_end)
  const int nch = int((LNG_RHI - LNG_RLO + C - 1) / C);
  const int64_t gwarp = int64_t(blockIdx.x) * WARPS + warp;
  const int64_t nwarps = int64_t(gridDim.x) * WARPS;
  const int64_t my_items = gwarp < p.M ? (p.M - 1 - gwarp) / nwarps + 1 : 0;
  const int jobs = int(my_items * nch);
  // partial 2 / 4: a route shard whose state leaves the sink to another shard
  const bool sink_in = p.partial != 2 && p.partial != 4 && (!SPLIT || blockIdx.y == 0);
  const int mem_dim = int(p.ts.mem_dim);

  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 32);
    fence_mbar_init();
  }
  // zero the pad after every stage (read by the last score k-step for rows near the end)
  for (int s = 0; s < STAGES; ++s)
    if (lane < 8) reinterpret_cast<uint32_t*>(stage_base + s * SB + C * ROWB)[lane] = 0u;
  __syncwarp();

  // Gather pipeline, lane = route within the chunk.  Job J's codes are loaded (prefetch) one
  // iteration before its row copies are issued, and copies run STAGES-1 jobs ahead of the math, so
  // neither the code loads nor the row loads sit on the critical path.  The stage of an item's
  // first chunk also receives the item's folded query (one bulk copy) and its query scale.
  int64_t pf_item = gwarp;  // prefetch cursor
  int pf_chunk = 0;
  ItemGeo pf_geo{};
  int32_t pend_c[MAXW];
  ItemGeo pend_geo{};
  int pend_chunk = 0;
  int64_t pend_item = 0;
  float pend_qs = 1.f;
  auto prefetch = [&]() {
    if (pf_chunk == 0) pf_geo = item_geometry(p.src, p.ts.order, p.ts.n_orders, pf_item);
    pend_geo = pf_geo;
    pend_chunk = pf_chunk;
    pend_item = pf_item;
    if (pf_chunk == 0) pend_qs = p.qscale ? __ldg(p.qscale + pf_item) : 1.f;
    const int64_t r = LNG_RLO + int64_t(pf_chunk) * C + lane;
    load_window_codes<CodeT>(p.src, pf_geo, r, r < LNG_RHI, pend_c);
    if (++pf_chunk == nch) {
      pf_chunk = 0;
      pf_item += nwarps;
    }
  };
  // The sum of squares of each gathered row (precomputed per table row) is loaded when the row's copy
  // is issued and written to the stage one iteration later, so its load latency is hidden too; the
  // lane that wrote it is the lane that reads it.
  const bool have_ss = p.ts.ss[0] != nullptr;
  float ss_pend[LNG_MAX_ORDERS];  // raw loaded values: summed only at flush time, after the loads landed
  int ss_stage = -1;
  auto flush_ss = [&]() {
    if (ss_stage >= 0) {
      float ss = 0.f;
#pragma unroll
      for (int o = 0; o < LNG_MAX_ORDERS; ++o)
        if (o < p.ts.n_orders) ss += ss_pend[o];
      reinterpret_cast<float*>(stage_base + ss_stage * SB + Cfg::SS_OFF)[lane] = ss;
    }
    ss_stage = -1;
  };
  const uint32_t qa_bytes = uint32_t(p.qh) * DT * 2;
  // Single-order tables: the chunk's 32 rows are copied cooperatively by the whole warp with 16-byte
  // cp.async copies (load/store path, about two rows per warp instruction).  One bulk copy (TMA
  // engine) per row measured slower: the engine's per-copy cost, not HBM, bounded the row rate.
  // Multi-order tokens keep one bulk copy per (route, order) row.
  const bool coop = p.ts.n_orders == 1 && p.rows32;
  const bool bulk_lane = !coop;
  auto issue = [&](int s) {
    flush_ss();
    const int64_t r = LNG_RLO + int64_t(pend_chunk) * C + lane;
    unsigned char* row_smem = stage_base + s * SB + lane * ROWB;
    int64_t rows[LNG_MAX_ORDERS];
    uint32_t bytes = 0;
#pragma unroll
    for (int o = 0; o < LNG_MAX_ORDERS; ++o) {
      if (o >= p.ts.n_orders) break;
      rows[o] = p.src.direct > 0 ? (r < LNG_RHI ? pend_item * p.src.direct + r : -1)
                                 : window_row(pend_c, p.ts.order[o], p.ts.bits, r,
                                              r < LNG_RHI && ((pend_geo.omask >> o) & 1u));
      ss_pend[o] = 0.f;
      if (rows[o] >= 0) {
        if (bulk_lane) bytes += uint32_t(mem_dim * 2);
        if (have_ss) ss_pend[o] = __ldg(p.ts.ss[o] + rows[o]);
      } else if (bulk_lane) {
        uint4* z = reinterpret_cast<uint4*>(row_smem + o * mem_dim * 2);
        for (int v = 0; v < mem_dim * 2 / 16; ++v) z[v] = make_uint4(0, 0, 0, 0);
      }
    }
    ss_stage = s;
    if (coop) {
      // 16-byte pieces: G lanes per row copy pieces 0..G-1 of 32 / G rows per instruction (the row
      // index comes from the lane that computed it); each lane copies the pieces G..DT/8-1 of its own
      // row; invalid rows are zero-filled (source size 0)
      constexpr int PPR = DT / 8;
      constexpr int G = PPR >= 16 ? 16 : (PPR >= 8 ? 8 : (PPR >= 4 ? 4 : (PPR >= 2 ? 2 : 1)));
      constexpr int RPI = 32 / G;
      const int32_t myrow = int32_t(rows[0]);
      const unsigned char* tbl = static_cast<const unsigned char*>(p.ts.tab[0]) + (lane % G) * 16;
      const uint32_t dst_l = smem_addr(stage_base + s * SB) + uint32_t((lane / G) * ROWB + (lane % G) * 16);
#pragma unroll
      for (int i = 0; i < C / RPI; ++i) {
        const int32_t rq = __shfl_sync(0xffffffffu, myrow, i * RPI + lane / G);
        cp_async16(dst_l + uint32_t(i * RPI * ROWB), tbl + uint64_t(uint32_t(rq < 0 ? 0 : rq)) * ROWB,
                   rq < 0 ? 0u : 16u);
      }
      const uint32_t dst_own = smem_addr(row_smem);
      const unsigned char* src_own = static_cast<const unsigned char*>(p.ts.tab[0]) +
                                     uint64_t(uint32_t(myrow < 0 ? 0 : myrow)) * ROWB;
#pragma unroll
      for (int pc = G; pc < PPR; ++pc) cp_async16(dst_own + pc * 16, src_own + pc * 16, myrow < 0 ? 0u : 16u);
      cp_async_mbar_arrive(&bars[s]);
    }
    const bool first = pend_chunk == 0 && lane == 0;
    if (first) {
      reinterpret_cast<float*>(stage_base + s * SB + Cfg::QS_OFF)[0] = pend_qs;
      bytes += qa_bytes;
    }
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&bars[s], bytes);
    if (first)
      bulk_g2s(stage_base + s * SB + Cfg::QA_OFF,
               static_cast<const unsigned char*>(p.qa) + pend_item * int64_t(qa_bytes), qa_bytes, &bars[s]);
#pragma unroll
    for (int o = 0; o < LNG_MAX_ORDERS; ++o) {
      if (o >= p.ts.n_orders) break;
      if (rows[o] >= 0 && bulk_lane) {
        const unsigned char* src = static_cast<const unsigned char*>(p.ts.tab[o]) + rows[o] * int64_t(mem_dim) * 2;
        bulk_g2s(row_smem + o * mem_dim * 2, src, uint32_t(mem_dim * 2), &bars[s]);
      }
    }
  };

  for (int j = 0; j < STAGES - 1 && j < jobs; ++j) {
    prefetch();
    issue(j % STAGES);
  }
  if (STAGES - 1 < jobs) prefetch();

  uint32_t qa_frag[KT][4];
  float uacc[NTU][4];
  float m_r[2], l_r[2];  // running offset (log2 units) and per-thread partial sums
  bool running_max = false;
  float qsl = 1.f;  // query scale x log2(e)
  const int g = lane >> 2, t4 = lane & 3;
  T* tag = nullptr;
  int64_t item = gwarp - nwarps;  // consume cursor
  int chunk = nch - 1;
  int s = STAGES - 1;
  uint32_t phase = 1;
  constexpr float LOG2E = 1.4426950408889634f;
  const float sink2 = p.sink * LOG2E;

  for (int j = 0; j < jobs; ++j) {
    if (j + STAGES - 1 < jobs) {
      issue((j + STAGES - 1) % STAGES);
      if (j + STAGES < jobs) prefetch();
    } else {
      flush_ss();
    }
    if (++s == STAGES) {
      s = 0;
      phase ^= 1u;
    }
    if (++chunk == nch) {
      chunk = 0;
      item += nwarps;
    }
    const bool landed = mbar_wait_bounded(&bars[s], phase, &g_error_word, DEV_ERR_WAIT_TIMEOUT);
    if (!__all_sync(0xffffffffu, landed)) return;
    const unsigned char* st = stage_base + s * SB;
    const uint32_t st_addr = smem_addr(st);
    if (chunk == 0) {
      // new item: its folded query as A fragments (rows = heads, k = token dims) from the stage,
      // rows >= qh and k >= DT zeroed
      const uint32_t qa_addr = st_addr + Cfg::QA_OFF + ((lane & 7) + ((lane >> 3) & 1) * 8) * ROWB;
#pragma unroll
      for (int kt = 0; kt < KT; ++kt) {
        if (kt == KT - 1 && (DT % 16) != 0) {
          ldsm_x2(qa_addr + kt * 32, qa_frag[kt][0], qa_frag[kt][1]);
          qa_frag[kt][2] = qa_frag[kt][3] = 0u;
        } else {
          ldsm_x4(qa_addr + kt * 32 + (lane >> 4) * 16, qa_frag[kt][0], qa_frag[kt][1], qa_frag[kt][2],
                  qa_frag[kt][3]);
        }
      }
      if (p.qh < 16) {
#pragma unroll
        for (int kt = 0; kt < KT; ++kt) {
          if (g >= p.qh) qa_frag[kt][0] = qa_frag[kt][2] = 0u;
          if (g + 8 >= p.qh) qa_frag[kt][1] = qa_frag[kt][3] = 0u;
        }
      }
      qsl = reinterpret_cast<const float*>(st + Cfg::QS_OFF)[0] * LOG2E;
#pragma unroll
      for (int nt = 0; nt < NTU; ++nt) uacc[nt][0] = uacc[nt][1] = uacc[nt][2] = uacc[nt][3] = 0.f;
      // every mode starts from the offset b0 (shards without the sink too, so that all shards'
      // states share one scale and combine without rescaling unless a score exceeded b0 + BIG)
      m_r[0] = m_r[1] = sink2;
      l_r[0] = l_r[1] = 0.f;  // the sink's 1 is added at the end
      running_max = false;
    }

    // inverse RMS of this lane's route token (row = lane)
    float rxl;
    if (have_ss) {
      rxl = rsqrtf(reinterpret_cast<const float*>(st + Cfg::SS_OFF)[lane] / float(DT) + p.eps);
    } else {
      const uint4* rowv = reinterpret_cast<const uint4*>(st + lane * ROWB);
      float ss = 0.f;
#pragma unroll
      for (int v = 0; v < DT / 8; ++v) {
        const uint4 w = rowv[v];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float lo, hi;
          if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            lo = __uint_as_float(ws[h] << 16);
            hi = __uint_as_float(ws[h] & 0xffff0000u);
          } else {
            __half2 h2 = *reinterpret_cast<const __half2*>(&ws[h]);
            float2 f = __half22float2(h2);
            lo = f.x;
            hi = f.y;
          }
          ss = fmaf(lo, lo, ss);
          ss = fmaf(hi, hi, ss);
        }
      }
      rxl = rsqrtf(ss / float(DT) + p.eps);
    }

    // scores S[16 heads x 32 routes] = qa . tok^T
    float sacc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
#pragma unroll
    for (int kt = 0; kt + 1 < KT; kt += 2) {
      // B fragments of two k16 steps for all four route tiles first, then the products one k-step at
      // a time across the tiles (four independent accumulators between dependent products)
      uint32_t bf[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
        ldsm_x4(st_addr + (nt * 8 + (lane & 7)) * ROWB + (kt * 16 + (lane >> 3) * 8) * 2, bf[nt][0], bf[nt][1],
                bf[nt][2], bf[nt][3]);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) mma16816<T>(sacc[nt], qa_frag[kt], bf[nt][0], bf[nt][1]);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) mma16816<T>(sacc[nt], qa_frag[kt + 1], bf[nt][2], bf[nt][3]);
    }
    if (KT & 1) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int rrow = nt * 8 + (lane & 7);
        const int kcol = (KT - 1) * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1;
        ldsm_x2(st_addr + rrow * ROWB + kcol * 2, b0, b1);
        mma16816<T>(sacc[nt], qa_frag[KT - 1], b0, b1);
      }
    }

    // softmax update in log2 units with the sink seed; rxv = this thread's 8 route columns' 1/rms.
    // The exponent offset stays the sink logit b0 (m_r's seed) while no score of the item has
    // exceeded b0 + BIG: p = 2^(s - b0) is then finite in the 16-bit P operand and the fp32 sums and
    // the normalised result is the same, with no per-chunk maximum or rescaling.  From the first
    // chunk with a larger score (a warp vote), the offset is the running maximum with online
    // rescaling.
    constexpr float BIG = std::is_same<T, __nv_bfloat16>::value ? 64.f : 4.f;  // f16 P: exp(BIG) * rx < 65504
    const float big2 = sink2 + BIG * LOG2E;
    const int64_t rbase = LNG_RLO + int64_t(chunk) * C;
    float rxv[4][2];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int b = 0; b < 2; ++b) rxv[nt][b] = __shfl_sync(0xffffffffu, rxl, nt * 8 + t4 * 2 + b);
    float sv[4][4];
    bool big = false;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const float c = qsl * rxv[nt][b];
        sv[nt][b] = sacc[nt][b] * c;
        sv[nt][b + 2] = sacc[nt][b + 2] * c;
      }
    }
    if (rbase + C > LNG_RHI) {  // the item's last chunk is ragged: routes past the end take no part
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int h = 0; h < 4; ++h)
          if (rbase + nt * 8 + t4 * 2 + (h & 1) >= LNG_RHI) sv[nt][h] = -INFINITY;
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int h = 0; h < 4; ++h) big = big || sv[nt][h] > big2;
    running_max = running_max || __any_sync(0xffffffffu, big);
    float alpha[2] = {1.f, 1.f};
    if (running_max) {
      float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int h = 0; h < 4; ++h) mx[h >> 1] = fmaxf(mx[h >> 1], sv[nt][h]);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        alpha[i] = ex2_approx(m_r[i] - mx[i]);
        m_r[i] = mx[i];
        l_r[i] *= alpha[i];
      }
    }
    uint32_t pa[2][4];  // P' as A fragments of the two k16 steps
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      float e[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float ex = ex2_approx(sv[nt][h] - m_r[h >> 1]);
        l_r[h >> 1] += ex;
        e[h] = ex * rxv[nt][h & 1];
      }
      pa[nt >> 1][(nt & 1) * 2 + 0] = pack2(e[0], e[1], tag);
      pa[nt >> 1][(nt & 1) * 2 + 1] = pack2(e[2], e[3], tag);
    }
    if (running_max) {
#pragma unroll
      for (int nt = 0; nt < NTU; ++nt) {
        uacc[nt][0] *= alpha[0];
        uacc[nt][1] *= alpha[0];
        uacc[nt][2] *= alpha[1];
        uacc[nt][3] *= alpha[1];
      }
    }
    // u += P' . tok   (B = tok rows as [k = route][n = dim], loaded transposed)
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      const int rrow = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int nt = 0; nt + 1 < NTU; nt += 2) {
        const int dcol = (nt + (lane >> 4)) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(st_addr + rrow * ROWB + dcol * 2, b0, b1, b2, b3);
        mma16816<T>(uacc[nt], pa[ks], b0, b1);
        mma16816<T>(uacc[nt + 1], pa[ks], b2, b3);
      }
      if (NTU & 1) {
        uint32_t b0, b1;
        ldsm_x2_t(st_addr + rrow * ROWB + (NTU - 1) * 8 * 2, b0, b1);
        mma16816<T>(uacc[NTU - 1], pa[ks], b0, b1);
      }
    }
    __syncwarp();

    if (chunk == nch - 1) {
      constexpr float LN2 = 0.6931471805599453f;
      float l[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        l[i] = l_r[i];
        l[i] += __shfl_xor_sync(0xffffffffu, l[i], 1);
        l[i] += __shfl_xor_sync(0xffffffffu, l[i], 2);
        if (sink_in) l[i] += ex2_approx(sink2 - m_r[i]);  // the sink's seed 1, rescaled to the final offset
      }
      const int64_t obase = item * int64_t(p.qh) * DT;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int row = g + i * 8;
        if (row >= p.qh) continue;
        if (p.partial >= 3) {
          // packed state (u, l) in bf16 [M, QH, DT + 1], ready for a SUM reduction across shards
          __nv_bfloat16* po = static_cast<__nv_bfloat16*>(p.u) + (item * int64_t(p.qh) + row) * (DT + 1);
#pragma unroll
          for (int nt = 0; nt < NTU; ++nt) {
            po[nt * 8 + t4 * 2] = __float2bfloat16_rn(uacc[nt][i * 2]);
            po[nt * 8 + t4 * 2 + 1] = __float2bfloat16_rn(uacc[nt][i * 2 + 1]);
          }
          if (t4 == 0) {
            po[DT] = __float2bfloat16_rn(l[i]);
            p.m_out[item * p.qh + row] = m_r[i] * LN2;
          }
        } else if (p.partial) {
          const int64_t ys = SPLIT ? int64_t(blockIdx.y) * p.M * p.qh : 0;  // state y of a route split
          float* uo = static_cast<float*>(p.u) + ys * DT + obase + row * DT;
#pragma unroll
          for (int nt = 0; nt < NTU; ++nt) {
            *reinterpret_cast<float2*>(uo + nt * 8 + t4 * 2) = make_float2(uacc[nt][i * 2], uacc[nt][i * 2 + 1]);
          }
          if (t4 == 0) {
            p.m_out[ys + item * p.qh + row] = m_r[i] * LN2;
            p.l_out[ys + item * p.qh + row] = l[i];
          }
        } else {
          const float inv = 1.f / fmaxf(l[i], 1.17549435e-38f);
          T* uo = static_cast<T*>(p.u) + obase + row * DT;
#pragma unroll
          for (int nt = 0; nt < NTU; ++nt) {
            *reinterpret_cast<uint32_t*>(uo + nt * 8 + t4 * 2) =
                pack2(uacc[nt][i * 2] * inv, uacc[nt][i * 2 + 1] * inv, tag);
          }
        }
      }
    }
  }
}
#undef LNG_RLO
#undef LNG_RHI

// The states of a route split (attend_mma_kernel with route_split, partial mode 1: u unnormalised,
// m the offset, l the weight sum with the sink in state 0) -> the normalised readout, as the unsplit
// kernel's mode 0 writes it: u = sum_y e^(m_y - m) u_y / sum_y e^(m_y - m) l_y, m = max_y m_y.
// One thread per (item, head, 4 dims); y in order, so the result does not depend on the schedule.
template <typename T>
__global__ void attend_split_combine_kernel(const float* __restrict__ u, const float* __restrict__ m,
                                            const float* __restrict__ l, int splits, int64_t M, int qh, int Dt,
                                            T* __restrict__ out) {
  const int64_t rows = M * qh;
  const int q4 = Dt / 4;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < rows * q4; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / q4;
    const int j = int(e - r * q4) * 4;
    float mx = -INFINITY;
    for (int y = 0; y < splits; ++y) mx = fmaxf(mx, m[y * rows + r]);
    float lsum = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int y = 0; y < splits; ++y) {
      const float ly = l[y * rows + r];
      if (ly == 0.f) continue;  // no valid route and no sink in this slice
      const float w = __expf(m[y * rows + r] - mx);
      const float4 v = *reinterpret_cast<const float4*>(u + (y * rows + r) * Dt + j);
      lsum = fmaf(w, ly, lsum);
      a0 = fmaf(w, v.x, a0);
      a1 = fmaf(w, v.y, a1);
      a2 = fmaf(w, v.z, a2);
      a3 = fmaf(w, v.w, a3);
    }
    const float inv = 1.f / fmaxf(lsum, 1.17549435e-38f);
    T* o = out + r * Dt + j;
    o[0] = from_f32<T>(a0 * inv);
    o[1] = from_f32<T>(a1 * inv);
    o[2] = from_f32<T>(a2 * inv);
    o[3] = from_f32<T>(a3 * inv);
  }
}

}  // namespace lng
