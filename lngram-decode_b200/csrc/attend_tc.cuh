// Fused n-gram gather + sink attention on the tcgen05 tensor cores, for 136-dim route tokens
// (bf16 / f16 tables), up to 192 routes and 16 heads per position (the SB / SD-B / scaled layers).
//
// Per position (item): tok [R, 136] = the gathered table rows, S^T [R, heads] = tok . qa^T,
// P = softmax over routes with the sink, u^T [136, heads] = tok^T . (P * rx)^T -- ffnmem/memory/
// lngram_v2.py:1944-2070 in the folded form (scores scaled by 1/rms(h) and 1/rms(token)).  Routes
// are the M dimension of the first MMA and the K dimension of the second, so both products run on
// the tensor cores with fp32 accumulators in TMEM, and the only per-route CUDA-core work left is
// the softmax (one thread per route).
//
// Persistent CTAs (one per SM), 17 warps, items (positions) in order, three item buffers in flight:
//   warps 8-15 producers, every item: window codes -> table rows ->
//              16-byte cp.async copies straight into the tensor-core operand layout (128-byte
//              swizzle for dims 0-127, 32-byte swizzle for dims 128-143), 16 lanes per row so a
//              warp instruction moves two whole 256-byte row prefixes; rows of invalid windows are
//              zero-filled; plus TMA loads of the item's folded query.  (Per-row TMA copies were
//              measured slower here: the TMA engine spends tens of cycles per small row.)
//   warp 16    TMEM allocation and the single MMA-issuing thread;
//   warps 0-7  two softmax / epilogue groups of four warps, alternating items (TMEM lane = route
//              for the softmax, token dim for the epilogue; each group owns half of TMEM).
// Every wait is a bounded mbarrier wait that records DEV_ERR_WAIT_TIMEOUT; after one expires, the
// remaining waits of the CTA return at once and the kernel runs out its loops.
#pragma once

#include "attend.cuh"
#include "gemm_tc.cuh"

namespace lng {

namespace atc {
constexpr int RP = 192;                          // routes per item, padded
constexpr int DT = 136;                          // token dims (one order of 136)
constexpr int QN = 16;                           // heads = MMA N
constexpr int NBUF = 3;                          // item buffers
constexpr uint32_t A_ATOM = RP * 128;            // tok dims 0-63 / 64-127: RP rows x 128 B, SW128
constexpr uint32_t T_OFF = 2 * A_ATOM;           // tok dims 128-143: RP rows x 32 B, SW32
constexpr uint32_t Q_OFF = T_OFF + RP * 32;      // query: 2 x (16 x 128 B) SW128 + 16 x 32 B SW32
constexpr uint32_t QT_OFF = Q_OFF + 2 * QN * 128;
constexpr uint32_t ROWS_OFF = QT_OFF + QN * 32;  // table row of every route [RP] i32 (-1: zero token)
constexpr uint32_t BUF = ((ROWS_OFF + RP * 4) + 1023) / 1024 * 1024;
constexpr uint32_t P_OFF = NBUF * BUF;           // (P * rx)^T per softmax group: RP routes x 16 heads, MN-major SW32
constexpr uint32_t P_BYTES = RP * 32;
constexpr uint32_t RED_OFF = P_OFF + 2 * P_BYTES;     // [group][16 heads][4 warps] maxima, [2][16] offsets (f32)
constexpr uint32_t INV_OFF = RED_OFF + 2 * 2 * 4 * QN * 4;  // [group][2 slots][16] f32: 1 / softmax denominator
constexpr uint32_t BAR_OFF = INV_OFF + 2 * 2 * QN * 4;
constexpr int NBARS = 3 * NBUF + 6 * 2;
constexpr uint32_t ABORT_OFF = BAR_OFF + NBARS * 8 + 8;  // u32: a bounded wait expired somewhere
constexpr uint32_t SMEM = ABORT_OFF + 8;
constexpr size_t SMEM_LAUNCH = SMEM + 1024;       // + alignment slack
constexpr int THREADS = 544;                      // 8 softmax/epilogue warps, 8 producer warps, 1 MMA warp
constexpr uint32_t TMEM_COLS = 128;               // per group: S tile0, S tile1, U dims 0-127, U dims 128+
static_assert(BUF % 1024 == 0 && Q_OFF % 1024 == 0 && T_OFF % 1024 == 0, "swizzle atom alignment");
static_assert(QT_OFF % 256 == 0 && P_OFF % 1024 == 0 && P_BYTES % 256 == 0, "32-byte swizzle atom alignment");
static_assert(SMEM_LAUNCH <= 227 * 1024, "shared memory per CTA");
}  // namespace atc

__device__ __forceinline__ void tma_load_2d_s(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void group_bar(int g) { asm volatile("bar.sync %0, 128;" ::"r"(1 + g) : "memory"); }
// Group barrier that also returns whether any of the group's threads passed pred = true.
__device__ __forceinline__ bool group_bar_or(int g, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred q, r;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred r, %2, 128, q;\n\tselp.u32 %0, 1, 0, r;\n\t}"
      : "=r"(out)
      : "r"(uint32_t(pred)), "r"(1 + g)
      : "memory");
  return out != 0;
}

// tcgen05.ld of 16 columns of this warp's 32 TMEM lanes without waiting, and the wait that makes
// the registers valid: it names them as operands, so no use can be scheduled above it.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// Shared-memory matrix descriptors (tcgen05): start, leading / stride byte offsets (16-byte units),
// version 1, layout type (2 = 128-byte swizzle, 6 = 32-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(layout) << 61);
}
// kind::f16 instruction descriptor with fp32 accumulation; a_mn / b_mn: operand is MN-major.
template <typename T>
__host__ __device__ constexpr uint32_t umma_idesc16(int M, int N, bool a_mn, bool b_mn) {
  constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// 16 values across a warp: on return lane L holds the reduction of value (L >> 1) & 15 over all 32
// lanes (a reduce-scatter butterfly: 16 shuffles instead of 16 x 5).
template <bool MAX>
__device__ __forceinline__ float warp_reduce16(float (&v)[16], int lane) {
  float a[8];
  const bool u4 = lane & 16;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float keep = u4 ? v[8 + j] : v[j], send = u4 ? v[j] : v[8 + j];
    const float o = __shfl_xor_sync(0xffffffffu, send, 16);
    a[j] = MAX ? fmaxf(keep, o) : keep + o;
  }
  float b[4];
  const bool u3 = lane & 8;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float keep = u3 ? a[4 + j] : a[j], send = u3 ? a[j] : a[4 + j];
    const float o = __shfl_xor_sync(0xffffffffu, send, 8);
    b[j] = MAX ? fmaxf(keep, o) : keep + o;
  }
  float c[2];
  const bool u2 = lane & 4;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float keep = u2 ? b[2 + j] : b[j], send = u2 ? b[j] : b[2 + j];
    const float o = __shfl_xor_sync(0xffffffffu, send, 4);
    c[j] = MAX ? fmaxf(keep, o) : keep + o;
  }
  const bool u1 = lane & 2;
  const float keep = u1 ? c[1] : c[0], send = u1 ? c[0] : c[1];
  const float o = __shfl_xor_sync(0xffffffffu, send, 2);
  float d = MAX ? fmaxf(keep, o) : keep + o;
  const float o2 = __shfl_xor_sync(0xffffffffu, d, 1);
  return MAX ? fmaxf(d, o2) : d + o2;
}

template <typename CodeT, typename T>
__global__ void __launch_bounds__(atc::THREADS, 1)
    attend_tc_kernel(const __grid_constant__ CUtensorMap tm_tab, const __grid_constant__ CUtensorMap tm_tab_tail,
                     const __grid_constant__ CUtensorMap tm_qa, const __grid_constant__ CUtensorMap tm_qa_tail,
                     AttendParams p) {
  using namespace atc;
  extern __shared__ uint8_t atc_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(atc_smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BAR_OFF);
  uint64_t* tok_full = bars;                 // [NBUF] gathered rows (cp.async) + query (TMA) landed
  uint64_t* rows_full = bars + NBUF;         // [NBUF] the item's row indices are in shared memory
  uint64_t* tok_empty = bars + 2 * NBUF;     // [NBUF] MMA done with the buffer (commit)
  uint64_t* s_full = bars + 3 * NBUF;        // [group] scores in TMEM (commit)
  uint64_t* s_free = s_full + 2;             // [group] softmax read the scores (128 arrivals)
  uint64_t* p_full = s_full + 4;             // [group] P written (128 arrivals)
  uint64_t* p_free = s_full + 6;             // [group] second MMA done with P (commit)
  uint64_t* u_full = s_full + 8;             // [group] u in TMEM (commit)
  uint64_t* u_free = s_full + 10;            // [group] epilogue read u (128 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(sm + ABORT_OFF);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Bounded wait; once any wait of the CTA has expired, every later wait returns at once, so all
  // roles run out their loops quickly (and each softmax group keeps its named barriers matched).
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait_bounded(bar, parity, &g_error_word, DEV_ERR_WAIT_TIMEOUT)) return true;
    *abort_flag = 1u;
    return false;
  };

  // zero every buffer once: padding dims, padding heads and padding routes stay zero for good
  for (uint32_t e = tid * 16; e < BAR_OFF; e += THREADS * 16) *reinterpret_cast<uint4*>(sm + e) = make_uint4(0, 0, 0, 0);
  if (tid == 0) {
    *abort_flag = 0u;
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(&tok_full[i], 256 + 1);  // the producers' cp.async completions + the query TMA
      mbar_init(&rows_full[i], 1);
      mbar_init(&tok_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_free[i], 1);
      mbar_init(&u_full[i], 1);
      mbar_init(&u_free[i], 128);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_tab);
    tma_prefetch_desc(&tm_tab_tail);
    tma_prefetch_desc(&tm_qa);
    tma_prefetch_desc(&tm_qa_tail);
  }
  if (warp == 16) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int64_t G = gridDim.x;
  const int64_t first = blockIdx.x;
  const int n_my = first < p.M ? int((p.M - 1 - first) / G + 1) : 0;
  const int R = int(p.route_end - p.route_start);
  const int QH = p.qh;
  const uint32_t qa_tx = 2 * QN * 128 + QN * 32;

  if (warp >= 8 && warp < 16) {
    // ------------------------------------------------------------------ producers: warps 8-15, every item
    const int pt = tid - 256, pwp = warp - 8;  // producer thread 0..255, producer warp 0..7
    int32_t pend_c[MAXW];                      // window codes of route pt, prefetched one item ahead
    ItemGeo geo{};
    auto load_codes = [&](int k) {
      geo = item_geometry(p.src, p.ts.order, p.ts.n_orders, first + int64_t(k) * G);
      load_window_codes<CodeT>(p.src, geo, p.route_start + pt, pt < R, pend_c);
    };
    const unsigned char* tab = static_cast<const unsigned char*>(p.ts.tab[0]);
    if (n_my > 0) load_codes(0);
    for (int k = 0; k < n_my; ++k) {
      const int b = k % NBUF;
      const int64_t item = first + int64_t(k) * G;
      const int32_t row =
          pt < R ? int32_t(window_row(pend_c, p.ts.order[0], p.ts.bits, p.route_start + pt, (geo.omask & 1u) != 0)) : -1;
      if (k + 1 < n_my) load_codes(k + 1);
      if (k >= NBUF) wait(&tok_empty[b], uint32_t(((k / NBUF) - 1) & 1));
      int32_t* rs = reinterpret_cast<int32_t*>(sm + b * BUF + ROWS_OFF);
      if (pt < RP) rs[pt] = row;
      asm volatile("bar.sync 3, 256;" ::: "memory");  // every route's row is in shared memory
      const uint32_t bb = sbase + uint32_t(b) * BUF;
      if (pt == 0) {
        mbar_arrive(&rows_full[b]);
        mbar_arrive_expect_tx(&tok_full[b], qa_tx);
        const int32_t qy = int32_t(item * QH);  // 16 query rows from here (rows past QH are ignored)
        tma_load_2d_s(bb + Q_OFF, &tm_qa, 0, qy, &tok_full[b]);
        tma_load_2d_s(bb + Q_OFF + QN * 128, &tm_qa, 64, qy, &tok_full[b]);
        tma_load_2d_s(bb + QT_OFF, &tm_qa_tail, 128, qy, &tok_full[b]);
      }
      // dims 0-127: lanes 0-15 copy route 2i, lanes 16-31 route 2i+1, lane = 16-byte chunk
      const int c = lane & 15;
      const uint32_t coff = c < 8 ? 0u : A_ATOM;
      const int cc = c & 7;
      for (int i = pwp; 2 * i < R; i += 8) {
        const int r = 2 * i + (lane >> 4);
        if (r < R) {
          const int32_t rw = rs[r];
          cp_async16(bb + coff + uint32_t(r) * 128u + (uint32_t(cc ^ (r & 7)) << 4),
                     tab + (rw >= 0 ? int64_t(rw) * (DT * 2) + c * 16 : 0), rw >= 0 ? 16u : 0u);
        }
      }
      // dims 128-135: one 16-byte chunk per route (dim 136 carries 1/rms, written by the softmax)
      if (pt < R)
        cp_async16(bb + T_OFF + uint32_t(pt) * 32u + (uint32_t((pt >> 2) & 1) << 4),
                   tab + (row >= 0 ? int64_t(row) * (DT * 2) + 256 : 0), row >= 0 ? 16u : 0u);
      cp_async_mbar_arrive_noinc(&tok_full[b]);
    }
    cp_async_wait_all();
  } else if (warp == 16) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = umma_idesc16<T>(128, QN, false, false);  // S^T = tok . qa^T
      constexpr uint32_t id_u = umma_idesc16<T>(128, QN, true, true);    // u^T = tok^T . P^T, both MN-major
      const int tiles = R > 128 ? 2 : 1;
      const int ksteps = (R + 15) / 16;
      bool ok = true;
      auto mma1 = [&](int k) {
        const int b = k % NBUF, ts = k & 1;
        ok = wait(&tok_full[b], uint32_t((k / NBUF) & 1));
        if (ok && k >= 2) ok = wait(&s_free[ts], uint32_t(((k >> 1) - 1) & 1));
        if (!ok) return;
        fence_proxy_async_smem();  // the producers' cp.async data -> visible to the tensor cores
        tc_fence_after();
        const uint32_t bb = sbase + uint32_t(b) * BUF;
        for (int t = 0; t < tiles; ++t) {
          const uint32_t d = tmem + uint32_t(ts * 64 + t * 16);
          uint32_t acc = 0;
#pragma unroll
          for (int a = 0; a < 2; ++a) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t da = umma_desc(bb + a * A_ATOM + t * 128 * 128 + kk * 32, 16, 1024, 2);
              const uint64_t db = umma_desc(bb + Q_OFF + a * QN * 128 + kk * 32, 16, 1024, 2);
              umma_bf16(d, da, db, id_s, acc);
              acc = 1;
            }
          }
          const uint64_t da = umma_desc(bb + T_OFF + t * 128 * 32, 16, 256, 6);
          const uint64_t db = umma_desc(bb + QT_OFF, 16, 256, 6);
          umma_bf16(d, da, db, id_s, 1u);
        }
        umma_commit(&s_full[ts]);
      };
      auto mma2 = [&](int k) {
        const int b = k % NBUF, ts = k & 1;
        ok = wait(&p_full[ts], uint32_t((k >> 1) & 1));
        if (ok && k >= 2) ok = wait(&u_free[ts], uint32_t(((k >> 1) - 1) & 1));
        if (!ok) return;
        tc_fence_after();
        const uint32_t bb = sbase + uint32_t(b) * BUF;
        const uint32_t pp = sbase + P_OFF + uint32_t(ts) * P_BYTES;
        for (int ks = 0; ks < ksteps; ++ks) {
          // B: 16 routes x 16 heads of (P * rx)^T, heads contiguous (MN-major, 32-byte swizzle)
          const uint64_t db = umma_desc(pp + ks * 512, 0, 256, 6);
          const uint32_t acc = ks ? 1u : 0u;
          // dims 0-127: the two 128-byte-swizzled atoms, A_ATOM apart along M
          umma_bf16(tmem + uint32_t(ts * 64 + 32), umma_desc(bb + ks * 2048, A_ATOM, 1024, 2), db, id_u, acc);
          // dims 128-255: the 32-byte-swizzled tail (dims 128-143) repeated along M (LBO = 0)
          umma_bf16(tmem + uint32_t(ts * 64 + 48), umma_desc(bb + T_OFF + ks * 512, 0, 256, 6), db, id_u, acc);
        }
        umma_commit(&u_full[ts]);
        umma_commit(&tok_empty[b]);
        umma_commit(&p_free[ts]);
      };
      if (n_my > 0) mma1(0);
      for (int k = 0; k < n_my && ok; ++k) {
        if (k + 1 < n_my) mma1(k + 1);
        if (!ok) break;
        mma2(k);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue: group g = warps 4g..4g+3,
    // items k = g mod 2; TMEM lane = route (softmax) or token dim (epilogue)
    //
    // The exponentials are offset by the sink logit b0 instead of the running maximum whenever no
    // score of the item exceeds b0 + BIG (one barrier-OR vote): p = exp(s - b0) then stays finite in
    // the 16-bit P operand and the fp32 accumulators, and p / (sum p + 1) is the same softmax.  Items
    // with a larger score take the exact maximum.  The sums over routes come out of the second MMA:
    // token dim 136 (zero padding, ignored by the first MMA's zero query column) carries 1 / rms of
    // each route, so u^T[136, h] = sum_r (p_rh * rx_r) / rx_r.
    constexpr float BIG = std::is_same<T, __nv_bfloat16>::value ? 64.f : 4.f;  // f16 P: p * rx < 65504
    const int g = warp >> 2, gw = warp & 3, gt = tid & 127;
    float* red = reinterpret_cast<float*>(sm + RED_OFF) + g * 2 * 4 * QN;  // [16][4] partial maxima (exact path)
    float* msm = red + 4 * QN;                                            // [slot][16] the item's exponent offset
    float* inv = reinterpret_cast<float*>(sm + INV_OFF) + g * 2 * QN;     // [slot][16] 1 / softmax denominator
    const uint32_t tl = tmem + (uint32_t(gw * 32) << 16) + uint32_t(g * 64);
    const int ra = gt, rb = 128 + gt;
    const bool va = ra < R, vb = rb < R;
    const float* ss0 = p.ts.ss[0];
    const float b0 = p.sink;
    uint32_t ua[16], ub[16];
    // epilogue, part 1: u of dims gt and 128 + gt; the lane of dim 136 turns the sums into 1 / l
    auto epi_load = [&](int k) {
      wait(&u_full[g], uint32_t((k >> 1) & 1));
      __syncwarp();
      tc_fence_after();
      tmem_ld16_issue(tl + 32u, ua);
      tmem_ld16_issue(tl + 48u, ub);
      tmem_ld_wait(ua);
      tmem_ld_wait(ub);
      tc_fence_before();
      mbar_arrive(&u_free[g]);
      if (gt == DT - 128) {
        const int sl = (k >> 1) & 1;
#pragma unroll
        for (int h = 0; h < QN; ++h)
          inv[sl * QN + h] = 1.f / fmaxf(__uint_as_float(ub[h]) + __expf(b0 - msm[sl * QN + h]), 1.17549435e-38f);
      }
    };
    // epilogue, part 2 (after a group barrier): u / l
    auto epi_store = [&](int k) {
      const int64_t item = first + int64_t(k) * G;
      T* out = static_cast<T*>(p.u) + item * int64_t(QH) * DT;
      const float* iv = inv + ((k >> 1) & 1) * QN;
#pragma unroll
      for (int h = 0; h < QN; ++h) {
        if (h < QH) {
          const float f = iv[h];
          out[h * DT + gt] = from_f32<T>(__uint_as_float(ua[h]) * f);
          if (gt < DT - 128) out[h * DT + 128 + gt] = from_f32<T>(__uint_as_float(ub[h]) * f);
        }
      }
    };
    int last = -1;
    for (int k = g; k < n_my; k += 2) {
      const int b = k % NBUF, sl = (k >> 1) & 1;
      const int64_t item = first + int64_t(k) * G;
      const float qs = p.qscale ? p.qscale[item] : 1.f;
      // the rows' sums of squares are loaded as soon as the producers have chosen the rows
      wait(&rows_full[b], uint32_t((k / NBUF) & 1));
      const int32_t* rs = reinterpret_cast<const int32_t*>(sm + b * BUF + ROWS_OFF);
      const int32_t rowa = va ? rs[ra] : -1, rowb = vb ? rs[rb] : -1;
      float ssa = 0.f, ssb = 0.f;
      if (ss0) {
        if (rowa >= 0) ssa = __ldg(ss0 + rowa);
        if (rowb >= 0) ssb = __ldg(ss0 + rowb);
      }
      wait(&s_full[g], uint32_t((k >> 1) & 1));
      __syncwarp();
      tc_fence_after();
      uint32_t sa_u[16], sb_u[16];
      tmem_ld16_issue(tl, sa_u);
      tmem_ld16_issue(tl + 16u, sb_u);  // (tile 1 scores: unused when R <= 128)
      tmem_ld_wait(sa_u);
      tmem_ld_wait(sb_u);
      tc_fence_before();
      mbar_arrive(&s_free[g]);
      const float rxa = rsqrtf(ssa / float(DT) + p.eps), rxb = rsqrtf(ssb / float(DT) + p.eps);
      float sa[16], sb[16];
      bool big = false;
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        sa[h] = va ? __uint_as_float(sa_u[h]) * (qs * rxa) : -INFINITY;
        sb[h] = (vb && R > 128) ? __uint_as_float(sb_u[h]) * (qs * rxb) : -INFINITY;
        big = big || sa[h] > b0 + BIG || sb[h] > b0 + BIG;
      }
      float m[16];
      if (!group_bar_or(g, big)) {
#pragma unroll
        for (int h = 0; h < 16; ++h) m[h] = b0;
      } else {  // exact maximum over routes per head: warp butterfly, then the group's four warps
        float mx[16];
#pragma unroll
        for (int h = 0; h < 16; ++h) mx[h] = fmaxf(sa[h], sb[h]);
        const float w = warp_reduce16<true>(mx, lane);
        if ((lane & 1) == 0) red[(lane >> 1) * 4 + gw] = w;
        group_bar(g);
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const float4 v = reinterpret_cast<const float4*>(red)[h];
          m[h] = fmaxf(fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)), b0);
        }
      }
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        sa[h] = va ? __expf(sa[h] - m[h]) * rxa : 0.f;
        sb[h] = vb ? __expf(sb[h] - m[h]) * rxb : 0.f;
      }
      // (P * rx)^T: route r's 16 heads are 32 contiguous bytes (two 16-byte chunks, 32-byte swizzle)
      if (k >= 2) wait(&p_free[g], uint32_t(((k >> 1) - 1) & 1));
      __syncwarp();
      uint8_t* pw = sm + P_OFF + g * P_BYTES;
      uint8_t* tail = sm + b * BUF + T_OFF;
      {
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = pack2(sa[2 * i], sa[2 * i + 1], static_cast<T*>(nullptr));
        const int sw = (ra >> 2) & 1;
        *reinterpret_cast<uint4*>(pw + ra * 32 + (sw << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(pw + ra * 32 + ((sw ^ 1) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
        if (va) *reinterpret_cast<T*>(tail + ra * 32 + ((sw ^ 1) << 4)) = from_f32<T>(1.f / rxa);  // dim 136
      }
      if (rb < RP) {
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = pack2(sb[2 * i], sb[2 * i + 1], static_cast<T*>(nullptr));
        const int sw = (rb >> 2) & 1;
        *reinterpret_cast<uint4*>(pw + rb * 32 + (sw << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(pw + rb * 32 + ((sw ^ 1) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
        if (vb) *reinterpret_cast<T*>(tail + rb * 32 + ((sw ^ 1) << 4)) = from_f32<T>(1.f / rxb);
      }
      if (gt == 0) {
#pragma unroll
        for (int h = 0; h < 16; ++h) msm[sl * QN + h] = m[h];
      }
      fence_proxy_async_smem();
      mbar_arrive(&p_full[g]);
      if (last >= 0) epi_load(last);
      group_bar(g);  // 1 / l of the previous item visible; this item's shared reductions consumed
      if (last >= 0) epi_store(last);
      last = k;
    }
    if (last >= 0) {
      epi_load(last);
      group_bar(g);
      epi_store(last);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 16) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

}  // namespace lng

namespace lng {
// 2D tensor map over a row-major [rows, cols] 16-bit matrix (row stride ld elements), box
// box_cols x box_rows, the given swizzle; rows / columns past the end read as zeros.
inline int make_tmap_16(CUtensorMap* map, int dtype, const void* ptr, int64_t rows, int64_t cols, int64_t ld,
                        int box_cols, int box_rows, CUtensorMapSwizzle swizzle) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(LNG_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (driver entry point)");
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  const cuuint32_t box[2] = {uint32_t(box_cols), uint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype == LNG_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LNG_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return LNG_OK;
}
}  // namespace lng
