// lngram_b200: the C ABI of include/lngram_b200.h (one translation unit, so every kernel shares
// the device error word and inlines the addressing helpers).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "address.cuh"
#include "attend.cuh"
#include "gemm_simt.cuh"
#include "gemm_tc.cuh"
#include "logits_tc.cuh"
#include "lookup.cuh"
#include "router.cuh"
#include "rowops.cuh"
#include "topk.cuh"
#include "drafter_ext.cuh"
#include "surrogate.cuh"
#include "online.cuh"

static int scratch_alloc(void** p, size_t bytes, cudaStream_t stream);

namespace lng {

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }
int fail(int status, const std::string& msg) {
  t_last_error = msg;
  return status;
}
int cuda_status(cudaError_t e, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return LNG_ERR_CUDA;
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

static int grid_for(int64_t work, int threads, int per_sm = 8) {
  const int64_t want = ceil_div(std::max<int64_t>(work, 1), threads);
  return int(std::max<int64_t>(1, std::min<int64_t>(want, int64_t(num_sms()) * per_sm)));
}

static cudaStream_t S(lng_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

static int check_tables(const lng_tables* t) {
  LNG_REQUIRE(t != nullptr, "tables descriptor is NULL");
  LNG_REQUIRE(t->n_orders >= 1 && t->n_orders <= LNG_MAX_ORDERS, "n_orders must be in [1, 4]");
  LNG_REQUIRE(t->bits >= 1 && t->bits <= 16, "bits_per_route must be in [1, 16]");
  LNG_REQUIRE(t->num_routes >= 1 && t->memory_dim >= 1, "num_routes and memory_dim must be positive");
  LNG_REQUIRE(t->table_dtype == LNG_F32 || t->table_dtype == LNG_BF16 || t->table_dtype == LNG_F16,
              "table dtype must be f32, bf16 or f16");
  for (int o = 0; o < t->n_orders; ++o) {
    LNG_REQUIRE(t->tables[o] != nullptr, "table pointer is NULL");
    LNG_REQUIRE(t->orders[o] >= 1 && int64_t(t->bits) * t->orders[o] <= 40, "order * bits must be in [1, 40]");
    if (o) LNG_REQUIRE(t->orders[o] > t->orders[o - 1], "orders must be ascending and distinct");
  }
  return LNG_OK;
}

static TableSet table_set(const lng_tables* t) {
  TableSet ts{};
  bool all_ss = true;
  for (int o = 0; o < t->n_orders; ++o) all_ss = all_ss && t->row_ss[o] != nullptr;
  for (int o = 0; o < t->n_orders; ++o) {
    ts.tab[o] = t->tables[o];
    ts.order[o] = t->orders[o];
    ts.ss[o] = all_ss ? t->row_ss[o] : nullptr;
  }
  ts.n_orders = t->n_orders;
  ts.bits = t->bits;
  ts.num_routes = t->num_routes;
  ts.mem_dim = t->memory_dim;
  return ts;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace lng

using namespace lng;

// ====================================================================== basics
extern "C" int lng_abi_version(void) { return 1; }
extern "C" const char* lng_last_error(void) { return t_last_error.c_str(); }

extern "C" int lng_device_ok(void) {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
  return major == 10 ? 1 : 0;
}

extern "C" int lng_device_error(int clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_error_word, sizeof(v)) != cudaSuccess) return -1;
  if (clear && v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_error_word, &z, sizeof(z));
  }
  return int(v);
}

// ====================================================================== router
extern "C" int lng_quantize_route_logits(const float* logits, int64_t n, int64_t routes, int32_t bits, void* codes,
                                         int32_t codes_dtype, lng_stream_t stream) {
  LNG_REQUIRE(n >= 0 && routes > 0, "bad shape");
  LNG_REQUIRE(bits >= 1 && bits <= 30, "bits_per_route must be in [1, 30]");
  LNG_REQUIRE(codes_dtype == LNG_I32 || (codes_dtype == LNG_U8 && bits <= 8), "codes dtype must be i32 or u8 (bits <= 8)");
  if (n == 0) return LNG_OK;
  LNG_REQUIRE(logits && codes, "NULL pointer");
  const int g = grid_for(n * routes, 256);
  if (codes_dtype == LNG_U8)
    quantize_logits_kernel<uint8_t><<<g, 256, 0, S(stream)>>>(logits, n, routes, bits, static_cast<uint8_t*>(codes));
  else
    quantize_logits_kernel<int32_t><<<g, 256, 0, S(stream)>>>(logits, n, routes, bits, static_cast<int32_t*>(codes));
  LNG_LAUNCHED("quantize_logits_kernel");
  return LNG_OK;
}

namespace lng {
// Sign-packed codes from split-K partial logits [splits, routes * bits, ldp >= n] (split order sum).
// Split-K reduce + sign pack of the small-batch router.  A 256-thread CTA owns 32 rows x RB routes
// (CB = RB * bits logit columns): thread (c, row) sums the `splits` partials of one logit in a fixed
// order (consecutive threads read consecutive rows of a partial), the logits meet in shared
// memory, and thread (route, row) packs that route's sign bits.
template <typename CodeT>
__global__ void __launch_bounds__(256) router_reduce_pack_kernel(const float* __restrict__ part, int splits, int64_t n,
                                                                 int64_t ldp, int64_t routes, int bits,
                                                                 CodeT* __restrict__ codes, float* __restrict__ logits) {
  __shared__ float lg[8][32];
  const int rb = bits <= 8 ? 8 / bits : 1;  // routes per CTA
  const int cb = rb * bits;                 // logit columns per CTA (<= 8)
  const int64_t cols = routes * bits;
  const int64_t row0 = int64_t(blockIdx.x) * 32, r0 = int64_t(blockIdx.y) * rb;
  const int t = threadIdx.x, row = t & 31, c = t >> 5;
  const int64_t grow = row0 + row, col = r0 * bits + c;
  if (c < cb && grow < n && col < cols) {
    const float* pp = part + col * ldp + grow;
    const int64_t sstride = cols * ldp;
    float acc = 0.f;
    int sp = 0;
    for (; sp + 4 <= splits; sp += 4) {  // four independent loads in flight, summed in split order
      const float v0 = pp[(sp + 0) * sstride], v1 = pp[(sp + 1) * sstride];
      const float v2 = pp[(sp + 2) * sstride], v3 = pp[(sp + 3) * sstride];
      acc += v0;
      acc += v1;
      acc += v2;
      acc += v3;
    }
    for (; sp < splits; ++sp) acc += pp[sp * sstride];
    lg[c][row] = acc;
    if (logits) logits[grow * cols + col] = acc;
  }
  __syncthreads();
  if (c < rb && grow < n && r0 + c < routes) {
    int v = 0;
    for (int j = 0; j < bits; ++j) v |= (lg[c * bits + j][row] > 0.f ? 1 : 0) << j;
    codes[grow * routes + r0 + c] = static_cast<CodeT>(v);
  }
}

// fp32 router for few rows on the tensor cores: x = x1 + x2 + x3 and W = W1 + W2 + W3 split into
// bf16 parts (each exact to ~2^-24 relative), logits^T = sum of the six products x_i . W_j^T with
// i + j <= 4 (the dropped ones are below 2^-24 of |x| |W|), as one split-K GEMM with the logit
// columns as M (so few rows still fill the GPU), partial sums reduced in a fixed order.
// Scratch (x parts, W parts, partials) comes from the library pool and is released on `stream`.
static int tc_router_small_f32(const float* x, int64_t n, int64_t in_dim, int64_t x_stride, const float* w,
                               int64_t routes, int32_t bits, void* codes, int codes_i32, float* logits,
                               cudaStream_t stream, const __nv_bfloat16* w_split = nullptr,
                               const __nv_bfloat16* x_split = nullptr) {
  if (in_dim % TC_BK != 0 || x_stride != in_dim || n < 1 || n > 256 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(x_split) & 15))
    return LNG_ERR_UNSUPPORTED;
  const int64_t cols = routes * bits;
  const int64_t m_tiles = (cols + TC_BM - 1) / TC_BM;
  const int npairs = 6;
  const int64_t KB = npairs * (in_dim / TC_BK);
  // whole waves only: m_tiles x splits CTAs on at most the SM count
  int splits = int(std::max<int64_t>(1, num_sms() / m_tiles));
  if (splits > KB) splits = int(KB);
  const int BN = n <= 64 ? 64 : n <= 128 ? 128 : 256;
  const int64_t ldp = (n + 3) & ~int64_t(3);  // partial rows padded so the epilogue's 16-byte stores stay aligned
  // x_split: the rows' bf16x3 parts [n, 3 in_dim] made by the caller (embed2 features write them)
  const size_t xs_b = x_split ? 0 : al256(size_t(n) * 3 * in_dim * 2),
               ws_b = w_split ? 0 : al256(size_t(cols) * 3 * in_dim * 2), ps_b = al256(size_t(splits) * cols * ldp * 4);
  void* scratch = nullptr;
  int st = scratch_alloc(&scratch, xs_b + ws_b + ps_b, stream);
  if (st) return st;
  auto* xs = x_split ? const_cast<__nv_bfloat16*>(x_split) : static_cast<__nv_bfloat16*>(scratch);
  auto* ws = w_split ? const_cast<__nv_bfloat16*>(w_split)
                     : reinterpret_cast<__nv_bfloat16*>(static_cast<unsigned char*>(scratch) + xs_b);
  auto* ps = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + xs_b + ws_b);
  if (!x_split) split_rows_bf16x3_kernel<<<grid_for(n * in_dim, 256, 16), 256, 0, stream>>>(x, n, in_dim, xs);
  if (!w_split) split_bf16x3_kernel<<<grid_for(cols * in_dim, 256, 16), 256, 0, stream>>>(w, cols, in_dim, ws);
  CUtensorMap ta, tb;
  st = make_tmap_bf16(&ta, ws, cols, 3 * in_dim, 3 * in_dim, TC_BM);
  if (!st) st = make_tmap_bf16(&tb, xs, n, 3 * in_dim, 3 * in_dim, BN);
  if (!st) {
    TcGemmParams p{};
    p.M = cols;
    p.N = n;
    p.K = npairs * in_dim;
    p.a_kperiod = p.K;
    p.C = ps;
    p.ldc = ldp;
    p.c_dtype = LNG_F32;
    p.npairs = npairs;
    const int ap[6] = {0, 1, 2, 0, 1, 0}, bp[6] = {0, 0, 0, 1, 1, 2};  // (W_j, x_i)
    for (int i = 0; i < npairs; ++i) {
      p.a_part[i] = ap[i];
      p.b_part[i] = bp[i];
    }
    p.part_k = in_dim;
    p.splits = splits;
    p.split_stride = cols * ldp;
    st = BN == 64 ? launch_tc_gemm<64, 0>(ta, tb, p, stream)
                  : BN == 128 ? launch_tc_gemm<128, 0>(ta, tb, p, stream) : launch_tc_gemm<256, 0>(ta, tb, p, stream);
  }
  if (!st) {
    const int rb = bits <= 8 ? 8 / bits : 1;
    const dim3 g(unsigned(ceil_div(n, 32)), unsigned(ceil_div(routes, rb)));
    if (codes_i32)
      router_reduce_pack_kernel<int32_t><<<g, 256, 0, stream>>>(ps, splits, n, ldp, routes, bits,
                                                                static_cast<int32_t*>(codes), logits);
    else
      router_reduce_pack_kernel<uint8_t><<<g, 256, 0, stream>>>(ps, splits, n, ldp, routes, bits,
                                                                static_cast<uint8_t*>(codes), logits);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) st = cuda_status(e, "router_reduce_pack_kernel");
  }
  cudaFreeAsync(scratch, stream);
  return st;
}

}  // namespace lng

namespace lng {
// Router codes of fp32 rows given the weight and its bf16x3 split (made once by the owner of a
// fixed weight, e.g. the drafter): the small-batch tensor-core path skips the per-call split.
static int route_codes_presplit(const float* x, int64_t n, int64_t in_dim, const float* w,
                                const __nv_bfloat16* w_split, int64_t routes, int32_t bits, uint8_t* codes,
                                cudaStream_t stream, const __nv_bfloat16* x_split = nullptr) {
  if (n >= 1 && n <= 256 && w_split) {
    const int st = tc_router_small_f32(x, n, in_dim, in_dim, w, routes, bits, codes, 0, nullptr, stream, w_split,
                                       x_split);
    if (st != LNG_ERR_UNSUPPORTED) return st;
  }
  return lng_route_codes(x, LNG_F32, n, in_dim, in_dim, w, routes, bits, codes, LNG_U8, nullptr,
                         reinterpret_cast<lng_stream_t>(stream));
}
}  // namespace lng

extern "C" int lng_route_codes(const void* x, int32_t x_dtype, int64_t n, int64_t in_dim, int64_t x_stride,
                               const float* weight, int64_t routes, int32_t bits, void* codes, int32_t codes_dtype,
                               float* logits, lng_stream_t stream) {
  LNG_REQUIRE(n >= 0 && in_dim > 0 && routes > 0 && x_stride >= in_dim, "bad router shape");
  LNG_REQUIRE(bits >= 1 && bits <= RT_MAXBITS, "router bits_per_route must be in [1, 8]");
  LNG_REQUIRE(codes_dtype == LNG_U8 || codes_dtype == LNG_I32, "codes dtype must be u8 or i32");
  LNG_REQUIRE(x_dtype == LNG_F32 || x_dtype == LNG_BF16, "router input dtype must be f32 or bf16");
  if (n == 0) return LNG_OK;
  LNG_REQUIRE(x && weight && codes, "NULL pointer");
  if (x_dtype == LNG_BF16 && codes_dtype == LNG_U8 && logits == nullptr) {
    const int st = tc_router_codes(static_cast<const __nv_bfloat16*>(x), n, in_dim, x_stride, weight, routes, bits,
                                   static_cast<uint8_t*>(codes), S(stream));
    if (st != LNG_ERR_UNSUPPORTED) return st;
  }
  if (x_dtype == LNG_F32 && n <= 256) {
    // few fp32 rows: six bf16 split products on the tensor cores, split-K over the GPU
    const int st = tc_router_small_f32(static_cast<const float*>(x), n, in_dim, x_stride, weight, routes, bits, codes,
                                       codes_dtype == LNG_I32, logits, S(stream));
    if (st != LNG_ERR_UNSUPPORTED) return st;
  }
  if (ceil_div(n, RT_ROWS) * ceil_div(routes, RT_ROUTES) < 2 * 148 && ceil_div(n, RS_ROWS) < 65536) {
    // few row tiles: split the features over a cluster instead
    dim3 grid(unsigned(ceil_div(routes, RS_RPC) * RS_SPLIT), unsigned(ceil_div(n, RS_ROWS)));
#define LNG_ROUTER_SMALL(XT, CT)                                                                             \
  router_small_kernel<XT, CT><<<grid, 256, 0, S(stream)>>>(static_cast<const XT*>(x), n, in_dim, x_stride, weight, \
                                                           routes, bits, static_cast<CT*>(codes), logits)
    if (x_dtype == LNG_F32) {
      if (codes_dtype == LNG_U8) LNG_ROUTER_SMALL(float, uint8_t); else LNG_ROUTER_SMALL(float, int32_t);
    } else {
      if (codes_dtype == LNG_U8) LNG_ROUTER_SMALL(__nv_bfloat16, uint8_t); else LNG_ROUTER_SMALL(__nv_bfloat16, int32_t);
    }
#undef LNG_ROUTER_SMALL
    LNG_LAUNCHED("router_small_kernel");
    return LNG_OK;
  }
  dim3 grid(unsigned(ceil_div(n, RT_ROWS)), unsigned(ceil_div(routes, RT_ROUTES)));
#define LNG_ROUTER(XT, CT)                                                                                   \
  router_simt_kernel<XT, CT><<<grid, 256, 0, S(stream)>>>(static_cast<const XT*>(x), n, in_dim, x_stride, weight, \
                                                          routes, bits, static_cast<CT*>(codes), logits)
  if (x_dtype == LNG_F32) {
    if (codes_dtype == LNG_U8) LNG_ROUTER(float, uint8_t); else LNG_ROUTER(float, int32_t);
  } else {
    if (codes_dtype == LNG_U8) LNG_ROUTER(__nv_bfloat16, uint8_t); else LNG_ROUTER(__nv_bfloat16, int32_t);
  }
#undef LNG_ROUTER
  LNG_LAUNCHED("router_simt_kernel");
  return LNG_OK;
}

extern "C" int lng_router_prepare(const float* weight, int64_t rows, int64_t in_dim, void* w_split,
                                  lng_stream_t stream) {
  LNG_REQUIRE(rows > 0 && in_dim > 0, "bad router shape");
  LNG_REQUIRE(weight && w_split, "NULL pointer");
  split_bf16x3_kernel<<<grid_for(rows * in_dim, 256, 16), 256, 0, S(stream)>>>(weight, rows, in_dim,
                                                                               static_cast<__nv_bfloat16*>(w_split));
  LNG_LAUNCHED("split_bf16x3_kernel");
  return LNG_OK;
}

extern "C" int lng_route_codes_split(const void* x_bf16, int64_t n, int64_t in_dim, int64_t x_stride,
                                     const void* w_split, int64_t routes, int32_t bits, uint8_t* codes,
                                     lng_stream_t stream) {
  LNG_REQUIRE(n >= 0 && in_dim > 0 && routes > 0 && x_stride >= in_dim, "bad router shape");
  LNG_REQUIRE(bits >= 1 && bits <= 6, "the tensor-core router takes bits_per_route in [1, 6]");
  LNG_REQUIRE(in_dim % TC_BK == 0, "the tensor-core router needs in_dim % 64 == 0");
  if (n == 0) return LNG_OK;
  LNG_REQUIRE(x_bf16 && w_split && codes, "NULL pointer");
  const int st = tc_router_split(static_cast<const __nv_bfloat16*>(x_bf16), n, in_dim, x_stride,
                                 static_cast<const __nv_bfloat16*>(w_split), routes, bits, codes, S(stream));
  if (st == LNG_ERR_UNSUPPORTED) return fail(st, "router operands violate the TMA alignment rules (16-byte rows)");
  return st;
}

namespace lng {
// embed2 features into rows of stride out_stride (the drafter appends its SSM state after them)
static int embed2_features(const int64_t* cur, const int64_t* prev, int64_t n, const void* embedding, int32_t e_dtype,
                           int64_t vocab, int64_t d, const float* prev_w, const float* cur_w, const float* start,
                           float eps, float* out, int64_t out_stride, cudaStream_t stream,
                           __nv_bfloat16* split = nullptr, int64_t split_width = 0) {
  LNG_REQUIRE(n >= 0 && vocab > 0 && d > 0, "bad shape");
  if (n == 0) return LNG_OK;
  LNG_REQUIRE(cur && embedding && prev_w && cur_w && start && out, "NULL pointer");
  const int g = int(n < (int64_t(1) << 20) ? n : (int64_t(1) << 20));
  switch (e_dtype) {
    case LNG_F32:
      embed2_features_kernel<float><<<g, 128, 0, stream>>>(cur, prev, n, static_cast<const float*>(embedding), vocab,
                                                               d, prev_w, cur_w, start, eps, out, out_stride, split,
                                                               split_width);
      break;
    case LNG_BF16:
      embed2_features_kernel<__nv_bfloat16><<<g, 128, 0, stream>>>(
          cur, prev, n, static_cast<const __nv_bfloat16*>(embedding), vocab, d, prev_w, cur_w, start, eps, out, out_stride,
          split, split_width);
      break;
    case LNG_F16:
      embed2_features_kernel<__half><<<g, 128, 0, stream>>>(cur, prev, n, static_cast<const __half*>(embedding),
                                                                vocab, d, prev_w, cur_w, start, eps, out, out_stride,
                                                                split, split_width);
      break;
    default:
      return fail(LNG_ERR_ARGUMENT, "embedding dtype must be f32, bf16 or f16");
  }
  LNG_LAUNCHED("embed2_features_kernel");
  return LNG_OK;
}
}  // namespace lng

extern "C" int lng_embed2_features(const int64_t* cur, const int64_t* prev, int64_t n, const void* embedding,
                                   int32_t e_dtype, int64_t vocab, int64_t d, const float* prev_w, const float* cur_w,
                                   const float* start, float eps, float* out, lng_stream_t stream) {
  return embed2_features(cur, prev, n, embedding, e_dtype, vocab, d, prev_w, cur_w, start, eps, out, 2 * d, S(stream));
}

// ====================================================================== lookup
extern "C" int lng_table_row_ss(const lng_tables* tables, float* const* row_ss, lng_stream_t stream) {
  int st = check_tables(tables);
  if (st) return st;
  LNG_REQUIRE(row_ss != nullptr, "row_ss is NULL");
  for (int o = 0; o < tables->n_orders; ++o) {
    LNG_REQUIRE(row_ss[o] != nullptr, "row_ss pointer is NULL");
    const int64_t rows = tables->num_routes << (int64_t(tables->bits) * tables->orders[o]);
    const int g = grid_for(rows * 32, 256, 16);
    switch (tables->table_dtype) {
      case LNG_F32:
        rms_rows_kernel<float, true><<<g, 256, 0, S(stream)>>>(static_cast<const float*>(tables->tables[o]), rows,
                                                                tables->memory_dim, 0.f, row_ss[o]);
        break;
      case LNG_BF16:
        rms_rows_kernel<__nv_bfloat16, true><<<g, 256, 0, S(stream)>>>(
            static_cast<const __nv_bfloat16*>(tables->tables[o]), rows, tables->memory_dim, 0.f, row_ss[o]);
        break;
      default:
        rms_rows_kernel<__half, true><<<g, 256, 0, S(stream)>>>(static_cast<const __half*>(tables->tables[o]), rows,
                                                                 tables->memory_dim, 0.f, row_ss[o]);
    }
    LNG_LAUNCHED("rms_rows_kernel (sum of squares)");
  }
  return LNG_OK;
}

template <typename CodeT>
static int launch_lookup(const lng_tables* t, const CodeSource& src, int64_t M, int64_t rs, int64_t re, void* out,
                         int32_t out_dtype, cudaStream_t stream) {
  const TableSet ts = table_set(t);
  const int64_t warps = M * (re - rs);
  if (warps == 0) return LNG_OK;
  const int g = grid_for(warps * 32, 256, 16);
  const int es = dtype_size(t->table_dtype);
  if (out_dtype == t->table_dtype && (t->memory_dim * es) % 16 == 0) {
    for (int o = 0; o < t->n_orders; ++o)
      LNG_REQUIRE((reinterpret_cast<uintptr_t>(t->tables[o]) & 15) == 0, "table pointers must be 16-byte aligned");
    LNG_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15) == 0, "output must be 16-byte aligned");
    lookup_vec_kernel<CodeT><<<g, 256, 0, stream>>>(ts, src, M, rs, re, es, static_cast<uint4*>(out));
    LNG_LAUNCHED("lookup_vec_kernel");
    return LNG_OK;
  }
#define LNG_LK(TT, OT) lookup_kernel<CodeT, TT, OT><<<g, 256, 0, stream>>>(ts, src, M, rs, re, static_cast<OT*>(out))
  if (out_dtype == LNG_F32) {
    if (t->table_dtype == LNG_F32) LNG_LK(float, float);
    else if (t->table_dtype == LNG_BF16) LNG_LK(__nv_bfloat16, float);
    else LNG_LK(__half, float);
  } else if (out_dtype == LNG_BF16 && t->table_dtype == LNG_BF16) {
    LNG_LK(__nv_bfloat16, __nv_bfloat16);
  } else if (out_dtype == LNG_F16 && t->table_dtype == LNG_F16) {
    LNG_LK(__half, __half);
  } else {
    return fail(LNG_ERR_ARGUMENT, "output dtype must be f32 or the table dtype");
  }
#undef LNG_LK
  LNG_LAUNCHED("lookup_kernel");
  return LNG_OK;
}

extern "C" int lng_lookup_route_chunk(const lng_tables* tables, const void* codes, int32_t codes_dtype, int64_t B,
                                      int64_t T, int64_t route_start, int64_t route_end, const int64_t* segment_ids,
                                      const uint8_t* valid_tokens, int64_t target_length, void* out, int32_t out_dtype,
                                      lng_stream_t stream) {
  int st = check_tables(tables);
  if (st) return st;
  LNG_REQUIRE(B >= 0 && T >= 0, "bad shape");
  LNG_REQUIRE(0 <= route_start && route_start <= route_end && route_end <= tables->num_routes, "bad route range");
  LNG_REQUIRE(codes_dtype == LNG_U8 || codes_dtype == LNG_I32, "codes dtype must be u8 or i32");
  const int64_t tout = target_length > 0 ? std::min(target_length, T) : T;
  if (B * tout == 0 || route_end == route_start) return LNG_OK;
  LNG_REQUIRE(codes && out, "NULL pointer");
  CodeSource src{codes, B, T, 0, tables->num_routes, segment_ids, valid_tokens, nullptr, T - tout, T};
  if (codes_dtype == LNG_U8)
    return launch_lookup<uint8_t>(tables, src, B * tout, route_start, route_end, out, out_dtype, S(stream));
  return launch_lookup<int32_t>(tables, src, B * tout, route_start, route_end, out, out_dtype, S(stream));
}

extern "C" int lng_lookup_windows(const lng_tables* tables, const void* codes, int32_t codes_dtype, int64_t M,
                                  int64_t W, const int32_t* seg, void* out, int32_t out_dtype, lng_stream_t stream) {
  int st = check_tables(tables);
  if (st) return st;
  LNG_REQUIRE(M >= 0 && W >= 1, "bad window shape");
  LNG_REQUIRE(codes_dtype == LNG_U8 || codes_dtype == LNG_I32, "codes dtype must be u8 or i32");
  if (M == 0) return LNG_OK;
  LNG_REQUIRE(codes && out, "NULL pointer");
  CodeSource src{codes, 0, 0, W, tables->num_routes, nullptr, nullptr, seg, 0, 0};
  if (codes_dtype == LNG_U8) return launch_lookup<uint8_t>(tables, src, M, 0, tables->num_routes, out, out_dtype, S(stream));
  return launch_lookup<int32_t>(tables, src, M, 0, tables->num_routes, out, out_dtype, S(stream));
}

// ====================================================================== training-mode lookup backward
extern "C" int lng_lookup_backward(const lng_tables* tables, const void* codes, int32_t codes_dtype, int64_t B,
                                   int64_t T, int64_t route_start, int64_t route_end, const int64_t* segment_ids,
                                   const uint8_t* valid_tokens, const void* grad_tokens, int32_t grad_dtype,
                                   const float* q_logits, int64_t q_routes, float temperature, float scale,
                                   int32_t exact, float* grad_q, float* const* grad_tables, lng_stream_t stream) {
  int st = check_tables(tables);
  if (st) return st;
  LNG_REQUIRE(codes_dtype == LNG_U8 || codes_dtype == LNG_I32, "codes dtype must be u8 or i32");
  LNG_REQUIRE(B >= 0 && T >= 0 && 0 <= route_start && route_start < route_end && route_end <= tables->num_routes,
              "bad shape or route range");
  LNG_REQUIRE(grad_dtype == LNG_F32 || grad_dtype == LNG_BF16 || grad_dtype == LNG_F16, "grad dtype must be float");
  LNG_REQUIRE(tables->memory_dim <= 32 * SG_MAXE, "memory_dim must be <= 256 for the backward");
  LNG_REQUIRE(!grad_q || (q_logits && q_routes >= route_end && tables->bits <= SG_MAXBITS),
              "the surrogate needs q_logits over the chunk's routes and bits <= 8");
  if (B == 0 || T == 0) return LNG_OK;
  LNG_REQUIRE(codes && grad_tokens, "NULL pointer");
  LookupGradParams p{};
  p.ts = table_set(tables);
  p.table_dtype = tables->table_dtype;
  p.src = CodeSource{codes, B, T, 0, tables->num_routes, segment_ids, valid_tokens, nullptr, 0, T, 0, 0};
  p.B = B;
  p.T = T;
  p.route_start = route_start;
  p.Rc = route_end - route_start;
  p.grad = grad_tokens;
  p.grad_dtype = grad_dtype;
  p.q = q_logits;
  p.Rq = q_routes;
  p.temperature = temperature;
  p.scale = scale;
  p.exact = exact != 0;
  p.grad_q = grad_q;
  bool any_tab = false;
  for (int o = 0; o < tables->n_orders; ++o) {
    p.gtab[o] = grad_tables ? grad_tables[o] : nullptr;
    any_tab = any_tab || p.gtab[o];
  }
  const int64_t warps = B * T * p.Rc;
  if (grad_q) {
    if (temperature == 0.f || scale == 0.f) {
      LNG_CUDA(cudaMemsetAsync(grad_q, 0, size_t(warps * tables->bits) * 4, S(stream)));
    } else {
      const int g = grid_for(warps * 32, 256, 16);
      if (codes_dtype == LNG_U8) surrogate_grad_kernel<uint8_t><<<g, 256, 0, S(stream)>>>(p);
      else surrogate_grad_kernel<int32_t><<<g, 256, 0, S(stream)>>>(p);
      LNG_LAUNCHED("surrogate_grad_kernel");
    }
  }
  if (any_tab) {
    const int g = grid_for(warps * tables->n_orders * 32, 256, 16);
    if (codes_dtype == LNG_U8) table_grad_kernel<uint8_t><<<g, 256, 0, S(stream)>>>(p);
    else table_grad_kernel<int32_t><<<g, 256, 0, S(stream)>>>(p);
    LNG_LAUNCHED("table_grad_kernel");
  }
  return LNG_OK;
}

// ====================================================================== host-RAM serving and incremental state
extern "C" int lng_lookup_serving_rows(const lng_tables* tables, const void* codes, int32_t codes_dtype, int64_t B,
                                       int64_t T, int64_t n, void* out, lng_stream_t stream) {
  int st = check_tables(tables);
  if (st) return st;
  LNG_REQUIRE(codes_dtype == LNG_U8 || codes_dtype == LNG_I32, "codes dtype must be u8 or i32");
  LNG_REQUIRE(B >= 0 && T >= 1 && n >= 1 && n <= T, "need 1 <= n <= T");
  if (B == 0) return LNG_OK;
  LNG_REQUIRE(codes && out, "NULL pointer");
  const int es = dtype_size(tables->table_dtype);
  LNG_REQUIRE((tables->memory_dim * es) % 16 == 0, "serving rows must be a whole number of 16-byte vectors");
  for (int o = 0; o < tables->n_orders; ++o)
    LNG_REQUIRE((reinterpret_cast<uintptr_t>(tables->tables[o]) & 15) == 0, "table pointers must be 16-byte aligned");
  LNG_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15) == 0, "output must be 16-byte aligned");
  TableSet ts = table_set(tables);
  CodeSource src{codes, B, T, 0, tables->num_routes, nullptr, nullptr, nullptr, T - n, T, 0, 1};
  const int64_t warps = B * n * tables->num_routes;
  const int g = grid_for(warps * 32, 256, 16);
  if (codes_dtype == LNG_U8)
    lookup_host_kernel<uint8_t><<<g, 256, 0, S(stream)>>>(ts, src, B * n, 0, tables->num_routes, es, static_cast<uint4*>(out));
  else
    lookup_host_kernel<int32_t><<<g, 256, 0, S(stream)>>>(ts, src, B * n, 0, tables->num_routes, es, static_cast<uint4*>(out));
  LNG_LAUNCHED("lookup_host_kernel");
  return LNG_OK;
}

extern "C" int lng_serving_permute(const void* src, void* dst, int32_t dtype, int64_t routes, int32_t order,
                                   int32_t bits, int64_t mem_dim, lng_stream_t stream) {
  LNG_REQUIRE(routes >= 1 && order >= 1 && bits >= 1 && int64_t(order) * bits <= 40 && mem_dim >= 1, "bad table shape");
  const int es = dtype_size(dtype);
  LNG_REQUIRE(es > 0 && (mem_dim * es) % 16 == 0, "rows must be a whole number of 16-byte vectors");
  LNG_REQUIRE(src && dst && src != dst, "src and dst must be distinct non-NULL buffers");
  LNG_REQUIRE(((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0,
              "buffers must be 16-byte aligned");
  const int64_t rows = routes << (int64_t(bits) * order);
  serving_permute_kernel<<<grid_for(rows * 32, 256, 16), 256, 0, S(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), rows, order, bits, mem_dim * es / 16);
  LNG_LAUNCHED("serving_permute_kernel");
  return LNG_OK;
}

namespace {
std::mutex g_host_map_mu;
std::vector<void*> g_host_registered;  // host ranges this library registered (and so unregisters)
}  // namespace

extern "C" int lng_host_map(void* host, size_t bytes, void** device_ptr) {
  LNG_REQUIRE(host && device_ptr && bytes > 0, "NULL pointer or empty range");
  *device_ptr = nullptr;
  cudaPointerAttributes attr{};
  LNG_CUDA(cudaPointerGetAttributes(&attr, host));
  if (attr.type != cudaMemoryTypeHost) {  // pageable: pin and map it (page-locked memory is already mapped)
    LNG_CUDA(cudaHostRegister(host, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable));
    std::lock_guard<std::mutex> lock(g_host_map_mu);
    g_host_registered.push_back(host);
  }
  LNG_CUDA(cudaHostGetDevicePointer(device_ptr, host, 0));
  return LNG_OK;
}

extern "C" int lng_host_unmap(void* host) {
  LNG_REQUIRE(host, "NULL pointer");
  std::lock_guard<std::mutex> lock(g_host_map_mu);
  for (size_t i = 0; i < g_host_registered.size(); ++i) {
    if (g_host_registered[i] == host) {
      g_host_registered.erase(g_host_registered.begin() + i);
      LNG_CUDA(cudaHostUnregister(host));
      return LNG_OK;
    }
  }
  return LNG_OK;  // memory the caller pinned itself stays pinned
}

extern "C" int lng_packed_suffix(const void* codes, int32_t codes_dtype, int64_t B, int64_t T, int64_t R,
                                 int32_t bits, int32_t maxn, const int32_t* packed_in, int32_t* packed_out,
                                 uint8_t* window_out, lng_stream_t stream) {
  LNG_REQUIRE(codes_dtype == LNG_U8 || codes_dtype == LNG_I32, "codes dtype must be u8 or i32");
  LNG_REQUIRE(B >= 0 && T >= 1 && R >= 1 && bits >= 1 && maxn >= 1 && int64_t(bits) * maxn <= 31,
              "bad packed-state shape (maxn * bits must fit 31 bits)");
  LNG_REQUIRE(!packed_in || T == 1, "advancing the packed state takes one position");
  if (B == 0) return LNG_OK;
  LNG_REQUIRE(codes && packed_out, "NULL pointer");
  const unsigned g = unsigned(ceil_div(B * R, 128));
  if (codes_dtype == LNG_U8)
    packed_suffix_kernel<uint8_t><<<g, 128, 0, S(stream)>>>(static_cast<const uint8_t*>(codes), B, T, R, bits, maxn,
                                                            packed_in, packed_in != nullptr, packed_out, window_out);
  else
    packed_suffix_kernel<int32_t><<<g, 128, 0, S(stream)>>>(static_cast<const int32_t*>(codes), B, T, R, bits, maxn,
                                                            packed_in, packed_in != nullptr, packed_out, window_out);
  LNG_LAUNCHED("packed_suffix_kernel");
  return LNG_OK;
}

// ====================================================================== attention core
// Warps per CTA and shared-memory stages per warp of the gather kernel come from the token width
// (AttendMmaCfg): two stages per warp, as many warps (at most 8) as the shared memory holds.
template <int DT, typename CodeT, typename T>
static int launch_attend_mma(const AttendParams& p, cudaStream_t stream) {
  using Cfg = AttendMmaCfg<DT>;
  constexpr int WARPS = Cfg::WARPS, STAGES = Cfg::STAGES;
  const size_t smem = size_t(WARPS) * STAGES * Cfg::STAGE_BYTES + size_t(WARPS) * STAGES * sizeof(uint64_t);
  auto kern = attend_mma_kernel<CodeT, T, DT, WARPS, STAGES>;
  LNG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  const int64_t blocks_needed = ceil_div(p.M, WARPS);
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(blocks_needed, num_sms())));
  kern<<<grid, WARPS * 32, smem, stream>>>(p);
  LNG_LAUNCHED("attend_mma_kernel");
  return LNG_OK;
}

// Few items leave most SMs idle with one warp per item walking every route chunk in turn (a 64-sequence
// draft step: 8 blocks of 8 warps, 6 chunks each), so the routes are split over block rows instead:
// row y takes a slice of whole 32-route chunks and writes its own (m, l, u) state, and
// attend_split_combine_kernel merges the slices.  Only as many slices as keep every block in one
// wave (one block per SM); none once the items alone fill half the SMs.
template <int DT, typename CodeT, typename T>
static int launch_attend_mma_split(const AttendParams& p, cudaStream_t stream, bool* used) {
  using Cfg = AttendMmaCfg<DT>;
  *used = false;
  const int64_t R = p.route_end - p.route_start;
  const int64_t chunks = ceil_div(R, int64_t(Cfg::C));
  const int64_t blocks = ceil_div(std::max<int64_t>(p.M, 1), int64_t(Cfg::WARPS));
  if (p.partial != 0 || 2 * blocks > num_sms()) return LNG_OK;
  int64_t splits = std::min<int64_t>(chunks, num_sms() / blocks);
  if (splits < 2) return LNG_OK;
  const int64_t per = ceil_div(chunks, splits) * Cfg::C;  // routes per slice, whole chunks
  splits = ceil_div(R, per);
  if (splits < 2) return LNG_OK;
  const size_t rows = size_t(p.M) * p.qh;
  const size_t bytes = al256(rows * splits * DT * 4) + 2 * al256(rows * splits * 4);
  void* buf = nullptr;
  int st = scratch_alloc(&buf, bytes, stream);
  if (st) return st;
  float* su = static_cast<float*>(buf);
  float* sm = reinterpret_cast<float*>(static_cast<unsigned char*>(buf) + al256(rows * splits * DT * 4));
  float* sl = sm + al256(rows * splits * 4) / 4;
  AttendParams q = p;
  q.partial = 1;
  q.route_split = per;
  q.u = su;
  q.m_out = sm;
  q.l_out = sl;
  constexpr int WARPS = Cfg::WARPS, STAGES = Cfg::STAGES;
  const size_t smem = size_t(WARPS) * STAGES * Cfg::STAGE_BYTES + size_t(WARPS) * STAGES * sizeof(uint64_t);
  auto kern = attend_mma_kernel<CodeT, T, DT, WARPS, STAGES, true>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e == cudaSuccess) {
    const dim3 grid{unsigned(blocks), unsigned(splits), 1u};
    kern<<<grid, WARPS * 32, smem, stream>>>(q);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    attend_split_combine_kernel<T><<<grid_for(int64_t(rows) * (DT / 4), 256, 8), 256, 0, stream>>>(
        su, sm, sl, int(splits), p.M, p.qh, DT, static_cast<T*>(p.u));
    e = cudaGetLastError();
  }
  cudaFreeAsync(buf, stream);
  if (e != cudaSuccess) return cuda_status(e, "attend_mma_kernel (route split)");
  *used = true;
  return LNG_OK;
}

template <int DT, typename CodeT, typename T>
static int launch_attend_mma_any(const AttendParams& p, cudaStream_t stream) {
  bool used = false;
  const int st = launch_attend_mma_split<DT, CodeT, T>(p, stream, &used);
  if (st || used) return st;
  return launch_attend_mma<DT, CodeT, T>(p, stream);
}

template <typename CodeT, typename T>
static int dispatch_attend_mma(int64_t Dt, const AttendParams& p, cudaStream_t stream) {
  switch (Dt) {
    case 32: return launch_attend_mma_any<32, CodeT, T>(p, stream);
    case 64: return launch_attend_mma_any<64, CodeT, T>(p, stream);
    case 128: return launch_attend_mma_any<128, CodeT, T>(p, stream);
    case 136: return launch_attend_mma_any<136, CodeT, T>(p, stream);
    case 256: return launch_attend_mma_any<256, CodeT, T>(p, stream);
    case 272: return launch_attend_mma_any<272, CodeT, T>(p, stream);
    default: return LNG_ERR_UNSUPPORTED;
  }
}

template <typename CodeT>
static int attend_impl(const lng_tables* t, const AttendParams& p, int32_t u_dtype, cudaStream_t stream) {
  const int64_t Dt = int64_t(t->n_orders) * t->memory_dim;
  const bool t16 = t->table_dtype == LNG_BF16 || t->table_dtype == LNG_F16;
  // qa dtype: the activations' in normalised mode; the tables' (16-bit) or f32 in partial mode
  const int qa_dtype = p.partial ? (t16 ? t->table_dtype : LNG_F32) : u_dtype;
  // tensor-core path: 16-bit tables, query of the same type, <= 16 heads, 16-byte rows
  const bool mma_ok = t16 && qa_dtype == t->table_dtype &&
                      (p.partial >= 3 ? u_dtype == LNG_BF16
                                      : (p.partial ? u_dtype == LNG_F32 : u_dtype == t->table_dtype)) &&
                      p.qh <= 16 && (t->memory_dim % 8) == 0 && t->orders[t->n_orders - 1] <= MAXW;
  if (mma_ok) {
    AttendParams q = p;
    q.rows32 = 1;
    if (p.src.direct > 0)
      q.rows32 = p.M * p.src.direct < (int64_t(1) << 31);
    else
      for (int o = 0; o < t->n_orders; ++o)
        q.rows32 = q.rows32 && (t->num_routes << (int64_t(t->bits) * t->orders[o])) < (int64_t(1) << 31);
    bool aligned = (reinterpret_cast<uintptr_t>(p.qa) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.u) & 15) == 0;
    for (int o = 0; o < t->n_orders; ++o) aligned = aligned && (reinterpret_cast<uintptr_t>(t->tables[o]) & 15) == 0;
    if (aligned) {
      const int st = t->table_dtype == LNG_BF16 ? dispatch_attend_mma<CodeT, __nv_bfloat16>(Dt, q, stream)
                                                : dispatch_attend_mma<CodeT, __half>(Dt, q, stream);
      if (st != LNG_ERR_UNSUPPORTED) return st;
    }
  }
  if (p.partial >= 3) return fail(LNG_ERR_UNSUPPORTED, "packed shard states need 16-bit tables and the tensor-core kernel");
  // CUDA-core path (fp32 tables / activations, partial shard states, any width)
  const int QH = p.qh;
  const size_t smem = sizeof(float) * (size_t(2 * QH + ATT_C) * Dt + ATT_C + size_t(QH) * ATT_C + 3 * QH);
  LNG_REQUIRE(smem <= 227 * 1024, "route token width too large for the CUDA-core readout");
  const int grid = int(std::min<int64_t>(p.M, int64_t(num_sms()) * 8));
#define LNG_AT(TT, QT, UT)                                                                                   \
  do {                                                                                                       \
    auto k = attend_simt_kernel<CodeT, TT, QT, UT>;                                                          \
    LNG_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));               \
    k<<<grid, 128, smem, stream>>>(p);                                                                       \
  } while (0)
  const int act = u_dtype;
  if (p.partial) {  // fp32 state out
    if (t->table_dtype == LNG_F32) LNG_AT(float, float, float);
    else if (t->table_dtype == LNG_BF16) LNG_AT(__nv_bfloat16, __nv_bfloat16, float);
    else LNG_AT(__half, __half, float);
  } else if (t->table_dtype == LNG_F32) {
    if (act == LNG_F32) LNG_AT(float, float, float);
    else if (act == LNG_BF16) LNG_AT(float, __nv_bfloat16, __nv_bfloat16);
    else return fail(LNG_ERR_ARGUMENT, "unsupported activation dtype");
  } else if (t->table_dtype == LNG_BF16) {
    if (act == LNG_F32) LNG_AT(__nv_bfloat16, float, float);
    else if (act == LNG_BF16) LNG_AT(__nv_bfloat16, __nv_bfloat16, __nv_bfloat16);
    else return fail(LNG_ERR_ARGUMENT, "unsupported activation dtype");
  } else {
    if (act == LNG_F32) LNG_AT(__half, float, float);
    else if (act == LNG_F16) LNG_AT(__half, __half, __half);
    else return fail(LNG_ERR_ARGUMENT, "unsupported activation dtype");
  }
#undef LNG_AT
  LNG_LAUNCHED("attend_simt_kernel");
  return LNG_OK;
}

extern "C" int lng_route_attend(const lng_tables* tables, const void* codes, int32_t codes_dtype, int64_t B, int64_t T,
                                int64_t window, const int64_t* segment_ids, const uint8_t* valid_tokens,
                                const int32_t* seg, int64_t target_length, int64_t route_start, int64_t route_end,
                                int32_t num_heads, float eps, float sink_logit, const void* qa, const float* qscale,
                                void* u, int32_t u_dtype, int32_t partial, float* m_out, float* l_out,
                                lng_stream_t stream) {
  int st = check_tables(tables);
  if (st) return st;
  LNG_REQUIRE(codes_dtype == LNG_U8 || codes_dtype == LNG_I32, "codes dtype must be u8 or i32");
  LNG_REQUIRE(num_heads >= 1 && num_heads <= 64, "num_heads must be in [1, 64]");
  LNG_REQUIRE(0 <= route_start && route_start < route_end && route_end <= tables->num_routes, "bad route range");
  LNG_REQUIRE(u_dtype == LNG_F32 || u_dtype == LNG_BF16 || u_dtype == LNG_F16, "u dtype must be f32, bf16 or f16");
  LNG_REQUIRE(partial >= 0 && partial <= 4, "partial must be 0 .. 4");
  LNG_REQUIRE(!(partial == 1 || partial == 2) || (u_dtype == LNG_F32 && m_out && l_out),
              "partial modes 1 / 2 need fp32 u, m_out and l_out");
  LNG_REQUIRE(partial < 3 || (u_dtype == LNG_BF16 && m_out), "partial modes 3 / 4 need a bf16 pack and m_out");
  const int64_t tout = (window <= 0 && target_length > 0) ? std::min(target_length, T) : T;
  const int64_t M = window > 0 ? B : B * tout;
  if (M == 0) return LNG_OK;
  LNG_REQUIRE(codes && qa && u, "NULL pointer");
  AttendParams p{};
  p.ts = table_set(tables);
  p.src = CodeSource{codes, window > 0 ? 0 : B, window > 0 ? 0 : T, window, tables->num_routes, segment_ids,
                     valid_tokens, seg, window > 0 ? 0 : T - tout, T};
  p.M = M;
  p.route_start = route_start;
  p.route_end = route_end;
  p.qh = num_heads;
  p.eps = eps;
  p.sink = sink_logit;
  p.qa = qa;
  p.qscale = qscale;
  p.u = u;
  p.partial = partial;
  p.m_out = m_out;
  p.l_out = l_out;
  if (codes_dtype == LNG_U8) return attend_impl<uint8_t>(tables, p, u_dtype, S(stream));
  return attend_impl<int32_t>(tables, p, u_dtype, S(stream));
}

extern "C" int lng_route_attend_rows(const void* tokens, int32_t tok_dtype, int64_t M, int64_t routes, int64_t Dt,
                                     int32_t num_heads, float eps, float sink_logit, const void* qa,
                                     const float* qscale, void* u, int32_t u_dtype, lng_stream_t stream) {
  LNG_REQUIRE(M >= 0 && routes >= 1 && Dt >= 1, "bad route-token shape");
  LNG_REQUIRE(num_heads >= 1 && num_heads <= 64, "num_heads must be in [1, 64]");
  LNG_REQUIRE(tok_dtype == LNG_F32 || tok_dtype == LNG_BF16 || tok_dtype == LNG_F16, "token dtype must be f32, bf16 or f16");
  LNG_REQUIRE(u_dtype == LNG_F32 || u_dtype == LNG_BF16 || u_dtype == LNG_F16, "u dtype must be f32, bf16 or f16");
  if (M == 0) return LNG_OK;
  LNG_REQUIRE(tokens && qa && u, "NULL pointer");
  // the tokens as a one-"order" table whose row of (item i, route r) is i * routes + r
  lng_tables t{};
  t.n_orders = 1;
  t.orders[0] = 1;
  t.tables[0] = tokens;
  t.table_dtype = tok_dtype;
  t.bits = 1;
  t.num_routes = routes;
  t.memory_dim = Dt;
  AttendParams p{};
  p.ts = table_set(&t);
  p.src = CodeSource{nullptr, 0, 0, 0, routes, nullptr, nullptr, nullptr, 0, 0, routes};
  p.M = M;
  p.route_start = 0;
  p.route_end = routes;
  p.qh = num_heads;
  p.eps = eps;
  p.sink = sink_logit;
  p.qa = qa;
  p.qscale = qscale;
  p.u = u;
  return attend_impl<uint8_t>(&t, p, u_dtype, S(stream));
}

// ====================================================================== GEMM
extern "C" int lng_gemm(const void* A, int32_t a_dtype, int64_t lda, const void* Bm, int32_t b_dtype, int64_t ldb,
                        void* C, int32_t c_dtype, int64_t ldc, int64_t M, int64_t N, int64_t K, const float* rowscale,
                        int32_t accumulate, lng_stream_t stream) {
  LNG_REQUIRE(M >= 0 && N >= 0 && K >= 0 && lda >= K && ldb >= K && ldc >= N, "bad GEMM shape");
  LNG_REQUIRE(is_float_dtype(a_dtype) && is_float_dtype(b_dtype) && is_float_dtype(c_dtype), "GEMM dtypes must be float");
  if (M == 0 || N == 0) return LNG_OK;
  LNG_REQUIRE(A && Bm && C, "NULL pointer");
  if (a_dtype == LNG_BF16 && b_dtype == LNG_BF16 && !accumulate) {
    const int splits = tc_gemm_small_m_splits(M, N, K);
    if (splits > 1 && (c_dtype == LNG_F32 || c_dtype == LNG_BF16) && N % 4 == 0) {
      void* part = nullptr;
      int st = scratch_alloc(&part, size_t(splits) * M * N * sizeof(float), S(stream));
      if (st) return st;
      st = tc_gemm_bf16_splitk(static_cast<const __nv_bfloat16*>(A), lda, static_cast<const __nv_bfloat16*>(Bm), ldb,
                               static_cast<float*>(part), splits, M, N, K, rowscale, S(stream));
      if (st == LNG_OK) {
        const int g = grid_for(M * (N / 4), 256, 8);
        if (c_dtype == LNG_F32)
          splitk_reduce_kernel<float><<<g, 256, 0, S(stream)>>>(static_cast<float*>(part), splits, M, N,
                                                                static_cast<float*>(C), ldc);
        else
          splitk_reduce_kernel<__nv_bfloat16><<<g, 256, 0, S(stream)>>>(static_cast<float*>(part), splits, M, N,
                                                                        static_cast<__nv_bfloat16*>(C), ldc);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) st = cuda_status(e, "splitk_reduce_kernel");
      }
      cudaFreeAsync(part, S(stream));
      if (st != LNG_ERR_UNSUPPORTED) return st;
    }
    const int st = tc_gemm_bf16(static_cast<const __nv_bfloat16*>(A), lda, static_cast<const __nv_bfloat16*>(Bm), ldb,
                                C, c_dtype, ldc, M, N, K, rowscale, S(stream));
    if (st != LNG_ERR_UNSUPPORTED) return st;
  }
  dim3 grid(unsigned(ceil_div(N, GS_TILE)), unsigned(ceil_div(M, GS_TILE)));
#define LNG_G(AT, BT, CT)                                                                                         \
  gemm_simt_kernel<AT, BT, CT><<<grid, 256, 0, S(stream)>>>(static_cast<const AT*>(A), lda, static_cast<const BT*>(Bm), \
                                                            ldb, static_cast<CT*>(C), ldc, M, N, K, rowscale, accumulate)
#define LNG_GC(AT, BT)                                             \
  do {                                                             \
    if (c_dtype == LNG_F32) LNG_G(AT, BT, float);                  \
    else if (c_dtype == LNG_BF16) LNG_G(AT, BT, __nv_bfloat16);    \
    else LNG_G(AT, BT, __half);                                    \
  } while (0)
  if (a_dtype == LNG_F32 && b_dtype == LNG_F32) LNG_GC(float, float);
  else if (a_dtype == LNG_BF16 && b_dtype == LNG_BF16) LNG_GC(__nv_bfloat16, __nv_bfloat16);
  else if (a_dtype == LNG_F32 && b_dtype == LNG_BF16) LNG_GC(float, __nv_bfloat16);
  else if (a_dtype == LNG_BF16 && b_dtype == LNG_F32) LNG_GC(__nv_bfloat16, float);
  else if (a_dtype == LNG_F16 && b_dtype == LNG_F16) LNG_GC(__half, __half);
  else if (a_dtype == LNG_F32 && b_dtype == LNG_F16) LNG_GC(float, __half);
  else return fail(LNG_ERR_UNSUPPORTED, "unsupported GEMM dtype combination");
#undef LNG_GC
#undef LNG_G
  LNG_LAUNCHED("gemm_simt_kernel");
  return LNG_OK;
}

// ====================================================================== row ops
extern "C" int lng_rms_rows(const void* x, int32_t x_dtype, int64_t n, int64_t d, float eps, float* rs,
                            lng_stream_t stream) {
  LNG_REQUIRE(n >= 0 && d > 0, "bad shape");
  if (n == 0) return LNG_OK;
  LNG_REQUIRE(x && rs, "NULL pointer");
  const int g = grid_for(n * 32, 256, 16);
  if (x_dtype == LNG_F32) rms_rows_kernel<float><<<g, 256, 0, S(stream)>>>(static_cast<const float*>(x), n, d, eps, rs);
  else if (x_dtype == LNG_BF16)
    rms_rows_kernel<__nv_bfloat16><<<g, 256, 0, S(stream)>>>(static_cast<const __nv_bfloat16*>(x), n, d, eps, rs);
  else if (x_dtype == LNG_F16) rms_rows_kernel<__half><<<g, 256, 0, S(stream)>>>(static_cast<const __half*>(x), n, d, eps, rs);
  else return fail(LNG_ERR_ARGUMENT, "x dtype must be float");
  LNG_LAUNCHED("rms_rows_kernel");
  return LNG_OK;
}

extern "C" int lng_rms_norm(const void* x, int32_t x_dtype, int64_t n, int64_t d, const float* w, float eps, void* y,
                            int32_t y_dtype, lng_stream_t stream) {
  LNG_REQUIRE(n >= 0 && d > 0, "bad shape");
  if (n == 0) return LNG_OK;
  LNG_REQUIRE(x && y, "NULL pointer");
  const int xsz = x_dtype == LNG_F32 ? 4 : 2;
  const int64_t vec_elems = 32 * (16 / xsz);
  if (d % vec_elems == 0 && d / vec_elems <= RN_NV && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    // rows that fit in registers: one read of x
    const int nv = int(d / vec_elems);
    const unsigned gr = unsigned(ceil_div(n, 8));
#define LNG_RNR(XT, YT) \
  rms_norm_reg_kernel<XT, YT><<<gr, 256, 0, S(stream)>>>(static_cast<const XT*>(x), n, d, nv, w, eps, static_cast<YT*>(y))
    bool done = true;
    if (x_dtype == LNG_F32 && y_dtype == LNG_F32) LNG_RNR(float, float);
    else if (x_dtype == LNG_BF16 && y_dtype == LNG_BF16) LNG_RNR(__nv_bfloat16, __nv_bfloat16);
    else if (x_dtype == LNG_BF16 && y_dtype == LNG_F32) LNG_RNR(__nv_bfloat16, float);
    else if (x_dtype == LNG_F32 && y_dtype == LNG_BF16) LNG_RNR(float, __nv_bfloat16);
    else done = false;
#undef LNG_RNR
    if (done) {
      LNG_LAUNCHED("rms_norm_reg_kernel");
      return LNG_OK;
    }
  }
  const int g = grid_for(n * 32, 256, 16);
#define LNG_RN(XT, YT) rms_norm_kernel<XT, YT><<<g, 256, 0, S(stream)>>>(static_cast<const XT*>(x), n, d, w, eps, static_cast<YT*>(y))
  if (x_dtype == LNG_F32 && y_dtype == LNG_F32) LNG_RN(float, float);
  else if (x_dtype == LNG_BF16 && y_dtype == LNG_BF16) LNG_RN(__nv_bfloat16, __nv_bfloat16);
  else if (x_dtype == LNG_BF16 && y_dtype == LNG_F32) LNG_RN(__nv_bfloat16, float);
  else if (x_dtype == LNG_F32 && y_dtype == LNG_BF16) LNG_RN(float, __nv_bfloat16);
  else if (x_dtype == LNG_F16 && y_dtype == LNG_F16) LNG_RN(__half, __half);
  else if (x_dtype == LNG_F16 && y_dtype == LNG_F32) LNG_RN(__half, float);
  else return fail(LNG_ERR_UNSUPPORTED, "unsupported RMSNorm dtype combination");
#undef LNG_RN
  LNG_LAUNCHED("rms_norm_kernel");
  return LNG_OK;
}

extern "C" int lng_rms_norm_model(const void* x, int32_t x_dtype, int64_t n, int64_t d, const void* w,
                                  int32_t w_dtype, float eps, void* y, int32_t y_dtype, lng_stream_t stream) {
  LNG_REQUIRE(n >= 0 && d > 0, "bad shape");
  LNG_REQUIRE(x_dtype == LNG_F32 || x_dtype == LNG_BF16 || x_dtype == LNG_F16, "x dtype must be f32, bf16 or f16");
  LNG_REQUIRE(!w || w_dtype == LNG_F32 || w_dtype == LNG_BF16, "weight dtype must be f32 or bf16");
  LNG_REQUIRE(y_dtype == LNG_F32 || y_dtype == LNG_BF16 || y_dtype == LNG_F16, "y dtype must be f32, bf16 or f16");
  if (n == 0) return LNG_OK;
  LNG_REQUIRE(x && y, "NULL pointer");
  const int64_t xsz = x_dtype == LNG_F32 ? 4 : 2;
  const int64_t vec_elems = 32 * (16 / xsz);
  const bool reg = d % vec_elems == 0 && d / vec_elems <= RN_NV && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  const int nv = reg ? int(d / vec_elems) : 0;
  const unsigned gr = unsigned(ceil_div(n, 8));
  const int wb = w && w_dtype == LNG_BF16;
#define LNG_RM(XT) rms_norm_model_kernel<XT><<<gr, 256, 0, S(stream)>>>(static_cast<const XT*>(x), n, d, nv, w, wb, eps, y, y_dtype)
  if (x_dtype == LNG_F32) LNG_RM(float);
  else if (x_dtype == LNG_BF16) LNG_RM(__nv_bfloat16);
  else LNG_RM(__half);
#undef LNG_RM
  LNG_LAUNCHED("rms_norm_model_kernel");
  return LNG_OK;
}

static int check_readout(const lng_readout* ro) {
  LNG_REQUIRE(ro != nullptr, "readout descriptor is NULL");
  LNG_REQUIRE(ro->hidden > 0 && ro->num_heads > 0 && ro->num_kv_heads > 0 && ro->head_dim > 0, "bad readout shape");
  LNG_REQUIRE(ro->num_heads % ro->num_kv_heads == 0, "num_heads must be divisible by num_kv_heads");
  LNG_REQUIRE(ro->conv_kernel >= 1 && ro->conv_dilation >= 1, "bad conv shape");
  LNG_REQUIRE(ro->act_dtype == LNG_F32 || ro->act_dtype == LNG_BF16, "activation dtype must be f32 or bf16");
  LNG_REQUIRE(ro->conv_norm && ro->conv_weight, "conv weights are NULL");
  return LNG_OK;
}

// Stream-ordered scratch for entry points without a workspace argument, from a memory pool owned by
// the library (one per device) that keeps freed blocks for reuse instead of returning them to the
// driver at every synchronisation.
namespace {
std::mutex g_pool_mu;
cudaMemPool_t g_pools[64] = {};
}  // namespace
static int scratch_alloc(void** p, size_t bytes, cudaStream_t stream) {
  int dev = 0;
  LNG_CUDA(cudaGetDevice(&dev));
  LNG_REQUIRE(dev >= 0 && dev < 64, "device ordinal out of range for the scratch pool table");
  cudaMemPool_t pool;
  {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    if (!g_pools[dev]) {
      cudaMemPoolProps props{};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      LNG_CUDA(cudaMemPoolCreate(&g_pools[dev], &props));
      uint64_t keep = ~uint64_t(0);
      LNG_CUDA(cudaMemPoolSetAttribute(g_pools[dev], cudaMemPoolAttrReleaseThreshold, &keep));
    }
    pool = g_pools[dev];
  }
  LNG_CUDA(cudaMallocFromPoolAsync(p, bytes, pool, stream));
  return LNG_OK;
}

static ConvParams conv_params(const lng_readout* ro) {
  return ConvParams{ro->hidden, ro->conv_kernel, ro->conv_dilation, ro->conv_norm, ro->conv_weight, ro->conv_bias};
}

static int conv_finish_ws(const lng_readout* ro, const void* mixed, int64_t B, int64_t T, const int64_t* seg,
                          const uint8_t* valid, void* out, void* conv_in, float* rs, cudaStream_t stream) {
  const int64_t M = B * T;
  int st = lng_rms_rows(mixed, ro->act_dtype, M, ro->hidden, ro->eps, rs, reinterpret_cast<lng_stream_t>(stream));
  if (st) return st;
  const ConvParams cp = conv_params(ro);
  const bool al16 = (reinterpret_cast<uintptr_t>(mixed) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(conv_in) & 15) == 0;
  if (ro->conv_kernel == 4 && ro->conv_dilation <= 1024 && al16 && M < (int64_t(1) << 31) - (int64_t(1) << 20) &&
      ro->hidden % (ro->act_dtype == LNG_F32 ? 4 : 8) == 0 && (ro->act_dtype == LNG_F32 || ro->act_dtype == LNG_BF16)) {
    const int64_t chunks = ro->hidden / (ro->act_dtype == LNG_F32 ? 4 : 8);
    const int64_t run = int64_t(CS_RUN) * ro->conv_dilation;
    const dim3 grid(unsigned(ceil_div(M, run)), unsigned(ro->conv_dilation), unsigned(ceil_div(chunks, 128)));
    if (ro->act_dtype == LNG_F32)
      conv_stream_kernel<float, 4><<<grid, 128, 0, stream>>>(cp, static_cast<const float*>(mixed), rs, int(M), int(T),
                                                             seg, valid, static_cast<float*>(out),
                                                             static_cast<float*>(conv_in));
    else
      conv_stream_kernel<__nv_bfloat16, 4><<<grid, 128, 0, stream>>>(
          cp, static_cast<const __nv_bfloat16*>(mixed), rs, int(M), int(T), seg, valid,
          static_cast<__nv_bfloat16*>(out), static_cast<__nv_bfloat16*>(conv_in));
    LNG_LAUNCHED("conv_stream_kernel");
    return LNG_OK;
  }
  const int64_t groups = ro->hidden / 8;
  if (ro->hidden % 8 == 0 && groups <= 256 && 256 % groups == 0 && ro->conv_kernel <= 8 && M < (int64_t(1) << 31) &&
      (reinterpret_cast<uintptr_t>(mixed) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(conv_in) & 15) == 0) {
    const int ppb = 32;
    const unsigned grid = unsigned(ceil_div(M, ppb));
    if (ro->act_dtype == LNG_F32)
      conv_seq_vec_kernel<float, 8><<<grid, 256, 0, stream>>>(cp, static_cast<const float*>(mixed), rs, int(M), int(T),
                                                               seg, valid, static_cast<float*>(out),
                                                               static_cast<float*>(conv_in), ppb);
    else
      conv_seq_vec_kernel<__nv_bfloat16, 8><<<grid, 256, 0, stream>>>(
          cp, static_cast<const __nv_bfloat16*>(mixed), rs, int(M), int(T), seg, valid,
          static_cast<__nv_bfloat16*>(out), static_cast<__nv_bfloat16*>(conv_in), ppb);
    LNG_LAUNCHED("conv_seq_vec_kernel");
    return LNG_OK;
  }
  const int g = grid_for(M * ro->hidden, 256, 16);
  if (ro->act_dtype == LNG_F32)
    conv_seq_kernel<float><<<g, 256, 0, stream>>>(cp, static_cast<const float*>(mixed), rs, B, T, seg, valid,
                                                  static_cast<float*>(out), static_cast<float*>(conv_in));
  else
    conv_seq_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(cp, static_cast<const __nv_bfloat16*>(mixed), rs, B, T, seg,
                                                          valid, static_cast<__nv_bfloat16*>(out),
                                                          static_cast<__nv_bfloat16*>(conv_in));
  LNG_LAUNCHED("conv_seq_kernel");
  return LNG_OK;
}

extern "C" int lng_conv_finish(const lng_readout* ro, const void* mixed, int64_t B, int64_t T,
                               const int64_t* segment_ids, const uint8_t* valid_tokens, void* out, void* conv_in,
                               lng_stream_t stream) {
  int st = check_readout(ro);
  if (st) return st;
  LNG_REQUIRE(B >= 0 && T >= 0, "bad shape");
  if (B * T == 0) return LNG_OK;
  LNG_REQUIRE(mixed && out && mixed != out, "mixed and out must be distinct non-NULL buffers");
  float* rs = nullptr;
  st = scratch_alloc(reinterpret_cast<void**>(&rs), sizeof(float) * B * T, S(stream));
  if (st) return st;
  st = conv_finish_ws(ro, mixed, B, T, segment_ids, valid_tokens, out, conv_in, rs, S(stream));
  cudaFreeAsync(rs, S(stream));
  return st;
}

extern "C" int lng_conv_window(const lng_readout* ro, const void* mixed, int64_t n, void* cache,
                               const int64_t* new_slot, const int64_t* slot, void* out, lng_stream_t stream) {
  int st = check_readout(ro);
  if (st) return st;
  if (n <= 0) return LNG_OK;
  LNG_REQUIRE(mixed && cache && new_slot && slot && out, "NULL pointer");
  float* rs = nullptr;
  st = scratch_alloc(reinterpret_cast<void**>(&rs), sizeof(float) * n, S(stream));
  if (st) return st;
  st = lng_rms_rows(mixed, ro->act_dtype, n, ro->hidden, ro->eps, rs, stream);
  if (st) {
    cudaFreeAsync(rs, S(stream));
    return st;
  }
  const ConvParams cp = conv_params(ro);
  const int g = grid_for(n * ro->hidden, 256, 16);
  if (ro->act_dtype == LNG_F32) {
    conv_cache_write_kernel<float><<<g, 256, 0, S(stream)>>>(cp, static_cast<const float*>(mixed), rs, n, new_slot,
                                                              static_cast<float*>(cache));
    conv_window_kernel<float><<<g, 256, 0, S(stream)>>>(cp, static_cast<const float*>(mixed), n,
                                                         static_cast<const float*>(cache), slot, static_cast<float*>(out));
  } else {
    conv_cache_write_kernel<__nv_bfloat16><<<g, 256, 0, S(stream)>>>(
        cp, static_cast<const __nv_bfloat16*>(mixed), rs, n, new_slot, static_cast<__nv_bfloat16*>(cache));
    conv_window_kernel<__nv_bfloat16><<<g, 256, 0, S(stream)>>>(cp, static_cast<const __nv_bfloat16*>(mixed), n,
                                                                 static_cast<const __nv_bfloat16*>(cache), slot,
                                                                 static_cast<__nv_bfloat16*>(out));
  }
  cudaFreeAsync(rs, S(stream));
  LNG_LAUNCHED("conv_window_kernel");
  return LNG_OK;
}

extern "C" int lng_sink_gqa(const void* q, const void* k, const void* v, int32_t dtype, int64_t M, int32_t num_kv_heads,
                            int32_t groups, int64_t routes, int32_t head_dim, float sink_logit, void* out,
                            lng_stream_t stream) {
  LNG_REQUIRE(M >= 0 && num_kv_heads > 0 && groups > 0 && routes > 0 && head_dim > 0, "bad shape");
  if (M == 0) return LNG_OK;
  LNG_REQUIRE(q && k && v && out, "NULL pointer");
  const size_t smem = sizeof(float) * (2 * size_t(routes) * head_dim + size_t(groups) * head_dim + size_t(groups) * routes);
  LNG_REQUIRE(smem <= 227 * 1024, "routes * head_dim too large for the explicit-K/V readout");
  const float scale = 1.0f / sqrtf(float(head_dim));
  const unsigned grid = unsigned(M * num_kv_heads);
#define LNG_SG(T)                                                                                          \
  do {                                                                                                     \
    auto kern = sink_gqa_kernel<T>;                                                                        \
    LNG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));          \
    kern<<<grid, 128, smem, S(stream)>>>(static_cast<const T*>(q), static_cast<const T*>(k),               \
                                         static_cast<const T*>(v), M, num_kv_heads, groups, int(routes),    \
                                         head_dim, scale, sink_logit, static_cast<T*>(out));               \
  } while (0)
  if (dtype == LNG_F32) LNG_SG(float);
  else if (dtype == LNG_BF16) LNG_SG(__nv_bfloat16);
  else if (dtype == LNG_F16) LNG_SG(__half);
  else return fail(LNG_ERR_ARGUMENT, "dtype must be float");
#undef LNG_SG
  LNG_LAUNCHED("sink_gqa_kernel");
  return LNG_OK;
}

// ====================================================================== fold / memory forward
extern "C" int lng_fold_readout(int64_t d, int64_t Dt, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                const float* q_norm, const float* q_proj, const float* mem_norm, const float* kv_proj,
                                const float* o_proj, void* w_qk, void* w_vo, int32_t act_dtype, lng_stream_t stream) {
  LNG_REQUIRE(d > 0 && Dt > 0 && num_heads > 0 && num_kv_heads > 0 && head_dim > 0, "bad readout shape");
  LNG_REQUIRE(num_heads % num_kv_heads == 0, "num_heads must be divisible by num_kv_heads");
  LNG_REQUIRE(act_dtype == LNG_F32 || act_dtype == LNG_BF16 || act_dtype == LNG_F16, "bad activation dtype");
  LNG_REQUIRE(mem_norm && kv_proj, "NULL pointer");
  const int G = num_heads / num_kv_heads;
  const float scale = 1.0f / sqrtf(float(head_dim));
  if (w_qk) {
    LNG_REQUIRE(q_norm && q_proj, "NULL pointer");
    const int g = grid_for(int64_t(num_heads) * Dt * d, 256, 16);
#define LNG_FQ(OT) fold_qk_kernel<OT><<<g, 256, 0, S(stream)>>>(d, Dt, num_heads, G, head_dim, scale, q_norm, q_proj, mem_norm, kv_proj, static_cast<OT*>(w_qk))
    if (act_dtype == LNG_F32) LNG_FQ(float); else if (act_dtype == LNG_BF16) LNG_FQ(__nv_bfloat16); else LNG_FQ(__half);
#undef LNG_FQ
    LNG_LAUNCHED("fold_qk_kernel");
  }
  if (w_vo) {
    LNG_REQUIRE(o_proj, "NULL pointer");
    const int g = grid_for(d * num_heads * Dt, 256, 16);
#define LNG_FV(OT) fold_vo_kernel<OT><<<g, 256, 0, S(stream)>>>(d, Dt, num_heads, G, head_dim, num_kv_heads, mem_norm, kv_proj, o_proj, static_cast<OT*>(w_vo))
    if (act_dtype == LNG_F32) LNG_FV(float); else if (act_dtype == LNG_BF16) LNG_FV(__nv_bfloat16); else LNG_FV(__half);
#undef LNG_FV
    LNG_LAUNCHED("fold_vo_kernel");
  }
  return LNG_OK;
}

namespace {
struct FwdLayout {
  size_t codes, qa, u, mixed, rs_h, rs_m, total;
};
FwdLayout fwd_layout(const lng_tables* t, const lng_readout* ro, int64_t M) {
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  const int64_t Dt = int64_t(t->n_orders) * t->memory_dim;
  const size_t es = size_t(dtype_size(ro->act_dtype));
  FwdLayout L{};
  size_t off = 0;
  L.codes = off; off += al(size_t(M) * t->num_routes);
  L.qa = off;    off += al(size_t(M) * ro->num_heads * Dt * es);
  L.u = off;     off += al(size_t(M) * ro->num_heads * Dt * es);
  L.mixed = off; off += al(size_t(M) * ro->hidden * es);
  L.rs_h = off;  off += al(size_t(M) * sizeof(float));
  L.rs_m = off;  off += al(size_t(M) * sizeof(float));
  L.total = off;
  return L;
}
}  // namespace

extern "C" size_t lng_memory_workspace_bytes(const lng_tables* tables, const lng_readout* ro, int64_t M) {
  if (!tables || !ro || M < 0) return 0;
  return fwd_layout(tables, ro, M).total;
}

extern "C" int lng_memory_forward(const lng_tables* tables, const lng_readout* ro, int64_t B, int64_t T, const void* h,
                                  const void* router_x, int32_t router_x_dtype, const void* codes_in,
                                  int32_t codes_in_dtype, const int64_t* segment_ids, const uint8_t* valid_tokens,
                                  void* out, uint8_t* codes_out, void* workspace, size_t workspace_bytes,
                                  lng_stream_t stream) {
  int st = check_tables(tables);
  if (st) return st;
  st = check_readout(ro);
  if (st) return st;
  LNG_REQUIRE(B >= 0 && T >= 0, "bad shape");
  const int64_t M = B * T;
  if (M == 0) return LNG_OK;
  LNG_REQUIRE(h && out && ro->w_qk && ro->w_vo, "NULL pointer");
  LNG_REQUIRE(tables->table_dtype == ro->act_dtype || tables->table_dtype == LNG_F32 ||
                  (ro->act_dtype == LNG_F32),
              "tables and activations must share a dtype (or be fp32)");
  const FwdLayout L = fwd_layout(tables, ro, M);
  LNG_REQUIRE(workspace && workspace_bytes >= L.total, "workspace too small (see lng_memory_workspace_bytes)");
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const int64_t Dt = int64_t(tables->n_orders) * tables->memory_dim;
  const int64_t QD = int64_t(ro->num_heads) * Dt;
  const int act = ro->act_dtype;
  // 1. codes
  const void* codes = codes_in;
  int32_t cdt = codes_in_dtype;
  if (!codes) {
    LNG_REQUIRE(router_x && ro->router_w, "router input and weight are needed when codes are not given");
    uint8_t* c = codes_out ? codes_out : reinterpret_cast<uint8_t*>(ws + L.codes);
    if (router_x_dtype == LNG_BF16 && ro->router_w_split && tables->bits <= 6 && ro->router_in_dim % TC_BK == 0)
      st = lng_route_codes_split(router_x, M, ro->router_in_dim, ro->router_in_dim, ro->router_w_split,
                                 tables->num_routes, tables->bits, c, stream);
    else
      st = lng_route_codes(router_x, router_x_dtype, M, ro->router_in_dim, ro->router_in_dim, ro->router_w,
                           tables->num_routes, tables->bits, c, LNG_U8, nullptr, stream);
    if (st) return st;
    codes = c;
    cdt = LNG_U8;
  }
  // 2. query scale 1/rms(h) and the folded query qa = h . w_qk^T
  float* rs_h = reinterpret_cast<float*>(ws + L.rs_h);
  st = lng_rms_rows(h, act, M, ro->hidden, ro->eps, rs_h, stream);
  if (st) return st;
  void* qa = ws + L.qa;
  st = lng_gemm(h, act, ro->hidden, ro->w_qk, act, ro->hidden, qa, act, QD, M, QD, ro->hidden, nullptr, 0, stream);
  if (st) return st;
  // 3. fused gather + sink attention over all routes
  void* u = ws + L.u;
  st = lng_route_attend(tables, codes, cdt, B, T, 0, segment_ids, valid_tokens, nullptr, 0, 0, tables->num_routes,
                        ro->num_heads, ro->eps, ro->sink_logit, qa, rs_h, u, act, 0, nullptr, nullptr, stream);
  if (st) return st;
  // 4. mixed = u . w_vo^T  (= o_proj(head))
  void* mixed = ws + L.mixed;
  st = lng_gemm(u, act, QD, ro->w_vo, act, QD, mixed, act, ro->hidden, M, ro->hidden, QD, nullptr, 0, stream);
  if (st) return st;
  // 5. out = mixed + SiLU(conv(RMSNorm(mixed))), masked by valid_tokens
  return conv_finish_ws(ro, mixed, B, T, segment_ids, valid_tokens, out, nullptr, reinterpret_cast<float*>(ws + L.rs_m),
                        S(stream));
}

namespace {
struct TreeLayout {
  size_t ctx, rs, qa, u, mixed, total;
};
TreeLayout tree_layout(const lng_tables* t, const lng_readout* ro, int64_t B, int64_t n, int64_t W) {
  const int64_t M = B * n, Dt = int64_t(t->n_orders) * t->memory_dim;
  const size_t es = size_t(dtype_size(ro->act_dtype));
  TreeLayout L{};
  size_t off = 0;
  L.ctx = off;   off += al256(size_t(M) * W * t->num_routes);
  L.rs = off;    off += al256(size_t(M) * 4);
  L.qa = off;    off += al256(size_t(M) * ro->num_heads * Dt * es);
  L.u = off;     off += al256(size_t(M) * ro->num_heads * Dt * es);
  L.mixed = off; off += al256(size_t(M) * ro->hidden * es);
  L.total = off;
  return L;
}
}  // namespace

extern "C" size_t lng_tree_workspace_bytes(const lng_tables* tables, const lng_readout* ro, int64_t B, int64_t n,
                                           int64_t W) {
  if (!tables || !ro || B < 0 || n < 0 || W < 1) return 0;
  return tree_layout(tables, ro, B, n, W).total;
}

extern "C" int lng_tree_memory_block(const lng_tables* tables, const lng_readout* ro, int64_t B, int64_t n, int64_t W,
                                     int64_t L, int64_t h0, int64_t max_len, const void* h, const uint8_t* codes_new,
                                     uint8_t* cache_codes, void* cache_conv, const int64_t* gidx, const uint8_t* gok,
                                     const int32_t* seg, const int64_t* slot, const int64_t* new_slot, void* out,
                                     void* workspace, size_t workspace_bytes, lng_stream_t stream) {
  int st = check_tables(tables);
  if (st) return st;
  st = check_readout(ro);
  if (st) return st;
  LNG_REQUIRE(B >= 0 && n >= 0 && W >= 1 && L >= 0 && h0 >= 0 && h0 <= L && L + n <= max_len, "bad tree shape");
  const int64_t M = B * n;
  if (M == 0) return LNG_OK;
  LNG_REQUIRE(h && codes_new && cache_codes && cache_conv && gidx && gok && seg && slot && new_slot && out && ro->w_qk &&
                  ro->w_vo, "NULL pointer");
  const TreeLayout Ly = tree_layout(tables, ro, B, n, W);
  LNG_REQUIRE(workspace && workspace_bytes >= Ly.total, "workspace too small (see lng_tree_workspace_bytes)");
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const int64_t R = tables->num_routes, Dt = int64_t(tables->n_orders) * tables->memory_dim;
  const int64_t QD = int64_t(ro->num_heads) * Dt;
  const int act = ro->act_dtype;
  cudaStream_t s = S(stream);
  uint8_t* ctx = ws + Ly.ctx;
  tree_windows_kernel<<<grid_for(M * (W + 1) * R, 256, 8), 256, 0, s>>>(codes_new, cache_codes, B, n, W, R, L, h0,
                                                                        max_len, gidx, gok, ctx);
  LNG_LAUNCHED("tree_windows_kernel");
  float* rs = reinterpret_cast<float*>(ws + Ly.rs);
  st = lng_rms_rows(h, act, M, ro->hidden, ro->eps, rs, stream);
  if (st) return st;
  void* qa = ws + Ly.qa;
  st = lng_gemm(h, act, ro->hidden, ro->w_qk, act, ro->hidden, qa, act, QD, M, QD, ro->hidden, nullptr, 0, stream);
  if (st) return st;
  void* u = ws + Ly.u;
  st = lng_route_attend(tables, ctx, LNG_U8, M, 0, W, nullptr, nullptr, seg, 0, 0, R, ro->num_heads, ro->eps,
                        ro->sink_logit, qa, rs, u, act, 0, nullptr, nullptr, stream);
  if (st) return st;
  void* mixed = ws + Ly.mixed;
  st = lng_gemm(u, act, QD, ro->w_vo, act, QD, mixed, act, ro->hidden, M, ro->hidden, QD, nullptr, 0, stream);
  if (st) return st;
  return lng_conv_window(ro, mixed, M, cache_conv, new_slot, slot, out, stream);
}

extern "C" int lng_attend_rescale(const float* m_local, const float* m_glob, float* l, float* u, int64_t M,
                                  int32_t num_heads, int64_t Dt, lng_stream_t stream) {
  LNG_REQUIRE(M >= 0 && num_heads > 0 && Dt > 0, "bad shape");
  if (M == 0) return LNG_OK;
  LNG_REQUIRE(m_local && m_glob && l && u, "NULL pointer");
  const int64_t MQ = M * num_heads;
  attend_rescale_kernel<<<grid_for(MQ * Dt, 256, 16), 256, 0, S(stream)>>>(m_local, m_glob, l, u, MQ, Dt);
  LNG_LAUNCHED("attend_rescale_kernel");
  return LNG_OK;
}

extern "C" int lng_attend_normalize(const float* l, const float* u, int64_t M, int32_t num_heads, int64_t Dt,
                                    void* u_out, int32_t u_dtype, lng_stream_t stream) {
  LNG_REQUIRE(M >= 0 && num_heads > 0 && Dt > 0, "bad shape");
  if (M == 0) return LNG_OK;
  LNG_REQUIRE(l && u && u_out, "NULL pointer");
  const int64_t MQ = M * num_heads;
  const int g = grid_for(MQ * Dt, 256, 16);
  if (u_dtype == LNG_F32) attend_normalize_kernel<float><<<g, 256, 0, S(stream)>>>(l, u, MQ, Dt, static_cast<float*>(u_out));
  else if (u_dtype == LNG_BF16)
    attend_normalize_kernel<__nv_bfloat16><<<g, 256, 0, S(stream)>>>(l, u, MQ, Dt, static_cast<__nv_bfloat16*>(u_out));
  else return fail(LNG_ERR_ARGUMENT, "u dtype must be f32 or bf16");
  LNG_LAUNCHED("attend_normalize_kernel");
  return LNG_OK;
}

extern "C" int lng_attend_pack(const float* m_local, const float* m_glob, const float* l, const float* o, int64_t M,
                               int32_t num_heads, int32_t head_dim, void* pack, int32_t pack_dtype, lng_stream_t stream) {
  LNG_REQUIRE(M >= 0 && num_heads > 0 && head_dim > 0, "bad shape");
  if (M == 0) return LNG_OK;
  LNG_REQUIRE(m_local && m_glob && l && o && pack, "NULL pointer");
  const int64_t MQ = M * num_heads;
  const int g = grid_for(MQ * (head_dim + 1), 256, 16);
  if (pack_dtype == LNG_F32)
    attend_pack_kernel<float><<<g, 256, 0, S(stream)>>>(m_local, m_glob, l, o, MQ, head_dim, static_cast<float*>(pack));
  else if (pack_dtype == LNG_BF16)
    attend_pack_kernel<__nv_bfloat16><<<g, 256, 0, S(stream)>>>(m_local, m_glob, l, o, MQ, head_dim,
                                                                static_cast<__nv_bfloat16*>(pack));
  else
    return fail(LNG_ERR_ARGUMENT, "pack dtype must be f32 or bf16");
  LNG_LAUNCHED("attend_pack_kernel");
  return LNG_OK;
}

extern "C" int lng_attend_unpack(const void* pack, int32_t pack_dtype, int64_t M, int32_t num_heads, int32_t head_dim,
                                 void* head, int32_t dtype, lng_stream_t stream) {
  LNG_REQUIRE(M >= 0 && num_heads > 0 && head_dim > 0, "bad shape");
  if (M == 0) return LNG_OK;
  LNG_REQUIRE(pack && head, "NULL pointer");
  LNG_REQUIRE(pack_dtype == LNG_F32 || pack_dtype == LNG_BF16, "pack dtype must be f32 or bf16");
  LNG_REQUIRE(dtype == LNG_F32 || dtype == LNG_BF16, "head dtype must be f32 or bf16");
  const int64_t MQ = M * num_heads;
  const int g = grid_for(MQ * head_dim, 256, 16);
#define LNG_UNPACK(PT, OT) \
  attend_unpack_kernel<PT, OT><<<g, 256, 0, S(stream)>>>(static_cast<const PT*>(pack), MQ, head_dim, static_cast<OT*>(head))
  if (pack_dtype == LNG_F32) {
    if (dtype == LNG_F32) LNG_UNPACK(float, float); else LNG_UNPACK(float, __nv_bfloat16);
  } else {
    if (dtype == LNG_F32) LNG_UNPACK(__nv_bfloat16, float); else LNG_UNPACK(__nv_bfloat16, __nv_bfloat16);
  }
#undef LNG_UNPACK
  LNG_LAUNCHED("attend_unpack_kernel");
  return LNG_OK;
}

extern "C" int lng_attend_pack_rescale(const float* m_local, const float* m_glob, int64_t M, int32_t num_heads,
                                       int32_t head_dim, void* pack, int32_t pack_dtype, lng_stream_t stream) {
  LNG_REQUIRE(M >= 0 && num_heads > 0 && head_dim > 0, "bad shape");
  if (M == 0) return LNG_OK;
  LNG_REQUIRE(m_local && m_glob && pack, "NULL pointer");
  const int64_t MQ = M * num_heads;
  const int g = grid_for(MQ, 256, 16);
  if (pack_dtype == LNG_F32)
    attend_pack_rescale_kernel<float><<<g, 256, 0, S(stream)>>>(m_local, m_glob, MQ, head_dim, static_cast<float*>(pack));
  else if (pack_dtype == LNG_BF16)
    attend_pack_rescale_kernel<__nv_bfloat16><<<g, 256, 0, S(stream)>>>(m_local, m_glob, MQ, head_dim,
                                                                        static_cast<__nv_bfloat16*>(pack));
  else
    return fail(LNG_ERR_ARGUMENT, "pack dtype must be f32 or bf16");
  LNG_LAUNCHED("attend_pack_rescale_kernel");
  return LNG_OK;
}

// ====================================================================== logits top-k
namespace {
size_t topk_cand_bytes(int64_t n, int64_t vocab, int32_t k) {
  return size_t(n) * ceil_div(vocab, TK_VC) * k * (sizeof(float) + sizeof(int64_t));
}
// The tensor-core path applies to a bf16 vocabulary matrix whose shapes meet the TMA rules.
bool logits_tc_ok(int64_t d, const void* embedding, int32_t e_dtype, int64_t vocab) {
  return e_dtype == LNG_BF16 && d % TC_BK == 0 && (reinterpret_cast<uintptr_t>(embedding) & 15) == 0 &&
         vocab < (int64_t(1) << 31);
}
size_t split_rows_bytes(int64_t n, int64_t d) { return size_t(n) * 3 * d * sizeof(__nv_bfloat16); }
}  // namespace

extern "C" size_t lng_logits_topk_scratch_bytes(int64_t n, int64_t d, int64_t vocab, int32_t k) {
  if (n <= 0 || d <= 0 || vocab <= 0 || k <= 0) return 0;
  // candidates, then (256-byte aligned) the three bf16 parts of h for the tensor cores
  return al256(topk_cand_bytes(n, vocab, k) + 256) + split_rows_bytes(n, d) + 256;
}

namespace {
// Per-tile candidates [n, ceil(vocab / 256), k] of h . E^T: the tcgen05 kernel (draft rows split
// into `split`, 16-byte aligned, n * 3d bf16) when `split` is given and the vocabulary matrix is
// bf16 with TMA-compatible shapes, the CUDA-core kernel otherwise.
int logits_chunks(const float* h, int64_t n, int64_t d, const void* embedding, int32_t e_dtype, int64_t vocab,
                  int32_t k, float* cand_v, int64_t* cand_i, float* logits, __nv_bfloat16* split,
                  cudaStream_t stream, bool presplit = false, bool dependent = false) {
  const int64_t nch = ceil_div(vocab, TK_VC);
  if (split && logits_tc_ok(d, embedding, e_dtype, vocab)) {
    if (!presplit) {  // presplit: the caller wrote the three parts of h to `split` already
      split_rows_bf16x3_kernel<<<grid_for(n * d, 256, 16), 256, 0, stream>>>(h, n, d, split);
      LNG_LAUNCHED("split_rows_bf16x3_kernel");
    }
    const int bn = n <= 32 ? 32 : n <= 64 ? 64 : 128;
    CUtensorMap te, th;
    int st = make_tmap_bf16(&te, embedding, vocab, d, d, LT_BM);
    if (st) return st;
    st = make_tmap_bf16(&th, split, n, 3 * d, 3 * d, bn);
    if (st) return st;
    dim3 grid(unsigned(ceil_div(n, bn)), unsigned(nch));
    // dependent: a programmatic dependent launch -- the kernel's start (set-up, first vocabulary tiles)
    // overlaps the kernel before it, which writes the split rows (griddepcontrol in both)
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
#define LNG_LT(BN)                                                                                          \
  do {                                                                                                      \
    auto kern = logits_tc_topk_kernel<BN>;                                                                  \
    LNG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(LtCfg<BN>::SMEM))); \
    if (dependent) {                                                                                        \
      cudaLaunchConfig_t cfg{};                                                                             \
      cfg.gridDim = grid;                                                                                   \
      cfg.blockDim = dim3(128);                                                                             \
      cfg.dynamicSmemBytes = LtCfg<BN>::SMEM;                                                               \
      cfg.stream = stream;                                                                                  \
      cfg.attrs = pdl;                                                                                      \
      cfg.numAttrs = 1;                                                                                     \
      LNG_CUDA(cudaLaunchKernelEx(&cfg, kern, te, th, n, d, vocab, k, cand_v, cand_i, logits));              \
    } else {                                                                                                \
      kern<<<grid, 128, LtCfg<BN>::SMEM, stream>>>(te, th, n, d, vocab, k, cand_v, cand_i, logits);           \
    }                                                                                                       \
  } while (0)
    if (bn == 32) LNG_LT(32);
    else if (bn == 64) LNG_LT(64);
    else LNG_LT(128);
#undef LNG_LT
    LNG_LAUNCHED("logits_tc_topk_kernel");
    return LNG_OK;
  }
  const size_t smem = sizeof(float) * (size_t(TK_ROWS) * d + size_t(TK_ROWS) * TK_VC);
  LNG_REQUIRE(smem <= 227 * 1024, "hidden size too large for the top-k kernel");
  dim3 grid(unsigned(nch), unsigned(ceil_div(n, TK_ROWS)));
#define LNG_TK(ET)                                                                                         \
  do {                                                                                                     \
    auto kern = logits_chunk_topk_kernel<ET>;                                                              \
    LNG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));          \
    kern<<<grid, 256, smem, stream>>>(h, n, d, static_cast<const ET*>(embedding), vocab, k, cand_v, cand_i, logits); \
  } while (0)
  if (e_dtype == LNG_F32) LNG_TK(float);
  else if (e_dtype == LNG_BF16) LNG_TK(__nv_bfloat16);
  else if (e_dtype == LNG_F16) LNG_TK(__half);
  else return fail(LNG_ERR_ARGUMENT, "embedding dtype must be float");
#undef LNG_TK
  LNG_LAUNCHED("logits_chunk_topk_kernel");
  return LNG_OK;
}
}  // namespace

extern "C" int lng_logits_topk(const float* h, int64_t n, int64_t d, const void* embedding, int32_t e_dtype,
                               int64_t vocab, int32_t k, int64_t* ids, float* vals, float* logits, void* scratch,
                               size_t scratch_bytes, lng_stream_t stream) {
  LNG_REQUIRE(n >= 0 && d > 0 && vocab > 0, "bad shape");
  LNG_REQUIRE(k >= 1 && k <= TK_MAXK, "k must be in [1, 8]");
  if (n == 0) return LNG_OK;
  LNG_REQUIRE(h && embedding && ids && vals, "NULL pointer");
  const int64_t nch = ceil_div(vocab, TK_VC);
  const size_t need = lng_logits_topk_scratch_bytes(n, d, vocab, k);
  LNG_REQUIRE(scratch && scratch_bytes >= need, "scratch too small (see lng_logits_topk_scratch_bytes)");
  uintptr_t base = (reinterpret_cast<uintptr_t>(scratch) + 255) & ~uintptr_t(255);
  int64_t* cand_i = reinterpret_cast<int64_t*>(base);
  float* cand_v = reinterpret_cast<float*>(cand_i + n * nch * k);
  auto* split = reinterpret_cast<__nv_bfloat16*>(base + al256(topk_cand_bytes(n, vocab, k)));
  int st = logits_chunks(h, n, d, embedding, e_dtype, vocab, k, cand_v, cand_i, logits, split, S(stream));
  if (st) return st;
  topk_merge_kernel<<<unsigned(ceil_div(n * 32, 256)), 256, 0, S(stream)>>>(cand_v, cand_i, n, nch, k, ids, vals);
  LNG_LAUNCHED("topk_merge_kernel");
  return LNG_OK;
}

// ====================================================================== allocation-free top-k
// Some callers cannot allocate device memory at the point where they draft: code running inside a
// captured or replayed CUDA graph, or a serving process whose allocator hands out no memory
// outside its own pools.  For them, lng_logits_topk_static runs the same two kernels as
// lng_logits_topk with the candidate scratch in this file-scope device array instead of a caller
// buffer.  The array is part of the library image: every GPU that loads the library holds its
// 4 MiB until the process exits.
static constexpr size_t kTopkStaticScratchBytes = size_t(4) << 20;
static __device__ __align__(256) unsigned char g_topk_static_scratch[kTopkStaticScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_topk_static_mu;
void* g_topk_static_base[kMaxDevices] = {};  // device address of the array, per device ordinal
}  // namespace

extern "C" int lng_logits_topk_static(const float* h, int64_t n, int64_t d, const void* embedding, int32_t e_dtype,
                                      int64_t vocab, int32_t k, int64_t* ids, float* vals, float* logits,
                                      lng_stream_t stream) {
  LNG_REQUIRE(n >= 0 && d > 0 && vocab > 0, "bad shape");
  LNG_REQUIRE(k >= 1 && k <= TK_MAXK, "k must be in [1, 8]");
  if (n == 0) return LNG_OK;
  LNG_REQUIRE(h && embedding && ids && vals, "NULL pointer");
  // candidates, plus the split draft rows when the tensor-core path applies
  const bool tc = logits_tc_ok(d, embedding, e_dtype, vocab);
  const size_t cand = al256(topk_cand_bytes(n, vocab, k));
  const size_t need = cand + (tc ? split_rows_bytes(n, d) : 0) + 256;
  if (need > kTopkStaticScratchBytes)
    return fail(LNG_ERR_ARGUMENT, "lng_logits_topk_static: n * ceil(vocab / 256) * k * 12 bytes" +
                                      std::string(tc ? " + n * d * 6 bytes (split rows)" : "") + " (+256) = " +
                                      std::to_string(need) + " exceeds the 4 MiB static scratch (" +
                                      std::to_string(kTopkStaticScratchBytes) +
                                      " bytes); use lng_logits_topk with a caller-provided buffer");
  int dev = 0;
  LNG_CUDA(cudaGetDevice(&dev));
  LNG_REQUIRE(dev >= 0 && dev < kMaxDevices, "device ordinal out of range for the static scratch table");
  void* base = nullptr;
  {
    // first call on a device: resolve the array's device address with that device current
    std::lock_guard<std::mutex> lock(g_topk_static_mu);
    if (!g_topk_static_base[dev]) {
      void* p = nullptr;
      LNG_CUDA(cudaGetSymbolAddress(&p, g_topk_static_scratch));
      g_topk_static_base[dev] = p;
    }
    base = g_topk_static_base[dev];
  }
  const int64_t nch = ceil_div(vocab, TK_VC);
  int64_t* cand_i = static_cast<int64_t*>(base);  // 256-byte aligned: no extra alignment step needed
  float* cand_v = reinterpret_cast<float*>(cand_i + n * nch * k);
  auto* split = tc ? reinterpret_cast<__nv_bfloat16*>(static_cast<unsigned char*>(base) + cand) : nullptr;
  int st = logits_chunks(h, n, d, embedding, e_dtype, vocab, k, cand_v, cand_i, logits, split, S(stream));
  if (st) return st;
  topk_merge_kernel<<<unsigned(ceil_div(n * 32, 256)), 256, 0, S(stream)>>>(cand_v, cand_i, n, nch, k, ids, vals);
  LNG_LAUNCHED("topk_merge_kernel (static scratch)");
  return LNG_OK;
}

// ====================================================================== online counts (acceptance harness)
extern "C" int lng_online_counts_mix(const int64_t* codes, int64_t T, int64_t R, const int32_t* orders_host,
                                     int32_t n_orders, int32_t bits, const int64_t* x, const int64_t* win,
                                     const uint8_t* real, int64_t N, int64_t W, const int64_t* deadline, const float* p,
                                     int64_t V, float kappa, float* out, lng_stream_t stream) {
  LNG_REQUIRE(T >= 0 && R > 0 && N >= 0 && V > 0 && W >= 1, "bad online-counts shape");
  LNG_REQUIRE(n_orders >= 1 && n_orders <= OC_MAX_ORDERS && orders_host, "n_orders must be in [1, 8]");
  LNG_REQUIRE(bits >= 1 && bits <= 16, "bits must be in [1, 16]");
  OnlineParams op{};
  for (int o = 0; o < n_orders; ++o) {
    LNG_REQUIRE(orders_host[o] >= 1 && orders_host[o] <= 8 && orders_host[o] <= W && int64_t(bits) * orders_host[o] <= 40,
                "orders must be in [1, min(8, W)] with bits x order <= 40");
    op.orders[o] = orders_host[o];
  }
  if (N == 0) return LNG_OK;
  LNG_REQUIRE(p && out && win && real && deadline, "NULL pointer");
  cudaStream_t s = S(stream);
  if (T < 2) {  // no verified pair: out = p
    if (out != p) LNG_CUDA(cudaMemcpyAsync(out, p, size_t(N * V) * 4, cudaMemcpyDeviceToDevice, s));
    return LNG_OK;
  }
  LNG_REQUIRE(codes && x, "NULL pointer");
  op.codes = codes;
  op.T = T;
  op.R = R;
  op.n_orders = n_orders;
  op.bits = bits;
  op.x = x;
  op.win = win;
  op.real = real;
  op.N = N;
  op.W = W;
  op.deadline = deadline;
  op.V = V;
  const int64_t T1 = T - 1;
  const size_t keys_b = al256(size_t(n_orders) * T1 * R * 8), q_b = al256(size_t(n_orders) * N * R * 8),
               tot_b = al256(size_t(N) * 4), sc_b = size_t(N) * V * 4;
  // p and out may alias: the votes go to a scratch of their own then
  const bool alias = p == out;
  void* buf = nullptr;
  int st = scratch_alloc(&buf, keys_b + q_b + tot_b + (alias ? sc_b : 0), s);
  if (st) return st;
  auto* keys = static_cast<int64_t*>(buf);
  auto* q = reinterpret_cast<int64_t*>(static_cast<unsigned char*>(buf) + keys_b);
  auto* tot = reinterpret_cast<float*>(static_cast<unsigned char*>(buf) + keys_b + q_b);
  float* sc = alias ? reinterpret_cast<float*>(static_cast<unsigned char*>(buf) + keys_b + q_b + tot_b) : out;
  cudaError_t e = cudaMemsetAsync(tot, 0, size_t(N) * 4, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(sc, 0, sc_b, s);
  if (e == cudaSuccess) {
    online_keys_kernel<<<grid_for(int64_t(n_orders) * T1 * R, 256, 8), 256, 0, s>>>(op, keys);
    online_queries_kernel<<<grid_for(int64_t(n_orders) * N * R, 256, 8), 256, 0, s>>>(op, q);
    const dim3 g(unsigned(std::min<int64_t>(ceil_div(T1, 128), 1024)), unsigned(N));
    online_votes_kernel<<<g, 128, 0, s>>>(op, keys, q, tot, sc);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && alias) {
    // the mix reads p and the votes element by element: move the votes into out after p is read
    online_mix_kernel<<<grid_for(N * V, 256, 8), 256, 0, s>>>(p, tot, N, V, float(R * n_orders), kappa, sc);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, sc, sc_b, cudaMemcpyDeviceToDevice, s);
  } else if (e == cudaSuccess) {
    online_mix_kernel<<<grid_for(N * V, 256, 8), 256, 0, s>>>(p, tot, N, V, float(R * n_orders), kappa, out);
    e = cudaGetLastError();
  }
  cudaFreeAsync(buf, s);
  if (e != cudaSuccess) return cuda_status(e, "online counts");
  return LNG_OK;
}

#include "drafter.cuh"
