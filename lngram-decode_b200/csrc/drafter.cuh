// GPU drafter: the state machine and API of the reference C++ drafter
// (drafting/cpu/drafter.cpp:150-595) with every per-token step on the device.
//
// Per token x[t] (the reference's drafting/cpu_drafter.py:1-33 steps 1-6, full vocabulary):
//   embed2 router features -> fp32 router -> sign codes (lng_embed2_features, lng_route_codes);
//   rows of the n-grams ending at t (window of the last max(ngrams) codes, zero rows before the
//   sequence start); the draft readout in folded form (w_qk / w_vo from W_q, the memory's norm +
//   kv_proj, W_o), RMSNorm(out_norm); logits against the embedding with a fused top-k.
// draft() keeps the drafted tokens on the device: step i+1 reads step i's argmax from device memory,
// so a gamma-token draft costs one host round trip at the end.  The committed state (tokens, codes)
// lives on the host, as in the reference, so truncate() is exact rollback.
#pragma once

namespace lng {

template <typename T>
__global__ void gather_rows_kernel(const int64_t* __restrict__ ids, int64_t n, const T* __restrict__ src, int64_t d,
                                   int64_t vocab, T* __restrict__ out) {
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n * d; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = e / d, j = e % d;
    const int64_t id = ids[i];
    if (id < 0 || id >= vocab) {
      if (j == 0) atomicCAS(&g_error_word, 0u, (unsigned int)DEV_ERR_TOKEN_RANGE);
      out[e] = from_f32<T>(0.f);
    } else {
      out[e] = src[id * d + j];
    }
  }
}

// dst[i] = src[i] (device scalars), used to chain a drafted token into the next step.
__global__ void copy_i64_kernel(const int64_t* __restrict__ src, int64_t* __restrict__ dst, int64_t n,
                                int64_t src_stride, int64_t dst_stride) {
  const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i < n) dst[i * dst_stride] = src[i * src_stride];
}

// The drafted tokens of one step: ids[s] -> toks[s * ts] and out[s * os] (one launch for both).
__global__ void store_draft_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t* __restrict__ toks,
                                   int64_t ts, int64_t* __restrict__ out, int64_t os) {
  const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i < n) {
    const int64_t v = ids[i];
    toks[i * ts] = v;
    out[i * os] = v;
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ in, int64_t n, __nv_bfloat16* __restrict__ out) {
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x)
    out[e] = __float2bfloat16_rn(in[e]);
}

}  // namespace lng

struct lng_drafter {
  // configuration
  int64_t d = 0, V = 0, R = 0, bits = 0, md = 0, kv = 0, hd = 0, qh = 0, Dt = 0, maxn = 0;
  int n_orders = 0;
  int orders[LNG_MAX_ORDERS] = {};
  float router_eps = 0, draft_eps = 0, mem_eps = 0, sink = 0;
  int act = LNG_F32;          // readout activations / folded maps
  int e_dtype = LNG_F32;      // embedding on the device
  int t_dtype = LNG_F32;      // tables on the device
  // device parameters
  void* E = nullptr;
  void* tab[LNG_MAX_ORDERS] = {};
  float* ss[LNG_MAX_ORDERS] = {};
  float *router_w = nullptr, *prev_norm = nullptr, *cur_norm = nullptr, *start = nullptr;
  __nv_bfloat16* router_w_split = nullptr;  // router weight as bf16 parts W1 | W2 | W3 (made once)
  float *out_norm = nullptr;
  void *w_qk = nullptr, *w_vo = nullptr;
  std::vector<void*> owned;
  // host state (the reference keeps the same: drafter.cpp:571-574)
  std::vector<int64_t> tokens;
  std::vector<uint8_t> codes;
  std::mutex mu;
  cudaStream_t stream = nullptr;
  // grow-on-demand device workspace
  void* ws = nullptr;
  size_t ws_bytes = 0;

  lng_tables tables() const {
    lng_tables t{};
    t.n_orders = n_orders;
    for (int o = 0; o < n_orders; ++o) {
      t.orders[o] = orders[o];
      t.tables[o] = tab[o];
      t.row_ss[o] = ss[o];
    }
    t.table_dtype = t_dtype;
    t.bits = int32_t(bits);
    t.num_routes = R;
    t.memory_dim = md;
    return t;
  }
  ~lng_drafter() {
    for (void* p : owned) cudaFree(p);
    if (ws) cudaFree(ws);
    if (stream) cudaStreamDestroy(stream);
  }
};

namespace lng {

static int drafter_alloc(lng_drafter* dr, size_t bytes, void** out) {
  void* p = nullptr;
  LNG_CUDA(cudaMalloc(&p, bytes > 0 ? bytes : 16));
  dr->owned.push_back(p);
  *out = p;
  return LNG_OK;
}

static const lng_array* find_array(const lng_array* arrays, int n, const char* name) {
  for (int i = 0; i < n; ++i)
    if (arrays[i].name && std::strcmp(arrays[i].name, name) == 0) return &arrays[i];
  return nullptr;
}

static int64_t array_numel(const lng_array* a) {
  int64_t n = 1;
  for (int i = 0; i < a->ndim; ++i) n *= a->shape[i];
  return n;
}

// Upload a host array as fp32 (from f32 / f16 / bf16).
static int upload_f32(lng_drafter* dr, const lng_array* a, int64_t expect, float** out) {
  if (!a) return fail(LNG_ERR_ARGUMENT, "bundle array missing");
  const int64_t n = array_numel(a);
  if (n != expect) return fail(LNG_ERR_ARGUMENT, std::string("bundle array ") + a->name + " has the wrong size");
  std::vector<float> tmp(static_cast<size_t>(n));
  if (a->dtype == LNG_F32) {
    std::memcpy(tmp.data(), a->data_host, size_t(n) * 4);
  } else if (a->dtype == LNG_F16) {
    const __half* s = static_cast<const __half*>(a->data_host);
    for (int64_t i = 0; i < n; ++i) tmp[size_t(i)] = __half2float(s[i]);
  } else if (a->dtype == LNG_BF16) {
    const __nv_bfloat16* s = static_cast<const __nv_bfloat16*>(a->data_host);
    for (int64_t i = 0; i < n; ++i) tmp[size_t(i)] = __bfloat162float(s[i]);
  } else {
    return fail(LNG_ERR_ARGUMENT, std::string("bundle array ") + a->name + " must be floating point");
  }
  void* p = nullptr;
  int st = drafter_alloc(dr, size_t(n) * 4, &p);
  if (st) return st;
  LNG_CUDA(cudaMemcpy(p, tmp.data(), size_t(n) * 4, cudaMemcpyHostToDevice));
  *out = static_cast<float*>(p);
  return LNG_OK;
}

// Upload a float host array in its own dtype (f32 / f16) or converted to bf16 when want_bf16.
static int upload_as(lng_drafter* dr, const lng_array* a, int64_t expect, bool want_bf16, void** out, int* dtype) {
  if (!a) return fail(LNG_ERR_ARGUMENT, "bundle array missing");
  const int64_t n = array_numel(a);
  if (n != expect) return fail(LNG_ERR_ARGUMENT, std::string("bundle array ") + a->name + " has the wrong size");
  if (!want_bf16 && (a->dtype == LNG_F32 || a->dtype == LNG_F16 || a->dtype == LNG_BF16)) {
    const size_t bytes = size_t(n) * dtype_size(a->dtype);
    int st = drafter_alloc(dr, bytes, out);
    if (st) return st;
    LNG_CUDA(cudaMemcpy(*out, a->data_host, bytes, cudaMemcpyHostToDevice));
    *dtype = a->dtype;
    return LNG_OK;
  }
  float* f = nullptr;
  int st = upload_f32(dr, a, expect, &f);
  if (st) return st;
  st = drafter_alloc(dr, size_t(n) * 2, out);
  if (st) return st;
  f32_to_bf16_kernel<<<grid_for(n, 256, 16), 256>>>(f, n, static_cast<__nv_bfloat16*>(*out));
  LNG_LAUNCHED("f32_to_bf16_kernel");
  LNG_CUDA(cudaDeviceSynchronize());
  *dtype = LNG_BF16;
  return LNG_OK;
}

struct ReadoutBufs {
  void* x;       // [M, d] embedding rows (E dtype)
  float* qs;     // [M]
  void* qa;      // [M, qh*Dt] act
  void* u;       // [M, qh*Dt] act
  float* hid;    // [M, d]
  float* hn;     // [M, d]
  int64_t* ids;  // [M, k]
  float* vals;   // [M, k]
  void* scratch; size_t scratch_bytes;
  float* feat;   // [M, 2d]
};

static int drafter_ws(lng_drafter* dr, int64_t M, int k, ReadoutBufs* b, size_t extra_bytes, void** extra) {
  const size_t es = size_t(dtype_size(dr->e_dtype)), as = size_t(dtype_size(dr->act));
  const size_t qd = size_t(dr->qh * dr->Dt);
  const size_t sizes[10] = {al256(size_t(M) * dr->d * es), al256(size_t(M) * 4), al256(size_t(M) * qd * as),
                            al256(size_t(M) * qd * as), al256(size_t(M) * dr->d * 4), al256(size_t(M) * dr->d * 4),
                            al256(size_t(M) * k * 8), al256(size_t(M) * k * 4),
                            al256(lng_logits_topk_scratch_bytes(M, dr->d, dr->V, k)), al256(size_t(M) * 2 * dr->d * 4)};
  size_t total = al256(extra_bytes);
  for (size_t s : sizes) total += s;
  if (total > dr->ws_bytes) {
    if (dr->ws) LNG_CUDA(cudaFree(dr->ws));
    dr->ws = nullptr;
    dr->ws_bytes = 0;
    LNG_CUDA(cudaMalloc(&dr->ws, total));
    dr->ws_bytes = total;
  }
  unsigned char* p = static_cast<unsigned char*>(dr->ws);
  void* ptrs[10];
  for (int i = 0; i < 10; ++i) {
    ptrs[i] = p;
    p += sizes[i];
  }
  b->x = ptrs[0];
  b->qs = static_cast<float*>(ptrs[1]);
  b->qa = ptrs[2];
  b->u = ptrs[3];
  b->hid = static_cast<float*>(ptrs[4]);
  b->hn = static_cast<float*>(ptrs[5]);
  b->ids = static_cast<int64_t*>(ptrs[6]);
  b->vals = static_cast<float*>(ptrs[7]);
  b->scratch = ptrs[8];
  b->scratch_bytes = sizes[8];
  b->feat = static_cast<float*>(ptrs[9]);
  if (extra) *extra = extra_bytes ? p : nullptr;
  return LNG_OK;
}

// Codes of M tokens given their previous tokens (device i64 arrays; prev = -1 -> start vector).
static int drafter_codes(lng_drafter* dr, const int64_t* cur, const int64_t* prev, int64_t M, float* feat,
                         uint8_t* codes_out, int64_t codes_stride) {
  lng_stream_t s = reinterpret_cast<lng_stream_t>(dr->stream);
  int st = lng_embed2_features(cur, prev, M, dr->E, dr->e_dtype, dr->V, dr->d, dr->prev_norm, dr->cur_norm,
                               dr->start, dr->router_eps, feat, s);
  if (st) return st;
  if (codes_stride == dr->R)
    return route_codes_presplit(feat, M, 2 * dr->d, dr->router_w, dr->router_w_split, dr->R, int32_t(dr->bits),
                                codes_out, dr->stream);
  for (int64_t i = 0; i < M; ++i) {  // strided destination (batched drafting): one row at a time
    st = route_codes_presplit(feat + i * 2 * dr->d, 1, 2 * dr->d, dr->router_w, dr->router_w_split, dr->R,
                              int32_t(dr->bits), codes_out + i * codes_stride, dr->stream);
    if (st) return st;
  }
  return LNG_OK;
}

// Readout of M items: embedding rows of `cur`, the item's code window per `src`, top-k (or full logits).
static int drafter_readout(lng_drafter* dr, const int64_t* cur, int64_t M, const CodeSource& src, int k,
                           ReadoutBufs& b, float* full_logits) {
  cudaStream_t s = dr->stream;
  lng_stream_t ls = reinterpret_cast<lng_stream_t>(s);
  const int64_t qd = dr->qh * dr->Dt;
#define LNG_GR(T) gather_rows_kernel<T><<<grid_for(M * dr->d, 256, 8), 256, 0, s>>>(cur, M, static_cast<const T*>(dr->E), dr->d, dr->V, static_cast<T*>(b.x))
  if (dr->e_dtype == LNG_F32) LNG_GR(float);
  else if (dr->e_dtype == LNG_BF16) LNG_GR(__nv_bfloat16);
  else LNG_GR(__half);
#undef LNG_GR
  LNG_LAUNCHED("gather_rows_kernel");
  int st = lng_rms_rows(b.x, dr->e_dtype, M, dr->d, dr->draft_eps, b.qs, ls);
  if (st) return st;
  st = lng_gemm(b.x, dr->e_dtype, dr->d, dr->w_qk, dr->act, dr->d, b.qa, dr->act, qd, M, qd, dr->d, nullptr, 0, ls);
  if (st) return st;
  const lng_tables t = dr->tables();
  AttendParams p{};
  p.ts = table_set(&t);
  p.src = src;
  p.M = M;
  p.route_start = 0;
  p.route_end = dr->R;
  p.qh = int(dr->qh);
  p.eps = dr->mem_eps;
  p.sink = dr->sink;
  p.qa = b.qa;
  p.qscale = b.qs;
  p.u = b.u;
  st = attend_impl<uint8_t>(&t, p, dr->act, s);
  if (st) return st;
  st = lng_gemm(b.u, dr->act, qd, dr->w_vo, dr->act, qd, b.hid, LNG_F32, dr->d, M, dr->d, qd, nullptr, 0, ls);
  if (st) return st;
  st = lng_rms_norm(b.hid, LNG_F32, M, dr->d, dr->out_norm, dr->draft_eps, b.hn, LNG_F32, ls);
  if (st) return st;
  return lng_logits_topk(b.hn, M, dr->d, dr->E, dr->e_dtype, dr->V, k, b.ids, b.vals, full_logits, b.scratch,
                         b.scratch_bytes, ls);
}

}  // namespace lng

extern "C" int lng_drafter_create(const lng_drafter_numbers* num, const lng_array* arrays, int32_t n_arrays,
                                  int32_t act_dtype, lng_drafter** out) {
  LNG_REQUIRE(num && arrays && out, "NULL pointer");
  *out = nullptr;
  LNG_REQUIRE(act_dtype == LNG_F32 || act_dtype == LNG_BF16, "act dtype must be f32 or bf16");
  if (num->ssm_dim > 0 || num->router_ssm || num->query_ssm)
    return fail(LNG_ERR_UNSUPPORTED, "SSM drafters (SD-C) are not implemented by lngram_b200");
  if (num->sketch_k > 0 && num->shortlist_cap > 0)
    return fail(LNG_ERR_UNSUPPORTED, "sketch shortlists are not implemented by lngram_b200 (full-vocabulary bundles)");
  LNG_REQUIRE(num->n_orders >= 1 && num->n_orders <= LNG_MAX_ORDERS, "n_orders must be in [1, 4]");
  LNG_REQUIRE(num->q_heads % num->kv_heads == 0 && num->q_heads <= 64, "q_heads must be a multiple of kv_heads");
  LNG_REQUIRE(num->bits >= 1 && num->bits <= 8, "bits must be in [1, 8]");
  std::unique_ptr<lng_drafter> dr(new lng_drafter());
  dr->d = num->d_model;
  dr->V = num->vocab;
  dr->R = num->routes;
  dr->bits = num->bits;
  dr->md = num->mem_dim;
  dr->kv = num->kv_heads;
  dr->hd = num->head_dim;
  dr->qh = num->q_heads;
  dr->n_orders = num->n_orders;
  for (int o = 0; o < num->n_orders; ++o) dr->orders[o] = num->orders[o];
  dr->maxn = *std::max_element(dr->orders, dr->orders + dr->n_orders);
  dr->Dt = int64_t(dr->n_orders) * dr->md;
  dr->router_eps = float(num->router_eps);
  dr->draft_eps = float(num->draft_eps);
  dr->mem_eps = float(num->mem_eps);
  dr->sink = float(num->sink_logit);
  dr->act = act_dtype;
  LNG_REQUIRE(std::fabs(num->softmax_scale * std::sqrt(double(num->head_dim)) - 1.0) < 1e-6,
              "softmax_scale must be head_dim^-1/2");
  LNG_CUDA(cudaStreamCreateWithFlags(&dr->stream, cudaStreamNonBlocking));
  lng_drafter* D = dr.get();
  const bool bf = act_dtype == LNG_BF16;
  int st = upload_as(D, find_array(arrays, n_arrays, "embedding"), D->V * D->d, bf, &D->E, &D->e_dtype);
  if (st) return st;
  for (int o = 0; o < D->n_orders; ++o) {
    const std::string name = "table_" + std::to_string(D->orders[o]);
    const int64_t rows = D->R << (D->bits * D->orders[o]);
    int tdt = 0;
    st = upload_as(D, find_array(arrays, n_arrays, name.c_str()), rows * D->md, bf, &D->tab[o], &tdt);
    if (st) return st;
    if (o && tdt != D->t_dtype) return fail(LNG_ERR_ARGUMENT, "all tables must share a dtype");
    D->t_dtype = tdt;
    void* p = nullptr;
    st = drafter_alloc(D, size_t(rows) * 4, &p);
    if (st) return st;
    D->ss[o] = static_cast<float*>(p);
  }
  {
    const lng_tables t = D->tables();
    float* ssp[LNG_MAX_ORDERS] = {D->ss[0], D->ss[1], D->ss[2], D->ss[3]};
    st = lng_table_row_ss(&t, ssp, nullptr);
    if (st) return st;
  }
  float *mem_norm = nullptr, *kv_proj = nullptr, *q_norm = nullptr, *w_q = nullptr, *w_o = nullptr;
  const int64_t KH = D->kv * D->hd, I = D->qh * D->hd;
  if ((st = upload_f32(D, find_array(arrays, n_arrays, "mem_norm"), D->Dt, &mem_norm))) return st;
  if ((st = upload_f32(D, find_array(arrays, n_arrays, "kv_proj"), 2 * KH * D->Dt, &kv_proj))) return st;
  if ((st = upload_f32(D, find_array(arrays, n_arrays, "router"), D->R * D->bits * 2 * D->d, &D->router_w))) return st;
  {  // the router weight's bf16x3 split, used by every small-batch code computation of this drafter
    const int64_t rows = D->R * D->bits, in_dim = 2 * D->d;
    void* wsp = nullptr;
    LNG_CUDA(cudaMalloc(&wsp, size_t(rows) * 3 * in_dim * sizeof(__nv_bfloat16)));
    D->owned.push_back(wsp);
    D->router_w_split = static_cast<__nv_bfloat16*>(wsp);
    split_bf16x3_kernel<<<grid_for(rows * in_dim, 256, 16), 256>>>(D->router_w, rows, in_dim, D->router_w_split);
    LNG_CUDA(cudaGetLastError());
    LNG_LAUNCHED("split_bf16x3_kernel");
  }
  if ((st = upload_f32(D, find_array(arrays, n_arrays, "router_prev_norm"), D->d, &D->prev_norm))) return st;
  if ((st = upload_f32(D, find_array(arrays, n_arrays, "router_cur_norm"), D->d, &D->cur_norm))) return st;
  if ((st = upload_f32(D, find_array(arrays, n_arrays, "router_start"), D->d, &D->start))) return st;
  if ((st = upload_f32(D, find_array(arrays, n_arrays, "q_norm"), D->d, &q_norm))) return st;
  if ((st = upload_f32(D, find_array(arrays, n_arrays, "w_q"), I * D->d, &w_q))) return st;
  if ((st = upload_f32(D, find_array(arrays, n_arrays, "w_o"), D->d * I, &w_o))) return st;
  if ((st = upload_f32(D, find_array(arrays, n_arrays, "out_norm"), D->d, &D->out_norm))) return st;
  const size_t as = size_t(dtype_size(act_dtype));
  if ((st = drafter_alloc(D, size_t(D->qh * D->Dt * D->d) * as, &D->w_qk))) return st;
  if ((st = drafter_alloc(D, size_t(D->d * D->qh * D->Dt) * as, &D->w_vo))) return st;
  st = lng_fold_readout(D->d, D->Dt, int32_t(D->qh), int32_t(D->kv), int32_t(D->hd), q_norm, w_q, mem_norm, kv_proj,
                        w_o, D->w_qk, D->w_vo, act_dtype, nullptr);
  if (st) return st;
  LNG_CUDA(cudaDeviceSynchronize());
  *out = dr.release();
  return LNG_OK;
}

extern "C" void lng_drafter_destroy(lng_drafter* d) { delete d; }

extern "C" int lng_drafter_reset(lng_drafter* d) {
  LNG_REQUIRE(d, "NULL drafter");
  std::lock_guard<std::mutex> lk(d->mu);
  d->tokens.clear();
  d->codes.clear();
  return LNG_OK;
}

extern "C" int64_t lng_drafter_length(const lng_drafter* d) { return d ? int64_t(d->tokens.size()) : -1; }

extern "C" int lng_drafter_truncate(lng_drafter* d, int64_t n) {
  LNG_REQUIRE(d, "NULL drafter");
  std::lock_guard<std::mutex> lk(d->mu);
  if (n < 0 || n > int64_t(d->tokens.size())) return fail(LNG_ERR_STATE, "cannot truncate to " + std::to_string(n));
  d->tokens.resize(size_t(n));
  d->codes.resize(size_t(n * d->R));
  return LNG_OK;
}

extern "C" int lng_drafter_committed_codes(const lng_drafter* d, uint8_t* codes_host) {
  LNG_REQUIRE(d, "NULL drafter");
  if (!d->codes.empty()) {
    LNG_REQUIRE(codes_host, "NULL pointer");
    std::memcpy(codes_host, d->codes.data(), d->codes.size());
  }
  return LNG_OK;
}

namespace lng {

// Codes of `n` new tokens after the committed state, on the device; written to codes_host [n, R].
static int drafter_codes_for(lng_drafter* d, const int64_t* toks_host, int64_t n, uint8_t* codes_host) {
  ReadoutBufs b;
  void* extra = nullptr;
  const size_t tb = al256(size_t(2 * n) * 8);
  int st = drafter_ws(d, n, 1, &b, tb + size_t(n * d->R), &extra);
  if (st) return st;
  int64_t* cur = static_cast<int64_t*>(extra);
  int64_t* prev = cur + n;
  uint8_t* cd = static_cast<uint8_t*>(extra) + tb;
  std::vector<int64_t> host(size_t(2 * n));
  for (int64_t i = 0; i < n; ++i) {
    host[size_t(i)] = toks_host[i];
    host[size_t(n + i)] = i > 0 ? toks_host[i - 1] : (d->tokens.empty() ? -1 : d->tokens.back());
  }
  LNG_CUDA(cudaMemcpyAsync(cur, host.data(), size_t(2 * n) * 8, cudaMemcpyHostToDevice, d->stream));
  st = drafter_codes(d, cur, prev, n, b.feat, cd, d->R);
  if (st) return st;
  LNG_CUDA(cudaMemcpyAsync(codes_host, cd, size_t(n * d->R), cudaMemcpyDeviceToHost, d->stream));
  LNG_CUDA(cudaStreamSynchronize(d->stream));
  const int derr = lng_device_error(1);
  if (derr) return fail(LNG_ERR_DEVICE, "device error " + std::to_string(derr) + " (token id out of range?)");
  return LNG_OK;
}

}  // namespace lng

extern "C" int lng_drafter_commit(lng_drafter* d, const int64_t* tokens_host, int64_t n, const int32_t* codes_host) {
  LNG_REQUIRE(d, "NULL drafter");
  LNG_REQUIRE(n >= 0, "bad length");
  if (n == 0) return LNG_OK;
  LNG_REQUIRE(tokens_host, "NULL pointer");
  std::lock_guard<std::mutex> lk(d->mu);
  for (int64_t i = 0; i < n; ++i)
    if (tokens_host[i] < 0 || tokens_host[i] >= d->V) return fail(LNG_ERR_STATE, "token id out of range");
  std::vector<uint8_t> c(size_t(n * d->R));
  if (codes_host) {
    for (int64_t i = 0; i < n * d->R; ++i) c[size_t(i)] = uint8_t(codes_host[i]);
  } else {
    int st = drafter_codes_for(d, tokens_host, n, c.data());
    if (st) return st;
  }
  d->tokens.insert(d->tokens.end(), tokens_host, tokens_host + n);
  d->codes.insert(d->codes.end(), c.begin(), c.end());
  return LNG_OK;
}

extern "C" int lng_drafter_draft(lng_drafter* d, int64_t gamma, const int64_t* hyp_host, int64_t n_hyp, int32_t topk,
                                 int32_t last_codes, int64_t* tokens_host, int64_t* ids_host, float* logits_host,
                                 uint8_t* codes_host) {
  LNG_REQUIRE(d, "NULL drafter");
  LNG_REQUIRE(gamma >= 0 && topk >= 1 && topk <= TK_MAXK, "need gamma >= 0 and 1 <= topk <= 8");
  LNG_REQUIRE(n_hyp >= 0 && (n_hyp == 0 || hyp_host), "bad hypothesis");
  std::lock_guard<std::mutex> lk(d->mu);
  const int64_t L = int64_t(d->tokens.size());
  if (L == 0 && n_hyp == 0) return fail(LNG_ERR_STATE, "draft needs at least one committed or hypothetical token");
  for (int64_t i = 0; i < n_hyp; ++i)
    if (hyp_host[i] < 0 || hyp_host[i] >= d->V) return fail(LNG_ERR_STATE, "token id out of range");
  const int64_t W = d->maxn, R = d->R;
  // slots: W-1 history slots, then hyp tokens, then drafted tokens (positions L-W+1 ..)
  const int64_t nslots = (W - 1) + 1 + n_hyp + gamma;  // +1: the last committed token's slot
  const int64_t n_codes = n_hyp + (last_codes ? gamma : std::max<int64_t>(gamma - 1, 0));
  ReadoutBufs b;
  void* extra = nullptr;
  const size_t tok_b = al256(size_t(nslots + 1) * 8), seg_b = al256(size_t(gamma * W) * 4), ids_b = al256(size_t(gamma * topk) * 8),
               val_b = al256(size_t(gamma * topk) * 4), code_b = al256(size_t(nslots * R));
  int st = drafter_ws(d, std::max<int64_t>(1, n_hyp), topk, &b, tok_b + seg_b + ids_b + val_b + code_b, &extra);
  if (st) return st;
  unsigned char* ex = static_cast<unsigned char*>(extra);
  int64_t* dtok = reinterpret_cast<int64_t*>(ex);            // dtok[s + 1] = token of slot s; dtok[0] = -1
  int32_t* dseg = reinterpret_cast<int32_t*>(ex + tok_b);
  int64_t* dids = reinterpret_cast<int64_t*>(ex + tok_b + seg_b);
  float* dvals = reinterpret_cast<float*>(ex + tok_b + seg_b + ids_b);
  uint8_t* dcodes = ex + tok_b + seg_b + ids_b + val_b;      // [nslots, R]
  // host-side initial slots: the last W committed positions (slot W-1 = position L-1)
  std::vector<int64_t> htok(size_t(nslots + 1), -1);
  std::vector<uint8_t> hcodes(size_t(nslots * R), 0);
  const int64_t first_pos = L - 1 - (W - 1);  // absolute position of slot 0
  for (int64_t s = 0; s < W; ++s) {
    const int64_t pos = first_pos + s;
    if (pos >= 0 && pos < L) {
      htok[size_t(s + 1)] = d->tokens[size_t(pos)];
      std::memcpy(&hcodes[size_t(s * R)], &d->codes[size_t(pos * R)], size_t(R));
    }
  }
  for (int64_t i = 0; i < n_hyp; ++i) htok[size_t(W + i + 1)] = hyp_host[i];
  std::vector<int32_t> hseg(size_t(std::max<int64_t>(gamma, 1) * W));
  for (int64_t g = 0; g < gamma; ++g)
    for (int64_t k = 0; k < W; ++k) {
      const int64_t pos = first_pos + n_hyp + g + k;  // window of step g: slots n_hyp+g .. W-1+n_hyp+g
      hseg[size_t(g * W + k)] = pos >= 0 ? 1 : 0;
    }
  LNG_CUDA(cudaMemcpyAsync(dtok, htok.data(), size_t(nslots + 1) * 8, cudaMemcpyHostToDevice, d->stream));
  LNG_CUDA(cudaMemcpyAsync(dcodes, hcodes.data(), size_t(nslots * R), cudaMemcpyHostToDevice, d->stream));
  if (gamma > 0)
    LNG_CUDA(cudaMemcpyAsync(dseg, hseg.data(), size_t(gamma * W) * 4, cudaMemcpyHostToDevice, d->stream));
  // hypothetical tokens: their codes in one batched router pass (prev of slot s is slot s-1)
  if (n_hyp > 0) {
    st = drafter_codes(d, dtok + W + 1, dtok + W, n_hyp, b.feat, dcodes + W * R, R);
    if (st) return st;
  }
  for (int64_t g = 0; g < gamma; ++g) {
    const int64_t end = W - 1 + n_hyp + g;  // slot of the current token
    CodeSource src{dcodes + (end - W + 1) * R, 0, 0, W, R, nullptr, nullptr, dseg + g * W, 0, 0};
    st = drafter_readout(d, dtok + end + 1, 1, src, topk, b, nullptr);
    if (st) return st;
    LNG_CUDA(cudaMemcpyAsync(dids + g * topk, b.ids, size_t(topk) * 8, cudaMemcpyDeviceToDevice, d->stream));
    LNG_CUDA(cudaMemcpyAsync(dvals + g * topk, b.vals, size_t(topk) * 4, cudaMemcpyDeviceToDevice, d->stream));
    if (g + 1 < gamma || last_codes) {
      copy_i64_kernel<<<1, 32, 0, d->stream>>>(b.ids, dtok + end + 2, 1, 1, 1);
      LNG_LAUNCHED("copy_i64_kernel");
      st = drafter_codes(d, dtok + end + 2, dtok + end + 1, 1, b.feat, dcodes + (end + 1) * R, R);
      if (st) return st;
    }
  }
  std::vector<int64_t> hids(size_t(std::max<int64_t>(gamma * topk, 1)));
  std::vector<float> hvals(size_t(std::max<int64_t>(gamma * topk, 1)));
  if (gamma > 0) {
    LNG_CUDA(cudaMemcpyAsync(hids.data(), dids, size_t(gamma * topk) * 8, cudaMemcpyDeviceToHost, d->stream));
    LNG_CUDA(cudaMemcpyAsync(hvals.data(), dvals, size_t(gamma * topk) * 4, cudaMemcpyDeviceToHost, d->stream));
  }
  std::vector<uint8_t> hc(size_t(std::max<int64_t>(n_codes * R, 1)));
  if (n_codes > 0)
    LNG_CUDA(cudaMemcpyAsync(hc.data(), dcodes + W * R, size_t(n_codes * R), cudaMemcpyDeviceToHost, d->stream));
  LNG_CUDA(cudaStreamSynchronize(d->stream));
  const int derr = lng_device_error(1);
  if (derr) return fail(LNG_ERR_DEVICE, "device error " + std::to_string(derr) + " during draft");
  for (int64_t g = 0; g < gamma; ++g) {
    if (tokens_host) tokens_host[g] = hids[size_t(g * topk)];
    for (int j = 0; j < topk; ++j) {
      if (ids_host) ids_host[g * topk + j] = hids[size_t(g * topk + j)];
      if (logits_host) logits_host[g * topk + j] = hvals[size_t(g * topk + j)];
    }
  }
  if (codes_host && n_codes > 0) std::memcpy(codes_host, hc.data(), size_t(n_codes * R));
  return LNG_OK;
}

extern "C" int lng_drafter_trace(lng_drafter* d, const int64_t* tokens_host, int64_t T, const int32_t* codes_host,
                                 int32_t full, int64_t S, uint8_t* codes_out_host, int64_t* ids_host,
                                 float* logits_host) {
  LNG_REQUIRE(d, "NULL drafter");
  LNG_REQUIRE(T >= 0 && S == d->V, "full-vocabulary trace: S must equal the vocabulary");
  (void)full;
  if (T == 0) return LNG_OK;
  LNG_REQUIRE(tokens_host, "NULL pointer");
  std::lock_guard<std::mutex> lk(d->mu);
  for (int64_t i = 0; i < T; ++i)
    if (tokens_host[i] < 0 || tokens_host[i] >= d->V) return fail(LNG_ERR_STATE, "token id out of range");
  const int64_t R = d->R;
  ReadoutBufs b;
  void* extra = nullptr;
  const size_t tok_b = al256(size_t(2 * T) * 8), code_b = al256(size_t(T * R)), lg_b = al256(size_t(T * d->V) * 4);
  int st = drafter_ws(d, T, 1, &b, tok_b + code_b + lg_b, &extra);
  if (st) return st;
  unsigned char* ex = static_cast<unsigned char*>(extra);
  int64_t* cur = reinterpret_cast<int64_t*>(ex);
  int64_t* prev = cur + T;
  uint8_t* dcodes = ex + tok_b;
  float* dlog = reinterpret_cast<float*>(ex + tok_b + code_b);
  std::vector<int64_t> host(size_t(2 * T));
  for (int64_t i = 0; i < T; ++i) {
    host[size_t(i)] = tokens_host[i];
    host[size_t(T + i)] = i > 0 ? tokens_host[i - 1] : -1;
  }
  LNG_CUDA(cudaMemcpyAsync(cur, host.data(), size_t(2 * T) * 8, cudaMemcpyHostToDevice, d->stream));
  if (codes_host) {
    std::vector<uint8_t> c(size_t(T * R));
    for (int64_t i = 0; i < T * R; ++i) c[size_t(i)] = uint8_t(codes_host[i]);
    LNG_CUDA(cudaMemcpyAsync(dcodes, c.data(), size_t(T * R), cudaMemcpyHostToDevice, d->stream));
    LNG_CUDA(cudaStreamSynchronize(d->stream));
  } else {
    st = drafter_codes(d, cur, prev, T, b.feat, dcodes, R);
    if (st) return st;
  }
  CodeSource src{dcodes, 1, T, 0, R, nullptr, nullptr, nullptr, 0, T};
  st = drafter_readout(d, cur, T, src, 1, b, dlog);
  if (st) return st;
  if (codes_out_host) LNG_CUDA(cudaMemcpyAsync(codes_out_host, dcodes, size_t(T * R), cudaMemcpyDeviceToHost, d->stream));
  if (logits_host)
    LNG_CUDA(cudaMemcpyAsync(logits_host, dlog, size_t(T * d->V) * 4, cudaMemcpyDeviceToHost, d->stream));
  LNG_CUDA(cudaStreamSynchronize(d->stream));
  const int derr = lng_device_error(1);
  if (derr) return fail(LNG_ERR_DEVICE, "device error " + std::to_string(derr) + " during trace");
  if (ids_host)
    for (int64_t t = 0; t < T; ++t)
      for (int64_t v = 0; v < d->V; ++v) ids_host[t * d->V + v] = v;
  return LNG_OK;
}

extern "C" int lng_drafter_draft_batch(lng_drafter* d, const int64_t* prefix, int64_t nseq, int64_t plen, int64_t gamma,
                                       int64_t* tokens_out, lng_stream_t stream) {
  LNG_REQUIRE(d, "NULL drafter");
  LNG_REQUIRE(nseq >= 0 && plen >= 1 && gamma >= 1, "need nseq >= 0, plen >= 1, gamma >= 1");
  if (nseq == 0) return LNG_OK;
  LNG_REQUIRE(prefix && tokens_out, "NULL pointer");
  std::lock_guard<std::mutex> lk(d->mu);
  const int64_t R = d->R, P = plen + gamma;  // positions per sequence in the working buffers
  // The drafts' code windows reach back n_max - 1 positions from the last prefix token, and the
  // embed2 router reads only a position's own and previous token (SSM routers are rejected at
  // create), so only the last `tail` prefix positions need codes; earlier rows of `codes` are never
  // read.
  int64_t n_max = 1;
  for (int o = 0; o < d->n_orders; ++o) n_max = std::max<int64_t>(n_max, d->orders[o]);
  const int64_t tail = std::min<int64_t>(plen, n_max);
  ReadoutBufs b;
  void* extra = nullptr;
  const size_t tok_b = al256(size_t(nseq * (P + 1)) * 8), prev_b = al256(size_t(nseq * std::max<int64_t>(2 * tail, 2)) * 8),
               code_b = al256(size_t(nseq * P * R));
  const int64_t M = nseq * tail;
  int st = drafter_ws(d, M, 1, &b, tok_b + prev_b + code_b, &extra);
  if (st) return st;
  unsigned char* ex = static_cast<unsigned char*>(extra);
  int64_t* toks = reinterpret_cast<int64_t*>(ex);  // [nseq, P + 1]: toks[s, 0] = -1, toks[s, 1 + p] = token p
  int64_t* scratch_i = reinterpret_cast<int64_t*>(ex + tok_b);  // [2, nseq * tail]: current, previous tokens
  uint8_t* codes = ex + tok_b + prev_b;             // [nseq, P, R]
  cudaStream_t us = reinterpret_cast<cudaStream_t>(stream);
  cudaEvent_t ev;
  LNG_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  LNG_CUDA(cudaEventRecord(ev, us));
  LNG_CUDA(cudaStreamWaitEvent(d->stream, ev, 0));
  // token matrix with a -1 column for the start vector, then prefix codes in one batched pass
  LNG_CUDA(cudaMemsetAsync(toks, 0xff, size_t(nseq * (P + 1)) * 8, d->stream));
  LNG_CUDA(cudaMemcpy2DAsync(toks + 1, size_t(P + 1) * 8, prefix, size_t(plen) * 8, size_t(plen) * 8, size_t(nseq),
                             cudaMemcpyDeviceToDevice, d->stream));
  // tokens of the last `tail` prefix positions (dense [nseq, tail]) and their previous tokens
  // (toks[s, p] is the token before position p, -1 at p = 0)
  const int64_t p0 = plen - tail;
  LNG_CUDA(cudaMemcpy2DAsync(scratch_i, size_t(tail) * 8, prefix + p0, size_t(plen) * 8, size_t(tail) * 8,
                             size_t(nseq), cudaMemcpyDeviceToDevice, d->stream));
  LNG_CUDA(cudaMemcpy2DAsync(scratch_i + nseq * tail, size_t(tail) * 8, toks + p0, size_t(P + 1) * 8,
                             size_t(tail) * 8, size_t(nseq), cudaMemcpyDeviceToDevice, d->stream));
  // their codes [nseq * tail, R] computed densely, then placed at rows p0 .. plen-1 with stride P * R
  uint8_t* dense = reinterpret_cast<uint8_t*>(b.u);  // reuse: nseq*tail*R bytes <= u's size (M = nseq*tail)
  const size_t dense_need = size_t(nseq * tail * R);
  const size_t u_bytes = size_t(M) * d->qh * d->Dt * dtype_size(d->act);
  LNG_REQUIRE(dense_need <= u_bytes, "internal: code staging buffer too small");
  st = drafter_codes(d, scratch_i, scratch_i + nseq * tail, nseq * tail, b.feat, dense, R);
  if (st) return st;
  LNG_CUDA(cudaMemcpy2DAsync(codes + p0 * R, size_t(P * R), dense, size_t(tail * R), size_t(tail * R), size_t(nseq),
                             cudaMemcpyDeviceToDevice, d->stream));
  for (int64_t g = 0; g < gamma; ++g) {
    const int64_t tpos = plen - 1 + g;  // position of the current token in every sequence
    // current tokens toks[s, 1 + tpos] -> gather into a dense [nseq] vector
    copy_i64_kernel<<<unsigned(ceil_div(nseq, 128)), 128, 0, d->stream>>>(toks + 1 + tpos, scratch_i, nseq, P + 1, 1);
    LNG_LAUNCHED("copy_i64_kernel");
    CodeSource src{codes, nseq, tpos + 1, 0, R, nullptr, nullptr, nullptr, tpos, P};
    st = drafter_readout(d, scratch_i, nseq, src, 1, b, nullptr);
    if (st) return st;
    // next tokens -> toks[s, 2 + tpos] and tokens_out[s, g]
    store_draft_kernel<<<unsigned(ceil_div(nseq, 128)), 128, 0, d->stream>>>(b.ids, nseq, toks + 2 + tpos, P + 1,
                                                                             tokens_out + g, gamma);
    LNG_LAUNCHED("store_draft_kernel");
    if (g + 1 < gamma) {
      // codes of the drafted tokens at position tpos + 1 (strided rows of the code buffer); their
      // previous tokens are this step's current tokens, still in scratch_i
      st = lng_embed2_features(b.ids, scratch_i, nseq, d->E, d->e_dtype, d->V, d->d, d->prev_norm,
                               d->cur_norm, d->start, d->router_eps, b.feat, reinterpret_cast<lng_stream_t>(d->stream));
      if (st) return st;
      st = route_codes_presplit(b.feat, nseq, 2 * d->d, d->router_w, d->router_w_split, R, int32_t(d->bits), dense,
                                d->stream);
      if (st) return st;
      LNG_CUDA(cudaMemcpy2DAsync(codes + (tpos + 1) * R, size_t(P * R), dense, size_t(R), size_t(R), size_t(nseq),
                                 cudaMemcpyDeviceToDevice, d->stream));
    }
  }
  LNG_CUDA(cudaEventRecord(ev, d->stream));
  LNG_CUDA(cudaStreamWaitEvent(us, ev, 0));
  LNG_CUDA(cudaEventDestroy(ev));
  return LNG_OK;
}
