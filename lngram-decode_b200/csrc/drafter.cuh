// GPU drafter: the state machine and API of the reference C++ drafter
// (drafting/cpu/drafter.cpp:150-595) with every per-token step on the device.
//
// Per token x[t] (drafter.cpp:396-545): the SD-C SSM step s = a s + (1 - a) W_in RMSNorm(E[x[t]]) when
// the bundle has one; embed2 router features [RMSNorm(E[x[t-1]] or start), RMSNorm(E[x[t]])] (+ s for
// the embed2_ssm router) -> fp32 router -> sign codes; the rows of the n-grams ending at t (window of
// the last max(ngrams) codes, zero rows before the sequence start); the draft readout in folded form
// (w_qk / w_vo from W_q, the memory's norm + kv_proj, W_o; + the folded W_sq s for query_ssm),
// RMSNorm(out_norm); then the logits against the embedding -- over the sketch shortlist when the
// bundle has sketches (drafter_ext.cuh), else over the whole vocabulary -- with a fused top-k.
// draft() keeps the drafted tokens on the device: step i+1 reads step i's argmax from device memory,
// so a gamma-token draft costs one host round trip at the end.  The committed state (tokens, codes,
// SSM states) lives on the host, as in the reference, so truncate() is exact rollback.
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

// The draft step's first two launches in one: item i's token ids[i * id_stride] (also copied to
// ids_dense[i] when given), its embedding row to out[i] and 1/rms of that row to rs[i] -- the row's
// sum of squares read back from `out` exactly as rms_rows_kernel reads it, so rs is bit-identical.
template <typename T>
__global__ void gather_rms_kernel(const int64_t* __restrict__ ids, int64_t id_stride, int64_t n,
                                  const T* __restrict__ E, int64_t d, int64_t vocab, float eps, T* __restrict__ out,
                                  float* __restrict__ rs, int64_t* __restrict__ ids_dense) {
  const int lane = threadIdx.x & 31;
  const bool vec = d % Vec16<T>::N == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  for (int64_t row = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; row < n;
       row += (int64_t(gridDim.x) * blockDim.x) >> 5) {
    const int64_t id = ids[row * id_stride];
    const bool ok = id >= 0 && id < vocab;
    if (lane == 0) {
      if (ids_dense) ids_dense[row] = id;
      if (!ok) atomicCAS(&g_error_word, 0u, (unsigned int)DEV_ERR_TOKEN_RANGE);
    }
    T* o = out + row * d;
    for (int64_t j = lane; j < d; j += 32) o[j] = ok ? E[id * d + j] : from_f32<T>(0.f);
    __syncwarp();
    const float ss = row_sumsq(o, d, vec, lane);
    if (lane == 0) rs[row] = rsqrtf(ss / float(d) + eps);
  }
}

// The draft head's output RMSNorm (rms_norm_reg_kernel's arithmetic, fp32 rows in registers) that
// also writes the normalised row's three bf16 parts (split_rows_bf16x3_kernel's arithmetic) for the
// tensor-core logits: parts [n, 3d] = (y1 | y2 | y3).
__global__ void __launch_bounds__(256) norm_split_kernel(const float* __restrict__ x, int64_t n, int64_t d, int nv,
                                                         const float* __restrict__ w, float eps, float* __restrict__ y,
                                                         __nv_bfloat16* __restrict__ parts) {
  constexpr int N = Vec16<float>::N;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the logits kernel may start its set-up
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= n) return;
  const float* xr = x + row * d;
  float v[RN_NV][N];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < RN_NV; ++i) {
    if (i < nv) {
      Vec16<float>::load(xr + (int64_t(i) * 32 + lane) * N, v[i]);
#pragma unroll
      for (int k = 0; k < N; ++k) ss = fmaf(v[i][k], v[i][k], ss);
    }
  }
  const float r = rsqrtf(warp_sum(ss) / float(d) + eps);
  float* yr = y + row * d;
  __nv_bfloat16* pr = parts + row * 3 * d;
#pragma unroll
  for (int i = 0; i < RN_NV; ++i) {
    if (i < nv) {
      const int64_t j0 = (int64_t(i) * 32 + lane) * N;
#pragma unroll
      for (int k = 0; k < N; ++k) {
        const float yv = w ? v[i][k] * r * w[j0 + k] : v[i][k] * r;
        yr[j0 + k] = yv;
        const __nv_bfloat16 a = __float2bfloat16_rn(yv);
        const float r1 = yv - __bfloat162float(a);
        const __nv_bfloat16 b = __float2bfloat16_rn(r1);
        pr[j0 + k] = a;
        pr[d + j0 + k] = b;
        pr[2 * d + j0 + k] = __float2bfloat16_rn(r1 - __bfloat162float(b));
      }
    }
  }
}

// Top-1 of each draft row from the per-tile candidates (topk_merge_kernel at k = 1: the best in
// (value desc, id asc) order), written to ids / vals and, for the batched draft, straight into the
// token matrix and the caller's output (store_draft_kernel's two stores).
__global__ void top1_merge_store_kernel(const float* __restrict__ cand_v, const int64_t* __restrict__ cand_i, int64_t n,
                                        int64_t nchunks, int64_t* __restrict__ ids, float* __restrict__ vals,
                                        int64_t* __restrict__ toks, int64_t ts, int64_t* __restrict__ out, int64_t os) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5;
  if (row >= n) return;
  const float* cv = cand_v + row * nchunks;
  const int64_t* ci = cand_i + row * nchunks;
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  for (int64_t c = lane; c < nchunks; c += 32) {
    const float v = cv[c];
    const int64_t id = ci[c];
    if (id >= 0 && tk_better(v, id, bv, bi)) {
      bv = v;
      bi = id;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (tk_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    const int64_t id = bi == INT64_MAX ? -1 : bi;
    ids[row] = id;
    vals[row] = bi == INT64_MAX ? -INFINITY : bv;
    if (toks) toks[row * ts] = id;
    if (out) out[row * os] = id;
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
  int64_t F = 0;              // router feature width: 2d (+ N for the embed2_ssm router)
  // SD-C SSM (N = 0: none)
  int64_t N = 0;
  bool router_ssm = false, query_ssm = false;
  float ssm_eps = 0;
  float *ssm_norm = nullptr, *ssm_w_in = nullptr, *ssm_a = nullptr;
  void* w_sqk = nullptr;      // folded query map of W_sq [qh*Dt, N] (act dtype)
  // sketch shortlist (K = 0 or cap = 0: full-vocabulary scoring)
  int64_t K = 0, cap = 0;
  int ht = 0;                 // hash slots per shortlist item
  int32_t* sk_ids[LNG_MAX_ORDERS] = {};
  int32_t* sk_cnt[LNG_MAX_ORDERS] = {};
  int32_t* fallback = nullptr;
  int n_fallback = 0;
  std::vector<void*> owned;
  // host state (the reference keeps the same: drafter.cpp:571-574)
  std::vector<int64_t> tokens;
  std::vector<uint8_t> codes;
  std::vector<float> ssm;     // SSM state after each committed token [length, N]
  std::mutex mu;
  cudaStream_t stream = nullptr;
  // grow-on-demand device workspace
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // draft_batch replays: per (shape, workspace), the calls seen and the CUDA graph of the launches
  // (captured at the second call; null: not yet, or the sequence could not be captured)
  struct BatchGraph {
    int calls = 0;
    cudaGraphExec_t exec = nullptr;
  };
  std::map<std::tuple<int64_t, int64_t, int64_t, const void*>, BatchGraph> graphs;

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
  bool has_sketch() const { return K > 0 && cap > 0; }
  ~lng_drafter() {
    for (auto& kv : graphs)
      if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
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

// Upload a host int32 array (sketch ids / counts, fallback list).
static int upload_i32(lng_drafter* dr, const lng_array* a, int64_t expect, int32_t** out) {
  if (!a) return fail(LNG_ERR_ARGUMENT, "bundle array missing");
  const int64_t n = array_numel(a);
  if (expect >= 0 && n != expect)
    return fail(LNG_ERR_ARGUMENT, std::string("bundle array ") + a->name + " has the wrong size");
  if (a->dtype != LNG_I32) return fail(LNG_ERR_ARGUMENT, std::string("bundle array ") + a->name + " must be int32");
  void* p = nullptr;
  int st = drafter_alloc(dr, size_t(n) * 4, &p);
  if (st) return st;
  if (n) LNG_CUDA(cudaMemcpy(p, a->data_host, size_t(n) * 4, cudaMemcpyHostToDevice));
  *out = static_cast<int32_t*>(p);
  return LNG_OK;
}

struct ReadoutBufs {
  int64_t rows;  // capacity in items of the per-item buffers below
  void* x;       // [rows, d] embedding rows (E dtype)
  float* qs;     // [rows]
  void* qa;      // [rows, qh*Dt] act
  void* u;       // [rows, qh*Dt] act
  float* hid;    // [rows, d]
  float* hn;     // [rows, d]
  int64_t* ids;  // [rows, k]
  float* vals;   // [rows, k]
  void* scratch; size_t scratch_bytes;
  float* feat;   // [rows, F]
  __nv_bfloat16* feat_parts;  // [rows, 3F] the router features' bf16x3 parts
};

static int drafter_ws(lng_drafter* dr, int64_t M, int k, ReadoutBufs* b, size_t extra_bytes, void** extra) {
  const size_t es = size_t(dtype_size(dr->e_dtype)), as = size_t(dtype_size(dr->act));
  const size_t qd = size_t(dr->qh * dr->Dt);
  const size_t sizes[11] = {al256(size_t(M) * dr->d * es), al256(size_t(M) * 4), al256(size_t(M) * qd * as),
                            al256(size_t(M) * qd * as), al256(size_t(M) * dr->d * 4), al256(size_t(M) * dr->d * 4),
                            al256(size_t(M) * k * 8), al256(size_t(M) * k * 4),
                            al256(lng_logits_topk_scratch_bytes(M, dr->d, dr->V, k)), al256(size_t(M) * dr->F * 4),
                            al256(size_t(M) * 3 * dr->F * 2)};
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
  void* ptrs[11];
  for (int i = 0; i < 11; ++i) {
    ptrs[i] = p;
    p += sizes[i];
  }
  b->rows = M;
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
  b->feat_parts = static_cast<__nv_bfloat16*>(ptrs[10]);
  if (extra) *extra = extra_bytes ? p : nullptr;
  return LNG_OK;
}

static int gather_embedding(lng_drafter* dr, const int64_t* tok, int64_t n, void* out) {
  cudaStream_t s = dr->stream;
#define LNG_GR(T) gather_rows_kernel<T><<<grid_for(n * dr->d, 256, 8), 256, 0, s>>>(tok, n, static_cast<const T*>(dr->E), dr->d, dr->V, static_cast<T*>(out))
  if (dr->e_dtype == LNG_F32) LNG_GR(float);
  else if (dr->e_dtype == LNG_BF16) LNG_GR(__nv_bfloat16);
  else LNG_GR(__half);
#undef LNG_GR
  LNG_LAUNCHED("gather_rows_kernel");
  return LNG_OK;
}

// SSM inputs u[i] = W_in RMSNorm(E[tok[i]]; ssm_norm) (fp32 [n, N]) in chunks of the workspace's rows
// (ffnmem/memory/ssm.py:40-43; drafter.cpp:399-401).
static int drafter_ssm_inputs(lng_drafter* dr, const int64_t* tok, int64_t n, ReadoutBufs& b, float* u) {
  lng_stream_t ls = reinterpret_cast<lng_stream_t>(dr->stream);
  for (int64_t c0 = 0; c0 < n; c0 += b.rows) {
    const int64_t m = std::min<int64_t>(b.rows, n - c0);
    int st = gather_embedding(dr, tok + c0, m, b.x);
    if (st) return st;
    st = lng_rms_norm(b.x, dr->e_dtype, m, dr->d, dr->ssm_norm, dr->ssm_eps, b.hid, LNG_F32, ls);
    if (st) return st;
    st = lng_gemm(b.hid, LNG_F32, dr->d, dr->ssm_w_in, LNG_F32, dr->d, u + c0 * dr->N, LNG_F32, dr->N, m, dr->N,
                  dr->d, nullptr, 0, ls);
    if (st) return st;
  }
  return LNG_OK;
}

// The recurrence over nseq sequences of L inputs each (u [nseq, L, N]) from s0 [nseq, N] (NULL =
// zeros): the states of positions >= out_from into states [nseq, L - out_from, N].
static int drafter_ssm_scan(lng_drafter* dr, const float* u, int64_t nseq, int64_t L, const float* s0,
                            int64_t out_from, float* states) {
  const int64_t n = nseq * dr->N;
  ssm_scan_kernel<<<unsigned(ceil_div(n, 128)), 128, 0, dr->stream>>>(u, nseq, L, dr->N, dr->ssm_a, s0, out_from,
                                                                       states);
  LNG_LAUNCHED("ssm_scan_kernel");
  return LNG_OK;
}

// Codes of M tokens given their previous tokens (device i64 arrays; prev = -1 -> start vector) and,
// for the embed2_ssm router, their SSM states s_rows [M, N].
static int drafter_codes(lng_drafter* dr, const int64_t* cur, const int64_t* prev, int64_t M, float* feat,
                         uint8_t* codes_out, int64_t codes_stride, const float* s_rows,
                         __nv_bfloat16* feat_parts = nullptr) {
  // the token-only router's features go to the tensor cores already split into bf16 parts
  __nv_bfloat16* parts = (!dr->router_ssm && codes_stride == dr->R && M <= 256) ? feat_parts : nullptr;
  int st = embed2_features(cur, prev, M, dr->E, dr->e_dtype, dr->V, dr->d, dr->prev_norm, dr->cur_norm, dr->start,
                           dr->router_eps, feat, dr->F, dr->stream, parts, dr->F);
  if (st) return st;
  if (dr->router_ssm) {
    LNG_REQUIRE(s_rows, "internal: the SSM router needs the states");
    copy_cols_kernel<<<grid_for(M * dr->N, 256, 8), 256, 0, dr->stream>>>(s_rows, M, dr->N, feat, dr->F, 2 * dr->d);
    LNG_LAUNCHED("copy_cols_kernel");
  }
  if (codes_stride == dr->R)
    return route_codes_presplit(feat, M, dr->F, dr->router_w, dr->router_w_split, dr->R, int32_t(dr->bits), codes_out,
                                dr->stream, parts);
  for (int64_t i = 0; i < M; ++i) {  // strided destination: one row at a time
    st = route_codes_presplit(feat + i * dr->F, 1, dr->F, dr->router_w, dr->router_w_split, dr->R, int32_t(dr->bits),
                              codes_out + i * codes_stride, dr->stream);
    if (st) return st;
  }
  return LNG_OK;
}

// How a readout scores the vocabulary: the sketch shortlist unless `full` (or no sketch); in trace
// mode (list_ids != NULL) the shortlist and its logits in list order [M, S].
struct Scoring {
  bool full = false;
  float* full_logits = nullptr;  // [M, V] when full-vocabulary logits are wanted
  int64_t S = 0;
  int64_t* list_ids = nullptr;
  float* list_lg = nullptr;
};

static int launch_shortlist(lng_drafter* dr, const CodeSource& src, int64_t M, const float* hn, int topk,
                            int64_t* ids, float* vals, const Scoring& sc) {
  ShortlistParams p{};
  p.src = src;
  for (int o = 0; o < dr->n_orders; ++o) {
    p.orders[o] = dr->orders[o];
    p.sk_ids[o] = dr->sk_ids[o];
    p.sk_cnt[o] = dr->sk_cnt[o];
  }
  p.n_orders = dr->n_orders;
  p.bits = int(dr->bits);
  p.R = dr->R;
  p.K = int(dr->K);
  p.fallback = dr->fallback;
  p.n_fallback = dr->n_fallback;
  p.cap = int(dr->cap);
  p.V = dr->V;
  p.d = dr->d;
  p.E = dr->E;
  p.e_dtype = dr->e_dtype;
  p.hn = hn;
  p.M = M;
  p.ht = dr->ht;
  p.topk = sc.list_ids ? 0 : topk;
  p.ids = ids;
  p.vals = vals;
  p.S = sc.S;
  p.list_ids = sc.list_ids;
  p.list_lg = sc.list_lg;
  const size_t smem = size_t(dr->ht) * 8 + size_t(dr->d) * 4 + size_t(dr->cap) * 8;
  auto kern = shortlist_kernel<uint8_t>;
  LNG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(M, int64_t(num_sms()))));
  kern<<<grid, SL_THREADS, smem, dr->stream>>>(p);
  LNG_LAUNCHED("shortlist_kernel");
  return LNG_OK;
}

// Where a batched draft stores each step's top-1 besides ids: the token matrix and the caller's output
// (strided), written by the merge kernel itself.
struct DraftStore {
  int64_t* toks = nullptr;
  int64_t ts = 0;
  int64_t* out = nullptr;
  int64_t os = 0;
};

// Draft-head logits + top-k over the whole vocabulary on lng_logits_topk's scratch layout; `presplit`:
// the three bf16 parts of hn are in place already (norm_split_kernel); with `store` and k = 1 the merge
// also writes the drafted tokens.
static int drafter_logits(lng_drafter* dr, ReadoutBufs& b, int64_t M, int k, float* full_logits, bool presplit,
                          const DraftStore* store) {
  const int64_t nch = ceil_div(dr->V, TK_VC);
  LNG_REQUIRE(b.scratch_bytes >= lng_logits_topk_scratch_bytes(M, dr->d, dr->V, k), "internal: logits scratch");
  const uintptr_t base = (reinterpret_cast<uintptr_t>(b.scratch) + 255) & ~uintptr_t(255);
  int64_t* cand_i = reinterpret_cast<int64_t*>(base);
  float* cand_v = reinterpret_cast<float*>(cand_i + M * nch * k);
  auto* split = reinterpret_cast<__nv_bfloat16*>(base + al256(topk_cand_bytes(M, dr->V, k)));
  int st = logits_chunks(b.hn, M, dr->d, dr->E, dr->e_dtype, dr->V, k, cand_v, cand_i, full_logits, split, dr->stream,
                         presplit, presplit);
  if (st) return st;
  if (store && k == 1) {
    top1_merge_store_kernel<<<unsigned(ceil_div(M * 32, 256)), 256, 0, dr->stream>>>(
        cand_v, cand_i, M, nch, b.ids, b.vals, store->toks, store->ts, store->out, store->os);
    LNG_LAUNCHED("top1_merge_store_kernel");
  } else {
    topk_merge_kernel<<<unsigned(ceil_div(M * 32, 256)), 256, 0, dr->stream>>>(cand_v, cand_i, M, nch, k, b.ids,
                                                                              b.vals);
    LNG_LAUNCHED("topk_merge_kernel");
    if (store) {
      store_draft_kernel<<<unsigned(ceil_div(M, 128)), 128, 0, dr->stream>>>(b.ids, M, store->toks, store->ts,
                                                                             store->out, store->os);
      LNG_LAUNCHED("store_draft_kernel");
    }
  }
  return LNG_OK;
}

// Readout of M items: embedding rows of the tokens cur[i * cur_stride] (copied densely to cur_dense
// when given), the item's code window per `src`, the SSM states s_rows [M, N] for query_ssm, then
// top-k (or the trace outputs) per `sc`; `store`: where the batched draft's top-1 goes as well.
static int drafter_readout(lng_drafter* dr, const int64_t* cur, int64_t M, const CodeSource& src, int k,
                           ReadoutBufs& b, const Scoring& sc, const float* s_rows, int64_t cur_stride = 1,
                           int64_t* cur_dense = nullptr, const DraftStore* store = nullptr) {
  cudaStream_t s = dr->stream;
  lng_stream_t ls = reinterpret_cast<lng_stream_t>(s);
  const int64_t qd = dr->qh * dr->Dt;
  int st = LNG_OK;
  {  // embedding rows and their 1/rms in one launch
    const int g = grid_for(M * 32, 256, 16);
#define LNG_GRMS(T)                                                                                            \
  gather_rms_kernel<T><<<g, 256, 0, s>>>(cur, cur_stride, M, static_cast<const T*>(dr->E), dr->d, dr->V,     \
                                         dr->draft_eps, static_cast<T*>(b.x), b.qs, cur_dense)
    if (dr->e_dtype == LNG_F32) LNG_GRMS(float);
    else if (dr->e_dtype == LNG_BF16) LNG_GRMS(__nv_bfloat16);
    else LNG_GRMS(__half);
#undef LNG_GRMS
    LNG_LAUNCHED("gather_rms_kernel");
  }
  const float* qscale = b.qs;
  if (dr->query_ssm) {
    // qa = rs(x) (x . w_qk^T) + s . w_sqk^T: the SSM term carries no RMS scale (drafter.cpp:505-508)
    LNG_REQUIRE(s_rows, "internal: the SSM query needs the states");
    st = lng_gemm(b.x, dr->e_dtype, dr->d, dr->w_qk, dr->act, dr->d, b.qa, dr->act, qd, M, qd, dr->d, b.qs, 0, ls);
    if (st) return st;
    st = lng_gemm(s_rows, LNG_F32, dr->N, dr->w_sqk, dr->act, dr->N, b.qa, dr->act, qd, M, qd, dr->N, nullptr, 1, ls);
    if (st) return st;
    qscale = nullptr;
  } else {
    st = lng_gemm(b.x, dr->e_dtype, dr->d, dr->w_qk, dr->act, dr->d, b.qa, dr->act, qd, M, qd, dr->d, nullptr, 0, ls);
    if (st) return st;
  }
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
  p.qscale = qscale;
  p.u = b.u;
  st = attend_impl<uint8_t>(&t, p, dr->act, s);
  if (st) return st;
  st = lng_gemm(b.u, dr->act, qd, dr->w_vo, dr->act, qd, b.hid, LNG_F32, dr->d, M, dr->d, qd, nullptr, 0, ls);
  if (st) return st;
  const bool shortlist = dr->has_sketch() && !sc.full;
  // full-vocabulary logits on the tensor cores: the output norm also writes the rows' bf16 parts
  const int64_t vec_elems = 32 * Vec16<float>::N;
  const bool fuse = !shortlist && logits_tc_ok(dr->d, dr->E, dr->e_dtype, dr->V) && dr->d % vec_elems == 0 &&
                    dr->d / vec_elems <= RN_NV;
  if (fuse) {
    const uintptr_t base = (reinterpret_cast<uintptr_t>(b.scratch) + 255) & ~uintptr_t(255);
    auto* parts = reinterpret_cast<__nv_bfloat16*>(base + al256(topk_cand_bytes(M, dr->V, k)));
    norm_split_kernel<<<unsigned(ceil_div(M, 8)), 256, 0, s>>>(b.hid, M, dr->d, int(dr->d / vec_elems), dr->out_norm,
                                                               dr->draft_eps, b.hn, parts);
    LNG_LAUNCHED("norm_split_kernel");
  } else {
    st = lng_rms_norm(b.hid, LNG_F32, M, dr->d, dr->out_norm, dr->draft_eps, b.hn, LNG_F32, ls);
    if (st) return st;
  }
  if (shortlist) {
    st = launch_shortlist(dr, src, M, b.hn, k, b.ids, b.vals, sc);
    if (st || !store) return st;
    store_draft_kernel<<<unsigned(ceil_div(M, 128)), 128, 0, s>>>(b.ids, M, store->toks, store->ts, store->out,
                                                                  store->os);
    LNG_LAUNCHED("store_draft_kernel");
    return LNG_OK;
  }
  return drafter_logits(dr, b, M, k, sc.full_logits, fuse, store);
}

}  // namespace lng

extern "C" int lng_drafter_create(const lng_drafter_numbers* num, const lng_array* arrays, int32_t n_arrays,
                                  int32_t act_dtype, lng_drafter** out) {
  LNG_REQUIRE(num && arrays && out, "NULL pointer");
  *out = nullptr;
  LNG_REQUIRE(act_dtype == LNG_F32 || act_dtype == LNG_BF16, "act dtype must be f32 or bf16");
  LNG_REQUIRE(num->n_orders >= 1 && num->n_orders <= LNG_MAX_ORDERS, "n_orders must be in [1, 4]");
  LNG_REQUIRE(num->q_heads % num->kv_heads == 0 && num->q_heads <= 64, "q_heads must be a multiple of kv_heads");
  LNG_REQUIRE(num->bits >= 1 && num->bits <= 8, "bits must be in [1, 8]");
  LNG_REQUIRE(num->ssm_dim >= 0 && num->sketch_k >= 0, "bad ssm_dim / sketch_k");
  LNG_REQUIRE(!(num->router_ssm || num->query_ssm) || num->ssm_dim > 0, "an SSM router / query needs ssm_dim > 0");
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
  dr->ssm_eps = float(num->ssm_eps);
  dr->sink = float(num->sink_logit);
  dr->act = act_dtype;
  dr->N = num->ssm_dim;
  dr->router_ssm = num->router_ssm != 0;
  dr->query_ssm = num->query_ssm != 0;
  dr->F = 2 * dr->d + (dr->router_ssm ? dr->N : 0);
  dr->K = num->sketch_k;
  dr->cap = num->shortlist_cap > 0 ? num->shortlist_cap : 0;
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
  if ((st = upload_f32(D, find_array(arrays, n_arrays, "router"), D->R * D->bits * D->F, &D->router_w))) return st;
  {  // the router weight's bf16x3 split, used by every small-batch code computation of this drafter
    const int64_t rows = D->R * D->bits, in_dim = D->F;
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
  if (D->N > 0) {  // SD-C: the SSM and, for query_ssm, the folded W_sq
    if ((st = upload_f32(D, find_array(arrays, n_arrays, "ssm_norm"), D->d, &D->ssm_norm))) return st;
    if ((st = upload_f32(D, find_array(arrays, n_arrays, "ssm_w_in"), D->N * D->d, &D->ssm_w_in))) return st;
    if ((st = upload_f32(D, find_array(arrays, n_arrays, "ssm_decay"), D->N, &D->ssm_a))) return st;
    if (D->query_ssm) {
      float* w_sq = nullptr;
      if ((st = upload_f32(D, find_array(arrays, n_arrays, "w_sq"), I * D->N, &w_sq))) return st;
      std::vector<float> ones(size_t(D->N), 1.f);
      void* onesd = nullptr;
      if ((st = drafter_alloc(D, size_t(D->N) * 4, &onesd))) return st;
      LNG_CUDA(cudaMemcpy(onesd, ones.data(), size_t(D->N) * 4, cudaMemcpyHostToDevice));
      if ((st = drafter_alloc(D, size_t(D->qh * D->Dt * D->N) * as, &D->w_sqk))) return st;
      st = lng_fold_readout(D->N, D->Dt, int32_t(D->qh), int32_t(D->kv), int32_t(D->hd), static_cast<float*>(onesd),
                            w_sq, mem_norm, kv_proj, nullptr, D->w_sqk, nullptr, act_dtype, nullptr);
      if (st) return st;
    }
  }
  if (D->has_sketch()) {  // the sketch shortlist
    const int64_t cand = int64_t(D->n_orders) * D->R * D->K;
    int64_t ht = 1;
    while (ht < 2 * cand) ht <<= 1;
    if (ht > SL_MAX_SLOTS)
      return fail(LNG_ERR_UNSUPPORTED, "sketch shortlist: orders x routes x sketch_k = " + std::to_string(cand) +
                                           " entries per position exceed the " + std::to_string(SL_MAX_SLOTS / 2) +
                                           " this build sums in shared memory");
    LNG_REQUIRE(D->V < (int64_t(1) << SL_ID_BITS) - 1, "sketch shortlist: vocabulary too large");
    LNG_REQUIRE(size_t(ht) * 8 + size_t(D->d) * 4 + size_t(D->cap) * 8 <= 227 * 1024,
                "sketch shortlist: shortlist_cap too large");
    D->ht = int(ht);
    for (int o = 0; o < D->n_orders; ++o) {
      const int64_t rows = D->R << (D->bits * D->orders[o]);
      const std::string n = std::to_string(D->orders[o]);
      if ((st = upload_i32(D, find_array(arrays, n_arrays, ("sketch_ids_" + n).c_str()), rows * D->K, &D->sk_ids[o])))
        return st;
      if ((st = upload_i32(D, find_array(arrays, n_arrays, ("sketch_counts_" + n).c_str()), rows * D->K,
                           &D->sk_cnt[o])))
        return st;
    }
    const lng_array* fb = find_array(arrays, n_arrays, "fallback");
    if (fb && array_numel(fb) > 0) {
      if ((st = upload_i32(D, fb, -1, &D->fallback))) return st;
      D->n_fallback = int(array_numel(fb));
    }
  }
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
  d->ssm.clear();
  return LNG_OK;
}

extern "C" int64_t lng_drafter_length(const lng_drafter* d) { return d ? int64_t(d->tokens.size()) : -1; }

extern "C" int lng_drafter_truncate(lng_drafter* d, int64_t n) {
  LNG_REQUIRE(d, "NULL drafter");
  std::lock_guard<std::mutex> lk(d->mu);
  if (n < 0 || n > int64_t(d->tokens.size())) return fail(LNG_ERR_STATE, "cannot truncate to " + std::to_string(n));
  d->tokens.resize(size_t(n));
  d->codes.resize(size_t(n * d->R));
  d->ssm.resize(size_t(n * d->N));
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

// Codes (and SSM states) of `n` new tokens after the committed state, on the device; written to
// codes_host [n, R] (unless the caller's codes replace them) and states_host [n, N].
static int drafter_codes_for(lng_drafter* d, const int64_t* toks_host, int64_t n, uint8_t* codes_host,
                             bool own_codes, float* states_host) {
  ReadoutBufs b;
  void* extra = nullptr;
  const size_t tb = al256(size_t(2 * n) * 8), cb = al256(size_t(n * d->R)), sb = al256(size_t(n * d->N) * 4);
  const size_t s0b = al256(size_t(d->N) * 4);
  int st = drafter_ws(d, std::min<int64_t>(n, 4096), 1, &b, tb + cb + 2 * sb + s0b, &extra);
  if (st) return st;
  unsigned char* ex = static_cast<unsigned char*>(extra);
  int64_t* cur = reinterpret_cast<int64_t*>(ex);
  int64_t* prev = cur + n;
  uint8_t* cd = ex + tb;
  float* u = reinterpret_cast<float*>(ex + tb + cb);
  float* states = reinterpret_cast<float*>(ex + tb + cb + sb);
  float* s0 = reinterpret_cast<float*>(ex + tb + cb + 2 * sb);
  std::vector<int64_t> host(size_t(2 * n));
  for (int64_t i = 0; i < n; ++i) {
    host[size_t(i)] = toks_host[i];
    host[size_t(n + i)] = i > 0 ? toks_host[i - 1] : (d->tokens.empty() ? -1 : d->tokens.back());
  }
  LNG_CUDA(cudaMemcpyAsync(cur, host.data(), size_t(2 * n) * 8, cudaMemcpyHostToDevice, d->stream));
  if (d->N > 0) {
    const bool have_prev = !d->ssm.empty();
    if (have_prev)
      LNG_CUDA(cudaMemcpyAsync(s0, d->ssm.data() + d->ssm.size() - size_t(d->N), size_t(d->N) * 4,
                               cudaMemcpyHostToDevice, d->stream));
    st = drafter_ssm_inputs(d, cur, n, b, u);
    if (st) return st;
    st = drafter_ssm_scan(d, u, 1, n, have_prev ? s0 : nullptr, 0, states);
    if (st) return st;
    LNG_CUDA(cudaMemcpyAsync(states_host, states, size_t(n * d->N) * 4, cudaMemcpyDeviceToHost, d->stream));
  }
  if (own_codes) {
    // the features of more rows than the workspace holds go in workspace-sized pieces
    for (int64_t c0 = 0; c0 < n; c0 += b.rows) {
      const int64_t m = std::min<int64_t>(b.rows, n - c0);
      st = drafter_codes(d, cur + c0, prev + c0, m, b.feat, cd + c0 * d->R, d->R, d->N > 0 ? states + c0 * d->N : nullptr);
      if (st) return st;
    }
    LNG_CUDA(cudaMemcpyAsync(codes_host, cd, size_t(n * d->R), cudaMemcpyDeviceToHost, d->stream));
  }
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
  std::vector<float> states(size_t(n * d->N));
  if (codes_host)
    for (int64_t i = 0; i < n * d->R; ++i) c[size_t(i)] = uint8_t(codes_host[i]);
  if (!codes_host || d->N > 0) {
    int st = drafter_codes_for(d, tokens_host, n, c.data(), codes_host == nullptr, states.data());
    if (st) return st;
  }
  d->tokens.insert(d->tokens.end(), tokens_host, tokens_host + n);
  d->codes.insert(d->codes.end(), c.begin(), c.end());
  d->ssm.insert(d->ssm.end(), states.begin(), states.end());
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
  const int64_t W = d->maxn, R = d->R, N = d->N;
  // slots: W-1 history slots, then hyp tokens, then drafted tokens (positions L-W+1 ..)
  const int64_t nslots = (W - 1) + 1 + n_hyp + gamma;  // +1: the last committed token's slot
  const int64_t n_codes = n_hyp + (last_codes ? gamma : std::max<int64_t>(gamma - 1, 0));
  ReadoutBufs b;
  void* extra = nullptr;
  // SSM states of the slots from W-1 on: row 0 = the last committed token's (zeros if none), then the
  // hypothesis tokens', then the drafted tokens'
  const int64_t srows = 1 + n_hyp + gamma;
  const size_t tok_b = al256(size_t(nslots + 1) * 8), seg_b = al256(size_t(gamma * W) * 4), ids_b = al256(size_t(gamma * topk) * 8),
               val_b = al256(size_t(gamma * topk) * 4), code_b = al256(size_t(nslots * R)),
               ssm_b = al256(size_t(srows * N) * 4), u_b = al256(size_t(std::max<int64_t>(n_hyp, 1) * N) * 4);
  int st = drafter_ws(d, std::max<int64_t>(1, n_hyp), topk, &b,
                      tok_b + seg_b + ids_b + val_b + code_b + ssm_b + u_b, &extra);
  if (st) return st;
  unsigned char* ex = static_cast<unsigned char*>(extra);
  int64_t* dtok = reinterpret_cast<int64_t*>(ex);            // dtok[s + 1] = token of slot s; dtok[0] = -1
  int32_t* dseg = reinterpret_cast<int32_t*>(ex + tok_b);
  int64_t* dids = reinterpret_cast<int64_t*>(ex + tok_b + seg_b);
  float* dvals = reinterpret_cast<float*>(ex + tok_b + seg_b + ids_b);
  uint8_t* dcodes = ex + tok_b + seg_b + ids_b + val_b;      // [nslots, R]
  float* dssm = reinterpret_cast<float*>(ex + tok_b + seg_b + ids_b + val_b + code_b);   // [srows, N]
  float* du = reinterpret_cast<float*>(ex + tok_b + seg_b + ids_b + val_b + code_b + ssm_b);
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
  if (N > 0) {
    if (L > 0)
      LNG_CUDA(cudaMemcpyAsync(dssm, d->ssm.data() + size_t((L - 1) * N), size_t(N) * 4, cudaMemcpyHostToDevice,
                               d->stream));
    else
      LNG_CUDA(cudaMemsetAsync(dssm, 0, size_t(N) * 4, d->stream));
  }
  // hypothetical tokens: their SSM states and codes in one batched pass (prev of slot s is slot s-1)
  if (n_hyp > 0) {
    if (N > 0) {
      st = drafter_ssm_inputs(d, dtok + W + 1, n_hyp, b, du);
      if (st) return st;
      st = drafter_ssm_scan(d, du, 1, n_hyp, dssm, 0, dssm + N);
      if (st) return st;
    }
    st = drafter_codes(d, dtok + W + 1, dtok + W, n_hyp, b.feat, dcodes + W * R, R, N > 0 ? dssm + N : nullptr);
    if (st) return st;
  }
  for (int64_t g = 0; g < gamma; ++g) {
    const int64_t end = W - 1 + n_hyp + g;  // slot of the current token
    const float* s_cur = N > 0 ? dssm + (n_hyp + g) * N : nullptr;
    CodeSource src{dcodes + (end - W + 1) * R, 0, 0, W, R, nullptr, nullptr, dseg + g * W, 0, 0};
    st = drafter_readout(d, dtok + end + 1, 1, src, topk, b, Scoring{}, s_cur);
    if (st) return st;
    LNG_CUDA(cudaMemcpyAsync(dids + g * topk, b.ids, size_t(topk) * 8, cudaMemcpyDeviceToDevice, d->stream));
    LNG_CUDA(cudaMemcpyAsync(dvals + g * topk, b.vals, size_t(topk) * 4, cudaMemcpyDeviceToDevice, d->stream));
    if (g + 1 < gamma || last_codes) {
      copy_i64_kernel<<<1, 32, 0, d->stream>>>(b.ids, dtok + end + 2, 1, 1, 1);
      LNG_LAUNCHED("copy_i64_kernel");
      float* s_next = N > 0 ? dssm + (n_hyp + g + 1) * N : nullptr;
      if (N > 0) {
        st = drafter_ssm_inputs(d, dtok + end + 2, 1, b, du);
        if (st) return st;
        st = drafter_ssm_scan(d, du, 1, 1, s_cur, 0, s_next);
        if (st) return st;
      }
      st = drafter_codes(d, dtok + end + 2, dtok + end + 1, 1, b.feat, dcodes + (end + 1) * R, R, s_next);
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
  // the reference's column count: the whole vocabulary unless the shortlist applies (drafter.cpp:333-334)
  const bool full_vocab = full || !d->has_sketch();
  const int64_t S_ref = full_vocab ? d->V : d->cap;
  LNG_REQUIRE(T >= 0 && S == S_ref, "trace: S must be the vocabulary (full or no sketch) or shortlist_cap");
  if (T == 0) return LNG_OK;
  LNG_REQUIRE(tokens_host, "NULL pointer");
  std::lock_guard<std::mutex> lk(d->mu);
  for (int64_t i = 0; i < T; ++i)
    if (tokens_host[i] < 0 || tokens_host[i] >= d->V) return fail(LNG_ERR_STATE, "token id out of range");
  const int64_t R = d->R, N = d->N;
  ReadoutBufs b;
  void* extra = nullptr;
  const size_t tok_b = al256(size_t(2 * T) * 8), code_b = al256(size_t(T * R)), lg_b = al256(size_t(T * S) * 4),
               li_b = full_vocab ? 0 : al256(size_t(T * S) * 8), ssm_b = al256(size_t(T * N) * 4);
  int st = drafter_ws(d, T, 1, &b, tok_b + code_b + lg_b + li_b + 2 * ssm_b, &extra);
  if (st) return st;
  unsigned char* ex = static_cast<unsigned char*>(extra);
  int64_t* cur = reinterpret_cast<int64_t*>(ex);
  int64_t* prev = cur + T;
  uint8_t* dcodes = ex + tok_b;
  float* dlog = reinterpret_cast<float*>(ex + tok_b + code_b);
  int64_t* dlist = full_vocab ? nullptr : reinterpret_cast<int64_t*>(ex + tok_b + code_b + lg_b);
  float* du = reinterpret_cast<float*>(ex + tok_b + code_b + lg_b + li_b);
  float* dstates = reinterpret_cast<float*>(ex + tok_b + code_b + lg_b + li_b + ssm_b);
  std::vector<int64_t> host(size_t(2 * T));
  for (int64_t i = 0; i < T; ++i) {
    host[size_t(i)] = tokens_host[i];
    host[size_t(T + i)] = i > 0 ? tokens_host[i - 1] : -1;
  }
  LNG_CUDA(cudaMemcpyAsync(cur, host.data(), size_t(2 * T) * 8, cudaMemcpyHostToDevice, d->stream));
  if (N > 0) {  // SSM states from the empty state
    st = drafter_ssm_inputs(d, cur, T, b, du);
    if (st) return st;
    st = drafter_ssm_scan(d, du, 1, T, nullptr, 0, dstates);
    if (st) return st;
  }
  if (codes_host) {
    std::vector<uint8_t> c(size_t(T * R));
    for (int64_t i = 0; i < T * R; ++i) c[size_t(i)] = uint8_t(codes_host[i]);
    LNG_CUDA(cudaMemcpyAsync(dcodes, c.data(), size_t(T * R), cudaMemcpyHostToDevice, d->stream));
    LNG_CUDA(cudaStreamSynchronize(d->stream));
  } else {
    st = drafter_codes(d, cur, prev, T, b.feat, dcodes, R, N > 0 ? dstates : nullptr);
    if (st) return st;
  }
  CodeSource src{dcodes, 1, T, 0, R, nullptr, nullptr, nullptr, 0, T};
  Scoring sc;
  sc.full = full_vocab;
  if (full_vocab) {
    sc.full_logits = dlog;
  } else {
    sc.S = S;
    sc.list_ids = dlist;
    sc.list_lg = dlog;
  }
  st = drafter_readout(d, cur, T, src, 1, b, sc, N > 0 ? dstates : nullptr);
  if (st) return st;
  if (codes_out_host) LNG_CUDA(cudaMemcpyAsync(codes_out_host, dcodes, size_t(T * R), cudaMemcpyDeviceToHost, d->stream));
  if (logits_host) LNG_CUDA(cudaMemcpyAsync(logits_host, dlog, size_t(T * S) * 4, cudaMemcpyDeviceToHost, d->stream));
  if (ids_host && !full_vocab)
    LNG_CUDA(cudaMemcpyAsync(ids_host, dlist, size_t(T * S) * 8, cudaMemcpyDeviceToHost, d->stream));
  LNG_CUDA(cudaStreamSynchronize(d->stream));
  const int derr = lng_device_error(1);
  if (derr) return fail(LNG_ERR_DEVICE, "device error " + std::to_string(derr) + " during trace");
  if (ids_host && full_vocab)
    for (int64_t t = 0; t < T; ++t)
      for (int64_t v = 0; v < d->V; ++v) ids_host[t * d->V + v] = v;
  return LNG_OK;
}

namespace lng {

struct DraftBatchPlan {
  int64_t nseq, plen, gamma, tail, P;
  size_t pre_b, out_b, tok_b, prev_b, code_b, u_b, st_b, cur_b;
  size_t total() const { return pre_b + out_b + tok_b + prev_b + code_b + u_b + st_b + cur_b; }
};

// Every device operation of one draft_batch call on d->stream (the workspace already sized): from the
// prefix copy in the workspace to the drafted tokens in the workspace, so a captured graph of it
// depends on the shape and the workspace only.
static int enqueue_draft_batch(lng_drafter* d, const DraftBatchPlan& pl, ReadoutBufs& b, void* extra) {
  const int64_t R = d->R, N = d->N, nseq = pl.nseq, plen = pl.plen, gamma = pl.gamma, tail = pl.tail, P = pl.P;
  int st = LNG_OK;
  const int64_t* prefix = static_cast<const int64_t*>(extra);                                      // [nseq, plen]
  int64_t* tokens_out = reinterpret_cast<int64_t*>(static_cast<unsigned char*>(extra) + pl.pre_b);  // [nseq, gamma]
  unsigned char* ex = static_cast<unsigned char*>(extra) + pl.pre_b + pl.out_b;
  int64_t* toks = reinterpret_cast<int64_t*>(ex);  // [nseq, P + 1]: toks[s, 0] = -1, toks[s, 1 + p] = token p
  int64_t* scratch_i = reinterpret_cast<int64_t*>(ex + pl.tok_b);  // [2, nseq * tail]: current, previous tokens
  uint8_t* codes = ex + pl.tok_b + pl.prev_b;             // [nseq, P, R]
  float* u = reinterpret_cast<float*>(ex + pl.tok_b + pl.prev_b + pl.code_b);                       // [nseq, plen, N]
  float* tail_states = reinterpret_cast<float*>(ex + pl.tok_b + pl.prev_b + pl.code_b + pl.u_b);    // [nseq, tail, N]
  float* s_cur = reinterpret_cast<float*>(ex + pl.tok_b + pl.prev_b + pl.code_b + pl.u_b + pl.st_b);  // [nseq, N] x 2
  float* s_next = s_cur + nseq * N;
  // token matrix with a -1 column for the start vector, then prefix codes in one batched pass
  LNG_CUDA(cudaMemsetAsync(toks, 0xff, size_t(nseq * (P + 1)) * 8, d->stream));
  LNG_CUDA(cudaMemcpy2DAsync(toks + 1, size_t(P + 1) * 8, prefix, size_t(plen) * 8, size_t(plen) * 8, size_t(nseq),
                             cudaMemcpyDeviceToDevice, d->stream));
  const int64_t p0 = plen - tail;
  if (N > 0) {  // the SSM over every prefix token; the states of the last `tail` positions are kept
    st = drafter_ssm_inputs(d, prefix, nseq * plen, b, u);
    if (st) return st;
    st = drafter_ssm_scan(d, u, nseq, plen, nullptr, p0, tail_states);
    if (st) return st;
    LNG_CUDA(cudaMemcpy2DAsync(s_cur, size_t(N) * 4, tail_states + (tail - 1) * N, size_t(tail * N) * 4,
                               size_t(N) * 4, size_t(nseq), cudaMemcpyDeviceToDevice, d->stream));
  }
  // tokens of the last `tail` prefix positions (dense [nseq, tail]) and their previous tokens
  // (toks[s, p] is the token before position p, -1 at p = 0)
  LNG_CUDA(cudaMemcpy2DAsync(scratch_i, size_t(tail) * 8, prefix + p0, size_t(plen) * 8, size_t(tail) * 8,
                             size_t(nseq), cudaMemcpyDeviceToDevice, d->stream));
  LNG_CUDA(cudaMemcpy2DAsync(scratch_i + nseq * tail, size_t(tail) * 8, toks + p0, size_t(P + 1) * 8,
                             size_t(tail) * 8, size_t(nseq), cudaMemcpyDeviceToDevice, d->stream));
  // their codes [nseq * tail, R] computed densely, then placed at rows p0 .. plen-1 with stride P * R
  uint8_t* dense = reinterpret_cast<uint8_t*>(b.u);  // reuse: nseq*tail*R bytes <= u's size (M = nseq*tail)
  const size_t dense_need = size_t(nseq * tail * R);
  const size_t u_bytes = size_t(b.rows) * d->qh * d->Dt * dtype_size(d->act);
  LNG_REQUIRE(dense_need <= u_bytes, "internal: code staging buffer too small");
  st = drafter_codes(d, scratch_i, scratch_i + nseq * tail, nseq * tail, b.feat, dense, R, N > 0 ? tail_states : nullptr,
                     b.feat_parts);
  if (st) return st;
  LNG_CUDA(cudaMemcpy2DAsync(codes + p0 * R, size_t(P * R), dense, size_t(tail * R), size_t(tail * R), size_t(nseq),
                             cudaMemcpyDeviceToDevice, d->stream));
  for (int64_t g = 0; g < gamma; ++g) {
    const int64_t tpos = plen - 1 + g;  // position of the current token in every sequence
    // the readout reads the current tokens toks[s, 1 + tpos] in place (copied densely to scratch_i)
    // and its merge stores the next tokens at toks[s, 2 + tpos] and tokens_out[s, g]
    CodeSource src{codes, nseq, tpos + 1, 0, R, nullptr, nullptr, nullptr, tpos, P};
    DraftStore store;
    store.toks = toks + 2 + tpos;
    store.ts = P + 1;
    store.out = tokens_out + g;
    store.os = gamma;
    st = drafter_readout(d, toks + 1 + tpos, nseq, src, 1, b, Scoring{}, N > 0 ? s_cur : nullptr, P + 1, scratch_i,
                         &store);
    if (st) return st;
    if (g + 1 < gamma) {
      // the drafted tokens' SSM states and their codes at position tpos + 1 (strided rows of the code
      // buffer); their previous tokens are this step's current tokens, still in scratch_i
      if (N > 0) {
        st = drafter_ssm_inputs(d, b.ids, nseq, b, u);
        if (st) return st;
        st = drafter_ssm_scan(d, u, nseq, 1, s_cur, 0, s_next);
        if (st) return st;
        std::swap(s_cur, s_next);
      }
      st = drafter_codes(d, b.ids, scratch_i, nseq, b.feat, dense, R, N > 0 ? s_cur : nullptr, b.feat_parts);
      if (st) return st;
      LNG_CUDA(cudaMemcpy2DAsync(codes + (tpos + 1) * R, size_t(P * R), dense, size_t(R), size_t(R), size_t(nseq),
                                 cudaMemcpyDeviceToDevice, d->stream));
    }
  }
  return LNG_OK;
}

}  // namespace lng

extern "C" int lng_drafter_draft_batch(lng_drafter* d, const int64_t* prefix, int64_t nseq, int64_t plen, int64_t gamma,
                                       int64_t* tokens_out, lng_stream_t stream) {
  LNG_REQUIRE(d, "NULL drafter");
  LNG_REQUIRE(nseq >= 0 && plen >= 1 && gamma >= 1, "need nseq >= 0, plen >= 1, gamma >= 1");
  if (nseq == 0) return LNG_OK;
  LNG_REQUIRE(prefix && tokens_out, "NULL pointer");
  std::lock_guard<std::mutex> lk(d->mu);
  const int64_t R = d->R, N = d->N;
  // The drafts' code windows reach back n_max - 1 positions from the last prefix token and the embed2
  // router reads a position's own and previous token (and, for SD-C, its SSM state), so only the last
  // `tail` prefix positions need codes; earlier rows of `codes` are never read.  The SSM state itself
  // runs over the whole prefix.
  int64_t n_max = 1;
  for (int o = 0; o < d->n_orders; ++o) n_max = std::max<int64_t>(n_max, d->orders[o]);
  DraftBatchPlan pl;
  pl.nseq = nseq;
  pl.plen = plen;
  pl.gamma = gamma;
  pl.tail = std::min<int64_t>(plen, n_max);
  pl.P = plen + gamma;  // positions per sequence in the working buffers
  pl.pre_b = al256(size_t(nseq * plen) * 8);
  pl.out_b = al256(size_t(nseq * gamma) * 8);
  pl.tok_b = al256(size_t(nseq * (pl.P + 1)) * 8);
  pl.prev_b = al256(size_t(nseq * std::max<int64_t>(2 * pl.tail, 2)) * 8);
  pl.code_b = al256(size_t(nseq * pl.P * R));
  pl.u_b = al256(size_t(N > 0 ? nseq * plen * N : 0) * 4);
  pl.st_b = al256(size_t(nseq * pl.tail * N) * 4);
  pl.cur_b = al256(size_t(2 * nseq * N) * 4);
  const int64_t M = nseq * pl.tail;
  ReadoutBufs b;
  void* extra = nullptr;
  int st = drafter_ws(d, std::max<int64_t>(M, N > 0 ? std::min<int64_t>(nseq * plen, 8192) : M), 1, &b, pl.total(),
                      &extra);
  if (st) return st;
  cudaStream_t us = reinterpret_cast<cudaStream_t>(stream);
  cudaEvent_t ev;
  LNG_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  LNG_CUDA(cudaEventRecord(ev, us));
  LNG_CUDA(cudaStreamWaitEvent(d->stream, ev, 0));
  LNG_CUDA(cudaMemcpyAsync(extra, prefix, size_t(nseq * plen) * 8, cudaMemcpyDeviceToDevice, d->stream));
  // The second call of a shape (same workspace) captures the launches as a CUDA graph and later calls
  // replay it (about sixty small kernels and copies per gamma = 4 draft): launch overhead instead of
  // launch latency.  One-off shapes run directly.
  const auto key = std::make_tuple(nseq, plen, gamma, static_cast<const void*>(d->ws));
  if (d->graphs.size() >= 16 && !d->graphs.count(key)) {
    for (auto& kv : d->graphs)
      if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    d->graphs.clear();
  }
  lng_drafter::BatchGraph& g = d->graphs[key];
  if (g.exec) {
    LNG_CUDA(cudaGraphLaunch(g.exec, d->stream));
  } else {
    st = enqueue_draft_batch(d, pl, b, extra);
    if (st) {
      cudaEventDestroy(ev);
      return st;
    }
    if (++g.calls == 2) {
      // capture the same launches for the next calls; a sequence that cannot be captured runs directly
      cudaGraph_t graph = nullptr;
      if (cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
        const int cst = enqueue_draft_batch(d, pl, b, extra);
        const cudaError_t ce = cudaStreamEndCapture(d->stream, &graph);
        if (cst == LNG_OK && ce == cudaSuccess && graph && cudaGraphInstantiate(&g.exec, graph, 0) != cudaSuccess)
          g.exec = nullptr;
        if (graph) cudaGraphDestroy(graph);
      }
      (void)cudaGetLastError();  // a failed capture leaves no error behind for the next call
    }
  }
  LNG_CUDA(cudaMemcpyAsync(tokens_out, static_cast<unsigned char*>(extra) + pl.pre_b, size_t(nseq * gamma) * 8,
                           cudaMemcpyDeviceToDevice, d->stream));
  LNG_CUDA(cudaEventRecord(ev, d->stream));
  LNG_CUDA(cudaStreamWaitEvent(us, ev, 0));
  LNG_CUDA(cudaEventDestroy(ev));
  return LNG_OK;
}
