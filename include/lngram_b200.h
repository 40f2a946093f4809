/*
 * lngram_b200 -- C ABI of the B200 (sm_100a) Lngram v2 route n-gram memory path.
 *
 * Every entry point takes plain device pointers, sizes, dtype codes and a CUDA stream, never a
 * framework tensor type, and returns an int status (LNG_OK = 0).  On failure the message of the
 * calling thread's last error is available from lng_last_error().  Work is enqueued on `stream`
 * (NULL = the legacy default stream); no entry point synchronises unless its comment says so.
 * Pointers named `*_host` are host memory; every other pointer is device memory of the current
 * CUDA device.  Arrays are dense row-major (C order) unless a stride argument says otherwise.
 *
 * Each declaration names the reference interface it replaces (path:line in the reference project
 * MorbiusPlexus/lngram-decode).  Integer results (codes, row indices, gathered rows, top-k ids)
 * are bit-exact against the reference; floating-point results follow the reference's math with
 * fp32 accumulation.
 */
#ifndef LNGRAM_B200_H_
#define LNGRAM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* lng_stream_t; /* == cudaStream_t */

enum lng_status {
  LNG_OK = 0,
  LNG_ERR_ARGUMENT = 1,    /* bad shape, dtype, pointer or configuration (the reference's ValueError) */
  LNG_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  LNG_ERR_UNSUPPORTED = 3, /* valid for the reference, not supported by this build */
  LNG_ERR_DEVICE = 4,      /* a kernel reported an error (bounded wait expired, bad index) */
  LNG_ERR_STATE = 5        /* drafter state error (the reference's RuntimeError) */
};

enum lng_dtype {
  LNG_F32 = 0,
  LNG_BF16 = 1,
  LNG_F16 = 2,
  LNG_U8 = 3,
  LNG_I32 = 4,
  LNG_I64 = 5,
  LNG_BOOL = 6 /* one byte per element, nonzero = true */
};

#define LNG_MAX_ORDERS 4

/* ABI version (bumped on any signature change) and the thread's last error message. */
int lng_abi_version(void);
const char* lng_last_error(void);
/* 1 when a CUDA device of compute capability 10.x is current and usable, else 0. */
int lng_device_ok(void);
/* The first error code a kernel recorded on the current device since the last clear (0 = none;
 * 1 = a route code >= 2^bits, 2 = a bounded wait expired, 3 = a token id out of range), or -1 when
 * it cannot be read.  Synchronises with the device.  clear != 0 resets it. */
int lng_device_error(int clear);

/* ------------------------------------------------------------------ router (a3, a4) */

/* codes[i, r] = sum_j (logits[i, r*bits + j] > 0) << j for n rows of routes*bits logits.
 * Replaces RouteNgramMemoryV2.quantize_route_logits / pack_bits_to_route_codes
 * (ffnmem/memory/lngram_v2.py:1012-1017, :74-89).  codes_dtype: LNG_U8 (bits <= 8) or LNG_I32. */
int lng_quantize_route_logits(const float* logits, int64_t n, int64_t routes, int32_t bits, void* codes,
                              int32_t codes_dtype, lng_stream_t stream);

/* Router GEMM in fp32 semantics followed by the sign pack: logits = x . W^T (x [n, in_dim] with row
 * stride x_stride elements, dtype LNG_F32 or LNG_BF16; W [routes*bits, in_dim] fp32), codes as
 * above.  `logits` (fp32 [n, routes*bits]) is optional (NULL = never materialised).
 * Replaces LngramMemory.route_logits + quantize (ffnmem/memory/wrapper.py:98-101, :106-112). */
int lng_route_codes(const void* x, int32_t x_dtype, int64_t n, int64_t in_dim, int64_t x_stride, const float* weight,
                    int64_t routes, int32_t bits, void* codes, int32_t codes_dtype, float* logits, lng_stream_t stream);

/* Split the fp32 router weight W [rows, in_dim] once into bf16 parts W1 | W2 | W3 ([rows, 3*in_dim],
 * W = W1 + W2 + W3) for the tensor-core router below (a load-time step; no reference counterpart). */
int lng_router_prepare(const float* weight, int64_t rows, int64_t in_dim, void* w_split, lng_stream_t stream);

/* The router of lng_route_codes on the tcgen05 tensor cores for bf16 inputs x [n, in_dim] (row stride
 * x_stride): logits = x.W1^T + x.W2^T + x.W3^T (each bf16 product exact, fp32 accumulation) sign-packed
 * to u8 codes [n, routes] in the GEMM epilogue.  bits in [1, 6], in_dim % 64 == 0, 16-byte rows.
 * Replaces LngramMemory.route_logits + quantize (ffnmem/memory/wrapper.py:98-101, :106-112). */
int lng_route_codes_split(const void* x_bf16, int64_t n, int64_t in_dim, int64_t x_stride, const void* w_split,
                          int64_t routes, int32_t bits, uint8_t* codes, lng_stream_t stream);

/* embed2 router features for token ids (ffnmem/memory/router.py:50-69): for item i with current
 * token cur[i] and previous token prev[i] (-1 = the learned start vector), writes
 * out[i] = concat(RMSNorm(E[prev] or start; prev_w), RMSNorm(E[cur]; cur_w)) in fp32 [n, 2*d].
 * E dtype: LNG_F32 / LNG_BF16 / LNG_F16; norm weights and start are fp32. */
int lng_embed2_features(const int64_t* cur, const int64_t* prev, int64_t n, const void* embedding, int32_t e_dtype,
                        int64_t vocab, int64_t d, const float* prev_w, const float* cur_w, const float* start,
                        float eps, float* out, lng_stream_t stream);

/* ------------------------------------------------------------------ tables and addressing (a5, a6) */

/* The n-gram tables of one memory layer: one table per order, [num_routes * 2^(bits*order), memory_dim]
 * (the reference's `tables["ngram_<n>"].weight`, lngram_v2.py:960-966). */
typedef struct {
  int32_t n_orders;
  int32_t orders[LNG_MAX_ORDERS]; /* ascending, as the reference sorts them (lngram_v2.py:934) */
  const void* tables[LNG_MAX_ORDERS];
  int32_t table_dtype; /* LNG_F32, LNG_BF16 or LNG_F16 */
  int32_t bits;        /* bits per route, 1..16 */
  int64_t num_routes;
  int64_t memory_dim;  /* route token width Dt = n_orders * memory_dim */
  /* Optional per-row sums of squares (fp32 [rows] per order, from lng_table_row_ss): the readout
   * kernels then read one float per gathered row instead of recomputing the row's RMS. */
  const float* row_ss[LNG_MAX_ORDERS];
} lng_tables;

/* row_ss[o][i] = sum_k tables[o][i, k]^2 in fp32 for every row of every order (a load-time step
 * for lng_route_attend / lng_memory_forward; no reference counterpart). */
int lng_table_row_ss(const lng_tables* tables, float* const* row_ss, lng_stream_t stream);

/* Route tokens [B, T_out, route_end-route_start, Dt] for codes [B, T, num_routes] (u8 or i32):
 * per order the row r*A^n + sum_k c[t-n+1+k] << (k*bits) (oldest code least significant), zero
 * where t < n-1, where segment_ids[t-n+1] != segment_ids[t], or where valid_tokens[t] is false;
 * orders concatenated on the feature axis; T_out = target_length (the last positions) or T when
 * target_length <= 0.  segment_ids (i64 [B, T]) and valid_tokens (bool [B, T]) may be NULL.
 * out_dtype: the table dtype or LNG_F32.
 * Replaces RouteNgramMemoryV2._lookup_route_chunk (lngram_v2.py:1047-1113). */
int lng_lookup_route_chunk(const lng_tables* tables, const void* codes, int32_t codes_dtype, int64_t B, int64_t T,
                           int64_t route_start, int64_t route_end, const int64_t* segment_ids,
                           const uint8_t* valid_tokens, int64_t target_length, void* out, int32_t out_dtype,
                           lng_stream_t stream);

/* Backward of the training-mode lookup (_lookup_route_chunk with the q surrogate, lngram_v2.py:1047-1113,
 * :326-447) for codes [B, T, num_routes] and the route chunk [route_start, route_end), given the route
 * tokens' gradient grad_tokens [B, T, route_end - route_start, Dt] (f32 / bf16 / f16):
 *   grad_tables[o] (fp32 [rows, memory_dim] per order, accumulated; the array or an entry may be NULL):
 *     the gathered rows' gradient of every valid window (the nn.Embedding backward);
 *   grad_q (fp32 [B, T, route_end - route_start, bits], written; NULL = none): the surrogate gradient of
 *     _LngramSurrogate.backward for q_logits [B, T, q_routes, bits] (fp32) -- exact == 0: one-bit
 *     counterfactuals (order x bits extra row gathers per window) times scale T p (1 - p), p =
 *     sigmoid(T q); exact != 0: the expectation over the whole alphabet per digit.  Zero when
 *     temperature or scale is 0.
 * The masks of lng_lookup_route_chunk apply (segment_ids, valid_tokens may be NULL).  memory_dim <= 256;
 * bits <= 8 for the surrogate. */
int lng_lookup_backward(const lng_tables* tables, const void* codes, int32_t codes_dtype, int64_t B, int64_t T,
                        int64_t route_start, int64_t route_end, const int64_t* segment_ids, const uint8_t* valid_tokens,
                        const void* grad_tokens, int32_t grad_dtype, const float* q_logits, int64_t q_routes,
                        float temperature, float scale, int32_t exact, float* grad_q, float* const* grad_tables,
                        lng_stream_t stream);

/* Route tokens [M, num_routes, Dt] of the n-grams ending at the LAST slot of explicit code windows
 * codes [M, W, num_routes] (u8 or i32; W >= max order) with per-slot segment ids seg [M, W] (i32,
 * NULL = all one segment): order n is valid iff seg[W-n] == seg[W-1].  This is the windowed lookup
 * of lookup_rows_at (ffnmem/memory/draft.py:26-47) and tree_route_tokens (drafting/tree.py:130-136). */
int lng_lookup_windows(const lng_tables* tables, const void* codes, int32_t codes_dtype, int64_t M, int64_t W,
                       const int32_t* seg, void* out, int32_t out_dtype, lng_stream_t stream);

/* ------------------------------------------------------------------ host-RAM serving, incremental state */

/* Route tokens [B, n, R, Dt] of the last n positions of codes [B, T, R] (T = h + n: h history codes, then
 * the n new ones) from tables in the SERVING layout (serving/layout.py:1-18: row r*A^n + sum_k c[t-k] A^k,
 * the newest code least significant; made by lng_serving_permute).  The tables may live in pinned host
 * memory mapped for the device (lng_host_map): each row is read across PCIe once with 16-byte loads, no
 * staging copy -- the zero-copy transfer mode serving/prefetch.py:579-586 leaves unimplemented, a
 * decode_step row_provider for tables larger than HBM (ffnmem/infer.py:238-240).  Windows that start before
 * position 0 of the context read zero rows (serving/prefetch.py:186-202).  out: the table dtype;
 * 16-byte rows. */
int lng_lookup_serving_rows(const lng_tables* tables, const void* codes, int32_t codes_dtype, int64_t B, int64_t T,
                            int64_t n, void* out, lng_stream_t stream);

/* The serving-layout copy of one order's v2 table (serving/layout.py:26-43, permute_table): within every
 * route's block of A^order rows, dst row j = src row reverse_digits(j).  src / dst: any memory the device
 * can read / write (device, or mapped host); distinct; 16-byte rows. */
int lng_serving_permute(const void* src, void* dst, int32_t dtype, int64_t routes, int32_t order, int32_t bits,
                        int64_t mem_dim, lng_stream_t stream);

/* The device address of host memory [host, host + bytes): page-locked memory is used as it is; pageable
 * memory is pinned and mapped first (cudaHostRegister) and lng_host_unmap releases it.  No reference
 * counterpart (the reference leaves the zero-copy mode unimplemented, serving/prefetch.py:579-586). */
int lng_host_map(void* host, size_t bytes, void** device_ptr);
int lng_host_unmap(void* host);

/* The packed n-gram suffix state of RouteNgramMemoryV2.forward_incremental (lngram_v2.py:1714-1760):
 * packed [B, R] int32 holds the codes of the last maxn positions, the newest in digit maxn - 1.  With
 * packed_in == NULL: _pack_suffix of the last min(T, maxn) positions of codes [B, T, R]; otherwise
 * _advance_packed: packed_in shifted down one digit, codes [B, 1, R] in the top digit.  window_out
 * (optional, u8 [B, maxn, R]) receives the digits unpacked (slot j = digit j, oldest first), the code
 * windows of lng_route_attend's window mode.  maxn * bits <= 31. */
int lng_packed_suffix(const void* codes, int32_t codes_dtype, int64_t B, int64_t T, int64_t R, int32_t bits,
                      int32_t maxn, const int32_t* packed_in, int32_t* packed_out, uint8_t* window_out,
                      lng_stream_t stream);

/* ------------------------------------------------------------------ readout (a7 - a11) */

/* A memory layer's readout in folded form.  The reference computes, per position,
 *   q = W_q RMSNorm(h; g_q);  K,V = W_kv RMSNorm(token_r; g_m);  p = sink-softmax(q.K * HD^-1/2)
 *   out = W_o (p . V);  out + SiLU(conv(RMSNorm(out; g_c)))
 * (lngram_v2.py:1115-1131, :1877-1920, :1354-1359).  Because both RMSNorms are a per-vector scale
 * and W_k, W_v are linear, the same function is computed with the maps
 *   w_qk[h*G+g][k, :] = HD^-1/2 g_m[k] sum_j W_k[h][j, k] W_q[h*G+g][j, :] g_q[:]   [QH*Dt, d]
 *   w_vo[:, (h*G+g)*Dt + k] = sum_j W_o[:, (h*G+g)*HD + j] W_v[h][j, k] g_m[k]          [d, QH*Dt]
 * applied to the raw hidden state and the raw route tokens (lng_fold_readout builds them). */
typedef struct {
  int64_t hidden;          /* d */
  int32_t num_heads;       /* QH (query heads) */
  int32_t num_kv_heads;    /* KV */
  int32_t head_dim;        /* HD */
  float eps;               /* RMSNorm epsilon of all readout norms */
  float sink_logit;        /* b0 = log(R (1 - mass) / mass) (lngram_v2.py:1865-1875) */
  int32_t conv_kernel;     /* short conv taps (k) */
  int32_t conv_dilation;   /* default max(ngrams) (lngram_v2.py:1000) */
  int32_t act_dtype;       /* LNG_F32 or LNG_BF16: hidden states, folded maps, outputs */
  const void* w_qk;        /* [QH*Dt, d] act_dtype */
  const void* w_vo;        /* [d, QH*Dt] act_dtype */
  const float* conv_norm;  /* [d] */
  const float* conv_weight;/* [d, k], taps oldest -> newest */
  const float* conv_bias;  /* [d] or NULL */
  const float* router_w;   /* [R*bits, router_in_dim] fp32, or NULL when codes are supplied */
  int64_t router_in_dim;
  const void* router_w_split; /* lng_router_prepare output, or NULL (bf16 router inputs then use CUDA cores) */
} lng_readout;

/* Build w_qk / w_vo (act_dtype) from the reference parameters (all fp32):
 * q_norm [d], q_proj [QH*HD, d], mem_norm [Dt], kv_proj [2*KV*HD, Dt], o_proj [d, QH*HD]. */
int lng_fold_readout(int64_t d, int64_t Dt, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                     const float* q_norm, const float* q_proj, const float* mem_norm, const float* kv_proj,
                     const float* o_proj, void* w_qk, void* w_vo, int32_t act_dtype, lng_stream_t stream);

/* Fused gather + sink attention over routes for M items (the core of _lookup_route_chunk +
 * _project_memory + _manual_gqa, lngram_v2.py:1047-1131, :1887-1920), in folded form:
 *   s[q, r] = qscale[i] * rms(tok_r)^-1 * (qa[i, q, :] . tok_r),  p = softmax with the sink b0,
 *   u[i, q, :] = sum_r p[q, r] rms(tok_r)^-1 tok_r.
 * qa: [M, QH, Dt] (act dtype of `u`); qscale: fp32 [M] or NULL (= 1).
 * Items address their codes in one of two modes:
 *   window == 0: sequence mode, item i = (b, t) of codes [B, T, R] with the masks of
 *                lng_lookup_route_chunk (segment_ids, valid_tokens may be NULL); with target_length
 *                > 0 only the last target_length positions of each row are items (M = B*target_length,
 *                the decode-step view of ffnmem/infer.py:169-174), else M = B*T;
 *   window  > 0: window mode, codes [M, window, R] and seg [M, window] as in lng_lookup_windows.
 * Routes [route_start, route_end) are attended.  partial == 0: u is normalised, in the dtype of qa.
 * partial == 1 or 2: the online-softmax state of these routes is written instead -- m [M, QH] and
 * l [M, QH] (fp32) and the unnormalised u in fp32 -- with the sink seeded in (1) or left out (2),
 * so that route shards (one of them with the sink) combine exactly as the streaming readout does
 * (lngram_v2.py:1944-2070); qa then has the tables' dtype (16-bit tables) or f32.
 * partial == 3 or 4 (16-bit tables): the same state as 1 / 2, written as the bf16 pack
 * [M, QH, Dt + 1] = (u, l) of lng_attend_pack plus m [M, QH]; the tensor-core kernel starts every
 * shard from the offset b0, so after the max all-reduce of m the packs of all shards usually share
 * one scale (lng_attend_pack_rescale fixes the rows that do not) and sum directly. */
int lng_route_attend(const lng_tables* tables, const void* codes, int32_t codes_dtype, int64_t B, int64_t T,
                     int64_t window, const int64_t* segment_ids, const uint8_t* valid_tokens, const int32_t* seg,
                     int64_t target_length, int64_t route_start, int64_t route_end, int32_t num_heads, float eps,
                     float sink_logit,
                     const void* qa, const float* qscale, void* u, int32_t u_dtype, int32_t partial, float* m_out,
                     float* l_out, lng_stream_t stream);

/* lng_route_attend (normalised output) over route tokens the CALLER supplies instead of table rows:
 * tokens [M, routes, Dt] (f32 / bf16 / f16; zero rows where an n-gram is not valid, as
 * _lookup_route_chunk gives them).  This is the readout of memory_step(..., route_tokens=)
 * (ffnmem/infer.py:168-173): the rows a decode_step row_provider returns (infer.py:238-240), e.g. from
 * host-RAM tables, skip the table lookup.  qa, qscale, u and u_dtype as for lng_route_attend. */
int lng_route_attend_rows(const void* tokens, int32_t tok_dtype, int64_t M, int64_t routes, int64_t Dt,
                          int32_t num_heads, float eps, float sink_logit, const void* qa, const float* qscale, void* u,
                          int32_t u_dtype, lng_stream_t stream);

/* Sink attention with explicit keys and values, the reference's _manual_gqa
 * (lngram_v2.py:1877-1920): q [M, KV*G, HD], k / v [M, KV, R, HD] (dtype f32/bf16/f16), scores
 * q.k * HD^-1/2 in fp32, p = exp(s - m) / (sum exp(s - m) + exp(b0 - m)), out = p . v [M, KV*G, HD]. */
int lng_sink_gqa(const void* q, const void* k, const void* v, int32_t dtype, int64_t M, int32_t num_kv_heads,
                 int32_t groups, int64_t routes, int32_t head_dim, float sink_logit, void* out, lng_stream_t stream);

/* C[M, N] = rowscale[m] * (A[M, K] . B[N, K]^T) (+ C when accumulate), fp32 accumulation.
 * A, B, C dtypes in {LNG_F32, LNG_BF16, LNG_F16}; lda/ldb/ldc are row strides in elements;
 * rowscale fp32 [M] or NULL.  bf16 x bf16 GEMMs run on the tcgen05 tensor cores. */
int lng_gemm(const void* A, int32_t a_dtype, int64_t lda, const void* Bm, int32_t b_dtype, int64_t ldb, void* C,
             int32_t c_dtype, int64_t ldc, int64_t M, int64_t N, int64_t K, const float* rowscale, int32_t accumulate,
             lng_stream_t stream);

/* rs[i] = 1 / sqrt(mean(x[i, :]^2) + eps) for n rows of width d (x dtype f32/bf16/f16). */
int lng_rms_rows(const void* x, int32_t x_dtype, int64_t n, int64_t d, float eps, float* rs, lng_stream_t stream);

/* y[i, :] = x[i, :] * rs(x[i]) * w (+ residual) -- RMSNorm of ffnmem/model.py:39-48 / F.rms_norm.
 * x, y dtypes f32/bf16/f16 (y may alias x); w fp32 [d] or NULL. */
int lng_rms_norm(const void* x, int32_t x_dtype, int64_t n, int64_t d, const float* w, float eps, void* y,
                 int32_t y_dtype, lng_stream_t stream);

/* The model block's RMSNorm with its rounding rule (ffnmem/model.py:39-48, the attn_norm that makes the
 * router input h_norm at ffnmem/model.py:114): y = cast_y(cast_x(x * rsqrt(mean(x^2) + eps)) * w), the
 * normalised row rounded to x's dtype BEFORE the weight multiply.  The reference's output dtype is the
 * promotion of x's and w's (bf16 x with an fp32 weight gives fp32 y; with a bf16 weight, bf16 y); y_dtype
 * selects it.  x f32 / bf16 / f16; w f32 / bf16 [d] or NULL (= 1); y may not alias x. */
int lng_rms_norm_model(const void* x, int32_t x_dtype, int64_t n, int64_t d, const void* w, int32_t w_dtype,
                       float eps, void* y, int32_t y_dtype, lng_stream_t stream);

/* The short-conv finish of the readout (lngram_v2.py:1354-1359, :207-286), sequence mode:
 * out[b, t] = mixed[b, t] + SiLU(bias + sum_tap w[:, tap] * RMSNorm(mixed)[b, t - lag(tap)] * same_segment)
 * with lag(tap) = (k-1-tap)*dilation and zero left padding, then * valid_tokens[b, t].
 * mixed/out dtype = act dtype (out may not alias mixed).  segment_ids, valid_tokens may be NULL.
 * conv_in (optional, same dtype) receives RMSNorm(mixed) (the decode cache of ffnmem/infer.py:176). */
int lng_conv_finish(const lng_readout* ro, const void* mixed, int64_t B, int64_t T, const int64_t* segment_ids,
                    const uint8_t* valid_tokens, void* out, void* conv_in, lng_stream_t stream);

/* Window form of the conv finish for decode and tree seams (ffnmem/infer.py:176-182,
 * drafting/tree.py:186-195): for item i, out[i] = mixed[i] + SiLU(bias + sum_tap w[:, tap] *
 * y[slot[i, tap]]) where y = RMSNorm(mixed) of the new items is first written to
 * cache[new_slot[i]] and slot = -1 reads zero.  cache: [S, d] act dtype (the cached conv inputs);
 * slot: i64 [n, k]; new_slot: i64 [n]. */
int lng_conv_window(const lng_readout* ro, const void* mixed, int64_t n, void* cache, const int64_t* new_slot,
                    const int64_t* slot, void* out, lng_stream_t stream);

/* A draft tree's memory block in one call (drafting/tree.py:178-195; the steps of tree_memory_block): the
 * n nodes of each of B sequences after L cached positions.  Node i's code window (W = history + 1 slots,
 * oldest first) reads slot gidx[i, w] of [the last h0 cached codes | the nodes' new codes], zero where
 * gok[i, w] == 0; seg [B*n, W] (i32) marks the window's valid slots for the row rule.  The nodes' codes
 * codes_new [B, n, R] (u8) are written to cache_codes [B, max_len, R] at L .. L+n-1; the readout (1/rms(h),
 * folded query, gather + sink attention over the windows, output map) gives mixed; lng_conv_window's
 * step then writes the nodes' conv inputs to cache_conv [B*max_len, d] at new_slot and gives out
 * [B, n, d] from the taps at slot [B*n, k].  h, out: act dtype; gidx: i64 [n, W]; gok: u8 [n, W]. */
size_t lng_tree_workspace_bytes(const lng_tables* tables, const lng_readout* ro, int64_t B, int64_t n, int64_t W);
int lng_tree_memory_block(const lng_tables* tables, const lng_readout* ro, int64_t B, int64_t n, int64_t W,
                          int64_t L, int64_t h0, int64_t max_len, const void* h, const uint8_t* codes_new,
                          uint8_t* cache_codes, void* cache_conv, const int64_t* gidx, const uint8_t* gok,
                          const int32_t* seg, const int64_t* slot, const int64_t* new_slot, void* out, void* workspace,
                          size_t workspace_bytes, lng_stream_t stream);

/* Workspace bytes needed by lng_memory_forward for M = B*T positions and Dt / R of `tables`. */
size_t lng_memory_workspace_bytes(const lng_tables* tables, const lng_readout* ro, int64_t M);

/* The whole memory layer forward (LngramMemory.forward, ffnmem/memory/wrapper.py:103-125, and
 * RouteNgramMemoryV2.forward, lngram_v2.py:1361-1407) for h [B, T, d] (act dtype):
 * codes = sign-pack(router_x . router_w^T) unless `codes_in` (u8/i32 [B, T, R]) is given, then the
 * fused gather/attention, w_vo, and the conv finish.  router_x [B, T, router_in_dim] (f32 or bf16).
 * codes_out (u8 [B, T, R]) is optional.  workspace: lng_memory_workspace_bytes bytes. */
int lng_memory_forward(const lng_tables* tables, const lng_readout* ro, int64_t B, int64_t T, const void* h,
                       const void* router_x, int32_t router_x_dtype, const void* codes_in, int32_t codes_in_dtype,
                       const int64_t* segment_ids, const uint8_t* valid_tokens, void* out, uint8_t* codes_out,
                       void* workspace, size_t workspace_bytes, lng_stream_t stream);

/* Combine per-shard online-softmax states (lng_route_attend partial == 1) given the global
 * per-(item, head) max m_glob: scale_i = exp(m_i - m_glob); l_i *= scale; u_i *= scale (in place).
 * After a SUM reduction across shards, lng_attend_normalize gives the head-space u. */
int lng_attend_rescale(const float* m_local, const float* m_glob, float* l, float* u, int64_t M, int32_t num_heads,
                       int64_t Dt, lng_stream_t stream);
int lng_attend_normalize(const float* l, const float* u, int64_t M, int32_t num_heads, int64_t Dt, void* u_out,
                         int32_t u_dtype, lng_stream_t stream);

/* Head-space form of the same combine, for route shards whose partial values were projected per
 * head (o = W_v g_m u, [M, QH, HD] fp32): pack [M, QH, HD+1] = (o, l) * exp(m_local - m_glob), ready
 * for a SUM reduction across shards; lng_attend_unpack then writes head = pack[.., :HD] / pack[.., HD]
 * (the streaming readout's final division, lngram_v2.py:2066-2070) in f32 or bf16.  The pack is f32
 * or bf16 (pack_dtype; bf16 halves the bytes a reduction moves between GPUs). */
int lng_attend_pack(const float* m_local, const float* m_glob, const float* l, const float* o, int64_t M,
                    int32_t num_heads, int32_t head_dim, void* pack, int32_t pack_dtype, lng_stream_t stream);
int lng_attend_unpack(const void* pack, int32_t pack_dtype, int64_t M, int32_t num_heads, int32_t head_dim, void* head,
                      int32_t dtype, lng_stream_t stream);
/* pack[i, q, :] *= exp(m_local[i, q] - m_glob[i, q]) for the rows where the two differ (packs written
 * by lng_route_attend partial 3 / 4), in place. */
int lng_attend_pack_rescale(const float* m_local, const float* m_glob, int64_t M, int32_t num_heads, int32_t head_dim,
                            void* pack, int32_t pack_dtype, lng_stream_t stream);

/* ------------------------------------------------------------------ draft head (a12) */

/* Top-k over V logits h[i] . E[v] for n rows without materialising the logits: ids i64 [n, k]
 * (ties -> lower id), vals fp32 [n, k]; logits (fp32 [n, V]) optional.  h fp32 [n, d];
 * E [V, d] f32/bf16/f16.  Replaces F.linear(h, E) + argmax / top-k
 * (ffnmem/memory/draft.py:88-91, drafting/cpu/drafter.cpp:537-556).  k <= 8.  A bf16 E with
 * d % 64 == 0 runs on the tensor cores with fp32-accurate logits (h split into three bf16 parts
 * inside `scratch`); other shapes on the CUDA cores.  scratch: lng_logits_topk_scratch_bytes. */
int lng_logits_topk(const float* h, int64_t n, int64_t d, const void* embedding, int32_t e_dtype, int64_t vocab,
                    int32_t k, int64_t* ids, float* vals, float* logits, void* scratch, size_t scratch_bytes,
                    lng_stream_t stream);
size_t lng_logits_topk_scratch_bytes(int64_t n, int64_t d, int64_t vocab, int32_t k);

/* lng_logits_topk without any allocation, for callers that cannot allocate device memory where they
 * draft (inside a captured or replayed CUDA graph, or under an allocator that only serves its own
 * pools).  No counterpart in the reference: it exists for those callers.  The scratch is a 4 MiB
 * array inside the library, held by every GPU that loads the library until the process exits;
 * sizes with n * ceil(vocab / 256) * k * 12 (candidates, rounded up to 256) + 256 -- plus
 * n * d * 6 (the split rows) when the tensor-core path applies -- above 4 MiB are rejected
 * (LNG_ERR_ARGUMENT): e.g. k = 3 at vocab 32000 allows n <= 932 rows on the CUDA-core path and
 * n <= 394 at d = 1024 on the tensor-core path.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current) and keeps it for the life of the
 * device's context (a cudaDeviceReset invalidates it), so make one call on each device before any
 * stream capture.  All calls share the array and it keeps the last call's contents
 * (every slot read is first written by the same call); calls that overlap on the GPU -- two streams,
 * or two threads -- race on it and must be serialised by the caller. */
int lng_logits_topk_static(const float* h, int64_t n, int64_t d, const void* embedding, int32_t e_dtype,
                           int64_t vocab, int32_t k, int64_t* ids, float* vals, float* logits, lng_stream_t stream);

/* ------------------------------------------------------------------ drafter (a15) */

/* A GPU drafter with the state machine and API of the reference C++ drafter
 * (drafting/cpu/drafter.cpp:150-595, Drafter(tensors, numbers, ngrams, threads)).  The bundle's
 * arrays are given as HOST pointers (the layout of drafting/export_drafter.py:25-34) and copied to
 * the device once.  Supports the embed2 router with full-vocabulary scoring or the sketch shortlist. */
typedef struct lng_drafter lng_drafter;

typedef struct {
  const char* name;    /* bundle array name ("embedding", "table_3", "router", ...) */
  const void* data_host;
  int32_t dtype;       /* LNG_F32 / LNG_F16 / LNG_BF16 / LNG_I32 */
  int32_t ndim;
  int64_t shape[4];
} lng_array;

typedef struct {
  int64_t d_model, vocab, routes, bits, mem_dim, kv_heads, head_dim, q_heads, ssm_dim, sketch_k, shortlist_cap;
  double router_eps, draft_eps, mem_eps, ssm_eps, softmax_scale, sink_logit;
  int32_t router_ssm, query_ssm;
  int32_t n_orders;
  int32_t orders[LNG_MAX_ORDERS];
} lng_drafter_numbers;

int lng_drafter_create(const lng_drafter_numbers* numbers, const lng_array* arrays, int32_t n_arrays,
                       int32_t act_dtype, lng_drafter** out);
void lng_drafter_destroy(lng_drafter* d);
int lng_drafter_reset(lng_drafter* d);
int64_t lng_drafter_length(const lng_drafter* d);
int lng_drafter_truncate(lng_drafter* d, int64_t n);
/* committed codes [length, R] u8 into codes_host. */
int lng_drafter_committed_codes(const lng_drafter* d, uint8_t* codes_host);
/* Append verified tokens; codes_host (i32 [n, R]) optionally replaces the drafter's own codes. */
int lng_drafter_commit(lng_drafter* d, const int64_t* tokens_host, int64_t n, const int32_t* codes_host);
/* gamma greedy drafts after the committed tokens + hyp (nothing committed): tokens [gamma], ids/logits
 * [gamma, topk] (-1 / -inf padded), codes [n_hyp + (last_codes ? gamma : gamma-1), R].  All host. */
int lng_drafter_draft(lng_drafter* d, int64_t gamma, const int64_t* hyp_host, int64_t n_hyp, int32_t topk,
                      int32_t last_codes, int64_t* tokens_host, int64_t* ids_host, float* logits_host,
                      uint8_t* codes_host);
/* Teacher-forced trace from an empty state: codes [T, R], ids / logits [T, S] with S = vocab (full)
 * or shortlist_cap. */
int lng_drafter_trace(lng_drafter* d, const int64_t* tokens_host, int64_t T, const int32_t* codes_host,
                      int32_t full, int64_t S, uint8_t* codes_out_host, int64_t* ids_host, float* logits_host);
/* Batched greedy drafting for nseq independent sequences (no reference counterpart: the reference
 * API is batch-1): each sequence's prefix tokens [nseq, plen] (device, i64) are committed in one
 * pass, then gamma argmax drafts per sequence are written to tokens_out (device i64 [nseq, gamma]).
 * The drafter's own committed state is not touched. */
int lng_drafter_draft_batch(lng_drafter* d, const int64_t* prefix, int64_t nseq, int64_t plen, int64_t gamma,
                            int64_t* tokens_out, lng_stream_t stream);

/* The in-context online-count mixer of the acceptance harness (drafting/drafters.py:117-143,
 * OnlineCounts(codes, x, orders, bits, vocab, kappa).mix(p, win, real, deadline)).  One record: codes
 * [T, R] (i64) and tokens x [T] (i64) give the verified pairs (t, x[t+1]), t < T-1, each keyed per order n
 * and route r by the row of the n-gram ending at t (drafting/build_sketches.py:186-197; -1 for t < n-1).
 * Query j's window win [N, W, R] (i64) with real [N, W] (u8) gives its rows (drafters.py:99-107; -1 unless
 * the last n slots are real).  w[j, t] = the (n, r) rows pair t shares with query j, for t <= deadline[j]
 * (i64 [N]); out [N, V] = (1 - lam) p + lam sc / max(tot, 1e-9) with sc[j, v] = sum of w[j, t] over pairs
 * whose next token is v, tot = sum_t w, lam = n_eff / (n_eff + kappa), n_eff = tot / (R n_orders), in
 * the reference's fp32 operation order (bit-identical results).  p, out: f32 [N, V], may alias.  All
 * device pointers; n_orders <= 8, orders in [1, 8], bits * order <= 40. */
int lng_online_counts_mix(const int64_t* codes, int64_t T, int64_t R, const int32_t* orders_host, int32_t n_orders,
                          int32_t bits, const int64_t* x, const int64_t* win, const uint8_t* real, int64_t N, int64_t W,
                          const int64_t* deadline, const float* p, int64_t V, float kappa, float* out,
                          lng_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LNGRAM_B200_H_ */
