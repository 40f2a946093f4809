// n-gram row addressing of the Lngram v2 tables, shared by every kernel that gathers rows.
//
// Reference: ffnmem/memory/lngram_v2.py:314-325 (_aligned_ngram_address: oldest code least
// significant), :1027-1045 (_valid_mask), :1075-1084 (route offsets r * A^n).
#pragma once

#include "common.cuh"

namespace lng {

__device__ unsigned int g_error_word;  // first device-side error code (0 = none)

enum DeviceError : unsigned int {
  DEV_ERR_CODE_RANGE = 1,   // a route code >= 2^bits (treated as an invalid window)
  DEV_ERR_WAIT_TIMEOUT = 2, // a bounded mbarrier wait expired
  DEV_ERR_TOKEN_RANGE = 3,  // a token id outside [0, vocab)
};

struct TableSet {
  const void* tab[LNG_MAX_ORDERS];
  const float* ss[LNG_MAX_ORDERS];  // per-row sums of squares, or null
  int order[LNG_MAX_ORDERS];
  int n_orders;
  int bits;
  int64_t num_routes;
  int64_t mem_dim;
};

// Where an item's codes live: sequence mode (item = b*T + t of codes [B, T, R]) or window mode
// (item = i of codes [M, W, R]).
struct CodeSource {
  const void* codes;
  int64_t B, T;          // sequence mode (window == 0)
  int64_t window;        // window mode when > 0
  int64_t R;             // routes in the codes array (row stride)
  const int64_t* segment_ids;  // sequence mode, [B, T] or null
  const uint8_t* valid_tokens; // sequence mode, [B, T] or null
  const int32_t* seg;          // window mode, [M, W] or null
  int64_t t_offset;      // sequence mode: item t is absolute position t + t_offset (target_length)
  int64_t bstride;       // sequence mode: positions between consecutive batch rows (>= T)
  int64_t direct;        // > 0: rows mode -- item i, route r reads row i * direct + r of table 0 (the
                         // caller's route tokens), always valid; codes, windows and masks are unused
  int serving;           // 1: the serving table layout (the newest code least significant,
                         // serving/layout.py:1-18) instead of the v2 layout (the oldest least significant)
};

// ---- pipelined form used by the gather kernels: an item's geometry once, then per-route codes.
constexpr int MAXW = 4;  // longest n-gram window (max order) the pipelined gather supports

struct ItemGeo {
  int64_t cur;     // codes row of the item's newest slot
  int avail;       // slots that exist at and before `cur` (capped at MAXW)
  uint32_t omask;  // bit o set: order o's window is valid for this item
};

__device__ __forceinline__ ItemGeo item_geometry(const CodeSource& s, const int* orders, int n_orders, int64_t item) {
  ItemGeo g;
  g.omask = 0;
  if (s.direct > 0) {
    g.cur = item;
    g.avail = 1;
    g.omask = 1u;
    return g;
  }
  if (s.window > 0) {
    const int64_t W = s.window;
    g.cur = item * W + W - 1;
    g.avail = int(W < MAXW ? W : MAXW);
    for (int o = 0; o < n_orders; ++o) {
      const int n = orders[o];
      bool ok = W >= n;
      if (ok && s.seg) ok = s.seg[item * W + W - n] == s.seg[item * W + W - 1];
      g.omask |= uint32_t(ok) << o;
    }
  } else {
    const int64_t Tout = s.T - s.t_offset;
    const int64_t b = item / Tout;
    const int64_t t = item - b * Tout + s.t_offset;
    const int64_t p = b * s.bstride + t;
    g.cur = p;
    g.avail = int(t + 1 < MAXW ? t + 1 : MAXW);
    const bool tok_ok = !s.valid_tokens || s.valid_tokens[p];
    for (int o = 0; o < n_orders; ++o) {
      const int n = orders[o];
      bool ok = tok_ok && t >= n - 1;
      if (ok && s.segment_ids) ok = s.segment_ids[p - n + 1] == s.segment_ids[p];
      g.omask |= uint32_t(ok) << o;
    }
  }
  return g;
}

// Codes of route r in the item's window, newest first (c[k] = code at slot cur - k); all loads are
// independent so they overlap, and their first use can be one pipeline step later.
template <typename CodeT>
__device__ __forceinline__ void load_window_codes(const CodeSource& s, const ItemGeo& g, int64_t r, bool route_ok,
                                                  int32_t (&c)[MAXW]) {
  const CodeT* codes = static_cast<const CodeT*>(s.codes);
  const bool read = route_ok && s.direct == 0;
#pragma unroll
  for (int k = 0; k < MAXW; ++k) c[k] = (read && k < g.avail) ? int32_t(codes[(g.cur - k) * s.R + r]) : 0;
}

// Table row of order n for window codes c (oldest code least significant), or -1.
__device__ __forceinline__ int64_t window_row(const int32_t (&c)[MAXW], int order, int bits, int64_t r, bool valid) {
  if (!valid) return -1;
  int64_t addr = 0;
  bool range_ok = true;
#pragma unroll
  for (int i = 0; i < MAXW; ++i) {
    if (i < order) {
      const int32_t v = c[order - 1 - i];
      range_ok = range_ok && (v >= 0) && (v < (1 << bits));
      addr |= int64_t(v) << (i * bits);
    }
  }
  if (!range_ok) {
    atomicCAS(&g_error_word, 0u, (unsigned int)DEV_ERR_CODE_RANGE);
    return -1;
  }
  return r * (int64_t(1) << (bits * order)) + addr;
}

template <typename CodeT>
__device__ __forceinline__ int64_t read_code(const CodeSource& s, int64_t pos_row, int64_t r) {
  return static_cast<int64_t>(static_cast<const CodeT*>(s.codes)[pos_row * s.R + r]);
}

// Global table row of (item, route r, order n), or -1 when the n-gram window is not valid.
// In sequence mode `item` indexes [B, T_out] with T_out = T - t_offset.
template <typename CodeT>
__device__ __forceinline__ int64_t ngram_row(const CodeSource& s, int64_t item, int64_t r, int order, int bits) {
  if (s.direct > 0) return item * s.direct + r;
  int64_t base;  // codes row of the window's first slot
  if (s.window > 0) {
    const int64_t W = s.window;
    if (W < order) return -1;
    if (s.seg) {
      const int32_t* sg = s.seg + item * W;
      if (sg[W - order] != sg[W - 1]) return -1;
    }
    base = item * W + (W - order);
  } else {
    const int64_t Tout = s.T - s.t_offset;
    const int64_t b = item / Tout;
    const int64_t t = item % Tout + s.t_offset;
    if (t < order - 1) return -1;
    const int64_t p = b * s.bstride + t;
    if (s.segment_ids && s.segment_ids[p - order + 1] != s.segment_ids[p]) return -1;
    if (s.valid_tokens && !s.valid_tokens[p]) return -1;
    base = p - order + 1;
  }
  int64_t addr = 0;
  const int64_t lim = int64_t(1) << bits;
  for (int k = 0; k < order; ++k) {
    const int64_t c = read_code<CodeT>(s, base + k, r);
    if (c < 0 || c >= lim) {
      atomicCAS(&g_error_word, 0u, (unsigned int)DEV_ERR_CODE_RANGE);
      return -1;
    }
    addr |= c << ((s.serving ? order - 1 - k : k) * bits);
  }
  return r * (int64_t(1) << (bits * order)) + addr;
}

}  // namespace lng
