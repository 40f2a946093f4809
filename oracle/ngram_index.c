/*
 * Plain-C oracle for the integer part of the Lngram v2 lookup (TEST INFRASTRUCTURE ONLY).
 *
 * Restates, for whole batches at once, the code packing and n-gram row addressing of
 *   ffnmem/memory/lngram_v2.py:74-89     pack_bits_to_route_codes (sign bits -> codes)
 *   ffnmem/memory/lngram_v2.py:314-325   _aligned_ngram_address (oldest code least significant)
 *   ffnmem/memory/lngram_v2.py:1027-1045 _valid_mask (t >= n-1, same segment, valid last token)
 *   ffnmem/memory/lngram_v2.py:1075-1084 route offsets r * A^n
 * so that tests can check the CUDA path bit-exactly at the full benchmark sizes in seconds.
 * Only tests/ and bench.py's CPU-baseline leg load the built library.
 */
#include <stdint.h>

/* codes[i, r] = sum_j (logits[i, r*bits + j] > 0) << j ; returns 0. */
int oracle_pack_codes(const float* logits, int64_t n, int64_t routes, int bits, uint8_t* codes) {
  for (int64_t i = 0; i < n; ++i) {
    const float* row = logits + i * routes * bits;
    for (int64_t r = 0; r < routes; ++r) {
      int v = 0;
      for (int j = 0; j < bits; ++j) v |= (row[r * bits + j] > 0.0f ? 1 : 0) << j;
      codes[i * routes + r] = (uint8_t)v;
    }
  }
  return 0;
}

/*
 * Row index of every (b, t, r) for one order: rows[b, t, r] = r * A^order + sum_k c[t-order+1+k] << (k*bits),
 * or -1 where the window is invalid (t < order-1, segment change, or invalid last token).
 * codes: uint8 [B, T, R]; segment_ids: int64 [B, T] or NULL; valid_tokens: uint8 [B, T] or NULL.
 */
int oracle_row_indices(const uint8_t* codes, int64_t B, int64_t T, int64_t R, int order, int bits,
                       const int64_t* segment_ids, const uint8_t* valid_tokens, int64_t* rows) {
  const int64_t span = (int64_t)1 << (bits * order);
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t t = 0; t < T; ++t) {
      int ok = t >= order - 1;
      if (ok && segment_ids) ok = segment_ids[b * T + t - order + 1] == segment_ids[b * T + t];
      if (ok && valid_tokens) ok = valid_tokens[b * T + t] != 0;
      for (int64_t r = 0; r < R; ++r) {
        int64_t out = -1;
        if (ok) {
          int64_t addr = 0;
          for (int k = 0; k < order; ++k)
            addr |= (int64_t)codes[(b * T + t - order + 1 + k) * R + r] << (k * bits);
          out = r * span + addr;
        }
        rows[(b * T + t) * R + r] = out;
      }
    }
  }
  return 0;
}
