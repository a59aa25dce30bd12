/*
 * naive.c — scalar oracle: a restatement of raya's Naive::attend
 * (crates/raya-kernels/src/naive.rs:13-65) and of Mask::key_range
 * (crates/raya-kernels/src/attention.rs:48-59), generalised to a batch
 * dimension, per-sequence valid_len, any block size and a halo.
 *
 * TEST INFRASTRUCTURE ONLY: this is the checker that the CUDA path is
 * compared against; nothing in the product links it.
 *
 * Numerics follow the reference exactly: a sequential fp32 dot product with
 * separate multiply and add (built with -ffp-contract=off; Rust never
 * contracts), then `* scale`, a running max, `expf(s - max)` from the C
 * library (what Rust's f32::exp calls on Linux), the sum, and per-weight
 * `p / sum` accumulation `o += w * v`.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

void oracle_key_range(const oracle_desc* d, int64_t i, int64_t valid_len,
                      int64_t* lo_out, int64_t* hi_out) {
  int64_t lo = 0, hi = 0;
  switch (d->mask) {
    case ORACLE_MASK_BLOCK: {
      /* attention.rs:50-53: b = i / BLOCK; (b.saturating_sub(1) * BLOCK,
       * (b + 2) * BLOCK), with BLOCK -> block and 1 -> halo. */
      int64_t b = i / d->block;
      int64_t first = b > d->halo ? b - d->halo : 0;
      lo = first * d->block;
      hi = (b + d->halo + 1) * d->block;
      break;
    }
    case ORACLE_MASK_WINDOW:
      /* attention.rs:54,56: (i.saturating_sub(w), i + w + 1) */
      lo = i > d->window ? i - d->window : 0;
      hi = i + d->window + 1;
      break;
    default: /* ORACLE_MASK_FULL, attention.rs:55 */
      lo = 0;
      hi = valid_len;
      break;
  }
  /* attention.rs:58: lo.min(valid_len)..hi.min(valid_len) */
  *lo_out = lo < valid_len ? lo : valid_len;
  *hi_out = hi < valid_len ? hi : valid_len;
}

void oracle_naive_range(const oracle_desc* d, const float* q, const float* k,
                        const float* v, float* out, const int32_t* valid_len,
                        int64_t bh0, int64_t bh1) {
  const int64_t L = d->seq, D = d->head_dim;
  float* scores = (float*)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1));
  for (int64_t bh = bh0; bh < bh1; ++bh) {
    const int64_t b = bh / d->heads;
    const int64_t valid = valid_len ? valid_len[b] : L;
    const int64_t base = bh * L * D;
    for (int64_t i = 0; i < L; ++i) {
      float* orow = out + base + i * D;
      /* naive.rs:29-32: zero the row; padded rows stay zero */
      for (int64_t c = 0; c < D; ++c) orow[c] = 0.0f;
      if (i >= valid) continue;
      int64_t lo, hi;
      oracle_key_range(d, i, valid, &lo, &hi);
      if (lo >= hi) continue; /* naive.rs:34-36 */
      const float* qrow = q + base + i * D;
      float max = -INFINITY;
      for (int64_t j = lo; j < hi; ++j) { /* naive.rs:40-49 */
        const float* krow = k + base + j * D;
        float s = 0.0f;
        for (int64_t c = 0; c < D; ++c) s += qrow[c] * krow[c];
        s = s * d->scale;
        max = fmaxf(max, s);
        scores[j - lo] = s;
      }
      float sum = 0.0f;
      for (int64_t j = lo; j < hi; ++j) { /* naive.rs:50-54 */
        scores[j - lo] = expf(scores[j - lo] - max);
        sum += scores[j - lo];
      }
      for (int64_t j = lo; j < hi; ++j) { /* naive.rs:55-61 */
        const float* vrow = v + base + j * D;
        const float w = scores[j - lo] / sum;
        for (int64_t c = 0; c < D; ++c) orow[c] += w * vrow[c];
      }
    }
  }
  free(scores);
}

void oracle_naive(const oracle_desc* d, const float* q, const float* k,
                  const float* v, float* out, const int32_t* valid_len) {
  oracle_naive_range(d, q, k, v, out, valid_len, 0, d->batch * d->heads);
}

void oracle_count(const oracle_desc* d, const int32_t* valid_len,
                  uint64_t* pairs, uint64_t* rows) {
  uint64_t p = 0, r = 0;
  for (int64_t b = 0; b < d->batch; ++b) {
    const int64_t valid = valid_len ? valid_len[b] : d->seq;
    uint64_t per_head = 0;
    for (int64_t i = 0; i < valid; ++i) {
      int64_t lo, hi;
      oracle_key_range(d, i, valid, &lo, &hi);
      if (hi > lo) per_head += (uint64_t)(hi - lo);
    }
    p += per_head * (uint64_t)d->heads;
    r += (uint64_t)valid * (uint64_t)d->heads;
  }
  *pairs = p;
  *rows = r;
}

void oracle_rand_vec(float* out, size_t n, uint64_t seed) {
  /* tests/common/mod.rs:6-18 */
  uint64_t s = (seed * 0x9E3779B97F4A7C15ull) | 1ull;
  for (size_t i = 0; i < n; ++i) {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    const float u = (float)(s >> 40) / (float)(1ull << 24);
    out[i] = 2.0f * u - 1.0f;
  }
}

void oracle_lcg_fill(float* out, size_t n, uint32_t seed) {
  /* tests/masks_edges.rs:6-14 */
  uint32_t s = seed;
  for (size_t i = 0; i < n; ++i) {
    s = s * 1664525u + 1013904223u;
    out[i] = (float)(s >> 8) / (float)(1u << 24) - 0.5f;
  }
}
