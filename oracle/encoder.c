/*
 * encoder.c — restatement of the caller's layout transforms around the
 * attention call, for checking the fused packed-layout entry point.
 * TEST INFRASTRUCTURE ONLY.
 *
 *   split_qkv     crates/raya-core/src/encoder.rs:34-53
 *   rope_in_place crates/raya-core/src/ops.rs:110-141 (rotate-half form, angles
 *                 in f32: inv_freq = 1/theta^(2i/head_dim), angle = pos*inv_freq)
 *   context back  crates/raya-core/src/encoder.rs:82-90
 *
 * Built with -ffp-contract=off like the rest of the oracle (Rust never fuses).
 */
#include <math.h>
#include <stdlib.h>

#include "oracle.h"

void oracle_split_qkv(const float* qkv, int64_t seq, int64_t heads, int64_t head_dim, float* q,
                      float* k, float* v) {
  const int64_t d = heads * head_dim;
  float* parts[3] = {q, k, v};
  for (int64_t t = 0; t < seq; ++t)
    for (int w = 0; w < 3; ++w)
      for (int64_t h = 0; h < heads; ++h) {
        const float* src = qkv + t * 3 * d + w * d + h * head_dim;
        float* dst = parts[w] + (h * seq + t) * head_dim;
        for (int64_t c = 0; c < head_dim; ++c) dst[c] = src[c];
      }
}

void oracle_rope_inplace(float* x, int64_t heads, int64_t seq, int64_t head_dim, float theta) {
  const int64_t half = head_dim / 2;
  float* inv_freq = (float*)malloc(sizeof(float) * (size_t)half);
  float* cs = (float*)malloc(sizeof(float) * (size_t)half);
  float* sn = (float*)malloc(sizeof(float) * (size_t)half);
  for (int64_t i = 0; i < half; ++i)
    inv_freq[i] = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
  for (int64_t pos = 0; pos < seq; ++pos) {
    for (int64_t i = 0; i < half; ++i) {
      const float angle = (float)pos * inv_freq[i];
      cs[i] = cosf(angle);
      sn[i] = sinf(angle);
    }
    for (int64_t h = 0; h < heads; ++h) {
      float* row = x + (h * seq + pos) * head_dim;
      for (int64_t i = 0; i < half; ++i) {
        const float a = row[i], b = row[i + half];
        row[i] = a * cs[i] - b * sn[i];
        row[i + half] = b * cs[i] + a * sn[i];
      }
    }
  }
  free(inv_freq);
  free(cs);
  free(sn);
}

void oracle_merge_ctx(const float* out, int64_t seq, int64_t heads, int64_t head_dim, float* ctx) {
  const int64_t d = heads * head_dim;
  for (int64_t h = 0; h < heads; ++h)
    for (int64_t t = 0; t < seq; ++t)
      for (int64_t c = 0; c < head_dim; ++c)
        ctx[t * d + h * head_dim + c] = out[(h * seq + t) * head_dim + c];
}
