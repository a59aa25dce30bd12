/*
 * tiled.c — CPU restatement of raya's Tiled kernel: the timed CPU baseline
 * ("CPU restatement of raya Tiled-AVX2") and a second checker.
 *
 * TEST / BASELINE INFRASTRUCTURE ONLY: nothing in the product links it.
 *
 * Restated from (paths relative to the raya project root):
 *   crates/raya-kernels/src/tiled/mod.rs:61-126  task list of (slice, query
 *       block) popped from a shared queue by `threads` workers
 *   crates/raya-kernels/src/tiled/tile.rs:27-62  run_block: MR=8 row micro
 *       tiles, padded rows filled with 0
 *   crates/raya-kernels/src/tiled/tile.rs:65-151 micro_tile: NC=64 key tiles,
 *       online softmax (scale, tile max, alpha = exp(m - new_m) or 0 when m
 *       is -inf, exp_shifted_sum, l = l*alpha + sum, acc *= alpha when the
 *       max rose), P.V accumulate, out = acc * (1/l) or 0
 *   crates/raya-kernels/src/simd/avx2.rs:23-74   dot_tile / axpy_rows
 *   crates/raya-kernels/src/simd/portable.rs:37-127 portable kernels
 *   crates/raya-kernels/src/simd/mod.rs:23-32,83-91 run-time AVX2+FMA check
 *
 * The vector exp the reference takes from the `wide` crate (1.7.1, not in
 * the reference tree) is replaced by the Cephes single-precision exp method
 * (S. L. Moshier): n = round(x log2 e), r = x - n ln2 in two parts, a
 * degree-6 polynomial, times 2^n.  Parity of this file with the oracle is
 * checked by the tests at the reference's 1e-5 bar.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

#if defined(__x86_64__)
#include <immintrin.h>
#endif

enum { MR = 8, NC = 64 };

int oracle_cpu_has_avx2_fma(void) {
#if defined(__x86_64__)
  __builtin_cpu_init();
  return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
#else
  return 0;
#endif
}

/* ---------------- portable micro-kernels (portable.rs) ---------------- */

static float dot_portable(const float* a, const float* b, int64_t d) {
  /* portable.rs:15-34: four 8-lane accumulators over chunks of 32, then the
   * 8-wide remainder into accumulator 0. */
  float acc[4][8];
  memset(acc, 0, sizeof acc);
  int64_t c = 0;
  for (; c + 32 <= d; c += 32)
    for (int t = 0; t < 4; ++t)
      for (int l = 0; l < 8; ++l) acc[t][l] += a[c + t * 8 + l] * b[c + t * 8 + l];
  for (; c + 8 <= d; c += 8)
    for (int l = 0; l < 8; ++l) acc[0][l] += a[c + l] * b[c + l];
  float s = 0.0f;
  for (int l = 0; l < 8; ++l) s += (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
  return s;
}

static void dot_tile_portable(const float* q, const float* k, int64_t d, int mr,
                              int nk, float* out) {
  for (int r = 0; r < mr; ++r)
    for (int j = 0; j < nk; ++j) out[r * NC + j] = dot_portable(q + r * d, k + j * d, d);
}

static void axpy_rows_portable(float* acc, const float* p, int n, const float* v,
                               int64_t d) {
  for (int j = 0; j < n; ++j) {
    const float pj = p[j];
    for (int64_t c = 0; c < d; ++c) acc[c] += pj * v[j * d + c];
  }
}

static float exp_shifted_sum_portable(float* x, int n, float shift) {
  float lanes[8] = {0};
  int i = 0;
  for (; i + 8 <= n; i += 8)
    for (int l = 0; l < 8; ++l) {
      x[i + l] = expf(x[i + l] - shift);
      lanes[l] += x[i + l];
    }
  float sum = ((lanes[0] + lanes[4]) + (lanes[2] + lanes[6])) +
              ((lanes[1] + lanes[5]) + (lanes[3] + lanes[7]));
  for (; i < n; ++i) {
    x[i] = expf(x[i] - shift);
    sum += x[i];
  }
  return sum;
}

/* ---------------- AVX2 + FMA micro-kernels (avx2.rs) ---------------- */
#if defined(__x86_64__)
__attribute__((target("avx2,fma"))) static float hsum256(__m256 x) {
  /* avx2.rs:9-17 */
  __m128 lo = _mm256_castps256_ps128(x);
  __m128 hi = _mm256_extractf128_ps(x, 1);
  __m128 s = _mm_add_ps(lo, hi);
  __m128 sh = _mm_movehdup_ps(s);
  __m128 s2 = _mm_add_ps(s, sh);
  __m128 hi2 = _mm_movehl_ps(sh, s2);
  return _mm_cvtss_f32(_mm_add_ss(s2, hi2));
}

__attribute__((target("avx2,fma"))) static void dot_tile_avx2(const float* q,
                                                              const float* k,
                                                              int64_t d, int mr,
                                                              int nk, float* out) {
  /* avx2.rs:23-47: per key, per row, two 8-lane FMA accumulators over
   * 16-column steps, an 8-column tail into the first. */
  for (int j = 0; j < nk; ++j) {
    const float* kj = k + j * d;
    for (int r = 0; r < mr; ++r) {
      const float* qr = q + r * d;
      __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
      int64_t c = 0;
      for (; c + 16 <= d; c += 16) {
        a0 = _mm256_fmadd_ps(_mm256_loadu_ps(qr + c), _mm256_loadu_ps(kj + c), a0);
        a1 = _mm256_fmadd_ps(_mm256_loadu_ps(qr + c + 8), _mm256_loadu_ps(kj + c + 8), a1);
      }
      if (c < d) a0 = _mm256_fmadd_ps(_mm256_loadu_ps(qr + c), _mm256_loadu_ps(kj + c), a0);
      out[r * NC + j] = hsum256(_mm256_add_ps(a0, a1));
    }
  }
}

__attribute__((target("avx2,fma"))) static void axpy_rows_avx2(float* acc,
                                                               const float* p, int n,
                                                               const float* v,
                                                               int64_t d) {
  /* avx2.rs:52-74: 64-column chunks held in eight registers. */
  for (int64_t c0 = 0; c0 < d; c0 += 64) {
    const int64_t w = d - c0 < 64 ? d - c0 : 64;
    const int nv = (int)(w / 8);
    __m256 r[8];
    for (int t = 0; t < nv; ++t) r[t] = _mm256_loadu_ps(acc + c0 + t * 8);
    for (int j = 0; j < n; ++j) {
      const float* vj = v + j * d + c0;
      const __m256 ps = _mm256_set1_ps(p[j]);
      for (int t = 0; t < nv; ++t) r[t] = _mm256_fmadd_ps(ps, _mm256_loadu_ps(vj + t * 8), r[t]);
    }
    for (int t = 0; t < nv; ++t) _mm256_storeu_ps(acc + c0 + t * 8, r[t]);
  }
}

/* Cephes single-precision exp (S. L. Moshier), eight lanes. */
__attribute__((target("avx2,fma"))) static __m256 exp8_cephes(__m256 x) {
  const __m256 hi = _mm256_set1_ps(88.3762626647949f);
  const __m256 lo = _mm256_set1_ps(-88.3762626647949f);
  const __m256 log2e = _mm256_set1_ps(1.44269504088896341f);
  const __m256 c1 = _mm256_set1_ps(0.693359375f);
  const __m256 c2 = _mm256_set1_ps(-2.12194440e-4f);
  const __m256 neg_inf_mask = _mm256_cmp_ps(x, _mm256_set1_ps(-INFINITY), _CMP_EQ_OQ);
  x = _mm256_min_ps(x, hi);
  x = _mm256_max_ps(x, lo);
  __m256 fx = _mm256_round_ps(_mm256_mul_ps(x, log2e), _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
  x = _mm256_fnmadd_ps(fx, c1, x);
  x = _mm256_fnmadd_ps(fx, c2, x);
  const __m256 z = _mm256_mul_ps(x, x);
  __m256 y = _mm256_set1_ps(1.9875691500e-4f);
  y = _mm256_fmadd_ps(y, x, _mm256_set1_ps(1.3981999507e-3f));
  y = _mm256_fmadd_ps(y, x, _mm256_set1_ps(8.3334519073e-3f));
  y = _mm256_fmadd_ps(y, x, _mm256_set1_ps(4.1665795894e-2f));
  y = _mm256_fmadd_ps(y, x, _mm256_set1_ps(1.6666665459e-1f));
  y = _mm256_fmadd_ps(y, x, _mm256_set1_ps(5.0000001201e-1f));
  y = _mm256_fmadd_ps(y, z, x);
  y = _mm256_add_ps(y, _mm256_set1_ps(1.0f));
  __m256i n = _mm256_cvtps_epi32(fx);
  n = _mm256_slli_epi32(_mm256_add_epi32(n, _mm256_set1_epi32(127)), 23);
  y = _mm256_mul_ps(y, _mm256_castsi256_ps(n));
  /* exp(-inf) = 0 exactly: masked scores never reach this kernel, but keep
   * the identity. */
  return _mm256_andnot_ps(neg_inf_mask, y);
}

__attribute__((target("avx2,fma"))) static float exp_shifted_sum_avx2(float* x, int n,
                                                                      float shift) {
  /* portable.rs:112-127 with the vector exp in AVX2 */
  const __m256 sh = _mm256_set1_ps(shift);
  __m256 acc = _mm256_setzero_ps();
  int i = 0;
  for (; i + 8 <= n; i += 8) {
    __m256 e = exp8_cephes(_mm256_sub_ps(_mm256_loadu_ps(x + i), sh));
    _mm256_storeu_ps(x + i, e);
    acc = _mm256_add_ps(acc, e);
  }
  float sum = hsum256(acc);
  for (; i < n; ++i) {
    x[i] = expf(x[i] - shift);
    sum += x[i];
  }
  return sum;
}
#endif

/* ---------------- tile driver (tile.rs) ---------------- */

typedef struct {
  const oracle_desc* d;
  const float *q, *k, *v;
  float* out;
  const int32_t* valid_len;
  int64_t bh0, nblocks_per_slice, rows_per_task;
  int64_t ntasks;
  atomic_llong next;
  int avx2;
} tiled_job;

static void micro_tile(const tiled_job* job, const float* q, const float* k,
                       const float* v, int64_t valid, int64_t gi0, int mr, float* out,
                       float* scores, float* acc) {
  const oracle_desc* d = job->d;
  const int64_t D = d->head_dim;
  int64_t rlo[MR], rhi[MR];
  for (int r = 0; r < MR; ++r) {
    const int rr = r < mr - 1 ? r : mr - 1; /* tile.rs:77-78 */
    oracle_key_range(d, gi0 + rr, valid, &rlo[r], &rhi[r]);
  }
  const int64_t ks = rlo[0], ke = rhi[mr - 1];
  float m[MR], l[MR];
  for (int r = 0; r < MR; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
  }
  memset(acc, 0, sizeof(float) * (size_t)(mr * D));
  const float* qt = q + gi0 * D;
  for (int64_t kt = ks; kt < ke; kt += NC) { /* tile.rs:87-141 */
    const int64_t kend = kt + NC < ke ? kt + NC : ke;
    const int nk = (int)(kend - kt);
#if defined(__x86_64__)
    if (job->avx2)
      dot_tile_avx2(qt, k + kt * D, D, mr, nk, scores);
    else
#endif
      dot_tile_portable(qt, k + kt * D, D, mr, nk, scores);
    int ba[MR], bz[MR];
    for (int r = 0; r < mr; ++r) {
      ba[r] = bz[r] = 0;
      const int64_t lo = rlo[r] > kt ? rlo[r] : kt;
      const int64_t hi = rhi[r] < kend ? rhi[r] : kend;
      if (lo >= hi) continue;
      const int a = (int)(lo - kt), z = (int)(hi - kt);
      ba[r] = a;
      bz[r] = z;
      float* row = scores + r * NC;
      float tmax = -INFINITY;
      for (int x = a; x < z; ++x) {
        row[x] *= d->scale;
        tmax = fmaxf(tmax, row[x]);
      }
      const float new_m = fmaxf(m[r], tmax);
      const float alpha = m[r] == -INFINITY ? 0.0f : expf(m[r] - new_m);
      float sum;
#if defined(__x86_64__)
      if (job->avx2)
        sum = exp_shifted_sum_avx2(row + a, z - a, new_m);
      else
#endif
        sum = exp_shifted_sum_portable(row + a, z - a, new_m);
      l[r] = l[r] * alpha + sum;
      const int raised = new_m > m[r];
      m[r] = new_m;
      if (raised)
        for (int64_t c = 0; c < D; ++c) acc[r * D + c] *= alpha;
    }
    for (int r = 0; r < mr; ++r) {
      if (ba[r] >= bz[r]) continue;
#if defined(__x86_64__)
      if (job->avx2)
        axpy_rows_avx2(acc + r * D, scores + r * NC + ba[r], bz[r] - ba[r],
                       v + (kt + ba[r]) * D, D);
      else
#endif
        axpy_rows_portable(acc + r * D, scores + r * NC + ba[r], bz[r] - ba[r],
                           v + (kt + ba[r]) * D, D);
    }
  }
  for (int r = 0; r < mr; ++r) { /* tile.rs:142-150 */
    const float inv = l[r] > 0.0f ? 1.0f / l[r] : 0.0f;
    for (int64_t c = 0; c < D; ++c) out[r * D + c] = acc[r * D + c] * inv;
  }
}

static void* tiled_worker(void* arg) {
  tiled_job* job = (tiled_job*)arg;
  const oracle_desc* d = job->d;
  const int64_t L = d->seq, D = d->head_dim;
  float* scores = (float*)malloc(sizeof(float) * MR * NC);
  float* acc = (float*)malloc(sizeof(float) * (size_t)(MR * D));
  for (;;) {
    const long long t = atomic_fetch_add(&job->next, 1);
    if (t >= job->ntasks) break;
    const int64_t bh = job->bh0 + t / job->nblocks_per_slice;
    const int64_t blk = t % job->nblocks_per_slice;
    const int64_t b = bh / d->heads;
    const int64_t valid = job->valid_len ? job->valid_len[b] : L;
    const float* q = job->q + bh * L * D;
    const float* k = job->k + bh * L * D;
    const float* v = job->v + bh * L * D;
    float* out = job->out + bh * L * D;
    /* tile.rs:27-62: MR-row micro tiles over the task's rows */
    const int64_t row0 = blk * job->rows_per_task;
    const int64_t rows_end = row0 + job->rows_per_task < L ? row0 + job->rows_per_task : L;
    for (int64_t gi0 = row0; gi0 < rows_end; gi0 += MR) {
      const int mr = (int)(rows_end - gi0 < MR ? rows_end - gi0 : MR);
      int64_t nvalid = valid - gi0;
      if (nvalid < 0) nvalid = 0;
      if (nvalid > mr) nvalid = mr;
      memset(out + (gi0 + nvalid) * D, 0, sizeof(float) * (size_t)((mr - nvalid) * D));
      if (nvalid > 0)
        micro_tile(job, q, k, v, valid, gi0, (int)nvalid, out + gi0 * D, scores, acc);
    }
  }
  free(scores);
  free(acc);
  return NULL;
}

int oracle_tiled(const oracle_desc* d, const float* q, const float* k,
                 const float* v, float* out, const int32_t* valid_len,
                 int64_t bh0, int64_t bh1, int threads, int backend) {
  tiled_job job;
  job.d = d;
  job.q = q;
  job.k = k;
  job.v = v;
  job.out = out;
  job.valid_len = valid_len;
  job.bh0 = bh0;
  /* tiled/mod.rs:82-88 splits each head into BLOCK-row tasks; with other
   * masks or block sizes the task stays 128 rows (the reference's BLOCK). */
  job.rows_per_task = d->mask == ORACLE_MASK_BLOCK ? d->block : 128;
  job.nblocks_per_slice =
      d->seq > 0 ? (d->seq + job.rows_per_task - 1) / job.rows_per_task : 0;
  job.ntasks = (bh1 - bh0) * job.nblocks_per_slice;
  atomic_init(&job.next, 0);
  job.avx2 = backend == 1 && oracle_cpu_has_avx2_fma();
  if (job.ntasks <= 0) return job.avx2;
  int workers = threads < 1 ? 1 : threads;
  if (workers > job.ntasks) workers = (int)job.ntasks;
  if (workers == 1) {
    tiled_worker(&job);
  } else {
    pthread_t* tids = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)workers);
    for (int w = 0; w < workers; ++w) pthread_create(&tids[w], NULL, tiled_worker, &job);
    for (int w = 0; w < workers; ++w) pthread_join(tids[w], NULL);
    free(tids);
  }
  return job.avx2;
}
