/*
 * oracle.h — CPU restatement of raya's block-local attention, used ONLY as a
 * checker by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference legs.  It is test infrastructure: the product path
 * (raya_b200/, libraya_attn.so) never links or calls it.
 *
 * Restated from the reference (paths relative to the raya project root):
 *   - naive.rs:13-65          Naive::attend (scalar oracle semantics)
 *   - attention.rs:48-69      Mask::key_range / Mask::allows
 *   - tiled/mod.rs:61-126     Tiled::attend_with_stages (task queue, threads)
 *   - tiled/tile.rs:27-151    run_block / micro_tile (online softmax tiles)
 *   - simd/avx2.rs:23-74      dot_tile / axpy_rows AVX2+FMA micro-kernels
 *   - simd/portable.rs:112-127 exp_shifted_sum
 *   - tests/common/mod.rs:6-18 xorshift rand_vec (test input generator)
 *   - tests/masks_edges.rs:6-14 LCG fill (test input generator)
 *
 * Generalisations (the reference accepts only block == 128, batch 1, one
 * scalar valid_len): a batch dimension with valid_len[batch], any block size,
 * a `halo` (query block b sees key blocks b-halo ..= b+halo; halo = 1 is the
 * reference's Block3), windows of any half width (Window64 = window 64,
 * Sliding(w)), and Full.  At block 128 / halo 1 / batch 1 the arithmetic is
 * the reference's.
 */
#ifndef RAYA_ORACLE_H
#define RAYA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORACLE_MASK_BLOCK = 0, ORACLE_MASK_WINDOW = 1, ORACLE_MASK_FULL = 2 };

typedef struct {
  int64_t batch, heads, seq, head_dim;
  int64_t block;  /* block size B (BLOCK masks) */
  int32_t mask;   /* ORACLE_MASK_* */
  int32_t halo;   /* BLOCK: key blocks on each side */
  int64_t window; /* WINDOW: half width */
  float scale;
} oracle_desc;

/* Keys [lo, hi) that query row i may attend, clipped to valid_len
 * (attention.rs:48-59 with BLOCK -> block and 1 -> halo). */
void oracle_key_range(const oracle_desc* d, int64_t i, int64_t valid_len,
                      int64_t* lo, int64_t* hi);

/* Naive::attend (naive.rs:13-65) over [batch][heads][seq][head_dim].
 * valid_len may be NULL (every sequence fully valid). */
void oracle_naive(const oracle_desc* d, const float* q, const float* k,
                  const float* v, float* out, const int32_t* valid_len);

/* Same, restricted to the flattened (batch*heads) slices [bh0, bh1); the
 * pointers address slice 0 of the full tensors. */
void oracle_naive_range(const oracle_desc* d, const float* q, const float* k,
                        const float* v, float* out, const int32_t* valid_len,
                        int64_t bh0, int64_t bh1);

/* Tiled::attend restated (tile.rs + avx2.rs micro-kernels), `threads`
 * workers pulling (slice, query block) tasks from a shared queue like
 * tiled/mod.rs:82-124.  backend: 0 = portable scalar, 1 = AVX2+FMA (falls
 * back to portable when the CPU lacks AVX2/FMA, simd/mod.rs:83-91).
 * Work is restricted to flattened slices [bh0, bh1).  Returns the backend
 * actually used. */
int oracle_tiled(const oracle_desc* d, const float* q, const float* k,
                 const float* v, float* out, const int32_t* valid_len,
                 int64_t bh0, int64_t bh1, int threads, int backend);

/* 1 if this CPU runs the AVX2+FMA kernels (simd/mod.rs:23-32). */
int oracle_cpu_has_avx2_fma(void);

/* Exact number of allowed (query < valid, key < valid, mask-allowed) pairs
 * and of valid query rows, summed over batch and heads. */
void oracle_count(const oracle_desc* d, const int32_t* valid_len,
                  uint64_t* pairs, uint64_t* rows);

/* The caller's layout transforms (encoder.c): split a packed [seq][3][heads]
 * [head_dim] projection into head-major q, k, v (encoder.rs:34-53); raya's
 * rotary embedding in place on [heads][seq][head_dim] (ops.rs:110-141); the
 * head-major output back to [seq][heads*head_dim] (encoder.rs:82-90). */
void oracle_split_qkv(const float* qkv, int64_t seq, int64_t heads, int64_t head_dim, float* q,
                      float* k, float* v);
void oracle_rope_inplace(float* x, int64_t heads, int64_t seq, int64_t head_dim, float theta);
void oracle_merge_ctx(const float* out, int64_t seq, int64_t heads, int64_t head_dim, float* ctx);

/* tests/common/mod.rs:6-18: xorshift values uniform in [-1, 1]. */
void oracle_rand_vec(float* out, size_t n, uint64_t seed);

/* tests/masks_edges.rs:6-14: LCG values in [-0.5, 0.5). */
void oracle_lcg_fill(float* out, size_t n, uint32_t seed);

#ifdef __cplusplus
}
#endif
#endif
