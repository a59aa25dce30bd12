/*
 * raya_attn.h — C ABI of the B200 (sm_100a) block-local attention library
 * (libraya_attn.so).  Plain pointers and sizes only: no CUDA or torch types
 * appear in these signatures (streams are passed as `void*` holding a
 * cudaStream_t, NULL meaning the legacy default stream).
 *
 * It replaces raya's `AttentionKernel` implementations for the block-local
 * path (paths relative to the raya project root):
 *   trait AttentionKernel::attend   crates/raya-kernels/src/attention.rs:113-125
 *   validate                        crates/raya-kernels/src/attention.rs:128-170
 *   Tiled::attend                   crates/raya-kernels/src/tiled/mod.rs:138-149
 * A Rust maintainer binds `raya_attn_forward_host` with `batch = 1` inside an
 * `impl AttentionKernel for Cuda`; the FFI crate crates/raya-kernels-cuda of
 * this repository is that binding.
 *
 * Layout contract (attention.rs:72-78, extended with a batch dimension):
 * q, k, v and out are row-major fp32 `[batch][heads][seq][head_dim]`; the
 * reference's `[heads][seq][head_dim]` is batch = 1.  valid_len holds one
 * int32 per batch entry: keys at or beyond it are padding and query rows at
 * or beyond it are written as +0.0f.  `out` is fully overwritten.
 *
 * Semantics (attention.rs:108-112, naive.rs:13-65): for row i < valid_len,
 * out[i] = sum_j softmax_j(scale * q_i . k_j) v_j over keys j < valid_len
 * allowed by the mask; rows with no allowed key are zero.
 */
#ifndef RAYA_ATTN_H
#define RAYA_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RAYA_ATTN_VERSION 1

/* Mirrors KernelError (attention.rs:8-20) plus device-side failures. */
typedef enum {
  RAYA_ATTN_OK = 0,
  RAYA_ATTN_ERR_SHAPE = 1,       /* KernelError::Shape */
  RAYA_ATTN_ERR_LENGTH = 2,      /* KernelError::Length { name, got, expected } */
  RAYA_ATTN_ERR_UNSUPPORTED = 3, /* KernelError::Unsupported */
  RAYA_ATTN_ERR_CUDA = 4,        /* a CUDA runtime call failed */
  RAYA_ATTN_ERR_TIMEOUT = 5      /* a device-side wait gave up (bounded spin) */
  /* The library runs no collective: raya_attn_forward_multi_gpu moves data
   * with peer copies (failures: RAYA_ATTN_ERR_CUDA), and the NCCL gather of
   * sharded outputs belongs to the caller's process group. */
} raya_attn_status;

/* Mask kinds (attention.rs:22-35, generalised):
 *   BLOCK  : |i/block - j/block| <= halo.  halo = 1, block = 128 is
 *            Mask::Block3 (Laya's block_local); halo = 0 is "own block only".
 *   WINDOW : |i - j| <= window.  window = 64 is Mask::Window64, any other
 *            value is Mask::Sliding(window).
 *   FULL   : every key below valid_len (Mask::Full).                       */
typedef enum {
  RAYA_MASK_BLOCK = 0,
  RAYA_MASK_WINDOW = 1,
  RAYA_MASK_FULL = 2
} raya_mask_kind;

/* AttnShape + AttnParams (attention.rs:72-106) with a batch dimension.
 * Rust's `AttnParams::new` sets scale = 1/sqrt(head_dim) in f32. */
typedef struct {
  int64_t batch;    /* >= 1 */
  int64_t heads;    /* >= 1 */
  int64_t seq;      /* >= 0 */
  int64_t head_dim; /* >= 8, multiple of 8 (validate), <= 256 (this library) */
  int64_t block;    /* BLOCK masks: block size, >= 1 (reference: only 128) */
  int32_t mask;     /* raya_mask_kind */
  int32_t halo;     /* BLOCK masks: key blocks on each side, >= 0 */
  int64_t window;   /* WINDOW masks: half width, >= 0 */
  float scale;      /* softmax scale applied to q.k */
} raya_attn_desc;

/* Kernel selection for raya_attn_forward_ex (tests and benchmarks). */
typedef enum {
  RAYA_KERNEL_AUTO = 0,     /* head_dim 64: the tensor-core kernel
                               RAYA_KERNEL_TC32_WS for Full, windows of half width >= 64,
                               other blocks >= 128 and block masks with a halo whose
                               allowed keys fill >= half of a 128-row CTA's key span, in
                               its two-tile form RAYA_KERNEL_TC32_WS2 for such blocks
                               below 128 with >= 1024 128-row tiles and for blocks >= 128
                               with >= 2048 tiles and at most 2048 keys per span; else the
                               tuned tiled kernel; other head_dims: rowwise */
  RAYA_KERNEL_TILED64 = 1,  /* the tuned tiled variant for the mask and block (head_dim 64):
                               W4R16_P2 for block <= 64 and windows, W4R32_P2 for
                               block >= 128 and Full */
  RAYA_KERNEL_ROWWISE = 2,  /* one warp per query row, any head_dim */
  /* Fixed variants of the tiled kernel for benchmarks and tests: 4 warps per
   * CTA of R = 32 or 16 query rows each; P2 = packed FFMA2 (two fused
   * multiply-adds per instruction) in QK^T and PV (R16) or PV only (R32). */
  RAYA_KERNEL_TILED64_W4R32 = 16,
  RAYA_KERNEL_TILED64_W4R16 = 19,
  RAYA_KERNEL_TILED64_W4R16_P2 = 20,
  RAYA_KERNEL_TILED64_W4R32_P2 = 21,
  /* Tensor cores (tcgen05, kind::tf32) in 3xTF32: each fp32 operand enters
   * as itself (read as TF32) and as its remainder, three products per tile,
   * fp32-level accuracy; head_dim 64, 128-row tiles.  Warp-specialised: a
   * split warp group prepares the K/V operand stages, QK^T and PV are issued
   * by two warps, and each key tile's PV product is added into the O rows in
   * fp32 registers (the tensor core's own accumulation truncates toward
   * zero, which over many tiles would exceed the parity bar). */
  RAYA_KERNEL_TC32_WS = 34,
  /* RAYA_KERNEL_TC32_WS with two 128-row tiles per CTA (four where a
   * (batch, head) slice is four row tiles, seq 385..512, so that a CTA runs
   * the whole slice, and where the slice's row tiles are a multiple of four
   * under a block mask of 128 keys or more, with at least 16384 row tiles in
   * all; head-major layout), one after
   * the other, each run as a CTA of its own (sharing only the CTA's launch,
   * tensor-memory allocation and valid_len loads). */
  RAYA_KERNEL_TC32_WS2 = 37,
  /* The same pipeline on tcgen05 kind::f16 in 3xFP16: each fp32 operand is
   * scaled by a power of two (per q row, per 64-key K or V tile) so that its
   * largest element lies in [2^14, 2^15), then split into two fp16 parts;
   * three products per tile at twice kind::tf32's rate per instruction.  The
   * softmax removes the scales exactly.  head_dim 64, 128-row tiles, one
   * per CTA; raya_attn_forward_ex only (the packed entry points use the TF32
   * kernels). */
  RAYA_KERNEL_TC16_WS = 40,
  /* RAYA_KERNEL_TC16_WS as a persistent grid: one CTA per SM walks its
   * 128-row tiles, every ring running on across them, so one tile's copies
   * and products overlap the previous tile's tail. */
  RAYA_KERNEL_TC16_WS2 = 41
} raya_kernel_id;

/* Argument checks of validate (attention.rs:128-170), extended to the batch
 * layout.  Buffer lengths are element counts, like the Rust slices' len();
 * valid_len is a HOST array of `batch` entries or NULL (every sequence fully
 * valid).  Returns OK or the error the reference would raise; the message is
 * available from raya_attn_last_error(). */
raya_attn_status raya_attn_validate(const raya_attn_desc* desc, const int32_t* valid_len,
                                    size_t q_len, size_t k_len, size_t v_len,
                                    size_t out_len);

/* Synchronous host-buffer call: the AttentionKernel::attend contract
 * (attention.rs:113-125, tiled/mod.rs:138-149).  q, k, v, out and valid_len
 * are HOST pointers (pageable or pinned).  Validates, copies the inputs to
 * device `device`, runs the kernel, copies `out` back and synchronises.
 * Thread-safe: concurrent callers serialise on the device's staging buffers. */
raya_attn_status raya_attn_forward_host(const raya_attn_desc* desc, const float* q,
                                        size_t q_len, const float* k, size_t k_len,
                                        const float* v, size_t v_len, float* out,
                                        size_t out_len, const int32_t* valid_len,
                                        int device);

/* The host-buffer call spread over several GPUs of this process: batch x
 * heads is the shard.  The flattened batch*heads slices are cut into
 * `ndevices` contiguous ranges balanced by allowed-pair count
 * (raya_attn_shard); device devices[r] receives range r's q, k and v rows,
 * runs the kernel on them and returns its part of the output, all devices at
 * once (one host thread each; the reference's counterpart is Tiled's task
 * split over (head, block) on host threads, tiled/mod.rs:82-124).  Slices are
 * independent, so the result is bit-identical to raya_attn_forward_host on
 * one device.  Outputs go to the HOST buffer `out` and, when `out_device0` is
 * not NULL, also to that DEVICE buffer of batch*heads*seq*head_dim floats on
 * devices[0]: the other devices' parts are copied into it device to device
 * (peer copies over NVLink).  `out` may be NULL when `out_device0` is given
 * (out_len is then ignored).  Device ids must be distinct.  Synchronous;
 * allocates staging buffers on each device like raya_attn_forward_host. */
raya_attn_status raya_attn_forward_multi_gpu(const raya_attn_desc* desc, const float* q, size_t q_len,
                                             const float* k, size_t k_len, const float* v, size_t v_len,
                                             float* out, size_t out_len, const int32_t* valid_len,
                                             const int* devices, int ndevices, float* out_device0);

/* Asynchronous device-buffer call on `stream` (the B200-native entry point,
 * no reference counterpart beyond the trait's semantics).  q, k, v, out are
 * DEVICE pointers holding batch*heads*seq*head_dim floats; valid_len is a
 * DEVICE array of `batch` int32 or NULL.  The shape is validated on the host;
 * valid_len values are not visible to the host here, so the kernel clamps
 * each into [0, seq] (use raya_attn_validate on a host copy for the
 * reference's error).  Launch errors are returned; device-side timeouts are
 * reported by raya_attn_sync_status.  Allocates nothing. */
raya_attn_status raya_attn_forward(const raya_attn_desc* desc, const float* q,
                                   const float* k, const float* v, float* out,
                                   const int32_t* valid_len, void* stream);

/* raya_attn_forward with an explicit kernel (raya_kernel_id). */
raya_attn_status raya_attn_forward_ex(const raya_attn_desc* desc, const float* q,
                                      const float* k, const float* v, float* out,
                                      const int32_t* valid_len, void* stream,
                                      int kernel_id);

/* The caller's layout, fused (§ "next" of the path: encoder.rs:34-92).
 * raya's encoder splits a packed projection qkv[seq][3][heads][head_dim] into
 * head-major q, k, v (split_qkv, encoder.rs:34-53), applies its rotary
 * embedding to q and k (ops.rs:110-141) and transposes the head-major output
 * back to ctx[seq][heads*head_dim] (encoder.rs:82-90).  This call does all of
 * it inside the attention kernel: qkv is the DEVICE tensor
 * [batch][seq][3][heads][64] (read in place by TMA), ctx the DEVICE tensor
 * [batch][seq][heads][64] it writes (padded rows +0.0f), valid_len a DEVICE
 * int32[batch] or NULL.  rope_theta > 0 rotates q and k first (angles in f32
 * as the reference computes them); 0 skips the rotation.  With rope_theta > 0
 * the call needs a DEVICE workspace of raya_attn_packed_workspace bytes (the
 * cos/sin table, written by the call); it may be NULL otherwise.  head_dim
 * must be 64.  Asynchronous on `stream`; allocates nothing.  Kernel: the
 * two-issuer tensor-core kernel (RAYA_KERNEL_TC32_WS) with this layout
 * wherever RAYA_KERNEL_AUTO picks a tensor-core kernel (its two-tile form
 * RAYA_KERNEL_TC32_WS2 where that is the choice and there is no rotation),
 * else the tuned tiled kernel (raya_attn_kernel_for with packed != 0 names
 * it). */
raya_attn_status raya_attn_forward_packed(const raya_attn_desc* desc, const float* qkv, float* ctx,
                                          const int32_t* valid_len, float rope_theta, void* workspace,
                                          size_t workspace_bytes, void* stream);

/* Workspace bytes raya_attn_forward_packed needs for this shape and theta. */
raya_attn_status raya_attn_packed_workspace(const raya_attn_desc* desc, float rope_theta, size_t* bytes);

/* raya_attn_forward_packed without a workspace: nothing is allocated.  No
 * counterpart in the reference.  For callers that cannot allocate device
 * memory: a serving runtime that owns all of the GPU's memory through its
 * own pool, a binding that only receives raw device pointers from its host,
 * or a latency-bound loop where cudaMalloc (which may synchronise the
 * device) must not run.  The rotary cos/sin table lives in a built-in device
 * array of 8192 positions (2 MiB, held on every GPU that loads the library
 * until the process exits); with rope_theta > 0 a seq above 8192 is
 * rejected with RAYA_ATTN_ERR_UNSUPPORTED.  The first call on each device
 * looks the array's address up (cudaGetSymbolAddress) with that device
 * current, so make that first call before any stream capture.  All calls
 * share the array: each rewrites the positions it reads, but calls whose
 * work overlaps on the GPU (other streams, other host threads) race on it.
 * Arguments and results as raya_attn_forward_packed. */
raya_attn_status raya_attn_forward_packed_noalloc(const raya_attn_desc* desc, const float* qkv, float* ctx,
                                                  const int32_t* valid_len, float rope_theta, void* stream);

/* Stage timing, the counterpart of Tiled::attend_with_stages / StageTimes
 * (tiled/mod.rs:60-126, tiled/stages.rs:1-31): raya_attn_forward_ex whose
 * kernel reads clock64 around each stage and adds the cycle counts into
 * stage_cycles, a DEVICE array of 8 uint64 that the caller zeroes.
 * kernel_id: RAYA_KERNEL_AUTO (the automatic choice), TILED64 or a
 * TILED64_* variant, or RAYA_KERNEL_TC32_WS / RAYA_KERNEL_TC32_WS2.
 * Tiled kernels (warp cycles summed over warps): [0] QK^T, [1] softmax,
 * [2] P.V, [3] K-tile wait, [4] V-tile wait, [5] next-tile refill,
 * [6] warp-tiles processed, [7] total cycles.
 * Tensor-core kernels (cycles per CTA, summed over CTAs): [0] QK^T products
 * in flight (issue to completion), [1] one softmax warp's work per key tile,
 * [2] P.V products in flight, [3] the QK^T issuer waiting for K's operands,
 * [4] the P.V issuer waiting for P and V's operands, [5] one split warp's
 * operand preparation, [6] key tiles, [7] cycles from a 128-row tile's start
 * to its output store.  These stages overlap in time.
 * Like the reference's stage-timing build, the clocks perturb the run
 * slightly: read the counters as proportions. */
raya_attn_status raya_attn_forward_timed(const raya_attn_desc* desc, const float* q,
                                         const float* k, const float* v, float* out,
                                         const int32_t* valid_len, void* stream,
                                         int kernel_id, uint64_t* stage_cycles);

/* Synchronises `stream` and returns RAYA_ATTN_ERR_TIMEOUT if any kernel of
 * this library on the current device recorded a bounded-wait timeout since
 * the last call (the record is then cleared), RAYA_ATTN_ERR_CUDA on a CUDA
 * error, else OK. */
raya_attn_status raya_attn_sync_status(void* stream);

/* Failure-detection probe (no reference counterpart): launches one warp that
 * waits on an mbarrier nothing arrives on, through the same bounded wait as
 * the attention kernels, limited to `timeout_cycles` (<= 2^31).  The wait
 * gives up and the kernel returns; the call then reports the recorded
 * timeout exactly as raya_attn_sync_status does (RAYA_ATTN_ERR_TIMEOUT, the
 * record cleared).  No GPU fault, trap or hang is involved. */
raya_attn_status raya_attn_probe_timeout(int64_t timeout_cycles, void* stream);

/* Message of the last error raised on the calling thread (KernelError's
 * Display text for the reference's errors).  Never NULL. */
const char* raya_attn_last_error(void);

/* The last error raised on the calling thread, as data: *kind is its status
 * code, RAYA_ATTN_OK if none; for RAYA_ATTN_ERR_LENGTH, *name is
 * the buffer ("q", "k", "v", "out" or "workspace") and *got / *expected its
 * element count and the count the shape asks for, the fields of
 * KernelError::Length { name, got, expected } (attention.rs:13-18); for other
 * kinds *name is "" and both counts 0.  Any output pointer may be NULL; the
 * name stays valid until the thread's next failing call.  Always returns
 * RAYA_ATTN_OK. */
raya_attn_status raya_attn_last_error_info(int* kind, const char** name, size_t* got, size_t* expected);

/* The kernel that raya_attn_forward, raya_attn_forward_host and
 * raya_attn_forward_ex(RAYA_KERNEL_AUTO) launch for this descriptor, or with
 * packed != 0 the packed entry points, without the rotation (packed = 1) or
 * with it (packed = 2) (a raya_kernel_id, the tiled kernel resolved to its
 * tuned variant).  Host-only: no device work.  No counterpart
 * in the reference, whose caller picks the kernel type itself
 * (crates/raya-kernels/src/attention.rs:113-125). */
raya_attn_status raya_attn_kernel_for(const raya_attn_desc* desc, int packed, int* kernel);

/* Exact algorithmic work of one call: allowed (query < valid, key < valid,
 * mask-allowed) pairs and valid query rows, summed over batch and heads.
 * valid_len is a HOST array or NULL.  FLOPs = 4 * head_dim * pairs. */
raya_attn_status raya_attn_work(const raya_attn_desc* desc, const int32_t* valid_len,
                                uint64_t* pairs, uint64_t* valid_rows);

/* Multi-GPU partition (batch x heads is the shard): the contiguous range
 * [*bh_begin, *bh_end) of flattened batch*heads slices that `rank` of
 * `world` owns, balanced by allowed-pair count.  valid_len is a HOST array or
 * NULL.  Every rank computes the same partition; ranges tile [0, batch*heads). */
raya_attn_status raya_attn_shard(const raya_attn_desc* desc, const int32_t* valid_len,
                                 int world, int rank, int64_t* bh_begin, int64_t* bh_end);

/* Fills DEVICE buffer dst[0..n) with seeded N(0, stddev^2) values:
 * splitmix64 of (seed, stream_id, pair index) -> two 24-bit uniforms ->
 * Box-Muller.  Element i is a function of (seed, stream_id, first_index + i)
 * only, so shards of a larger tensor can be generated independently. */
raya_attn_status raya_attn_fill_normal(float* dst, int64_t n, uint64_t seed,
                                       uint32_t stream_id, int64_t first_index,
                                       float stddev, void* stream);

/* FP32 FFMA throughput probe on the current device: a kernel of dependent-
 * chain-free FFMAs over every SM, timed with CUDA events (best of `reps`).
 * Writes the achieved FFMA rate in TFLOP/s (2 flops per FFMA). */
raya_attn_status raya_attn_ffma_peak(int reps, double* tflops);

/* Library ABI version (RAYA_ATTN_VERSION). */
int raya_attn_version(void);

#ifdef __cplusplus
}
#endif
#endif /* RAYA_ATTN_H */
