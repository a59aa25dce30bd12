// raya_attn.cu — the C ABI of libraya_attn.so (include/raya_attn.h):
// argument validation mirroring raya's `validate`, the host-buffer and
// device-buffer entry points, kernel launch, exact work counts, the
// batch x heads shard partition, the seeded device generator and the FFMA
// throughput probe.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/raya_attn.h"
#include "common.cuh"
#include "rowwise.cuh"
#include "tc16_ws.cuh"
#include "tc32_common.cuh"
#include "tc32_ws.cuh"
#include "tiled64.cuh"

namespace raya {
namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxHeadDim = 256;
constexpr long long kMaxSeq = 1ll << 29;
constexpr long long kDefaultTimeoutCycles = 1ll << 31;  // ~1 s at B200 clocks
// Host-buffer call: chunks through three streams (copies in, kernels, copies
// out).  Each chunk costs ~30 us on the copy-in path; the last chunk's kernel
// and copy out form a tail that shrinks as chunks do.  Time ~ copies + n *
// 30 us + tail / n is least near n = sqrt(bytes / kHostChunkUnit): measured
// on c2 (302 MB in, 101 MB out; copies alone 5.66 ms) 16 equal chunks 6.50
// ms, 8 equal 6.30, 8 with the last two at half size 6.21.
constexpr int kHostStreams = 3;
constexpr int64_t kMaxHostChunks = 128;
constexpr double kHostChunkUnit = 6.0 * (1 << 20);

// The tiled kernel's instantiations: (warps per CTA, K/V stages).
using TiledFn = void (*)(AttnArgs, tiled64::TmaMaps);
struct TiledVariant {
  int id;
  int warps;
  int rows_per_warp;
  int stages;
  TiledFn fn;
  TiledFn timed;  // the same kernel with per-stage clocks
  size_t smem;
};
template <int W, int R, int S, bool PQK, bool PPV>
constexpr TiledVariant variant(int id) {
  return {id, W, R, S, tiled64::tiled64_fwd<W, R, S, PQK, PPV, false>,
          tiled64::tiled64_fwd<W, R, S, PQK, PPV, true>, tiled64::smem_bytes<W, R, S>()};
}
const TiledVariant kTiled[] = {
    variant<4, 32, 1, false, false>(RAYA_KERNEL_TILED64_W4R32),
    variant<4, 16, 1, false, false>(RAYA_KERNEL_TILED64_W4R16),
    variant<4, 16, 1, true, true>(RAYA_KERNEL_TILED64_W4R16_P2),
    variant<4, 32, 1, false, true>(RAYA_KERNEL_TILED64_W4R32_P2)};

// The packed-layout (caller's [b*seq][3][heads][64] -> [b*seq][heads][64])
// instantiations of the two tuned variants, without and with rotary embedding.
struct PackedVariant {
  int id;
  int warps;
  int rows_per_warp;
  TiledFn plain;
  TiledFn rope;
  size_t smem;
};
template <int W, int R, bool PQK, bool PPV>
constexpr PackedVariant packed_variant(int id) {
  return {id, W, R, tiled64::tiled64_fwd<W, R, 1, PQK, PPV, false, tiled64::kPacked, false>,
          tiled64::tiled64_fwd<W, R, 1, PQK, PPV, false, tiled64::kPacked, true>, tiled64::smem_bytes<W, R, 1>()};
}
const PackedVariant kPacked[] = {packed_variant<4, 16, true, true>(RAYA_KERNEL_TILED64_W4R16_P2),
                                 packed_variant<4, 32, false, true>(RAYA_KERNEL_TILED64_W4R32_P2)};

// The tuned choice (measured on B200, profiles/): 64-row CTAs of 16-row warps
// with packed QK^T and PV for short key spans (block <= 64, windows), 128-row
// CTAs of 32-row warps with packed PV for long ones (block >= 128, Full).
int tuned_tiled(const raya_attn_desc* d) {
  const bool long_span = d->mask == RAYA_MASK_FULL || (d->mask == RAYA_MASK_BLOCK && d->block >= 128);
  return long_span ? RAYA_KERNEL_TILED64_W4R32_P2 : RAYA_KERNEL_TILED64_W4R16_P2;
}

// The automatic choice for head_dim 64 (measured on B200 over block 32..256,
// halo 0..2, Window64 and Full).  The two-issuer tensor-core kernel computes
// every key of a 128-row CTA's key span for every row of the CTA; it wins
// for Full, windows of half width >= 64, blocks >= 128, and block masks with
// a halo whose allowed keys per row, (2*halo + 1) * block, are at least half
// of that span.  With halo 0 and blocks below 128 the 64-row tiles of the
// tuned FFMA kernel waste less and win.
constexpr long long kTwoTileMinTiles = 1024;
constexpr long long kTwoTileMinTilesLong = 2048;
int auto_kernel(const raya_attn_desc* d) {
  if (d->head_dim != 64) return RAYA_KERNEL_ROWWISE;
  if (d->mask == RAYA_MASK_FULL) return RAYA_KERNEL_TC32_WS;
  if (d->mask == RAYA_MASK_WINDOW) return d->window >= 64 ? RAYA_KERNEL_TC32_WS : tuned_tiled(d);
  const long long blk = d->block, halo = d->halo;
  const long long tiles = d->batch * d->heads * ((d->seq + tc32::kBM - 1) / tc32::kBM);
  if (blk >= tc32::kBM) {
    // Two tiles per CTA pay off with many tiles (>= ~14 waves of 148 SMs)
    // and key spans of at most 32 key tiles (c5: 138 against 134 TFLOP/s;
    // Block3 at seq 2048 x 8: 147.7 against 141.6); with fewer tiles or
    // longer spans the single-tile form wins (Block3 at seq 8192 x 1: 133.8
    // against 129.3).
    const long long span_keys = (2 * halo + 1) * blk;
    return tiles >= kTwoTileMinTilesLong && span_keys <= 32 * tc32::kBN ? RAYA_KERNEL_TC32_WS2 : RAYA_KERNEL_TC32_WS;
  }
  if (halo == 0) return tuned_tiled(d);
  const long long spanned = (tc32::kBM + blk - 1) / blk + (tc32::kBM % blk != 0 ? 1 : 0);
  const long long span = ((spanned + 2 * halo) * blk + tc32::kBN - 1) / tc32::kBN * tc32::kBN;
  const long long allowed = (2 * halo + 1) * blk;
  if (2 * allowed < span) return tuned_tiled(d);
  // Short key ranges (blocks below 128) and many 128-row tiles (>= ~7 waves
  // of 148 SMs): two tiles per CTA share its launch and set-up (c2, c3-b64,
  // c4: +1.5-2.6%; with fewer tiles the halved CTA count costs more).
  return tiles >= kTwoTileMinTiles ? RAYA_KERNEL_TC32_WS2 : RAYA_KERNEL_TC32_WS;
}

// The packed entry points' kernel: the two-issuer tensor-core kernel with the
// packed layout where the automatic choice is a tensor-core kernel, else the
// tuned tiled kernel.  Its two-tile form where that is the choice (two tiles
// per CTA in this layout), except with the rotation (whose two-tile form
// spills registers and measured slower).
int packed_kernel(const raya_attn_desc* d, bool rope) {
  const int id = auto_kernel(d);
  if (id == RAYA_KERNEL_TC32_WS2 && !rope) return id;
  return id == RAYA_KERNEL_TC32_WS || id == RAYA_KERNEL_TC32_WS2 ? RAYA_KERNEL_TC32_WS : tuned_tiled(d);
}

// Device status word: bit 0 = a bounded wait gave up.  One per device that
// loads the library; its device address is looked up once per device.
__device__ int g_status;

thread_local std::string t_error = "no error";
// The last error as data (raya_attn_last_error_info): its status, and for
// RAYA_ATTN_ERR_LENGTH the buffer name and the two element counts.
struct ErrorInfo {
  int kind = RAYA_ATTN_OK;
  std::string name;
  size_t got = 0, expected = 0;
};
thread_local ErrorInfo t_info;

// cuTensorMapEncodeTiled, fetched once from the driver through the runtime
// (no libcuda link dependency).
std::once_flag g_encode_once;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

raya_attn_status fail(raya_attn_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_error = buf;
  t_info = ErrorInfo{};
  t_info.kind = st;
  return st;
}

// KernelError::Length { name, got, expected } with its Display text
// (attention.rs:13-18, 159-168).
raya_attn_status fail_length(const char* name, size_t got, size_t expected) {
  fail(RAYA_ATTN_ERR_LENGTH, "buffer `%s` has length %zu, expected %zu", name, got, expected);
  t_info.name = name;
  t_info.got = got;
  t_info.expected = expected;
  return RAYA_ATTN_ERR_LENGTH;
}

raya_attn_status cuda_fail(cudaError_t e, const char* what) {
  return fail(RAYA_ATTN_ERR_CUDA, "cuda: %s: %s", what, cudaGetErrorString(e));
}

// Per-device state: status-word address, kernel attributes, staging buffers
// of the host-buffer entry point.
struct DeviceCtx {
  std::mutex mu;
  bool ready = false;
  int* status = nullptr;
  int sms = 0;
  cudaStream_t streams[kHostStreams] = {};  // host-buffer call: copies in, kernels, copies out
  cudaEvent_t valid_ready = nullptr;
  cudaEvent_t chunk_in[kMaxHostChunks] = {};    // chunk c's inputs are on the device
  cudaEvent_t chunk_done[kMaxHostChunks] = {};  // chunk c's output is written
  float* buf[4] = {nullptr, nullptr, nullptr, nullptr};  // q, k, v, out
  size_t cap = 0;                                        // floats per buffer
  int32_t* dvalid = nullptr;                             // valid length per slice
  size_t vcap = 0;
  std::vector<int32_t> slice_valid;
};
DeviceCtx g_ctx[kMaxDevices];

raya_attn_status ensure_ready(int dev, DeviceCtx** out) {
  if (dev < 0 || dev >= kMaxDevices) return fail(RAYA_ATTN_ERR_CUDA, "cuda: device %d out of range", dev);
  DeviceCtx& c = g_ctx[dev];
  std::lock_guard<std::mutex> lock(c.mu);
  if (!c.ready) {
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&c.status), g_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    e = cudaDeviceGetAttribute(&c.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SMs)");
    for (const TiledVariant& tv : kTiled) {
      for (auto fn : {tv.fn, tv.timed}) {
        e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(tv.smem));
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tiled64 smem)");
      }
    }
    for (auto fn : {tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 1>, tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 2>,
                    tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 4>,
                    tc32::tc32_ws_fwd<tiled64::kPacked, false, 1>, tc32::tc32_ws_fwd<tiled64::kPacked, true, 1>,
                    tc32::tc32_ws_fwd<tiled64::kPacked, false, 2>, tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 1, true>,
                    tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 2, true>,
                    tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 4, true>}) {
      e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(tc32::pipe_smem_bytes()));
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tc32_ws smem)");
    }
    for (auto fn : {tc16::tc16_ws_fwd<tiled64::kHeadMajor>, tc16::tc16_ws_fwd<tiled64::kHeadMajor, true>}) {
      e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(tc16::smem_bytes()));
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tc16_ws smem)");
    }
    for (const PackedVariant& pv : kPacked) {
      for (auto fn : {pv.plain, pv.rope}) {
        e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(pv.smem));
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(packed smem)");
      }
    }
    c.ready = true;
  }
  *out = &c;
  return RAYA_ATTN_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
raya_attn_status load_encoder() {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return fail(RAYA_ATTN_ERR_CUDA, "cuda: cuTensorMapEncodeTiled is unavailable");
  return RAYA_ATTN_OK;
}

// A 2-D tensor map over a [rows][64] fp32 tensor with boxes of
// [box_rows][32 floats], zero fill out of bounds; 128-byte swizzle of
// 16-byte chunks unless another swizzle is asked for.
raya_attn_status encode_rows64(CUtensorMap* map, const float* base, uint64_t rows, uint32_t box_rows,
                               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  raya_attn_status st = load_encoder();
  if (st != RAYA_ATTN_OK) return st;
  const cuuint64_t gdim[2] = {64, rows};
  const cuuint64_t gstride[1] = {64 * sizeof(float)};
  const cuuint32_t box[2] = {32, box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), gdim,
                              gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(RAYA_ATTN_ERR_CUDA, "cuda: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return RAYA_ATTN_OK;
}

// A 3-D tensor map over a [slices][seq][64] fp32 tensor with boxes of
// [1][64 rows][32 floats], 128-byte swizzle: a store clips rows past seq.
raya_attn_status encode_slices3d(CUtensorMap* map, float* base, uint64_t slices, uint64_t seq) {
  raya_attn_status st = load_encoder();
  if (st != RAYA_ATTN_OK) return st;
  const cuuint64_t gdim[3] = {64, seq, slices};
  const cuuint64_t gstride[2] = {64 * sizeof(float), seq * 64 * sizeof(float)};
  const cuuint32_t box[3] = {32, 64, 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, gdim, gstride, box, estride,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(RAYA_ATTN_ERR_CUDA, "cuda: cuTensorMapEncodeTiled (slices) failed (%d)", static_cast<int>(r));
  return RAYA_ATTN_OK;
}

// A 4-D tensor map over the packed projection [rows][3][heads][64] fp32
// (rows = batch*seq) with boxes of [box_rows][1][1][32 floats]: one head of
// one of q/k/v at box_rows consecutive positions, 128-byte swizzle.
raya_attn_status encode_packed(CUtensorMap* map, const float* base, uint64_t rows, uint64_t heads,
                               uint32_t box_rows, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  raya_attn_status st = load_encoder();
  if (st != RAYA_ATTN_OK) return st;
  const cuuint64_t gdim[4] = {64, heads, 3, rows};
  const cuuint64_t gstride[3] = {64 * sizeof(float), heads * 64 * sizeof(float), 3 * heads * 64 * sizeof(float)};
  const cuuint32_t box[4] = {32, 1, 1, box_rows};
  const cuuint32_t estride[4] = {1, 1, 1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), gdim, gstride,
                              box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(RAYA_ATTN_ERR_CUDA, "cuda: cuTensorMapEncodeTiled (packed) failed (%d)", static_cast<int>(r));
  return RAYA_ATTN_OK;
}

// A 4-D tensor map over the context tensor [batch][seq][heads][64] with boxes
// of [1][64 rows][1][32 floats], 128-byte swizzle: a store clips rows past seq.
raya_attn_status encode_context(CUtensorMap* map, float* base, uint64_t batch, uint64_t seq, uint64_t heads) {
  raya_attn_status st = load_encoder();
  if (st != RAYA_ATTN_OK) return st;
  const cuuint64_t gdim[4] = {64, heads, seq, batch};
  const cuuint64_t gstride[3] = {64 * sizeof(float), heads * 64 * sizeof(float), seq * heads * 64 * sizeof(float)};
  const cuuint32_t box[4] = {32, 1, 64, 1};
  const cuuint32_t estride[4] = {1, 1, 1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, gdim, gstride, box, estride,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(RAYA_ATTN_ERR_CUDA, "cuda: cuTensorMapEncodeTiled (context) failed (%d)", static_cast<int>(r));
  return RAYA_ATTN_OK;
}

// Shape checks of validate (attention.rs:136-158), in the reference's order,
// plus this library's own limits.
raya_attn_status check_shape(const raya_attn_desc* d) {
  if (!d) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: null descriptor");
  if (d->heads <= 0 || d->head_dim <= 0)
    return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: heads and head_dim must be at least 1");
  if (d->head_dim % 8 != 0)
    return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: head_dim %lld is not a multiple of 8",
                static_cast<long long>(d->head_dim));
  if (d->batch <= 0) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: batch must be at least 1");
  if (d->seq < 0) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: seq %lld is negative",
                              static_cast<long long>(d->seq));
  if (d->mask == RAYA_MASK_BLOCK) {
    if (d->block < 1)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: block %lld (must be at least 1)",
                  static_cast<long long>(d->block));
    if (d->halo < 0) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: halo %d is negative", d->halo);
  } else if (d->mask == RAYA_MASK_WINDOW) {
    if (d->window < 0)
      return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: window %lld is negative",
                  static_cast<long long>(d->window));
  } else if (d->mask != RAYA_MASK_FULL) {
    return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: mask kind %d", d->mask);
  }
  if (d->head_dim > kMaxHeadDim)
    return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: head_dim %lld (at most %d)",
                static_cast<long long>(d->head_dim), kMaxHeadDim);
  if (d->seq >= kMaxSeq)
    return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: seq %lld (below %lld)",
                static_cast<long long>(d->seq), kMaxSeq);
  if (!std::isfinite(d->scale)) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: scale is not finite");
  return RAYA_ATTN_OK;
}

raya_attn_status check_valid(const raya_attn_desc* d, const int32_t* valid_len) {
  if (!valid_len) return RAYA_ATTN_OK;
  for (int64_t b = 0; b < d->batch; ++b) {
    if (valid_len[b] < 0)
      return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: valid_len %d is negative", valid_len[b]);
    if (valid_len[b] > d->seq)  // attention.rs:147-152
      return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: valid_len %d exceeds seq %lld",
                  valid_len[b], static_cast<long long>(d->seq));
  }
  return RAYA_ATTN_OK;
}

size_t numel(const raya_attn_desc* d) {
  return static_cast<size_t>(d->batch) * d->heads * d->seq * d->head_dim;
}

AttnArgs make_args(const raya_attn_desc* d, const float* q, const float* k, const float* v,
                   float* out, const int32_t* valid_len, int* status) {
  AttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.out = out;
  a.valid_len = valid_len;
  a.status = status;
  a.batch = static_cast<int>(d->batch);
  a.heads = static_cast<int>(d->heads);
  a.seq = static_cast<int>(d->seq);
  a.head_dim = static_cast<int>(d->head_dim);
  a.mask = d->mask;
  // Clamp the mask parameters to the sequence (same key ranges, no int32
  // overflow): a block >= seq puts every row in block 0, a halo past the
  // block count or a window past seq allows everything.
  const long long seq = std::max<long long>(d->seq, 1);
  a.block = static_cast<int>(std::min<long long>(std::max<long long>(d->block, 1), seq));
  const long long nblocks = (seq + a.block - 1) / a.block;
  a.halo = static_cast<int>(std::min<long long>(std::max(d->halo, 0), nblocks));
  a.window = static_cast<int>(std::min<long long>(std::max<long long>(d->window, 0), seq));
  a.qscale = static_cast<float>(static_cast<double>(d->scale) * 1.4426950408889634);
  a.row_tiles = 1;
  a.timeout_cycles = kDefaultTimeoutCycles;
  return a;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launches on the current device, whose context `ctx` is ready.
raya_attn_status launch_on(DeviceCtx* ctx, const raya_attn_desc* d, const float* q, const float* k,
                           const float* v, float* out, const int32_t* valid_len, cudaStream_t stream,
                           int kernel_id, unsigned long long* stage_cycles = nullptr) {
  if (d->seq == 0) return RAYA_ATTN_OK;  // nothing to write (tiled/mod.rs:79-81)
  if (!q || !k || !v || !out)
    return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: tensors must be 16-byte aligned");
  cudaError_t e;
  AttnArgs a = make_args(d, q, k, v, out, valid_len, ctx->status);
  a.stage_cycles = stage_cycles;

  if (kernel_id == RAYA_KERNEL_AUTO) kernel_id = auto_kernel(d);
  if (kernel_id == RAYA_KERNEL_TILED64) kernel_id = tuned_tiled(d);
  const TiledVariant* tv = nullptr;
  for (const TiledVariant& t : kTiled)
    if (t.id == kernel_id) tv = &t;
  if (tv) {
    if (d->head_dim != 64)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: the tiled kernel needs head_dim 64, got %lld",
                  static_cast<long long>(d->head_dim));
    const int bm = tv->warps * tv->rows_per_warp;
    a.row_tiles = static_cast<int>((d->seq + bm - 1) / bm);
    const long long grid = static_cast<long long>(d->batch) * d->heads * a.row_tiles;
    if (grid > 0x7fffffffll)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: %lld CTAs exceed the grid limit", grid);
    tiled64::TmaMaps maps;
    const uint64_t rows = static_cast<uint64_t>(d->batch) * d->heads * d->seq;
    raya_attn_status st = encode_rows64(&maps.q, q, rows, static_cast<uint32_t>(bm));
    if (st == RAYA_ATTN_OK) st = encode_rows64(&maps.k, k, rows, tiled64::kBN);
    if (st == RAYA_ATTN_OK) st = encode_rows64(&maps.v, v, rows, tiled64::kBN);
    if (st != RAYA_ATTN_OK) return st;
    auto fn = stage_cycles ? tv->timed : tv->fn;
    fn<<<static_cast<unsigned>(grid), tv->warps * 32, tv->smem, stream>>>(a, maps);
  } else if (kernel_id == RAYA_KERNEL_TC32_WS || kernel_id == RAYA_KERNEL_TC32_WS2) {
    if (d->head_dim != 64)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: the tensor-core kernel needs head_dim 64, got %lld",
                  static_cast<long long>(d->head_dim));
    a.row_tiles = static_cast<int>((d->seq + tc32::kBM - 1) / tc32::kBM);
    const long long grid = static_cast<long long>(d->batch) * d->heads * a.row_tiles;
    if (grid > 0x7fffffffll)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: %lld CTAs exceed the grid limit", grid);
    tc32::PipeMaps maps;
    const uint64_t rows = static_cast<uint64_t>(d->batch) * d->heads * d->seq;
    raya_attn_status st = encode_rows64(&maps.k, k, rows, tc32::kBN);
    if (st == RAYA_ATTN_OK) st = encode_rows64(&maps.v, v, rows, tc32::kBN, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (st == RAYA_ATTN_OK)
      st = encode_slices3d(&maps.o, out, static_cast<uint64_t>(d->batch) * d->heads, static_cast<uint64_t>(d->seq));
    if (st == RAYA_ATTN_OK) st = encode_rows64(&maps.q, q, rows, tc32::kBN);
    if (st != RAYA_ATTN_OK) return st;
    if (rows > 0x7fffffffull)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: %llu rows exceed the tensor-map row limit",
                  static_cast<unsigned long long>(rows));
    {
      // UNITS row tiles per CTA: 1 (kernel 34); for kernel 37 4 where a slice
      // is four row tiles, or a multiple of four with blocks of 128 keys or
      // more and at least 16384 row tiles in all (c5: +0.7% over 2, same box;
      // c3 at 3072 row tiles -3 to -4%: a partial last wave of 768 CTAs;
      // c2's 64-key blocks -1.2%), else 2; the stage-timing build where asked.
      const bool four = a.row_tiles == 4 || (a.row_tiles % 4 == 0 && d->mask == RAYA_MASK_BLOCK &&
                                             d->block >= 128 && grid >= 16384);
      const int units = kernel_id == RAYA_KERNEL_TC32_WS ? 1 : four ? 4 : 2;
      using WsFn = void (*)(AttnArgs, tc32::PipeMaps);
      WsFn fn = nullptr;
      if (units == 1)
        fn = stage_cycles ? tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 1, true>
                          : tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 1>;
      else if (units == 4)
        fn = stage_cycles ? tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 4, true>
                          : tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 4>;
      else
        fn = stage_cycles ? tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 2, true>
                          : tc32::tc32_ws_fwd<tiled64::kHeadMajor, false, 2>;
      fn<<<static_cast<unsigned>((grid + units - 1) / units), tc32::kWsThreads, tc32::pipe_smem_bytes(), stream>>>(
          a, maps);
    }
  } else if (kernel_id == RAYA_KERNEL_TC16_WS || kernel_id == RAYA_KERNEL_TC16_WS2) {
    if (d->head_dim != 64)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: the tensor-core kernel needs head_dim 64, got %lld",
                  static_cast<long long>(d->head_dim));
    a.row_tiles = static_cast<int>((d->seq + tc16::kBM - 1) / tc16::kBM);
    const long long grid = static_cast<long long>(d->batch) * d->heads * a.row_tiles;
    if (grid > 0x7fffffffll)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: %lld CTAs exceed the grid limit", grid);
    const uint64_t rows = static_cast<uint64_t>(d->batch) * d->heads * d->seq;
    if (rows > 0x7fffffffull)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: %llu rows exceed the tensor-map row limit",
                  static_cast<unsigned long long>(rows));
    tc32::PipeMaps maps;  // k, v and q all [64 rows][32] boxes under the 128-byte swizzle of 16-byte chunks
    raya_attn_status st = encode_rows64(&maps.k, k, rows, tc16::kBN);
    if (st == RAYA_ATTN_OK) st = encode_rows64(&maps.v, v, rows, tc16::kBN);
    if (st == RAYA_ATTN_OK)
      st = encode_slices3d(&maps.o, out, static_cast<uint64_t>(d->batch) * d->heads, static_cast<uint64_t>(d->seq));
    if (st == RAYA_ATTN_OK) st = encode_rows64(&maps.q, q, rows, tc16::kBN);
    if (st != RAYA_ATTN_OK) return st;
    // kernel 40: one unit (128-row tile) per CTA; kernel 41: persistent, one
    // CTA per SM walking its units.
    const long long ctas = kernel_id == RAYA_KERNEL_TC16_WS ? grid : std::min<long long>(grid, ctx->sms);
    auto fn = stage_cycles ? tc16::tc16_ws_fwd<tiled64::kHeadMajor, true>
                           : tc16::tc16_ws_fwd<tiled64::kHeadMajor>;
    fn<<<static_cast<unsigned>(std::max<long long>(ctas, 1)), tc16::kThreads, tc16::smem_bytes(), stream>>>(a, maps);
  } else if (stage_cycles) {
    return fail(RAYA_ATTN_ERR_UNSUPPORTED,
                "unsupported: stage timing needs a tiled kernel or the two-issuer tensor-core kernel");
  } else if (kernel_id == RAYA_KERNEL_ROWWISE) {
    const long long rows = static_cast<long long>(d->batch) * d->heads * d->seq;
    const long long want = (rows + rowwise::kWarps - 1) / rowwise::kWarps;
    const long long grid = std::min<long long>(want, static_cast<long long>(ctx->sms) * 16);
    rowwise::rowwise_fwd<<<static_cast<unsigned>(grid), rowwise::kThreads, 0, stream>>>(a);
  } else {
    return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: kernel id %d", kernel_id);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return RAYA_ATTN_OK;
}

raya_attn_status launch(const raya_attn_desc* d, const float* q, const float* k, const float* v,
                        float* out, const int32_t* valid_len, cudaStream_t stream, int kernel_id,
                        unsigned long long* stage_cycles = nullptr) {
  if (d->seq == 0) return RAYA_ATTN_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  DeviceCtx* ctx = nullptr;
  raya_attn_status st = ensure_ready(dev, &ctx);
  if (st != RAYA_ATTN_OK) return st;
  return launch_on(ctx, d, q, k, v, out, valid_len, stream, kernel_id, stage_cycles);
}

uint64_t row_pairs(const AttnArgs& a, int valid, int i) {
  int lo, hi;
  key_range(a, i, valid, lo, hi);
  return hi > lo ? static_cast<uint64_t>(hi - lo) : 0;
}

// Allowed pairs of one (batch entry, head) slice with `valid` valid rows.
uint64_t slice_pairs(const AttnArgs& a, int valid) {
  uint64_t p = 0;
  for (int i = 0; i < valid; ++i) p += row_pairs(a, valid, i);
  return p;
}

// splitmix64 (Steele, Lea, Flood 2014) — the generator's mixing function.
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__global__ void fill_normal_kernel(float* dst, long long n, uint64_t key, long long first,
                                   float stddev) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long idx = first + i;
    const uint64_t h = splitmix64(key + static_cast<uint64_t>(idx >> 1));
    const float u1 = (static_cast<float>(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (static_cast<float>(h & 0xFFFFFFull) + 0.5f) * (1.0f / 16777216.0f);
    const float r = sqrtf(-2.0f * logf(u1));
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    dst[i] = stddev * r * ((idx & 1) ? sn : cs);
  }
}

// FFMA throughput probe: 16 independent FMA chains per thread.
__global__ void __launch_bounds__(256) ffma_probe_kernel(float* sink, int iters, float mul, float add) {
  float x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = 1e-3f * threadIdx.x + static_cast<float>(i);
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = fmaf(x[i], mul, add);
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) s += x[i];
  if (s == 1234.5f) sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

// raya's rotary table (ops.rs:118-131): cs[pos][i] = (cos, sin) of
// angle = pos * inv_freq[i] in f32, inv_freq computed on the host with the C
// library's powf exactly as the reference computes it.
struct RopeFreq {
  float inv_freq[32];
};
// 64-bit element count and a grid-stride loop: seq * 32 passes 2^31 from
// seq = 2^26 on, below the library's sequence limit.
__global__ void rope_table_kernel(float2* cs, long long seq, const __grid_constant__ RopeFreq f) {
  const long long n = seq * 32;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < n;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float angle = __fmul_rn(static_cast<float>(idx >> 5), f.inv_freq[idx & 31]);
    cs[idx] = make_float2(cosf(angle), sinf(angle));
  }
}

// The rotary table's launch: enough CTAs for one element each, at most 32
// per SM (the loop strides over the rest).
raya_attn_status launch_rope_table(float2* cs, int64_t seq, const RopeFreq& f, int sms, cudaStream_t s) {
  const long long n = static_cast<long long>(seq) * 32;
  const long long blocks = std::max<long long>(1, std::min<long long>((n + 255) / 256, static_cast<long long>(sms) * 32));
  rope_table_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(cs, seq, f);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "rope table launch");
  return RAYA_ATTN_OK;
}

// Failure-detection probe: one warp waits on an mbarrier that nothing ever
// arrives on, through the same bounded wait the attention kernels use, with a
// short limit.  The wait gives up, records bit 0 of the status word and the
// kernel returns; the context stays usable.
__global__ void timeout_probe_kernel(int* status, long long timeout_cycles) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  mbar_wait_bounded(&bar, 0, &abort_flag, status, timeout_cycles);
}

// ---- Allocation-free rotary table ----
// Some callers cannot allocate device memory for the rotary table that
// raya_attn_forward_packed takes as a workspace: a serving runtime that owns
// all of the GPU's memory through its own pool, a binding that only receives
// raw device pointers from its host and holds no allocator, or a
// latency-bound loop in which cudaMalloc (which may synchronise the device)
// must not run.  raya_attn_forward_packed_noalloc keeps the table in this
// file-scope array instead: kStaticRopeMaxSeq positions x 32 (cos, sin)
// pairs = 2 MiB, held by every GPU that loads the library until the process
// exits.
constexpr int kStaticRopeMaxSeq = 8192;
static __device__ __align__(256) float2 g_rope_static[kStaticRopeMaxSeq * 32];

// The array's device address on each device, looked up once per device with
// that device current (host code cannot use the symbol itself: in host code
// it names a host-side stand-in, not device memory).
std::mutex g_rope_static_mu;
float2* g_rope_static_ptr[kMaxDevices] = {};

raya_attn_status rope_static_table(int dev, float2** out) {
  if (dev < 0 || dev >= kMaxDevices) return fail(RAYA_ATTN_ERR_CUDA, "cuda: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_rope_static_mu);
  if (!g_rope_static_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_rope_static);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(rotary table)");
    g_rope_static_ptr[dev] = static_cast<float2*>(p);
  }
  *out = g_rope_static_ptr[dev];
  return RAYA_ATTN_OK;
}

// One valid length per (batch, head) slice, so that any range of slices is
// an independent call (batch = #slices, heads = 1).
std::vector<int32_t> slice_valid_lengths(const raya_attn_desc* d, const int32_t* valid_len) {
  const int64_t nbh = d->batch * d->heads;
  std::vector<int32_t> sv(static_cast<size_t>(nbh));
  for (int64_t bh = 0; bh < nbh; ++bh)
    sv[bh] = valid_len ? valid_len[bh / d->heads] : static_cast<int32_t>(d->seq);
  return sv;
}

// The slices [bh0, bh1) of a validated call, run through one device:
// host inputs q/k/v (whole tensors; the range is read at its offset), host
// output `out` (or NULL), and optionally a DEVICE output `gather` of the
// whole tensor on device `gather_dev` that receives this range (written by
// the kernel itself when gather_dev is this device, else by peer copies).
struct HostJob {
  const raya_attn_desc* desc;
  const int32_t* slice_valid;  // [batch*heads]
  int64_t bh0, bh1;
  const float *q, *k, *v;
  float* out;
  float* gather;
  int gather_dev;
};

raya_attn_status host_pipeline(int device, const HostJob& job) {
  const raya_attn_desc* desc = job.desc;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  DeviceCtx* ctx = nullptr;
  raya_attn_status st = ensure_ready(device, &ctx);
  if (st != RAYA_ATTN_OK) return st;
  const bool direct = job.gather && job.gather_dev == device;  // the kernel writes into the gather buffer
  const bool peer = job.gather && !direct;
  if (peer) {
    int can = 0;
    e = cudaDeviceCanAccessPeer(&can, device, job.gather_dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceCanAccessPeer");
    if (can) {
      e = cudaDeviceEnablePeerAccess(job.gather_dev, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();  // already on: not an error
      } else if (e != cudaSuccess) {
        return cuda_fail(e, "cudaDeviceEnablePeerAccess");
      }
    }
  }
  std::lock_guard<std::mutex> lock(ctx->mu);  // one host call per device at a time
  if (!ctx->streams[0]) {
    for (auto& sm : ctx->streams) {
      e = cudaStreamCreateWithFlags(&sm, cudaStreamNonBlocking);
      if (e != cudaSuccess) return cuda_fail(e, "cudaStreamCreate");
    }
    e = cudaEventCreateWithFlags(&ctx->valid_ready, cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
    for (int64_t c = 0; c < kMaxHostChunks; ++c) {
      e = cudaEventCreateWithFlags(&ctx->chunk_in[c], cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->chunk_done[c], cudaEventDisableTiming);
      if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
    }
  }
  const int64_t nbh = job.bh1 - job.bh0;
  const size_t slice = static_cast<size_t>(desc->seq) * desc->head_dim;
  const size_t n = static_cast<size_t>(nbh) * slice;
  if (ctx->cap < n) {
    for (auto& p : ctx->buf) {
      if (p) cudaFree(p);
      p = nullptr;
    }
    ctx->cap = 0;
    for (auto& p : ctx->buf) {
      e = cudaMalloc(&p, n * sizeof(float));
      if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(staging)");
    }
    ctx->cap = n;
  }
  if (ctx->vcap < static_cast<size_t>(nbh)) {
    if (ctx->dvalid) cudaFree(ctx->dvalid);
    ctx->dvalid = nullptr;
    ctx->vcap = 0;
    e = cudaMalloc(&ctx->dvalid, nbh * sizeof(int32_t));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(valid_len)");
    ctx->vcap = nbh;
  }
  ctx->slice_valid.assign(job.slice_valid + job.bh0, job.slice_valid + job.bh1);
  e = cudaMemcpyAsync(ctx->dvalid, ctx->slice_valid.data(), nbh * sizeof(int32_t), cudaMemcpyHostToDevice,
                      ctx->streams[0]);
  if (e != cudaSuccess) return cuda_fail(e, "copy valid_len to device");
  e = cudaEventRecord(ctx->valid_ready, ctx->streams[0]);
  if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");

  // Pipeline over chunks of slices: stream 0 copies every chunk in, back to
  // back; stream 1 runs chunk c's kernel once its inputs are in; stream 2
  // copies chunk c out once its kernel is done.  The host-to-device copy
  // engine (the bound: 3/4 of the bytes) never waits for a kernel or an
  // outgoing copy, which one stream per chunk made it do.
  const size_t bytes_total = 4 * n * sizeof(float);
  const int64_t nchunks = std::max<int64_t>(
      1, std::min<int64_t>({nbh, kMaxHostChunks,
                            static_cast<int64_t>(std::llround(std::sqrt(static_cast<double>(bytes_total) / kHostChunkUnit)))}));
  const float* src[3] = {job.q, job.k, job.v};
  for (int64_t c = 0; c < nchunks; ++c) {
    // Chunk c spans weight 2, the last two (with 3+ chunks) weight 1: a shorter tail.
    auto cum = [&](int64_t i) {
      const int64_t big = nchunks >= 3 ? nchunks - 2 : nchunks;
      return 2 * std::min(i, big) + std::max<int64_t>(0, i - big);
    };
    const int64_t wt = cum(nchunks);
    const int64_t c0 = nbh * cum(c) / wt, c1 = nbh * cum(c + 1) / wt;  // slices of this range
    if (c1 <= c0) continue;
    cudaStream_t s_in = ctx->streams[0], s_run = ctx->streams[1], s_out = ctx->streams[2];
    const size_t off = static_cast<size_t>(c0) * slice;              // in the staging buffers
    const size_t abs = static_cast<size_t>(job.bh0 + c0) * slice;    // in the caller's tensors
    const size_t cnt = static_cast<size_t>(c1 - c0) * slice;
    // Only the valid rows of each slice go in: no kernel reads q, k or v rows
    // at or past valid_len (keys there are masked, V rows there are zeroed in
    // shared memory, q rows there are read as zero), so whatever the staging
    // buffers hold there does not reach the output.  One 2-D copy per run of
    // slices with the same valid length (rows of `valid` * head_dim floats,
    // pitch seq * head_dim).
    for (int64_t r0 = c0; r0 < c1;) {
      const int32_t vl = ctx->slice_valid[r0];
      int64_t r1 = r0 + 1;
      while (r1 < c1 && ctx->slice_valid[r1] == vl) ++r1;
      if (vl > 0) {
        const size_t pitch = slice * sizeof(float);
        const size_t width = static_cast<size_t>(vl) * desc->head_dim * sizeof(float);
        const size_t o = static_cast<size_t>(r0) * slice;
        const size_t oa = static_cast<size_t>(job.bh0 + r0) * slice;
        for (int i = 0; i < 3; ++i) {
          e = cudaMemcpy2DAsync(ctx->buf[i] + o, pitch, src[i] + oa, pitch, width, static_cast<size_t>(r1 - r0),
                                cudaMemcpyHostToDevice, s_in);
          if (e != cudaSuccess) return cuda_fail(e, "copy inputs to device");
        }
      }
      r0 = r1;
    }
    e = cudaEventRecord(ctx->chunk_in[c], s_in);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s_run, ctx->chunk_in[c], 0);
    if (e == cudaSuccess && c == 0) e = cudaStreamWaitEvent(s_run, ctx->valid_ready, 0);
    if (e != cudaSuccess) return cuda_fail(e, "chunk events");
    raya_attn_desc sub = *desc;
    sub.batch = c1 - c0;
    sub.heads = 1;
    float* kout = direct ? job.gather + abs : ctx->buf[3] + off;
    st = launch_on(ctx, &sub, ctx->buf[0] + off, ctx->buf[1] + off, ctx->buf[2] + off, kout, ctx->dvalid + c0,
                   s_run, RAYA_KERNEL_AUTO);
    if (st != RAYA_ATTN_OK) return st;
    e = cudaEventRecord(ctx->chunk_done[c], s_run);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s_out, ctx->chunk_done[c], 0);
    if (e != cudaSuccess) return cuda_fail(e, "chunk events");
    if (job.out) {
      e = cudaMemcpyAsync(job.out + abs, kout, cnt * sizeof(float), cudaMemcpyDeviceToHost, s_out);
      if (e != cudaSuccess) return cuda_fail(e, "copy out to host");
    }
    if (peer) {
      e = cudaMemcpyPeerAsync(job.gather + abs, job.gather_dev, kout, device, cnt * sizeof(float), s_out);
      if (e != cudaSuccess) return cuda_fail(e, "peer copy to the gather buffer");
    }
  }
  for (auto& sm : ctx->streams) {
    e = cudaStreamSynchronize(sm);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  }
  int flag = 0;
  e = cudaMemcpy(&flag, ctx->status, sizeof flag, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  if (flag != 0) {
    const int zero = 0;
    cudaMemcpy(ctx->status, &zero, sizeof zero, cudaMemcpyHostToDevice);
    return fail(RAYA_ATTN_ERR_TIMEOUT, "timeout: a device-side wait gave up (status 0x%x)", flag);
  }
  return RAYA_ATTN_OK;
}

}  // namespace
}  // namespace raya

using namespace raya;

extern "C" {

int raya_attn_version(void) { return RAYA_ATTN_VERSION; }

const char* raya_attn_last_error(void) { return t_error.c_str(); }

raya_attn_status raya_attn_last_error_info(int* kind, const char** name, size_t* got, size_t* expected) {
  if (kind) *kind = t_info.kind;
  if (name) *name = t_info.name.c_str();
  if (got) *got = t_info.got;
  if (expected) *expected = t_info.expected;
  return RAYA_ATTN_OK;
}

raya_attn_status raya_attn_validate(const raya_attn_desc* desc, const int32_t* valid_len,
                                    size_t q_len, size_t k_len, size_t v_len, size_t out_len) {
  raya_attn_status st = check_shape(desc);
  if (st != RAYA_ATTN_OK) return st;
  st = check_valid(desc, valid_len);
  if (st != RAYA_ATTN_OK) return st;
  const size_t expected = numel(desc);
  const struct { const char* name; size_t got; } bufs[4] = {
      {"q", q_len}, {"k", k_len}, {"v", v_len}, {"out", out_len}};
  for (const auto& b : bufs)  // attention.rs:159-168
    if (b.got != expected) return fail_length(b.name, b.got, expected);
  return RAYA_ATTN_OK;
}

raya_attn_status raya_attn_forward_ex(const raya_attn_desc* desc, const float* q, const float* k,
                                      const float* v, float* out, const int32_t* valid_len,
                                      void* stream, int kernel_id) {
  raya_attn_status st = check_shape(desc);
  if (st != RAYA_ATTN_OK) return st;
  return launch(desc, q, k, v, out, valid_len, static_cast<cudaStream_t>(stream), kernel_id);
}

raya_attn_status raya_attn_forward(const raya_attn_desc* desc, const float* q, const float* k,
                                   const float* v, float* out, const int32_t* valid_len,
                                   void* stream) {
  return raya_attn_forward_ex(desc, q, k, v, out, valid_len, stream, RAYA_KERNEL_AUTO);
}

raya_attn_status raya_attn_forward_timed(const raya_attn_desc* desc, const float* q, const float* k,
                                         const float* v, float* out, const int32_t* valid_len,
                                         void* stream, int kernel_id, uint64_t* stage_cycles) {
  raya_attn_status st = check_shape(desc);
  if (st != RAYA_ATTN_OK) return st;
  if (!stage_cycles) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: null stage counter buffer");
  return launch(desc, q, k, v, out, valid_len, static_cast<cudaStream_t>(stream), kernel_id,
                reinterpret_cast<unsigned long long*>(stage_cycles));
}

// The packed layout's attention launch (rope_cs: the (cos, sin) table, or
// NULL for no rotation), shared by both packed entry points.
raya_attn_status launch_packed(DeviceCtx* ctx_dev, const raya_attn_desc* desc, const float* qkv, float* ctx,
                               const int32_t* valid_len, const float* rope_cs, cudaStream_t s) {
  const bool rope = rope_cs != nullptr;
  AttnArgs a = make_args(desc, qkv, qkv, qkv, ctx, valid_len, ctx_dev->status);
  a.rope_cs = rope_cs;
  const uint64_t rows = static_cast<uint64_t>(desc->batch) * desc->seq;
  raya_attn_status st;
  const int pk = packed_kernel(desc, rope);
  if (pk == RAYA_KERNEL_TC32_WS || pk == RAYA_KERNEL_TC32_WS2) {
    a.row_tiles = static_cast<int>((desc->seq + tc32::kBM - 1) / tc32::kBM);
    const long long grid = static_cast<long long>(desc->batch) * desc->heads * a.row_tiles;
    if (grid > 0x7fffffffll)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: %lld CTAs exceed the grid limit", grid);
    if (rows > 0x7fffffffull)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: %llu rows exceed the tensor-map row limit",
                  static_cast<unsigned long long>(rows));
    tc32::PipeMaps maps;
    st = encode_packed(&maps.q, qkv, rows, desc->heads, tc32::kBN);
    if (st == RAYA_ATTN_OK)
      st = encode_packed(&maps.v, qkv, rows, desc->heads, tc32::kBN, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (st == RAYA_ATTN_OK)
      st = encode_context(&maps.o, ctx, static_cast<uint64_t>(desc->batch), static_cast<uint64_t>(desc->seq),
                          static_cast<uint64_t>(desc->heads));
    if (st != RAYA_ATTN_OK) return st;
    maps.k = maps.q;  // the same [64 rows][32] boxes of the packed tensor
    if (pk == RAYA_KERNEL_TC32_WS2)  // two 128-row tiles per CTA (no rotation)
      tc32::tc32_ws_fwd<tiled64::kPacked, false, 2>
          <<<static_cast<unsigned>((grid + 1) / 2), tc32::kWsThreads, tc32::pipe_smem_bytes(), s>>>(a, maps);
    else
      (rope ? tc32::tc32_ws_fwd<tiled64::kPacked, true, 1> : tc32::tc32_ws_fwd<tiled64::kPacked, false, 1>)
          <<<static_cast<unsigned>(grid), tc32::kWsThreads, tc32::pipe_smem_bytes(), s>>>(a, maps);
  } else {
    const int id = tuned_tiled(desc);
    const PackedVariant* pv = nullptr;
    for (const PackedVariant& v : kPacked)
      if (v.id == id) pv = &v;
    const int bm = pv->warps * pv->rows_per_warp;
    a.row_tiles = static_cast<int>((desc->seq + bm - 1) / bm);
    const long long grid = static_cast<long long>(desc->batch) * desc->heads * a.row_tiles;
    if (grid > 0x7fffffffll)
      return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: %lld CTAs exceed the grid limit", grid);
    tiled64::TmaMaps maps;
    st = encode_packed(&maps.q, qkv, rows, desc->heads, static_cast<uint32_t>(bm));
    if (st == RAYA_ATTN_OK) st = encode_packed(&maps.k, qkv, rows, desc->heads, tiled64::kBN);
    if (st != RAYA_ATTN_OK) return st;
    maps.v = maps.k;
    (rope ? pv->rope : pv->plain)<<<static_cast<unsigned>(grid), pv->warps * 32, pv->smem, s>>>(a, maps);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "packed kernel launch");
  return RAYA_ATTN_OK;
}

raya_attn_status raya_attn_packed_workspace(const raya_attn_desc* desc, float rope_theta, size_t* bytes) {
  raya_attn_status st = check_shape(desc);
  if (st != RAYA_ATTN_OK) return st;
  if (!bytes) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: null output");
  *bytes = rope_theta > 0.f ? static_cast<size_t>(desc->seq) * 32 * 2 * sizeof(float) : 0;
  return RAYA_ATTN_OK;
}

raya_attn_status raya_attn_forward_packed(const raya_attn_desc* desc, const float* qkv, float* ctx,
                                          const int32_t* valid_len, float rope_theta, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  raya_attn_status st = check_shape(desc);
  if (st != RAYA_ATTN_OK) return st;
  if (desc->head_dim != 64)
    return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: the packed layout needs head_dim 64, got %lld",
                static_cast<long long>(desc->head_dim));
  if (!std::isfinite(rope_theta) || rope_theta < 0.f)
    return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: rope_theta %g", static_cast<double>(rope_theta));
  if (desc->seq == 0) return RAYA_ATTN_OK;
  if (!qkv || !ctx) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: null tensor pointer");
  if (!aligned16(qkv) || !aligned16(ctx) || (workspace && !aligned16(workspace)))
    return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: tensors must be 16-byte aligned");
  const bool rope = rope_theta > 0.f;
  size_t need = 0;
  raya_attn_packed_workspace(desc, rope_theta, &need);
  if (rope && (!workspace || workspace_bytes < need))
    return fail_length("workspace", workspace_bytes, need);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  DeviceCtx* ctx_dev = nullptr;
  st = ensure_ready(dev, &ctx_dev);
  if (st != RAYA_ATTN_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rope) {
    RopeFreq f;
    for (int i = 0; i < 32; ++i)  // ops.rs:120-122, in f32 with the C library's powf
      f.inv_freq[i] = 1.0f / powf(rope_theta, static_cast<float>(2 * i) / 64.0f);
    st = launch_rope_table(static_cast<float2*>(workspace), desc->seq, f, ctx_dev->sms, s);
    if (st != RAYA_ATTN_OK) return st;
  }
  return launch_packed(ctx_dev, desc, qkv, ctx, valid_len, rope ? static_cast<const float*>(workspace) : nullptr, s);
}

raya_attn_status raya_attn_forward_packed_noalloc(const raya_attn_desc* desc, const float* qkv, float* ctx,
                                                  const int32_t* valid_len, float rope_theta, void* stream) {
  raya_attn_status st = check_shape(desc);
  if (st != RAYA_ATTN_OK) return st;
  if (desc->head_dim != 64)
    return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: the packed layout needs head_dim 64, got %lld",
                static_cast<long long>(desc->head_dim));
  if (!std::isfinite(rope_theta) || rope_theta < 0.f)
    return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: rope_theta %g", static_cast<double>(rope_theta));
  const bool rope = rope_theta > 0.f;
  if (rope && desc->seq > kStaticRopeMaxSeq)
    return fail(RAYA_ATTN_ERR_UNSUPPORTED,
                "unsupported: seq %lld exceeds the %d positions of the built-in rotary table "
                "(use raya_attn_forward_packed with a workspace)",
                static_cast<long long>(desc->seq), kStaticRopeMaxSeq);
  if (desc->seq == 0) return RAYA_ATTN_OK;
  if (!qkv || !ctx) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: null tensor pointer");
  if (!aligned16(qkv) || !aligned16(ctx))
    return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: tensors must be 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  DeviceCtx* ctx_dev = nullptr;
  st = ensure_ready(dev, &ctx_dev);
  if (st != RAYA_ATTN_OK) return st;
  float2* table = nullptr;
  if (rope) {
    st = rope_static_table(dev, &table);
    if (st != RAYA_ATTN_OK) return st;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rope) {
    // Rewrites positions [0, seq) of the shared table; the attention kernel
    // below reads only those (rows past valid_len <= seq are not rotated), so
    // nothing left by an earlier call is read and nothing needs clearing.
    RopeFreq f;
    for (int i = 0; i < 32; ++i)  // ops.rs:120-122, in f32 with the C library's powf
      f.inv_freq[i] = 1.0f / powf(rope_theta, static_cast<float>(2 * i) / 64.0f);
    st = launch_rope_table(table, desc->seq, f, ctx_dev->sms, s);
    if (st != RAYA_ATTN_OK) return st;
  }
  return launch_packed(ctx_dev, desc, qkv, ctx, valid_len, rope ? reinterpret_cast<const float*>(table) : nullptr, s);
}

raya_attn_status raya_attn_probe_timeout(int64_t timeout_cycles, void* stream) {
  if (timeout_cycles < 0 || timeout_cycles > kDefaultTimeoutCycles)
    return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: timeout of %lld cycles", static_cast<long long>(timeout_cycles));
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  DeviceCtx* ctx = nullptr;
  raya_attn_status st = ensure_ready(dev, &ctx);
  if (st != RAYA_ATTN_OK) return st;
  timeout_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(ctx->status, timeout_cycles);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "timeout probe launch");
  return raya_attn_sync_status(stream);
}

raya_attn_status raya_attn_sync_status(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  DeviceCtx* ctx = nullptr;
  raya_attn_status st = ensure_ready(dev, &ctx);
  if (st != RAYA_ATTN_OK) return st;
  int flag = 0;
  e = cudaMemcpy(&flag, ctx->status, sizeof flag, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  if (flag != 0) {
    const int zero = 0;
    e = cudaMemcpy(ctx->status, &zero, sizeof zero, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "clear status");
    return fail(RAYA_ATTN_ERR_TIMEOUT, "timeout: a device-side wait gave up (status 0x%x)", flag);
  }
  return RAYA_ATTN_OK;
}

raya_attn_status raya_attn_forward_host(const raya_attn_desc* desc, const float* q, size_t q_len,
                                        const float* k, size_t k_len, const float* v, size_t v_len,
                                        float* out, size_t out_len, const int32_t* valid_len,
                                        int device) {
  raya_attn_status st = raya_attn_validate(desc, valid_len, q_len, k_len, v_len, out_len);
  if (st != RAYA_ATTN_OK) return st;
  if (numel(desc) == 0) return RAYA_ATTN_OK;
  if (!q || !k || !v || !out) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: null buffer");
  const std::vector<int32_t> sv = slice_valid_lengths(desc, valid_len);
  HostJob job{desc, sv.data(), 0, desc->batch * desc->heads, q, k, v, out, nullptr, -1};
  return host_pipeline(device, job);
}

raya_attn_status raya_attn_forward_multi_gpu(const raya_attn_desc* desc, const float* q, size_t q_len,
                                             const float* k, size_t k_len, const float* v, size_t v_len,
                                             float* out, size_t out_len, const int32_t* valid_len,
                                             const int* devices, int ndevices, float* out_device0) {
  raya_attn_status st = check_shape(desc);
  if (st != RAYA_ATTN_OK) return st;
  if (!out && !out_device0) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: no output buffer");
  st = raya_attn_validate(desc, valid_len, q_len, k_len, v_len, out ? out_len : numel(desc));
  if (st != RAYA_ATTN_OK) return st;
  if (!devices || ndevices < 1 || ndevices > kMaxDevices)
    return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: %d devices (1 to %d)", ndevices, kMaxDevices);
  for (int i = 0; i < ndevices; ++i) {
    if (devices[i] < 0 || devices[i] >= kMaxDevices)
      return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: device id %d", devices[i]);
    for (int j = 0; j < i; ++j)
      if (devices[j] == devices[i])
        return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: device %d listed twice", devices[i]);
  }
  if (numel(desc) == 0) return RAYA_ATTN_OK;
  if (!q || !k || !v) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: null buffer");
  if (out_device0 && !aligned16(out_device0))
    return fail(RAYA_ATTN_ERR_UNSUPPORTED, "unsupported: tensors must be 16-byte aligned");
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  for (int i = 0; i < ndevices; ++i)
    if (devices[i] >= count)
      return fail(RAYA_ATTN_ERR_CUDA, "cuda: device %d of %d", devices[i], count);
  const std::vector<int32_t> sv = slice_valid_lengths(desc, valid_len);
  // The partition of raya_attn_shard, one range per device.
  std::vector<int64_t> lo(ndevices), hi(ndevices);
  for (int r = 0; r < ndevices; ++r) {
    int64_t b = 0, en = 0;
    st = raya_attn_shard(desc, valid_len, ndevices, r, &b, &en);
    if (st != RAYA_ATTN_OK) return st;
    lo[r] = b;
    hi[r] = en;
  }
  // One host thread per device; each runs the host-buffer pipeline on its
  // range.  Errors are raised on the worker's thread and handed back here.
  struct Result {
    raya_attn_status st = RAYA_ATTN_OK;
    std::string msg;
    ErrorInfo info;
  };
  std::vector<Result> res(ndevices);
  std::vector<std::thread> pool;
  pool.reserve(ndevices);
  for (int r = 0; r < ndevices; ++r) {
    pool.emplace_back([&, r] {
      if (hi[r] <= lo[r]) return;
      HostJob job{desc, sv.data(), lo[r], hi[r], q, k, v, out, out_device0, devices[0]};
      res[r].st = host_pipeline(devices[r], job);
      if (res[r].st != RAYA_ATTN_OK) {
        res[r].msg = t_error;
        res[r].info = t_info;
      }
    });
  }
  for (auto& t : pool) t.join();
  for (int r = 0; r < ndevices; ++r)
    if (res[r].st != RAYA_ATTN_OK) {
      t_error = res[r].msg;
      t_info = res[r].info;
      return res[r].st;
    }
  return RAYA_ATTN_OK;
}

raya_attn_status raya_attn_kernel_for(const raya_attn_desc* desc, int packed, int* kernel) {
  raya_attn_status st = check_shape(desc);
  if (st != RAYA_ATTN_OK) return st;
  if (!kernel) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: null kernel pointer");
  *kernel = packed ? packed_kernel(desc, packed == 2) : auto_kernel(desc);
  return RAYA_ATTN_OK;
}

raya_attn_status raya_attn_work(const raya_attn_desc* desc, const int32_t* valid_len, uint64_t* pairs,
                                uint64_t* valid_rows) {
  raya_attn_status st = check_shape(desc);
  if (st != RAYA_ATTN_OK) return st;
  st = check_valid(desc, valid_len);
  if (st != RAYA_ATTN_OK) return st;
  const AttnArgs a = make_args(desc, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr);
  std::vector<uint64_t> memo(static_cast<size_t>(desc->seq) + 1, UINT64_MAX);
  uint64_t p = 0, r = 0;
  for (int64_t b = 0; b < desc->batch; ++b) {
    const int valid = valid_len ? valid_len[b] : static_cast<int>(desc->seq);
    if (memo[valid] == UINT64_MAX) memo[valid] = slice_pairs(a, valid);
    p += memo[valid] * static_cast<uint64_t>(desc->heads);
    r += static_cast<uint64_t>(valid) * desc->heads;
  }
  if (pairs) *pairs = p;
  if (valid_rows) *valid_rows = r;
  return RAYA_ATTN_OK;
}

raya_attn_status raya_attn_shard(const raya_attn_desc* desc, const int32_t* valid_len, int world,
                                 int rank, int64_t* bh_begin, int64_t* bh_end) {
  raya_attn_status st = check_shape(desc);
  if (st != RAYA_ATTN_OK) return st;
  st = check_valid(desc, valid_len);
  if (st != RAYA_ATTN_OK) return st;
  if (world < 1 || rank < 0 || rank >= world)
    return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: rank %d of world %d", rank, world);
  const AttnArgs a = make_args(desc, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr);
  const int64_t nbh = desc->batch * desc->heads;
  // Cost of a slice: its allowed pairs plus one unit per row for the stores.
  std::vector<double> prefix(static_cast<size_t>(nbh) + 1, 0.0);
  std::vector<double> memo(static_cast<size_t>(desc->seq) + 1, -1.0);
  for (int64_t bh = 0; bh < nbh; ++bh) {
    const int valid = valid_len ? valid_len[bh / desc->heads] : static_cast<int>(desc->seq);
    if (memo[valid] < 0) memo[valid] = static_cast<double>(slice_pairs(a, valid)) + desc->seq;
    prefix[bh + 1] = prefix[bh] + memo[valid];
  }
  auto cut = [&](int r) -> int64_t {  // first slice whose prefix reaches r/world of the total
    if (r <= 0) return 0;
    if (r >= world) return nbh;
    const double target = prefix[nbh] * r / world;
    const auto it = std::lower_bound(prefix.begin(), prefix.end(), target);
    int64_t idx = it - prefix.begin();
    if (idx > 0 && target - prefix[idx - 1] < prefix[idx] - target) --idx;
    return std::min<int64_t>(idx, nbh);
  };
  *bh_begin = cut(rank);
  *bh_end = std::max(*bh_begin, cut(rank + 1));
  return RAYA_ATTN_OK;
}

raya_attn_status raya_attn_fill_normal(float* dst, int64_t n, uint64_t seed, uint32_t stream_id,
                                       int64_t first_index, float stddev, void* stream) {
  if (n <= 0) return RAYA_ATTN_OK;
  if (!dst) return fail(RAYA_ATTN_ERR_SHAPE, "invalid shape: null destination");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t key = splitmix64(seed * 0x100000001B3ull + stream_id);
  const long long blocks = std::min<long long>((n + 255) / 256, static_cast<long long>(sms) * 8);
  fill_normal_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      dst, n, key, first_index, stddev);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fill_normal launch");
  return RAYA_ATTN_OK;
}

raya_attn_status raya_attn_ffma_peak(int reps, double* tflops) {
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  const int blocks = sms * 8, threads = 256, iters = 16384;
  float* sink = nullptr;
  e = cudaMalloc(&sink, sizeof(float) * blocks * threads);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(sink)");
  cudaEvent_t t0, t1;
  cudaEventCreate(&t0);
  cudaEventCreate(&t1);
  ffma_probe_kernel<<<blocks, threads>>>(sink, iters, 0.99999f, 1e-6f);  // warm-up
  double best = 0.0;
  for (int r = 0; r < std::max(reps, 1); ++r) {
    cudaEventRecord(t0);
    ffma_probe_kernel<<<blocks, threads>>>(sink, iters, 0.99999f, 1e-6f);
    cudaEventRecord(t1);
    cudaEventSynchronize(t1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, t0, t1);
    const double flops = 2.0 * 16 * 8 * static_cast<double>(iters) * blocks * threads;
    best = std::max(best, flops / (ms * 1e-3) / 1e12);
  }
  e = cudaGetLastError();
  cudaEventDestroy(t0);
  cudaEventDestroy(t1);
  cudaFree(sink);
  if (e != cudaSuccess) return cuda_fail(e, "ffma probe");
  *tflops = best;
  return RAYA_ATTN_OK;
}

}  // extern "C"
