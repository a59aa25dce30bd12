// tiled64.cuh — the block-local attention kernel for head_dim 64 on sm_100a.
//
// The reference's Tiled kernel (crates/raya-kernels/src/tiled/tile.rs:65-151)
// runs 8-row micro tiles over 64-key tiles with an online softmax; this is
// the same algorithm laid out for a B200 SM:
//
//   * one CTA per (batch*head slice, 32*WARPS query rows); 32 rows per warp;
//   * the CTA's key span (union of its rows' key ranges) is walked in 64-key
//     tiles.  Q, K and V tiles are staged into shared memory by tensor-map
//     TMA (cp.async.bulk.tensor.2d, no multicast): each tile is two boxes of
//     [rows][32 floats] with the 128-byte swizzle, so one tile is two TMA
//     requests and every LDS.128 below is bank-conflict-free;
//   * QK^T and PV are FP32 FFMA register tiles: each lane owns 8 rows x 8 keys
//     of S and 8 rows x 8 columns of O (rows lane/8 + 4m, keys lane%8 + 8n,
//     columns 4*(lane%8) + {0..3, 32..35}); every LDS.128 feeds 16 FFMAs;
//   * online softmax per 64-key tile in registers: row max by three xor
//     shuffles, p = 2^(s*scale*log2e - m) on the SFU, per-lane partial row
//     sums (reduced once at the end), O rescaled by alpha;
//   * P goes through a per-warp shared buffer (stride 72: conflict-free
//     scalar stores and broadcast LDS.128 loads) into the PV tile;
//   * K and V have STAGES buffers each; the last warp to finish with a buffer
//     (an acq_rel shared-memory counter) refills it with the tile STAGES
//     ahead, so K loads overlap softmax/PV and V loads overlap QK.
//
// Padding: a tile may extend past valid_len (or past the slice).  Keys there
// are masked to -inf before the softmax, and the PV loop stops at valid_len,
// so no value from a padded K/V row reaches the output — as in the reference,
// whose key loops stop at valid_len (naive.rs:37, tile.rs:80-87).  Padded
// query rows are written as +0.0f; a row with no allowed key is 0.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace raya {
namespace tiled64 {

constexpr int kD = 64;          // head_dim
constexpr int kBN = 64;         // keys per tile
constexpr int kHalfCols = 32;   // floats per swizzled box row (128 bytes)
constexpr int kPS = kBN + 8;    // padded row stride of the P buffer (floats)

// Shared-memory layout for WARPS warps of RPW query rows each.  Q, K and V
// are stored as two column halves of [rows][32 floats], each row 128 bytes
// with the TMA 128-byte swizzle (16-byte chunk c of row r lives at chunk
// c ^ (r & 7)); every half starts on a 1024-byte boundary.
template <int WARPS, int RPW, int STAGES>
struct Smem {
  float q[2][WARPS * RPW][kHalfCols];
  float k[STAGES][2][kBN][kHalfCols];
  float v[STAGES][2][kBN][kHalfCols];
  float p[WARPS][RPW][kPS];
  uint64_t qbar;
  uint64_t kbar[STAGES];
  uint64_t vbar[STAGES];
  uint64_t kready[STAGES];  // rotary kernels: every warp has rotated its part of K
  int kdone[STAGES];
  int vdone[STAGES];
  int kissued[STAGES];
  int vissued[STAGES];
  int abort_flag;
};

// Tensor maps of the launch: q with boxes of [WARPS*RPW rows][32 floats], k and
// v with boxes of [64 rows][32 floats]; all over the [batch*heads*seq][64]
// fp32 view of the tensors, 128-byte swizzle, zero fill out of bounds.
struct TmaMaps {
  CUtensorMap q;
  CUtensorMap k;
  CUtensorMap v;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            int w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar))
      : "memory");
}

// Tensor layouts the kernel reads and writes.
//   kHeadMajor: q, k, v, out are [batch*heads*seq][64] (raya's [heads][seq][head_dim]
//               per batch entry); 2-D tensor maps, coordinates (column, slice*seq + pos).
//   kPacked:    q, k, v are the packed projection [batch*seq][3][heads][64]
//               (encoder.rs:34-53 before split_qkv); 4-D tensor maps, coordinates
//               (column, head, which, b*seq + pos); out is the context
//               [batch*seq][heads][64] (encoder.rs:82-90 after the transpose back).
enum Layout : int { kHeadMajor = 0, kPacked = 1 };

// One thread: post the byte count of a [rows x 64] tile and issue its two
// column-half boxes (`which` selects q/k/v in the packed layout).
template <int LAYOUT>
__device__ __forceinline__ void stage_tile(float* half0, float* half1, const CUtensorMap* map,
                                           int head, int which, int y, int rows, uint64_t* bar) {
  fence_proxy_async_smem();
  mbar_arrive_expect_tx(bar, static_cast<uint32_t>(rows) * kD * 4);
  if constexpr (LAYOUT == kHeadMajor) {
    tma_load_2d(half0, map, 0, y, bar);
    tma_load_2d(half1, map, kHalfCols, y, bar);
  } else {
    tma_load_4d(half0, map, 0, head, which, y, bar);
    tma_load_4d(half1, map, kHalfCols, head, which, y, bar);
  }
}

// raya's rotary embedding (ops.rs:110-141, rotate-half form) on rows
// [r0, r0 + nrows) of a staged [rows][64] tile whose row r holds position
// pos0 + r: element i and i + 32 of a row become a*cos - b*sin and
// b*cos + a*sin, with (cos, sin) of that position and i from the table
// cs[pos][32][2], in unfused f32 arithmetic as the reference computes it.
// Rows at or past `valid` are left as they are (their keys are masked and
// their outputs are zero).  Warp-collective; the caller synchronises.
__device__ __forceinline__ void rope_rows(uint32_t half0, uint32_t half1, int r0, int nrows, int pos0,
                                          int valid, const float* __restrict__ cs, int lane) {
  for (int idx = lane; idx < nrows * 8; idx += 32) {
    const int r = r0 + (idx >> 3), ch = idx & 7;
    const int pos = pos0 + r;
    if (pos >= valid) continue;
    const uint32_t off = static_cast<uint32_t>(r * 128 + ((ch ^ (r & 7)) << 4));
    float4 a = lds128(half0 + off), b = lds128(half1 + off);
    const float4* t = reinterpret_cast<const float4*>(cs + (static_cast<size_t>(pos) * 32 + 4 * ch) * 2);
    const float4 t0 = __ldg(t), t1 = __ldg(t + 1);  // (cos, sin) of i = 4ch .. 4ch+3
    auto rot = [](float& x, float& y, float c, float sn) {
      const float nx = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, sn));
      const float ny = __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, sn));
      x = nx;
      y = ny;
    };
    rot(a.x, b.x, t0.x, t0.y);
    rot(a.y, b.y, t0.z, t0.w);
    rot(a.z, b.z, t1.x, t1.y);
    rot(a.w, b.w, t1.z, t1.w);
    sts128(half0 + off, a);
    sts128(half1 + off, b);
  }
}

__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "r"(smem_addr(p)), "r"(v)
               : "memory");
  return old;
}

// Returns true in every lane of the warp that is the last of the CTA's WARPS
// warps to finish with a buffer (the WARPS-th increment of its counter in this
// round).  __syncwarp orders the warp's shared reads before lane 0's release.
template <int WARPS>
__device__ __forceinline__ bool arrive_last(int* counter, int lane) {
  __syncwarp();
  int old = 0;
  if (lane == 0) old = atom_add_acq_rel(counter, 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  return old % WARPS == WARPS - 1;
}

// S[m][n] = q_row(m) . k_key(n) over the 64 columns for the lane's MR rows
// and 8 keys.  q0: shared address of Q half 0, row (warp rows + rg); rows of
// m step 4 (512 bytes).  k0: shared address of K half 0, row cg; keys of n
// step 8 (1024 bytes).  QH: byte size of one Q column half.  Swizzle: row
// r's chunk c is at c ^ (r & 7); for Q r & 7 = rg + 4*(m & 1) (warp rows
// start on a multiple of 8), for K r & 7 = cg.
//
// P2 = false: one FFMA per product, sequential in c.
// P2 = true: packed FFMA2 (two FMAs per instruction): even and odd columns
// accumulate in the two halves of a float2 (both operands are the aligned
// register pairs of the float4 loads), summed once at the end.
template <int MR, uint32_t QH, bool P2>
__device__ __forceinline__ void qk_tile(float (&s)[MR][8], uint32_t q0, uint32_t k0, int rg, int cg) {
  constexpr uint32_t KH = kBN * kHalfCols * 4;
  float2 acc[MR][P2 ? 8 : 1];
  if constexpr (P2) {
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int n = 0; n < 8; ++n) acc[m][n] = make_float2(0.f, 0.f);
  } else {
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int n = 0; n < 8; ++n) s[m][n] = 0.f;
  }
#pragma unroll 1
  for (int c4 = 0; c4 < kD / 4; ++c4) {
    const uint32_t half = static_cast<uint32_t>(c4 >> 3);
    const uint32_t cc = static_cast<uint32_t>(c4 & 7);
    const uint32_t qe = q0 + half * QH + ((cc ^ static_cast<uint32_t>(rg)) << 4);
    const uint32_t qo = q0 + half * QH + ((cc ^ static_cast<uint32_t>(rg + 4)) << 4);
    const uint32_t ka = k0 + half * KH + ((cc ^ static_cast<uint32_t>(cg)) << 4);
    float4 qv[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) qv[m] = lds128((m & 1 ? qo : qe) + m * 4 * 128);
    if constexpr (P2) {
      // Two keys at a time, so that the two FFMA2s into one accumulator are
      // 2*MR instructions apart.
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        const float4 k0v = lds128(ka + n * 8 * 128);
        const float4 k1v = lds128(ka + (n + 1) * 8 * 128);
#pragma unroll
        for (int m = 0; m < MR; ++m)
          acc[m][n] = __ffma2_rn(make_float2(qv[m].x, qv[m].y), make_float2(k0v.x, k0v.y), acc[m][n]);
#pragma unroll
        for (int m = 0; m < MR; ++m)
          acc[m][n + 1] = __ffma2_rn(make_float2(qv[m].x, qv[m].y), make_float2(k1v.x, k1v.y), acc[m][n + 1]);
#pragma unroll
        for (int m = 0; m < MR; ++m)
          acc[m][n] = __ffma2_rn(make_float2(qv[m].z, qv[m].w), make_float2(k0v.z, k0v.w), acc[m][n]);
#pragma unroll
        for (int m = 0; m < MR; ++m)
          acc[m][n + 1] = __ffma2_rn(make_float2(qv[m].z, qv[m].w), make_float2(k1v.z, k1v.w), acc[m][n + 1]);
      }
    } else {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float4 kv = lds128(ka + n * 8 * 128);
#pragma unroll
        for (int m = 0; m < MR; ++m) s[m][n] = fmaf(qv[m].x, kv.x, s[m][n]);
#pragma unroll
        for (int m = 0; m < MR; ++m) s[m][n] = fmaf(qv[m].y, kv.y, s[m][n]);
#pragma unroll
        for (int m = 0; m < MR; ++m) s[m][n] = fmaf(qv[m].z, kv.z, s[m][n]);
#pragma unroll
        for (int m = 0; m < MR; ++m) s[m][n] = fmaf(qv[m].w, kv.w, s[m][n]);
      }
    }
  }
  if constexpr (P2) {
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int n = 0; n < 8; ++n) s[m][n] = acc[m][n].x + acc[m][n].y;
  }
}

// o[m][i] += p[m] * (V row at shared byte address va, columns
// 4cg + {0,1}, {2,3} of half 0 and 32 + 4cg + {0,1}, {2,3} of half 1, already
// swizzled for that row).  O is held as column pairs; with P2 each pair is
// one packed FFMA2 (the same per-element FMA as two FFMAs).
template <int MR, bool P2>
__device__ __forceinline__ void pv_row(float2 (&o)[MR][4], const float (&p)[MR], uint32_t va) {
  constexpr uint32_t VH = kBN * kHalfCols * 4;
  const float4 x = lds128(va);
  const float4 y = lds128(va + VH);
  const float2 v[4] = {make_float2(x.x, x.y), make_float2(x.z, x.w), make_float2(y.x, y.y),
                       make_float2(y.z, y.w)};
#pragma unroll
  for (int m = 0; m < MR; ++m) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (P2) {
        o[m][i] = __ffma2_rn(make_float2(p[m], p[m]), v[i], o[m][i]);
      } else {
        o[m][i].x = fmaf(p[m], v[i].x, o[m][i].x);
        o[m][i].y = fmaf(p[m], v[i].y, o[m][i].y);
      }
    }
  }
}

// O[m][:] += sum_{j < nv} P[m][j] V[j][:].  pa: shared address of this lane's
// first P row (row stride 4 rows); v0: shared address of V half 0 row 0 plus
// (cg << 4).  Keys go 8 at a time (rows 8*j8 + u hold chunk cg at cg ^ u);
// keys at or past nv (valid_len inside a partial tile) are never read.
template <int MR, bool P2>
__device__ __forceinline__ void pv_tile(float2 (&o)[MR][4], uint32_t pa, uint32_t v0, int nv) {
  const int groups = nv >> 3;
#pragma unroll 1
  for (int j8 = 0; j8 < groups; ++j8) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float4 pv[MR];
#pragma unroll
      for (int m = 0; m < MR; ++m) pv[m] = lds128(pa + (m * 4 * kPS + j8 * 8 + h * 4) * 4);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int u = h * 4 + jj;
        float p[MR];
#pragma unroll
        for (int m = 0; m < MR; ++m)
          p[m] = jj == 0 ? pv[m].x : jj == 1 ? pv[m].y : jj == 2 ? pv[m].z : pv[m].w;
        pv_row<MR, P2>(o, p, (v0 + (j8 * 8 + u) * 128) ^ static_cast<uint32_t>(u << 4));
      }
    }
  }
  // Tail of a partial tile: the last nv % 8 valid keys, one at a time.
  for (int j = groups * 8; j < nv; ++j) {
    float p[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) p[m] = lds32(pa + (m * 4 * kPS + j) * 4);
    pv_row<MR, P2>(o, p, (v0 + j * 128) ^ static_cast<uint32_t>((j & 7) << 4));
  }
}

// Per-warp stage clock (lane 0 only); compiles to nothing unless TIMED.
template <bool TIMED>
struct StageClock {
  __device__ __forceinline__ void start() {}
  __device__ __forceinline__ void lap(int) {}
  __device__ __forceinline__ void tile() {}
  __device__ __forceinline__ void flush(unsigned long long*, int) {}
};

template <>
struct StageClock<true> {
  long long last = 0, first = 0;
  unsigned long long acc[kStageSlots] = {};
  __device__ __forceinline__ void start() { first = last = clock64(); }
  __device__ __forceinline__ void lap(int slot) {
    const long long now = clock64();
    acc[slot] += static_cast<unsigned long long>(now - last);
    last = now;
  }
  __device__ __forceinline__ void tile() { acc[kStageTiles] += 1; }
  __device__ __forceinline__ void flush(unsigned long long* out, int lane) {
    acc[kStageTotal] = static_cast<unsigned long long>(clock64() - first);
    if (out && lane == 0)
      for (int i = 0; i < kStageSlots; ++i) atomicAdd(out + i, acc[i]);
  }
};

template <int WARPS, int RPW, int STAGES>
constexpr size_t smem_bytes() {
  return sizeof(Smem<WARPS, RPW, STAGES>) + 1024;  // + slack to align the base to 1024 bytes
}

template <int WARPS, int RPW, int STAGES>
constexpr int min_blocks() {
  // CTAs per SM that the shared memory allows (228 KB per SM, 1 KB reserved
  // per CTA), which also sets the register cap of __launch_bounds__.
  return (228 * 1024) / (static_cast<int>(smem_bytes<WARPS, RPW, STAGES>()) + 1024);
}

// WARPS warps of RPW (32 or 16) query rows; each lane owns MR = RPW/4 rows.
// PQK / PPV: packed FFMA2 in the QK^T / PV tiles.  LAYOUT: Layout above.
// ROPE: rotate q and k in shared memory before use (packed layout).
template <int WARPS, int RPW, int STAGES, bool PQK, bool PPV, bool TIMED, int LAYOUT = kHeadMajor,
          bool ROPE = false>
__global__ void __launch_bounds__(WARPS * 32, min_blocks<WARPS, RPW, STAGES>())
    tiled64_fwd(const __grid_constant__ AttnArgs a, const __grid_constant__ TmaMaps maps) {
  static_assert(RPW == 16 || RPW == 32, "rows per warp");
  constexpr int MR = RPW / 4;
  constexpr int kRowsPerWarp = RPW;
  constexpr int kBM = WARPS * kRowsPerWarp;
  constexpr int kThreads = WARPS * 32;
  constexpr uint32_t kQHalf = kBM * kHalfCols * 4;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  Smem<WARPS, RPW, STAGES>& sm =
      *reinterpret_cast<Smem<WARPS, RPW, STAGES>*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int rg = lane >> 3, cg = lane & 7;
  const int tile = static_cast<int>(blockIdx.x % static_cast<unsigned>(a.row_tiles));
  const long long bh = blockIdx.x / static_cast<unsigned>(a.row_tiles);
  const int b = static_cast<int>(bh / a.heads);
  const int seq = a.seq;
  int valid = a.valid_len ? a.valid_len[b] : seq;
  valid = valid < 0 ? 0 : (valid > seq ? seq : valid);
  const int r0 = tile * kBM;
  const int head = static_cast<int>(bh - static_cast<long long>(b) * a.heads);
  // First TMA row of this slice: slice*seq (head-major) or b*seq (packed).
  const long long row_base = LAYOUT == kHeadMajor ? bh * seq : static_cast<long long>(b) * seq;
  // Output row `pos` of this slice lives at outp + pos * ostride floats.
  const size_t ostride = LAYOUT == kHeadMajor ? static_cast<size_t>(kD) : static_cast<size_t>(a.heads) * kD;
  float* __restrict__ outp = a.out + (LAYOUT == kHeadMajor ? static_cast<size_t>(row_base) * kD
                                                           : static_cast<size_t>(row_base) * ostride +
                                                                 static_cast<size_t>(head) * kD);

  if (r0 >= valid) {  // the whole tile is padding: exact zeros, no loads
    const int rows = min(kBM, seq - r0);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int idx = tid; idx < rows * 16; idx += kThreads)
      st_stream(outp + static_cast<size_t>(r0 + (idx >> 4)) * ostride + (idx & 15) * 4, zero);
    return;
  }

  // CTA key span [klo, khi) and its 64-key tiles.
  const int last = min(r0 + kBM, valid) - 1;
  int klo, khi, unused;
  key_range(a, r0, valid, klo, unused);
  key_range(a, last, valid, unused, khi);
  const int t_begin = klo / kBN;
  const int ntiles = (khi + kBN - 1) / kBN - t_begin;

  // This warp's rows and the key ranges of its first and last valid row.
  const int wr0 = r0 + warp * kRowsPerWarp;
  const int wrows = max(0, min(kRowsPerWarp, valid - wr0));
  const int wlast = wr0 + max(wrows, 1) - 1;
  int lo_f = 0, hi_f = 0, lo_l = 0, hi_l = 0;
  if (wrows > 0) {
    key_range(a, wr0, valid, lo_f, hi_f);
    key_range(a, wlast, valid, lo_l, hi_l);
  }

  if (tid == 0) {
    mbar_init(&sm.qbar, 1);
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.kbar[s], 1);
      mbar_init(&sm.vbar[s], 1);
      mbar_init(&sm.kready[s], WARPS);
      sm.kdone[s] = sm.vdone[s] = 0;
      sm.kissued[s] = sm.vissued[s] = 0;
    }
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (tid == 0) {
    stage_tile<LAYOUT>(&sm.q[0][0][0], &sm.q[1][0][0], &maps.q, head, 0, static_cast<int>(row_base + r0), kBM,
                       &sm.qbar);
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      if (s < ntiles) {
        const int y = static_cast<int>(row_base + (t_begin + s) * kBN);
        stage_tile<LAYOUT>(&sm.k[s][0][0][0], &sm.k[s][1][0][0], &maps.k, head, 1, y, kBN, &sm.kbar[s]);
        stage_tile<LAYOUT>(&sm.v[s][0][0][0], &sm.v[s][1][0][0], &maps.v, head, 2, y, kBN, &sm.vbar[s]);
        sm.kissued[s] = 1;
        sm.vissued[s] = 1;
      }
    }
  }

  volatile int* abort_flag = &sm.abort_flag;
  const float qscale = a.qscale;
  float2 o[MR][4];  // column pairs (4cg, 4cg+1), (4cg+2, 4cg+3), (32+4cg, ..), (34+4cg, ..)
  float msc[MR], lrow[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    msc[m] = -INFINITY;
    lrow[m] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) o[m][c] = make_float2(0.f, 0.f);
  }

  const uint32_t q0 = smem_addr(&sm.q[0][warp * kRowsPerWarp + rg][0]);
  const uint32_t pa_store = smem_addr(&sm.p[warp][rg][cg]);
  const uint32_t pa = smem_addr(&sm.p[warp][rg][0]);
  StageClock<TIMED> clk;
  clk.start();
  bool ok = mbar_wait_bounded(&sm.qbar, 0, abort_flag, a.status, a.timeout_cycles);
  if constexpr (ROPE) {
    // Each warp rotates its own query rows, then reads only those.
    if (ok)
      rope_rows(smem_addr(&sm.q[0][0][0]), smem_addr(&sm.q[1][0][0]), warp * kRowsPerWarp, kRowsPerWarp, r0,
                valid, a.rope_cs, lane);
    __syncwarp();
  }

  for (int t = 0; ok && t < ntiles; ++t) {
    const int s = STAGES == 1 ? 0 : t % STAGES;
    const uint32_t par = static_cast<uint32_t>(t / STAGES) & 1u;
    const int kt = (t_begin + t) * kBN;
    const bool active = wrows > 0 && kt < hi_l && kt + kBN > lo_f;
    const bool whole = lo_l <= kt && hi_f >= kt + kBN;

    if (!mbar_wait_bounded(&sm.kbar[s], par, abort_flag, a.status, a.timeout_cycles)) { ok = false; break; }
    if constexpr (ROPE) {
      // The K tile is shared: each warp rotates kBN/WARPS of its rows, then
      // all warps wait until every part is rotated.
      constexpr int kRot = kBN / WARPS;
      rope_rows(smem_addr(&sm.k[s][0][0][0]), smem_addr(&sm.k[s][1][0][0]), warp * kRot, kRot, kt, valid,
                a.rope_cs, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.kready[s]);
      if (!mbar_wait_bounded(&sm.kready[s], par, abort_flag, a.status, a.timeout_cycles)) { ok = false; break; }
    }
    clk.lap(kStageKWait);
    float sc[MR][8];
    if (active) {
      clk.tile();
      qk_tile<MR, kQHalf, PQK>(sc, q0, smem_addr(&sm.k[s][0][cg][0]), rg, cg);
      if (!whole) {
        // Per-element mask: key j allowed for row i iff lo(i) <= j < hi(i)
        // (hi <= valid_len, so padded keys are always masked).  Rows past
        // valid_len reuse the last valid row's range (their output is
        // overwritten with zeros).
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          const int i = min(wr0 + rg + 4 * m, wlast);
          int lo, hi;
          key_range(a, i, valid, lo, hi);
#pragma unroll
          for (int n = 0; n < 8; ++n) {
            const int j = kt + cg + 8 * n;
            if (static_cast<unsigned>(j - lo) >= static_cast<unsigned>(hi - lo)) sc[m][n] = -INFINITY;
          }
        }
      }
    }
    clk.lap(kStageQk);
    // Done reading K buffer s: the last warp refills it with tile t+STAGES.
    if (arrive_last<WARPS>(&sm.kdone[s], lane) && t + STAGES < ntiles && lane == 0) {
      const int y = static_cast<int>(row_base + (t_begin + t + STAGES) * kBN);
      stage_tile<LAYOUT>(&sm.k[s][0][0][0], &sm.k[s][1][0][0], &maps.k, head, 1, y, kBN, &sm.kbar[s]);
      sm.kissued[s] += 1;
    }
    clk.lap(kStageRefill);

    if (active) {
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        float tmax = sc[m][0];
#pragma unroll
        for (int n = 1; n < 8; ++n) tmax = fmaxf(tmax, sc[m][n]);
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
        // Running max kept pre-scaled (scale*log2e > 0 keeps the order).
        const float mnew = fmaxf(msc[m], tmax * qscale);
        const float mbase = mnew == -INFINITY ? 0.f : mnew;
        const float alpha = ex2(msc[m] - mbase);  // 0 while nothing was seen
        msc[m] = mnew;
        float rs = 0.f;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const float p = ex2(fmaf(sc[m][n], qscale, -mbase));
          rs += p;
          sts32(pa_store + ((4 * m) * kPS + 8 * n) * 4, p);
        }
        lrow[m] = fmaf(lrow[m], alpha, rs);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if constexpr (PPV) {
            o[m][c] = __fmul2_rn(o[m][c], make_float2(alpha, alpha));
          } else {
            o[m][c].x *= alpha;
            o[m][c].y *= alpha;
          }
        }
      }
    }
    __syncwarp();
    clk.lap(kStageSoftmax);

    if (!mbar_wait_bounded(&sm.vbar[s], par, abort_flag, a.status, a.timeout_cycles)) { ok = false; break; }
    clk.lap(kStageVWait);
    if (active) pv_tile<MR, PPV>(o, pa, smem_addr(&sm.v[s][0][0][0]) + (cg << 4), min(kBN, valid - kt));
    clk.lap(kStagePv);
    if (arrive_last<WARPS>(&sm.vdone[s], lane) && t + STAGES < ntiles && lane == 0) {
      const int y = static_cast<int>(row_base + (t_begin + t + STAGES) * kBN);
      stage_tile<LAYOUT>(&sm.v[s][0][0][0], &sm.v[s][1][0][0], &maps.v, head, 2, y, kBN, &sm.vbar[s]);
      sm.vissued[s] += 1;
    }
    clk.lap(kStageRefill);
  }
  clk.flush(a.stage_cycles, lane);

  // Epilogue: reduce the per-lane row sums, normalise, store (+0.0f for
  // padded rows; rows past seq are not ours).
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    float l = lrow[m];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    l += __shfl_xor_sync(0xffffffffu, l, 4);
    const int row = wr0 + rg + 4 * m;
    if (row < seq) {
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f), y = x;
      if (row < valid) {
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        x = make_float4(o[m][0].x * inv, o[m][0].y * inv, o[m][1].x * inv, o[m][1].y * inv);
        y = make_float4(o[m][2].x * inv, o[m][2].y * inv, o[m][3].x * inv, o[m][3].y * inv);
      }
      float* orow = outp + static_cast<size_t>(row) * ostride;
      st_stream(orow + 4 * cg, x);
      st_stream(orow + 32 + 4 * cg, y);
    }
  }

  // After a timeout, wait (bounded) for copies still in flight into this
  // CTA's shared memory before it is released.
  __syncthreads();
  if (*abort_flag && tid == 0) {
    const long long t0 = clock64();
    auto drain = [&](uint64_t* bar, int issued) {
      if (issued <= 0) return;
      const uint32_t par = static_cast<uint32_t>(issued - 1) & 1u;
      while (!mbar_try_wait(bar, par) && clock64() - t0 < a.timeout_cycles) {
      }
    };
    drain(&sm.qbar, 1);
    for (int s = 0; s < STAGES; ++s) {
      drain(&sm.kbar[s], sm.kissued[s]);
      drain(&sm.vbar[s], sm.vissued[s]);
    }
  }
}

}  // namespace tiled64
}  // namespace raya
