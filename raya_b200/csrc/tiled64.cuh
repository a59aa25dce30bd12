// tiled64.cuh — the block-local attention kernel for head_dim 64 on sm_100a.
//
// The reference's Tiled kernel (crates/raya-kernels/src/tiled/tile.rs:65-151)
// runs 8-row micro tiles over 64-key tiles with an online softmax; this is
// the same algorithm laid out for a B200 SM:
//
//   * one CTA per (batch*head slice, 128 query rows); 4 warps of 32 rows;
//   * the CTA's key span (union of its rows' key ranges) is walked in 64-key
//     tiles.  K and V tiles are staged into shared memory by TMA bulk copies
//     (one 256-byte row each, into rows padded to 68 floats), and only rows
//     below valid_len are copied, so padding is never read — as in the
//     reference, whose key loops stop at valid_len;
//   * QK^T and PV are FP32 FFMA register tiles: each lane owns 8 rows x 8 keys
//     of S and 8 rows x 8 columns of O (rows lane/8 + 4m, keys lane%8 + 8n,
//     columns 4*(lane%8) + {0..3, 32..35}); every LDS.128 feeds 16 FFMAs and
//     the padded strides make all shared loads conflict-free;
//   * online softmax per 64-key tile in registers: row max by three xor
//     shuffles, p = 2^(s*scale*log2e - m) on the SFU, per-lane partial row
//     sums (reduced once at the end), O rescaled by alpha;
//   * P goes through a per-warp shared buffer (stride 72: conflict-free
//     scalar stores and broadcast LDS.128 loads) into the PV tile;
//   * K and V are single-buffered per stage; the last warp to finish with a
//     stage (shared-memory counter) refills it with the next tile, so loads
//     of K(t+S) overlap softmax/PV(t) and loads of V(t+S) overlap QK(t+S).
//     Two CTAs fit per SM (106.5 KB shared memory, <= 255 registers).
//
// Semantics kept from the reference: scale applied to q.k (here folded into
// the exponent), masked keys weigh exactly 0 (ex2(-inf) = +0), padded query
// rows are written as +0.0f, a row with no allowed key is 0, out is fully
// overwritten.
#pragma once

#include "common.cuh"

namespace raya {
namespace tiled64 {

constexpr int kD = 64;          // head_dim
constexpr int kRowsPerWarp = 32;
constexpr int kBN = 64;         // keys per tile
constexpr int kQS = kD + 4;     // padded row stride (floats) of Q, K, V tiles
constexpr int kPS = kBN + 8;    // padded row stride of the P buffer
constexpr int kRowBytes = kD * 4;

// WARPS warps of 32 query rows per CTA (CTA rows = 32 * WARPS); STAGES K/V
// tile buffers.
template <int WARPS, int STAGES>
struct Smem {
  float q[WARPS * kRowsPerWarp][kQS];
  float k[STAGES][kBN][kQS];
  float v[STAGES][kBN][kQS];
  float p[WARPS][kRowsPerWarp][kPS];
  uint64_t qbar;
  uint64_t kbar[STAGES];
  uint64_t vbar[STAGES];
  int kdone[STAGES];
  int vdone[STAGES];
  int kissued[STAGES];
  int vissued[STAGES];
  int abort_flag;
};

// Warp-collective: zero rows [nvalid, nrows) of a padded tile, then stage
// rows [0, nvalid) from global memory with one TMA bulk copy per row, all
// completing on `bar`.  Lane 0 posts the byte count.
__device__ __forceinline__ void stage_rows(float* dst, const float* src, int nvalid,
                                           int nrows, uint64_t* bar, int lane) {
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int idx = nvalid * 16 + lane; idx < nrows * 16; idx += 32)
    *reinterpret_cast<float4*>(dst + (idx >> 4) * kQS + (idx & 15) * 4) = zero;
  __syncwarp();
  if (lane == 0) {
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nvalid) * kRowBytes);
  }
  __syncwarp();
  for (int r = lane; r < nvalid; r += 32)
    tma_load_1d(dst + r * kQS, src + static_cast<size_t>(r) * kD, kRowBytes, bar);
}

// Returns true in every lane of the warp that is the last of the CTA's WARPS
// warps to finish with a stage (the WARPS-th increment of its counter for
// this round).
template <int WARPS>
__device__ __forceinline__ bool arrive_last(int* counter, int lane) {
  __syncwarp();
  int old = 0;
  if (lane == 0) {
    __threadfence_block();
    old = atomicAdd(counter, 1);
    __threadfence_block();
  }
  old = __shfl_sync(0xffffffffu, old, 0);
  return old % WARPS == WARPS - 1;
}

// S[m][n] = q_row(m) . k_key(n) over the 64 columns, sequential in c.
// qa: shared address of this lane's first Q row (row stride 4 rows);
// ka: shared address of its first K row (row stride 8 rows).  The four
// column components are applied component-major so that consecutive FFMAs
// hit different accumulators.
__device__ __forceinline__ void qk_tile(float (&s)[8][8], uint32_t qa, uint32_t ka) {
#pragma unroll
  for (int m = 0; m < 8; ++m)
#pragma unroll
    for (int n = 0; n < 8; ++n) s[m][n] = 0.f;
#pragma unroll 1
  for (int c4 = 0; c4 < kD / 4; ++c4) {
    float4 qv[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) qv[m] = lds128(qa + (m * 4 * kQS + c4 * 4) * 4);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float4 kv = lds128(ka + (n * 8 * kQS + c4 * 4) * 4);
#pragma unroll
      for (int m = 0; m < 8; ++m) s[m][n] = fmaf(qv[m].x, kv.x, s[m][n]);
#pragma unroll
      for (int m = 0; m < 8; ++m) s[m][n] = fmaf(qv[m].y, kv.y, s[m][n]);
#pragma unroll
      for (int m = 0; m < 8; ++m) s[m][n] = fmaf(qv[m].z, kv.z, s[m][n]);
#pragma unroll
      for (int m = 0; m < 8; ++m) s[m][n] = fmaf(qv[m].w, kv.w, s[m][n]);
    }
  }
}

// O[m][0..3] += sum_j P[m][j] V[j][4cg..4cg+3]; O[m][4..7] likewise at +32.
// pa: shared address of this lane's first P row (row stride 4 rows);
// va: shared address of V row 0, column 4*cg.
__device__ __forceinline__ void pv_tile(float (&o)[8][8], uint32_t pa, uint32_t va) {
#pragma unroll 2
  for (int j4 = 0; j4 < kBN / 4; ++j4) {
    float4 pv[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) pv[m] = lds128(pa + (m * 4 * kPS + j4 * 4) * 4);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const float4 x = lds128(va + ((j4 * 4 + jj) * kQS) * 4);
      const float4 y = lds128(va + ((j4 * 4 + jj) * kQS + 32) * 4);
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const float p = jj == 0 ? pv[m].x : jj == 1 ? pv[m].y : jj == 2 ? pv[m].z : pv[m].w;
        o[m][0] = fmaf(p, x.x, o[m][0]);
        o[m][1] = fmaf(p, x.y, o[m][1]);
        o[m][2] = fmaf(p, x.z, o[m][2]);
        o[m][3] = fmaf(p, x.w, o[m][3]);
        o[m][4] = fmaf(p, y.x, o[m][4]);
        o[m][5] = fmaf(p, y.y, o[m][5]);
        o[m][6] = fmaf(p, y.z, o[m][6]);
        o[m][7] = fmaf(p, y.w, o[m][7]);
      }
    }
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

template <int WARPS, int STAGES>
constexpr int min_blocks() {
  // CTAs per SM that the shared memory allows (228 KB per SM, 1 KB reserved
  // per CTA), which also sets the register cap of __launch_bounds__.
  return (228 * 1024) / (static_cast<int>(sizeof(Smem<WARPS, STAGES>)) + 1024);
}

template <int WARPS, int STAGES, bool TIMED>
__global__ void __launch_bounds__(WARPS * 32, min_blocks<WARPS, STAGES>())
    tiled64_fwd(const __grid_constant__ AttnArgs a) {
  constexpr int kBM = WARPS * kRowsPerWarp;
  constexpr int kThreads = WARPS * 32;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Smem<WARPS, STAGES>& sm = *reinterpret_cast<Smem<WARPS, STAGES>*>(smem_raw);

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
  const size_t base = static_cast<size_t>(bh) * seq * kD;
  float* __restrict__ outp = a.out + base;

  if (r0 >= valid) {  // the whole tile is padding: exact zeros, no loads
    const int rows = min(kBM, seq - r0);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int idx = tid; idx < rows * 16; idx += kThreads)
      st_stream(outp + static_cast<size_t>(r0 + (idx >> 4)) * kD + (idx & 15) * 4, zero);
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
      sm.kdone[s] = sm.vdone[s] = 0;
      sm.kissued[s] = sm.vissued[s] = 0;
    }
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const float* __restrict__ kbase = a.k + base;
  const float* __restrict__ vbase = a.v + base;
  if (warp == 0) {
    stage_rows(&sm.q[0][0], a.q + base + static_cast<size_t>(r0) * kD, last - r0 + 1,
               last - r0 + 1, &sm.qbar, lane);
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      if (s < ntiles) {
        const int kt = (t_begin + s) * kBN;
        const int nv = min(kBN, valid - kt);
        stage_rows(&sm.k[s][0][0], kbase + static_cast<size_t>(kt) * kD, nv, kBN, &sm.kbar[s], lane);
        stage_rows(&sm.v[s][0][0], vbase + static_cast<size_t>(kt) * kD, nv, kBN, &sm.vbar[s], lane);
        if (lane == 0) { sm.kissued[s] = 1; sm.vissued[s] = 1; }
      }
    }
  }

  volatile int* abort_flag = &sm.abort_flag;
  const float qscale = a.qscale;
  float o[8][8];
  float msc[8], lrow[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    msc[m] = -INFINITY;
    lrow[m] = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) o[m][c] = 0.f;
  }

  const uint32_t qa = smem_addr(&sm.q[warp * kRowsPerWarp + rg][0]);
  const uint32_t pa_store = smem_addr(&sm.p[warp][rg][cg]);
  const uint32_t pa = smem_addr(&sm.p[warp][rg][0]);
  StageClock<TIMED> clk;
  clk.start();
  bool ok = mbar_wait_bounded(&sm.qbar, 0, abort_flag, a.status, a.timeout_cycles);

  for (int t = 0; ok && t < ntiles; ++t) {
    const int s = STAGES == 1 ? 0 : t % STAGES;
    const uint32_t par = static_cast<uint32_t>(t / STAGES) & 1u;
    const int kt = (t_begin + t) * kBN;
    const bool active = wrows > 0 && kt < hi_l && kt + kBN > lo_f;
    const bool whole = lo_l <= kt && hi_f >= kt + kBN;

    if (!mbar_wait_bounded(&sm.kbar[s], par, abort_flag, a.status, a.timeout_cycles)) { ok = false; break; }
    clk.lap(kStageKWait);
    float sc[8][8];
    if (active) {
      clk.tile();
      qk_tile(sc, qa, smem_addr(&sm.k[s][cg][0]));
      if (!whole) {
        // Per-element mask: key j allowed for row i iff lo(i) <= j < hi(i).
        // Rows past valid_len reuse the last valid row's range (their
        // output is overwritten with zeros).
#pragma unroll
        for (int m = 0; m < 8; ++m) {
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
    // Done reading K stage s: the last warp refills it with tile t+STAGES.
    if (arrive_last<WARPS>(&sm.kdone[s], lane) && t + STAGES < ntiles) {
      const int kn = (t_begin + t + STAGES) * kBN;
      stage_rows(&sm.k[s][0][0], kbase + static_cast<size_t>(kn) * kD, min(kBN, valid - kn), kBN,
                 &sm.kbar[s], lane);
      if (lane == 0) sm.kissued[s] += 1;
    }
    clk.lap(kStageRefill);

    if (active) {
#pragma unroll
      for (int m = 0; m < 8; ++m) {
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
        for (int c = 0; c < 8; ++c) o[m][c] *= alpha;
      }
    }
    __syncwarp();
    clk.lap(kStageSoftmax);

    if (!mbar_wait_bounded(&sm.vbar[s], par, abort_flag, a.status, a.timeout_cycles)) { ok = false; break; }
    clk.lap(kStageVWait);
    if (active) pv_tile(o, pa, smem_addr(&sm.v[s][0][4 * cg]));
    clk.lap(kStagePv);
    if (arrive_last<WARPS>(&sm.vdone[s], lane) && t + STAGES < ntiles) {
      const int kn = (t_begin + t + STAGES) * kBN;
      stage_rows(&sm.v[s][0][0], vbase + static_cast<size_t>(kn) * kD, min(kBN, valid - kn), kBN,
                 &sm.vbar[s], lane);
      if (lane == 0) sm.vissued[s] += 1;
    }
    clk.lap(kStageRefill);
  }
  clk.flush(a.stage_cycles, lane);

  // Epilogue: reduce the per-lane row sums, normalise, store (+0.0f for
  // padded rows; rows past seq are not ours).
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float l = lrow[m];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    l += __shfl_xor_sync(0xffffffffu, l, 4);
    const int row = wr0 + rg + 4 * m;
    if (row < seq) {
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f), y = x;
      if (row < valid) {
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        x = make_float4(o[m][0] * inv, o[m][1] * inv, o[m][2] * inv, o[m][3] * inv);
        y = make_float4(o[m][4] * inv, o[m][5] * inv, o[m][6] * inv, o[m][7] * inv);
      }
      float* orow = outp + static_cast<size_t>(row) * kD;
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

template <int WARPS, int STAGES>
constexpr size_t smem_bytes() {
  return sizeof(Smem<WARPS, STAGES>);
}

}  // namespace tiled64
}  // namespace raya
