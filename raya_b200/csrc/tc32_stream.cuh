// tc32_stream.cuh — the tc32_ws_fwd pipeline in one resident CTA per SM that
// streams its row tiles back to back (sm_100a).
//
// A "unit" is 128 query rows of one (sequence, head) slice, the work of one
// tc32_ws_fwd CTA.  With short key ranges (block-local masks: 2-6 key tiles
// per unit) a tc32_ws_fwd CTA spends most of its life outside the steady
// state: barrier and tensor-memory set-up, the first copies' latency, the
// first QK^T, the epilogue and the launch of the next CTA (per-CTA clocks on
// a 4-tile unit: ~11k of ~18k cycles).  Here one CTA per SM walks units
// blockIdx.x, blockIdx.x + gridDim.x, ... and every ring carries on from one
// unit to the next, so unit u+1's copies, splits and first QK^T overlap unit
// u's last tiles and its epilogue.
//
// Arithmetic and per-tile protocol are those of tc32_ws_fwd (3xTF32: raw fp32
// tiles as hi operands, lo = x - trunc(x); O in tensor memory with the lazy
// 2^8 rescale).  What changes:
//
//   * The raw ring (4 stages of 32 KB) carries a sequence of items: for each
//     unit with work, its q tile ([half][128 rows][32], the size of one K/V
//     stage), then the K/V tiles of its key range.  A producer thread (warp
//     9) copies items in order, each as soon as the item four places earlier
//     has been released, independently of the split warps (warps 4-8).
//   * Split warps 4-7 (which together reach all 128 tensor-memory lanes)
//     move each q tile into tensor memory, as q and q - trunc(q), as soon
//     as QK(u-1, last) has completed and the softmax warps have used unit
//     u-1's q_ready phase (q_free takes one arrival from each); so QK(u, 0)
//     needs nothing from the softmax warps and runs while they finish unit
//     u-1.
//   * The softmax warps write unit u-1's output after its last P: once
//     PV(u-1, last) is complete and unit u's q tile has been read, O / l is
//     staged in that q tile's slot and stored by TMA; the slot goes back to
//     the producer once the store has read it (checked after the next P).
//     PV(u, 0), which overwrites O, waits for P(u, 0), i.e. after that read.
//   * P is double-buffered as in tc32_ws_fwd (P(g) waits for PV(g-2)).
//   * Barrier phases come from per-CTA running counts (key tiles g, ring
//     items, units with work k), so each barrier advances as in one long
//     tc32_ws_fwd CTA; every role reads the next unit's valid length one unit
//     ahead.
//   * Padding-only units (rows at or past valid_len) are written as zeros by
//     the softmax warps and add no items.
//
// Tensor memory (512 columns): as tc32_ws_fwd: S [0,64), Q hi [64,128), Q lo
// [128,192), P0 hi/lo [192,320), P1 hi/lo [320,448), O [448,512).
//
// Roles (384 threads): softmax warps 0-3, split warps 4-8 (160 threads),
// copy producer warp 9 (lane 0), QK^T issuer warp 10, PV issuer warp 11.
// Work done once per unit (the output write, the q tile into tensor memory,
// the unit decode, the spin of a bounded wait) lives in out-of-line
// functions: inlined, it spread the per-tile loops over more instruction-
// cache lines and multiplied the instruction-fetch stalls.
//
// Measured against tc32_ws_fwd on B200: faster where units have two key
// tiles (block masks with halo 0 and block 128: ~1.2x), slower where they
// have more (the rings carried across units hold slots that the next unit's
// copies wait for; per-tile period ~2.9k cycles against ~2.3k).
//
// Shutdown: every issuing thread waits for the last arrival of each barrier
// it feeds with tcgen05.commit and the producer waits for the release of
// every ring slot, so no arrival lands after tensor memory is freed.  After a
// timeout a softmax warp leaves the key loop, every warp still runs each
// unit's output write (so the named barriers match), and the copies and MMAs
// in flight are drained (bounded) before tensor memory is freed.
#pragma once

#include "tc32_ws.cuh"

namespace raya {
namespace tc32 {

constexpr int kStSplitThreads = 160;  // split warps 4-8
constexpr int kStProducer = 288;      // warp 9, lane 0: the copy producer

struct StreamSmem {
  float raw[kRawStages][2][2][kBN][32];  // ring items: a q tile [half][128][32] or K/V [K, V][half][key][32]
  float lo[kLoStages][2][2][kBN][32];    // [stage][K lo, V lo][half][key][32]
  uint64_t raw_full[kRawStages], raw_free[kRawStages];
  uint64_t k_ready[kLoStages], v_ready[kLoStages], k_free[kLoStages], v_free[kLoStages];
  uint64_t s_full, s_free, p_ready[2], pv_done[2], q_ready, q_free;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t stream_smem_bytes() { return sizeof(StreamSmem) + 1024; }
static_assert(stream_smem_bytes() <= 232448, "more shared memory than one sm_100 block may hold");
static_assert(sizeof(float) * 2 * kBM * 32 == sizeof(float) * 2 * 2 * kBN * 32, "a q tile fills one raw stage");


// One unit: rows [r0, r0 + 128) of slice bh, its valid length and key tiles.
struct StreamUnit {
  int bh;       // slice (batch * heads + head)
  int r0;       // first row
  int valid;    // valid rows of the slice, clamped to [0, seq]
  int t_begin;  // first key tile
  int ntiles;   // key tiles (0: padding only)
};

// The raw valid length of unit u's sequence (the host keeps batch * heads *
// row_tiles below 2^31).
__device__ __forceinline__ int stream_valid(const AttnArgs& a, unsigned u) {
  if (!a.valid_len) return a.seq;
  const unsigned bh = u / static_cast<unsigned>(a.row_tiles);
  return a.valid_len[bh / static_cast<unsigned>(a.heads)];
}

__device__ __noinline__ StreamUnit stream_unit(const AttnArgs& a, unsigned u, int v) {
  StreamUnit s;
  const unsigned rt = static_cast<unsigned>(a.row_tiles);
  s.bh = static_cast<int>(u / rt);
  s.r0 = static_cast<int>(u - static_cast<unsigned>(s.bh) * rt) * kBM;
  s.valid = v < 0 ? 0 : (v > a.seq ? a.seq : v);
  int klo = 0, khi = 0, unused = 0;
  if (s.r0 < s.valid) {
    key_range(a, s.r0, s.valid, klo, unused);
    key_range(a, min(s.r0 + kBM, s.valid) - 1, s.valid, unused, khi);
  }
  s.t_begin = klo / kBN;
  s.ntiles = (s.r0 < s.valid && khi > klo) ? (khi + kBN - 1) / kBN - s.t_begin : 0;
  return s;
}

// The bounded mbarrier wait with its spin loop out of line: one try_wait
// inline, the loop in one shared function, so that the per-tile loops stay
// compact in the instruction cache.
__device__ __noinline__ bool stream_wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                              long long timeout_cycles) {
  return mbar_wait_bounded(bar, parity, abort_flag, status, timeout_cycles);
}
__device__ __forceinline__ bool stream_wait(uint64_t* bar, uint32_t parity, const AttnArgs& a,
                                            volatile int* abort_flag) {
  return mbar_try_wait(bar, parity) || stream_wait_slow(bar, parity, abort_flag, a.status, a.timeout_cycles);
}

// Bounded wait for a barrier's completion number `count` (0-based), when no
// later completion can follow; true when it completed.
__device__ __forceinline__ bool stream_tail_wait(uint64_t* bar, int count, const AttnArgs& a,
                                                 volatile int* abort_flag) {
  return stream_wait(bar, static_cast<uint32_t>(count) & 1u, a, abort_flag);
}

// The last of `n` events 0..n-1 that fall on stage s of a ring of `stages`
// (-1 if none).
__device__ __forceinline__ int stream_last_on(int n, int s, int stages) {
  if (n <= s) return -1;
  return n - 1 - (n - 1 - s) % stages;
}


// Once-per-unit work lives in out-of-line functions: inlined, it would sit in
// the middle of the per-tile loops and spread their instructions over more
// instruction-cache lines (measured: several times the instruction-fetch
// stalls of tc32_ws_fwd).

// The output of a finished unit, kept by the softmax warps until its write.
struct StreamOut {
  int bh, r0;
  int row_valid;     // this thread's row is below valid_len
  float lsum;        // this thread's row sum
  int glast;         // the unit's last key tile
};

// Softmax warps (thread t = row t): O / l of unit `o` -> staged at `stage`
// ([half][128][32], 128-byte swizzle) once `stage_bar` (if any) has completed
// phase `stage_par` -> TMA store, issued and committed by thread 0.  Returns
// false after a timeout (then zeros are staged and stored).
__device__ __noinline__ bool stream_write_out(StreamSmem& sm, const AttnArgs& a, const PipeMaps& maps,
                                              uint32_t tmem_row, StreamOut o, float* stage, uint64_t* stage_bar,
                                              uint32_t stage_par, bool ok, volatile int* abort_flag) {
  const int tid = threadIdx.x;
  float acc[64];
#pragma unroll
  for (int c = 0; c < 64; ++c) acc[c] = 0.f;
  bool w = ok && stream_wait(&sm.pv_done[o.glast & 1], static_cast<uint32_t>(o.glast >> 1) & 1u, a, abort_flag);
  if (__any_sync(0xffffffffu, !w)) {
    ok = false;
  } else {
    tc_fence_after();
    tmem_ld32(tmem_row + kWsColO, acc);
    tmem_ld32(tmem_row + kWsColO + 32, acc + 32);
  }
  if (stage_bar) {
    w = ok && stream_wait(stage_bar, stage_par, a, abort_flag);
    if (__any_sync(0xffffffffu, !w)) ok = false;
  }
  // Rows at or past valid_len (and everything after a timeout) are +0.0f
  // exactly (a product with 0 would give -0.0f for negative O).
  const bool live = ok && o.row_valid;
  const float inv = (live && o.lsum > 0.f) ? 1.0f / o.lsum : 0.f;
#pragma unroll
  for (int c4 = 0; c4 < 16; ++c4)
    sts128(smem_addr(stage) + chunk_offset<kBM>(tid, c4),
           live ? make_float4(acc[4 * c4] * inv, acc[4 * c4 + 1] * inv, acc[4 * c4 + 2] * inv, acc[4 * c4 + 3] * inv)
                : make_float4(0.f, 0.f, 0.f, 0.f));
  fence_proxy_async_smem();
  bar_named(kSoftmaxBarrier, 128);
  if (tid == 0) {
#pragma unroll
    for (int half = 0; half < 2; ++half)
#pragma unroll
      for (int rb = 0; rb < 2; ++rb)
        if (o.r0 + 64 * rb < a.seq)  // (a box starting past the slice would be clipped whole; skip it)
          tma_store_3d(&maps.o, stage + half * kBM * 32 + rb * 64 * 32, 32 * half, o.r0 + 64 * rb, o.bh);
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
  return ok;
}

// Split warps: unit k's q tile (ring item qitem) -> tensor memory as q and
// q - trunc(q), once QK(k-1, last) is complete and unit k-1's q_ready phase
// has been used (q_free).  Warps 4-7 (rows st = 0..127) reach the 128 lanes.
// Returns false on a timeout (decided collectively).
__device__ __noinline__ bool stream_q_to_tmem(StreamSmem& sm, const AttnArgs& a, uint32_t tmem, int st, int r0,
                                              int valid, int qitem, int k, volatile int* abort_flag) {
  const int s4 = static_cast<int>(qitem & 3);
  bool w = stream_wait(&sm.raw_full[s4], static_cast<uint32_t>(qitem >> 2) & 1u, a, abort_flag);
  if (w && k >= 1)
    w = stream_wait(&sm.q_free, static_cast<uint32_t>(k - 1) & 1u, a, abort_flag);
  if (bar_any(kSplitBarrier, kStSplitThreads, !w)) return false;
  if (st < 128) {
    const bool rv = r0 + st < valid;
    const uint32_t qs = smem_addr(&sm.raw[s4][0][0][0][0]);
    const uint32_t lane_off = static_cast<uint32_t>(st & ~31) << 16;
    float qf[64];
#pragma unroll
    for (int c4 = 0; c4 < 16; ++c4) {
      const float4 x = rv ? lds128(qs + chunk_offset<kBM>(st, c4)) : make_float4(0.f, 0.f, 0.f, 0.f);
      qf[4 * c4] = x.x;
      qf[4 * c4 + 1] = x.y;
      qf[4 * c4 + 2] = x.z;
      qf[4 * c4 + 3] = x.w;
    }
    tmem_st32(tmem + lane_off + kWsColQh, qf);
    tmem_st32(tmem + lane_off + kWsColQh + 32, qf + 32);
#pragma unroll
    for (int i = 0; i < 64; ++i) qf[i] = tf32_lo(qf[i]);
    tmem_st32(tmem + lane_off + kWsColQl, qf);
    tmem_st32(tmem + lane_off + kWsColQl + 32, qf + 32);
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&sm.q_ready);  // QK(u, 0) may start; the softmax warps may stage over the slot
  }
  return true;
}

__global__ void __launch_bounds__(kWsThreads, 1)
    tc32_stream_fwd(const __grid_constant__ AttnArgs a, const __grid_constant__ PipeMaps maps) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  StreamSmem& sm = *reinterpret_cast<StreamSmem*>(smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr));

  const int tid = threadIdx.x, warp = tid >> 5;
  const int seq = a.seq;
  const unsigned nunits = static_cast<unsigned>(a.batch) * static_cast<unsigned>(a.heads) *
                          static_cast<unsigned>(a.row_tiles);
  const unsigned ustep = gridDim.x;

  if (warp == 10) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&sm.tmem_base)),
                 "r"(kPipeTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < kRawStages; ++s) {
      mbar_init(&sm.raw_full[s], 1);
      mbar_init(&sm.raw_free[s], 1);
    }
    for (int s = 0; s < kLoStages; ++s) {
      mbar_init(&sm.k_ready[s], kStSplitThreads);
      mbar_init(&sm.v_ready[s], kStSplitThreads);
      mbar_init(&sm.k_free[s], 1);
      mbar_init(&sm.v_free[s], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_free, 128);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.p_ready[b], 128);
      mbar_init(&sm.pv_done[b], 1);
    }
    mbar_init(&sm.q_ready, 128);  // split warps 4-7
    mbar_init(&sm.q_free, 2);     // QK(u, last) commit + softmax thread 0
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_flag = &sm.abort_flag;

  // Abort drains (registers of the threads that own them).
  int issued = 0;     // producer: ring items copied
  int mma_tiles = 0;  // QK / PV thread: key tiles whose products were issued

  // Every role walks the same units; the next unit's valid length is loaded
  // one unit ahead.
  unsigned u = blockIdx.x;
  int vcur = u < nunits ? stream_valid(a, u) : 0, vnext = 0;

  if (warp < 4) {
    // ---------------- softmax warpgroup ----------------
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float qscale = a.qscale;
    int g = 0, item = 0;  // key tiles and ring items of this CTA so far
    int k = 0;                  // units with work so far
    bool ok = true;             // false after a timeout: the unit skeleton (named barriers) still runs
    bool have_prev = false;     // a unit whose output is still in tensor memory
    StreamOut prev{};
    int release_slot = -1;  // thread 0: ring slot holding an output store still reading it

    for (; u < nunits; u += ustep, vcur = vnext) {
      const StreamUnit un = stream_unit(a, u, vcur);
      vnext = u + ustep < nunits ? stream_valid(a, u + ustep) : 0;
      if (un.ntiles == 0) {  // padding only: exact zeros
        float* outp = a.out + (static_cast<size_t>(un.bh) * seq + un.r0) * kD;
        const int rows = min(kBM, seq - un.r0);
        const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int idx = tid; idx < rows * 16; idx += 128)
          st_stream(outp + static_cast<size_t>(idx >> 4) * kD + (idx & 15) * 4, zero);
        continue;
      }
      const int row = un.r0 + tid;
      const int last = min(un.r0 + kBM, un.valid) - 1;
      const bool row_valid = row < un.valid;
      int rlo = 0, rhi = 0;
      key_range(a, min(row, last), un.valid, rlo, rhi);

      // Unit u's q tile has left its slot once q_ready completes (phase k).
      const int qslot = static_cast<int>(item & 3);
      const uint32_t qpar = static_cast<uint32_t>(k) & 1u;
      if (have_prev) {  // staged over that q tile
        ok = stream_write_out(sm, a, maps, tmem + lane_off, prev, &sm.raw[qslot][0][0][0][0], &sm.q_ready, qpar, ok,
                              abort_flag);
        if (tid == 0) release_slot = qslot;
      } else {
        bool w = true;
        if (tid == 0) {
          w = ok && stream_wait(&sm.q_ready, qpar, a, abort_flag);
          if (w) mbar_arrive(&sm.raw_free[qslot]);
        }
        if (__any_sync(0xffffffffu, !w)) ok = false;  // (warp-uniform)
      }
      if (tid == 0 && ok) mbar_arrive(&sm.q_free);  // this q_ready phase has been used
      item += 1;
      k += 1;

      float m_used = -INFINITY, lsum = 0.f;
      // (After a timeout a warp leaves the key loop; the loop has no named
      // barriers, and each unit's output write still runs.)
      for (int j = 0; ok && j < un.ntiles; ++j, ++g, ++item) {
        const int pb = static_cast<int>(g & 1);  // P buffer
        const int kt = (un.t_begin + j) * kBN;
        bool w = stream_wait(&sm.s_full, static_cast<uint32_t>(g) & 1u, a, abort_flag);
        if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
        tc_fence_after();
        float sv[64];
        tmem_ld32(tmem + lane_off + kWsColS, sv);
        tmem_ld32(tmem + lane_off + kWsColS + 32, sv + 32);
        tc_fence_before();
        mbar_arrive(&sm.s_free);  // QK(g+1) may overwrite S

        if (!(rlo <= kt && rhi >= kt + kBN)) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (static_cast<unsigned>(kt + c - rlo) >= static_cast<unsigned>(rhi - rlo)) sv[c] = -INFINITY;
        }
        float m4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
        for (int c = 4; c < 64; ++c) m4[c & 3] = fmaxf(m4[c & 3], sv[c]);
        const float mc = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * qscale;
        // Lazy rescale (as tc32_ws_fwd): move the running max only when it
        // grows by more than 2^8 (or is first set).
        float alpha = 1.f;
        if (mc > m_used + kRescaleLog2) {
          alpha = ex2(m_used - mc);  // 0 when m_used was -inf
          m_used = mc;
        }
        const float mbase = m_used == -INFINITY ? 0.f : m_used;
        float rs = 0.f;
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
          sv[c] = ex2(fmaf(sv[c], qscale, -mbase));
          sv[c + 1] = ex2(fmaf(sv[c + 1], qscale, -mbase));
          sv[c + 2] = ex2(fmaf(sv[c + 2], qscale, -mbase));
          sv[c + 3] = ex2(fmaf(sv[c + 3], qscale, -mbase));
          rs += (sv[c] + sv[c + 1]) + (sv[c + 2] + sv[c + 3]);
        }
        lsum = fmaf(lsum, alpha, rs);

        if (__any_sync(0xffffffffu, j > 0 && alpha != 1.f)) {
          // O row *= alpha once PV(g-1) is complete (O then holds this unit's tiles 0..j-1).
          w = stream_wait(&sm.pv_done[(g - 1) & 1], static_cast<uint32_t>((g - 1) >> 1) & 1u, a, abort_flag);
          if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 64; c += 32) {
            float t[32];
            tmem_ld32(tmem + lane_off + kWsColO + c, t);
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] *= alpha;
            tmem_st32(tmem + lane_off + kWsColO + c, t);
          }
        }
        if (g >= 2) {  // P buffer pb is free once PV(g-2) is complete
          w = stream_wait(&sm.pv_done[pb], static_cast<uint32_t>((g - 2) >> 1) & 1u, a, abort_flag);
          if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
          tc_fence_after();
        }
        const uint32_t ph = tmem + lane_off + ws_col_ph(pb);
        tmem_st32(ph, sv);
        tmem_st32(ph + 32, sv + 32);
#pragma unroll
        for (int c = 0; c < 64; ++c) sv[c] = tf32_lo(sv[c]);
        tmem_st32(ph + 64, sv);
        tmem_st32(ph + 96, sv + 32);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&sm.p_ready[pb]);
        if (j == 0 && tid == 0 && release_slot >= 0) {
          // The previous output store has long been issued: once it has read
          // its staging slot, the producer may refill it.
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
          mbar_arrive(&sm.raw_free[release_slot]);
          release_slot = -1;
        }
      }
      have_prev = true;
      prev.bh = un.bh;
      prev.r0 = un.r0;
      prev.row_valid = row_valid;
      prev.lsum = lsum;
      prev.glast = g - 1;
    }
    if (have_prev) {
      // Every copy has been consumed and every product is complete once
      // PV(last) is: raw stage 0 is idle.
      ok = stream_write_out(sm, a, maps, tmem + lane_off, prev, &sm.raw[0][0][0][0][0], nullptr, 0u, ok, abort_flag);
      if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      // The other P buffer's last PV commit (the final write waited for this one's).
      if (tid == 0 && ok && g >= 2) ok = stream_tail_wait(&sm.pv_done[(g - 2) & 1], (g - 2) >> 1, a, abort_flag);
    }
  } else if (warp < 9) {
    // ---------------- split warps ----------------
    const int st = tid - 128;
    constexpr int kPer = (kBN * 16 + kStSplitThreads - 1) / kStSplitThreads;  // float4s per thread per tile
    int g = 0, item = 0;
    int k = 0;
    bool ok = true;
    for (; ok && u < nunits; u += ustep, vcur = vnext) {
      const StreamUnit un = stream_unit(a, u, vcur);
      vnext = u + ustep < nunits ? stream_valid(a, u + ustep) : 0;
      if (un.ntiles == 0) continue;
      const int qitem = item;  // the unit's q tile; moved after the first key tile's K split
      item += 1;
      for (int j = 0; j < un.ntiles; ++j, ++g, ++item) {
        const int s3 = static_cast<int>(g % kLoStages), s4 = static_cast<int>(item & 3);
        const uint32_t ph = static_cast<uint32_t>(g / kLoStages - 1) & 1u;  // phase of tile g-3's release
        bool w = stream_wait(&sm.raw_full[s4], static_cast<uint32_t>(item >> 2) & 1u, a, abort_flag);
        if (w && g >= kLoStages) w = stream_wait(&sm.k_free[s3], ph, a, abort_flag);
        if (bar_any(kSplitBarrier, kStSplitThreads, !w)) { ok = false; break; }
        const int nv = min(kBN, un.valid - (un.t_begin + j) * kBN);
        float4* kr = reinterpret_cast<float4*>(&sm.raw[s4][0][0][0][0]);
        float4* vr = reinterpret_cast<float4*>(&sm.raw[s4][1][0][0][0]);
        float4* kl = reinterpret_cast<float4*>(&sm.lo[s3][0][0][0][0]);
        float4* vl = reinterpret_cast<float4*>(&sm.lo[s3][1][0][0][0]);
        {
          float4 x[kPer];
#pragma unroll
          for (int i = 0; i < kPer; ++i)
            if (st + i * kStSplitThreads < kBN * 16) x[i] = kr[st + i * kStSplitThreads];
#pragma unroll
          for (int i = 0; i < kPer; ++i)
            if (st + i * kStSplitThreads < kBN * 16)
              kl[st + i * kStSplitThreads] =
                  make_float4(tf32_lo(x[i].x), tf32_lo(x[i].y), tf32_lo(x[i].z), tf32_lo(x[i].w));
        }
        fence_proxy_async_smem();      // generic-proxy writes -> visible to the tensor core
        mbar_arrive(&sm.k_ready[s3]);  // QK(g) may start
        if (j == 0) {
          if (!stream_q_to_tmem(sm, a, tmem, st, un.r0, un.valid, qitem, k, abort_flag)) { ok = false; break; }
          k += 1;
        }
        w = true;
        if (g >= kLoStages) w = stream_wait(&sm.v_free[s3], ph, a, abort_flag);
        if (bar_any(kSplitBarrier, kStSplitThreads, !w)) { ok = false; break; }
        {
          float4 x[kPer];
#pragma unroll
          for (int i = 0; i < kPer; ++i)
            if (st + i * kStSplitThreads < kBN * 16) x[i] = vr[st + i * kStSplitThreads];
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            const int f = st + i * kStSplitThreads;
            if (f < kBN * 16) {
              if (((f % (kBN * 8)) >> 3) < nv) {
                vl[f] = make_float4(tf32_lo(x[i].x), tf32_lo(x[i].y), tf32_lo(x[i].z), tf32_lo(x[i].w));
              } else {  // the tail tile: V rows at or past valid_len become exact zeros in both parts
                vr[f] = make_float4(0.f, 0.f, 0.f, 0.f);
                vl[f] = make_float4(0.f, 0.f, 0.f, 0.f);
              }
            }
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&sm.v_ready[s3]);
      }
    }
  } else if (tid == kStProducer) {
    // ---------------- copy producer ----------------
    // Every ring item in order, each into slot issued % 4 as soon as the item
    // four places earlier has been released (raw_free: PV of a K/V item; the
    // softmax warps for a q tile, once it has been read and, when it staged
    // an output, once that store has read it).
    bool ok = true;
    for (; ok && u < nunits; u += ustep, vcur = vnext) {
      const StreamUnit un = stream_unit(a, u, vcur);
      vnext = u + ustep < nunits ? stream_valid(a, u + ustep) : 0;
      if (un.ntiles == 0) continue;
      const int row_base = un.bh * seq;
      for (int j = -1; ok && j < un.ntiles; ++j) {  // j = -1: the q tile (units with work only)
        const int s = issued & 3;
        if (issued >= kRawStages)
          ok = stream_wait(&sm.raw_free[s], static_cast<uint32_t>((issued >> 2) - 1) & 1u, a, abort_flag);
        if (!ok) break;
        uint64_t* bar = &sm.raw_full[s];
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(bar, 2u * kBN * kD * 4u);  // = kBM * kD * 4 for a q tile
        if (j < 0) {
          float* qs = &sm.raw[s][0][0][0][0];  // [half][128 rows][32]
#pragma unroll
          for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int rb = 0; rb < 2; ++rb)
              tiled64::tma_load_2d(qs + half * kBM * 32 + rb * 64 * 32, &maps.q, 32 * half, row_base + un.r0 + 64 * rb,
                                   bar);
        } else {
          const int y = row_base + (un.t_begin + j) * kBN;
          tiled64::tma_load_2d(&sm.raw[s][0][0][0][0], &maps.k, 0, y, bar);
          tiled64::tma_load_2d(&sm.raw[s][0][1][0][0], &maps.k, 32, y, bar);
          tiled64::tma_load_2d(&sm.raw[s][1][0][0][0], &maps.v, 0, y, bar);
          tiled64::tma_load_2d(&sm.raw[s][1][1][0][0], &maps.v, 32, y, bar);
        }
        ++issued;
      }
    }
    // Tail: the release of every ring slot's last item (the PV commits among
    // them included).
    for (int s = 0; ok && s < kRawStages; ++s) {
      const int t = stream_last_on(issued, s, kRawStages);
      if (t >= 0) ok = stream_tail_wait(&sm.raw_free[s], t >> 2, a, abort_flag);
    }
  } else if (tid == kWsQkThread) {
    // ---------------- QK^T issuer ----------------
    int item = 0;
    int k = 0;
    bool ok = true;
    for (; ok && u < nunits; u += ustep, vcur = vnext) {
      const StreamUnit un = stream_unit(a, u, vcur);
      vnext = u + ustep < nunits ? stream_valid(a, u + ustep) : 0;
      if (un.ntiles == 0) continue;
      ok = stream_wait(&sm.q_ready, static_cast<uint32_t>(k) & 1u, a, abort_flag);
      item += 1;
      const uint32_t qh = tmem + kWsColQh, ql = tmem + kWsColQl;
      for (int j = 0; ok && j < un.ntiles; ++j, ++item) {
        const int g = mma_tiles;
        const int s3 = static_cast<int>(g % kLoStages);
        ok = stream_wait(&sm.k_ready[s3], static_cast<uint32_t>(g / kLoStages) & 1u, a, abort_flag);
        if (ok && g >= 1)  // the softmax has read S(g-1)
          ok = stream_wait(&sm.s_free, static_cast<uint32_t>(g - 1) & 1u, a, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t khi = smem_addr(&sm.raw[item & 3][0][0][0][0]);
        const uint32_t klo = smem_addr(&sm.lo[s3][0][0][0][0]);
        const uint32_t d = tmem + kWsColS;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) mma_tf32_ts(d, qh + 8 * kk, k_desc(klo, kk), kIdescQK, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) mma_tf32_ts(d, ql + 8 * kk, k_desc(khi, kk), kIdescQK, 1u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) mma_tf32_ts(d, qh + 8 * kk, k_desc(khi, kk), kIdescQK, 1u);
        mma_commit(&sm.s_full);
        mma_commit(&sm.k_free[s3]);
        if (j + 1 == un.ntiles) mma_commit(&sm.q_free);  // tensor memory may take unit k+1's q
        ++mma_tiles;
      }
      k += 1;
    }
    // Tail: the last commits nobody else waits for: k_free of each lo stage
    // and the last q_free.
    for (int s = 0; ok && s < kLoStages; ++s) {
      const int t = stream_last_on(mma_tiles, s, kLoStages);
      if (t >= 0) ok = stream_tail_wait(&sm.k_free[s], t / kLoStages, a, abort_flag);
    }
    if (ok && k > 0) ok = stream_tail_wait(&sm.q_free, k - 1, a, abort_flag);
  } else if (tid == kWsPvThread) {
    // ---------------- PV issuer ----------------
    int item = 0;
    bool ok = true;
    for (; ok && u < nunits; u += ustep, vcur = vnext) {
      const StreamUnit un = stream_unit(a, u, vcur);
      vnext = u + ustep < nunits ? stream_valid(a, u + ustep) : 0;
      if (un.ntiles == 0) continue;
      item += 1;
      for (int j = 0; ok && j < un.ntiles; ++j, ++item) {
        const int g = mma_tiles;
        const int s3 = static_cast<int>(g % kLoStages);
        const int pb = static_cast<int>(g & 1);
        ok = stream_wait(&sm.p_ready[pb], static_cast<uint32_t>(g >> 1) & 1u, a, abort_flag) &&
             stream_wait(&sm.v_ready[s3], static_cast<uint32_t>(g / kLoStages) & 1u, a, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t vh = smem_addr(&sm.raw[item & 3][1][0][0][0]);
        const uint32_t vl = smem_addr(&sm.lo[s3][1][0][0][0]);
        const uint32_t d = tmem + kWsColO, aph = tmem + ws_col_ph(pb), apl = aph + 64;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // the unit's first product overwrites O
          mma_tf32_ts(d, aph + 8 * kk, v_desc(vl, kk), kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) mma_tf32_ts(d, apl + 8 * kk, v_desc(vh, kk), kIdescPV, 1u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) mma_tf32_ts(d, aph + 8 * kk, v_desc(vh, kk), kIdescPV, 1u);
        mma_commit(&sm.pv_done[pb]);
        mma_commit(&sm.v_free[s3]);
        mma_commit(&sm.raw_free[item & 3]);
        ++mma_tiles;
      }
    }
    // Tail: the last v_free commit of each lo stage (raw_free: the producer's
    // tail; pv_done: the softmax warps').
    for (int s = 0; ok && s < kLoStages; ++s) {
      const int t = stream_last_on(mma_tiles, s, kLoStages);
      if (t >= 0) ok = stream_tail_wait(&sm.v_free[s], t / kLoStages, a, abort_flag);
    }
  }
  __syncwarp();

  // Release tensor memory (every path); after a timeout first drain this
  // CTA's copies and MMAs still in flight (bounded).
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    const long long t0 = clock64();
    auto drain = [&](uint64_t* bar, uint32_t parity) {
      while (!mbar_try_wait(bar, parity) && clock64() - t0 < a.timeout_cycles) {
      }
    };
    if (tid == kStProducer) {  // the last item copied into each raw slot
#pragma unroll
      for (int s = 0; s < kRawStages; ++s) {
        const int t = stream_last_on(issued, s, kRawStages);
        if (t >= 0) drain(&sm.raw_full[s], static_cast<uint32_t>(t >> 2) & 1u);
      }
    }
    if (tid == kWsQkThread && mma_tiles > 0) drain(&sm.s_full, static_cast<uint32_t>(mma_tiles - 1) & 1u);
    if (tid == kWsPvThread && mma_tiles > 0)
      drain(&sm.pv_done[(mma_tiles - 1) & 1], static_cast<uint32_t>((mma_tiles - 1) >> 1) & 1u);
    if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  __syncthreads();
  if (warp == 10) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPipeTmemCols) : "memory");
  }
}

}  // namespace tc32
}  // namespace raya
