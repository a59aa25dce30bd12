// tc32_pair.cuh — 3xTF32 tensor-core attention over PAIRS of 128-row tiles
// that share one K/V stream (sm_100a).
//
// One CTA per (slice, 256 query rows): unit A = rows [r0, r0 + 128), unit B =
// rows [r0 + 128, r0 + 256).  Their key ranges overlap (a block-local mask at
// halo 1 gives A tiles t..t+5 and B tiles t+2..t+7 at block 128), so each K/V
// tile of the union is loaded and split into its TF32 hi/lo operands once
// and feeds up to four products (QK^T and PV of A and of B).  Two softmax
// warpgroups, one per unit, run side by side: while one works on its scores
// the tensor core runs the other's products, and one unit's output store
// overlaps the other's last tiles.
//
// Accuracy.  The tensor core's accumulation into tensor memory is biased
// toward zero (measured: outputs shrink by ~2e-6 relative per 64-key tile
// when every tile's PV accumulates into one tensor-memory block, 5.7e-5 at
// 128 tiles).  Here each tile's PV goes into a fresh per-unit partial (one
// 24-product chain), and every softmax thread adds the partial into its O
// row in fp32 registers with round-to-nearest adds.
//
// Roles (384 threads):
//   warps 0-3   softmax of unit A: one query row per thread (TMEM lane = row
//               within the unit): S row -> mask -> online softmax (running
//               log2-domain max moved only when it grows by more than 2^8)
//               -> P and its lo part into tensor memory -> the previous
//               tile's PV partial into the O row in registers; at the end
//               O / l staged in shared memory (over the unit's q tile) and
//               stored by TMA.
//   warps 4-7   the same for unit B.
//   warps 8-9   split: per key tile the lo parts of K and of V (V rows at or
//               past valid_len zeroed in both), the K chain one tile ahead of
//               the V chain, and the TMA copies of the tiles after them.
//               (Each softmax thread takes its own q row's lo part first.)
//   warp 10     QK issuer (and tensor-memory allocation): QK(A, g), QK(B, g)
//               once K's lo part of tile g is ready and each unit's previous
//               S has been read; q tiles are shared-memory operands.
//   warp 11     PV issuer: PV(A, g), PV(B, g) into the units' partials once
//               their P and V's lo part are ready.
//               Both issuers run their loops on the whole warp and issue from
//               one elected lane: a chain of MMAs into one accumulator then
//               runs at ~64 cycles per MMA instead of ~120 (one lane in a
//               divergent branch), and the two chains together keep the
//               tensor core at its ~32.
//
// Shared memory (224 KB): both units' q tiles and their lo parts (the A
// operands of QK^T, 128 KB), rings of two raw K and two raw V tiles (TMA
// targets, the hi operands), one K lo and one V lo stage.  K and V are
// released separately (k_free by QK, v_free by PV), so the copy of K(g+2)
// leaves as soon as both QK(g) are done.
// Tensor memory (512 columns), per unit u at 256 u: S [0, 64), P hi
// [64, 128), P lo [128, 192), PV partial [192, 256).
// Every wait is bounded; every group's exit is a collective decision of that
// group; after a timeout the issuing threads drain their copies and MMAs
// (bounded) before tensor memory is freed.
#pragma once

#include "tc32_common.cuh"

namespace raya {
namespace tc32 {

constexpr int kPairThreads = 384;
constexpr int kPairSplitThreads = 64;  // warps 8-9
constexpr int kPairSplitTid0 = 256;
constexpr int kPairQkThread = 320;  // warp 10, lane 0
constexpr int kPairPvThread = 352;  // warp 11, lane 0
constexpr int kPairSplitBarrier = 1;
constexpr int kPairSoftmaxBarrier = 2;  // + unit
constexpr uint32_t kPairColUnit = 256, kPairColS = 0, kPairColPh = 64, kPairColPl = 128, kPairColPv = 192;
constexpr float kPairRescaleLog2 = 8.0f;
// Register split (setmaxnreg): the two softmax warp groups hold an O row
// (64 floats) next to a score row; the split/issue warp group needs few.
// 2 * 128 * 200 + 128 * 104 = 64,512 = 384 threads * the 168 registers a
// thread of this launch gets, so the increase never waits on the pool.
#ifndef RAYA_PAIR_SOFTMAX_REGS
#define RAYA_PAIR_SOFTMAX_REGS 200
#define RAYA_PAIR_OTHER_REGS 104
#endif
constexpr int kPairSoftmaxRegs = RAYA_PAIR_SOFTMAX_REGS, kPairOtherRegs = RAYA_PAIR_OTHER_REGS;
static_assert(2 * 128 * kPairSoftmaxRegs + 128 * kPairOtherRegs <= kPairThreads * 168,
              "register split above the launch's allocation");

struct PairSmem {
  float q[2][2][2][kBM][32];  // [unit][hi, lo][column half][row][32]: A operands of QK^T
  float kraw[2][2][kBN][32];  // [stage][half][key][32]: K tiles (TMA), the hi operands
  float vraw[2][2][kBN][32];  // V tiles (TMA, 32-byte-granule swizzle)
  float klo[2][kBN][32];      // K lo (one stage)
  float vlo[2][kBN][32];      // V lo (one stage)
  uint64_t q_full, q_ready[2];
  uint64_t k_full[2], v_full[2];
  uint64_t k_ready, v_ready, k_free, v_free;
  uint64_t s_full[2], s_free[2], p_ready[2], pv_done[2];
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t pair_smem_bytes() { return sizeof(PairSmem) + 1024; }
static_assert(pair_smem_bytes() <= 232448, "more shared memory than one sm_100 block may hold");

// a.row_tiles = 256-row pairs per (batch, head) slice; grid = batch * heads * pairs.
// TIMED: the stage-timing build (the counterpart of the reference's
// StageTimes, tiled/stages.rs:1-31), cycles added per unit into
// a.stage_cycles: [kStageQk] QK^T products in flight (first issue to
// completion, seen by the QK issuer, which in this build waits for each QK),
// [kStageSoftmax] one softmax warp's work per tile (S read to P stored),
// [kStagePv] PV products in flight (the PV issuer waits for each), [kStageKWait]
// the QK issuer waiting for K's split, [kStageVWait] the PV issuer waiting for
// P and V's split, [kStageRefill] one split warp's operand preparation,
// [kStageTiles] unit key tiles, [kStageTotal] a softmax warp's cycles from the
// CTA's start to its output store.  The stages overlap in time.
template <bool TIMED = false>
__global__ void __launch_bounds__(kPairThreads, 1)
    tc32_pair_fwd(const __grid_constant__ AttnArgs a, const __grid_constant__ PipeMaps maps) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  PairSmem& sm = *reinterpret_cast<PairSmem*>(smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr));

  const int tid = threadIdx.x, warp = tid >> 5;
  const int seq = a.seq;
  // 32-bit index math (the host keeps batch * heads * pairs below 2^31).
  const unsigned pairs = static_cast<unsigned>(a.row_tiles);
  const unsigned bh32 = blockIdx.x / pairs;
  const int pt = static_cast<int>(blockIdx.x - bh32 * pairs);
  const unsigned b32 = bh32 / static_cast<unsigned>(a.heads);
  const int valid_raw = a.valid_len ? a.valid_len[b32] : seq;
  const long long row_base = static_cast<long long>(bh32) * seq;  // this slice's first row

  if (tid == 0) {  // barrier set-up needs no valid length: it overlaps that load
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_free[s], 128);
      mbar_init(&sm.p_ready[s], 128);
      mbar_init(&sm.pv_done[s], 1);
      mbar_init(&sm.q_ready[s], 128);
    }
    mbar_init(&sm.k_ready, kPairSplitThreads);
    mbar_init(&sm.v_ready, kPairSplitThreads);
    mbar_init(&sm.k_free, 1);
    mbar_init(&sm.v_free, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  const int valid = valid_raw < 0 ? 0 : (valid_raw > seq ? seq : valid_raw);

  // The two units: rows, activity, key-tile ranges [t0, t1); the union [g0, g0 + n).
  int r0[2], t0[2], t1[2], lastrow[2];
  bool act[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    r0[u] = pt * 2 * kBM + u * kBM;
    act[u] = r0[u] < valid;
    t0[u] = t1[u] = 0;
    lastrow[u] = 0;
    if (act[u]) {
      int lo = 0, hi = 0, x = 0;
      lastrow[u] = min(r0[u] + kBM, valid) - 1;
      key_range(a, r0[u], valid, lo, x);
      key_range(a, lastrow[u], valid, x, hi);
      if (hi > lo) {
        t0[u] = lo / kBN;
        t1[u] = (hi + kBN - 1) / kBN;
      } else {
        act[u] = false;
      }
    }
  }
  const int g0 = act[0] ? (act[1] ? min(t0[0], t0[1]) : t0[0]) : t0[1];
  const int g1 = act[0] ? (act[1] ? max(t1[0], t1[1]) : t1[0]) : t1[1];
  const int n = (act[0] || act[1]) ? g1 - g0 : 0;
  float* __restrict__ outp = a.out + static_cast<size_t>(row_base) * kD;

  if (n <= 0) {  // padding only: exact zeros, no loads, no tensor memory
    const int rend = min(r0[0] + 2 * kBM, seq);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int idx = tid; idx < (rend - r0[0]) * 16; idx += kPairThreads)
      st_stream(outp + static_cast<size_t>(r0[0] + (idx >> 4)) * kD + (idx & 15) * 4, zero);
    return;
  }

  if (warp == 10) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&sm.tmem_base)),
                 "r"(kPipeTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Copies of K/V tile gg of the union into raw stage gg % 2.
  auto copy_k = [&](int gg) {
    const int s = gg & 1;
    const int y = static_cast<int>(row_base + static_cast<long long>(g0 + gg) * kBN);
    mbar_arrive_expect_tx(&sm.k_full[s], kBN * kD * 4u);
    tiled64::tma_load_2d(&sm.kraw[s][0][0][0], &maps.k, 0, y, &sm.k_full[s]);
    tiled64::tma_load_2d(&sm.kraw[s][1][0][0], &maps.k, 32, y, &sm.k_full[s]);
  };
  auto copy_v = [&](int gg) {
    const int s = gg & 1;
    const int y = static_cast<int>(row_base + static_cast<long long>(g0 + gg) * kBN);
    mbar_arrive_expect_tx(&sm.v_full[s], kBN * kD * 4u);
    tiled64::tma_load_2d(&sm.vraw[s][0][0][0], &maps.v, 0, y, &sm.v_full[s]);
    tiled64::tma_load_2d(&sm.vraw[s][1][0][0], &maps.v, 32, y, &sm.v_full[s]);
  };
  if (tid == 0) {
    // The active units' q tiles (four [64 rows][32] boxes each), then K/V tile 0.
    mbar_arrive_expect_tx(&sm.q_full, (act[0] + act[1]) * kBM * kD * 4u);
#pragma unroll
    for (int u = 0; u < 2; ++u)
      if (act[u])
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
          for (int rb = 0; rb < 2; ++rb)
            tiled64::tma_load_2d(&sm.q[u][0][half][rb * 64][0], &maps.q, 32 * half,
                                 static_cast<int>(row_base + r0[u] + 64 * rb), &sm.q_full);
    copy_k(0);
    copy_v(0);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0 && n > 1) {
    copy_k(1);
    copy_v(1);
  }
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_flag = &sm.abort_flag;
  long long c_start = 0;
  if constexpr (TIMED) c_start = clock64();

  // Drain bookkeeping (registers of the issuing threads).
  int last_k = min(2, n) - 1, last_v = min(2, n) - 1;  // split thread 0: last tiles copied (the first two by thread 0)
  uint64_t* last_commit = nullptr;
  uint32_t last_commit_parity = 0;
  auto commit = [&](uint64_t* bar, uint32_t parity) {  // the issuing warps: one elected lane commits
    mma_commit_e(bar);
    last_commit = bar;
    last_commit_parity = parity;
  };
  // A bounded wait whose outcome is the same on every lane of the warp.
  auto warp_wait = [&](uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, a.status, a.timeout_cycles));
  };
  // Whether unit u uses union tile g, and the unit's own index of it.
  auto uses = [&](int u, int g) { return act[u] && g0 + g >= t0[u] && g0 + g < t1[u]; };

  if (warp < 8)
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPairSoftmaxRegs));
  else
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPairOtherRegs));
  if (warp < 8) {
    // ---------------- softmax warpgroups (unit u = warp / 4) ----------------
    const int u = warp >> 2;
    const int r = (warp & 3) * 32 + (tid & 31);  // row within the unit = TMEM lane
    const int row = r0[u] + r;
    const int nu = act[u] ? t1[u] - t0[u] : 0;
    int rlo = 0, rhi = 0;
    if (act[u]) key_range(a, min(row, lastrow[u]), valid, rlo, rhi);
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t ucol = tmem + lane_off + kPairColUnit * static_cast<uint32_t>(u);
    const float qscale = a.qscale;
    bool ok = true;
    if (act[u]) {  // this row's q lo (the tensor core reads the raw q tile as q's hi part)
      const bool w = mbar_wait_bounded(&sm.q_full, 0, abort_flag, a.status, a.timeout_cycles);
      if (__any_sync(0xffffffffu, !w)) ok = false;
      if (ok) {
        const uint32_t qh = smem_addr(&sm.q[u][0][0][0][0]), ql = smem_addr(&sm.q[u][1][0][0][0]);
#pragma unroll
        for (int c4 = 0; c4 < 16; ++c4) {
          const uint32_t off = chunk_offset<kBM>(r, c4);
          const float4 x = lds128(qh + off);
          sts128(ql + off, make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w)));
        }
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        mbar_arrive(&sm.q_ready[u]);
      }
    }
    float o[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) o[c] = 0.f;
    float m_used = -INFINITY, lsum = 0.f;
    unsigned long long c_sm = 0;
    for (int j = 0; ok && j < nu; ++j) {
      const int kt = (t0[u] + j) * kBN;
      bool w = mbar_wait_bounded(&sm.s_full[u], static_cast<uint32_t>(j) & 1u, abort_flag, a.status,
                                 a.timeout_cycles);
      if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
      tc_fence_after();
      long long c_s0 = 0;
      if constexpr (TIMED) c_s0 = clock64();
      float sv[64];
      tmem_ld32(ucol + kPairColS, sv);
      tmem_ld32(ucol + kPairColS + 32, sv + 32);
      tc_fence_before();
      mbar_arrive(&sm.s_free[u]);  // QK(u, j+1) may overwrite S

      if (!(rlo <= kt && rhi >= kt + kBN)) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (static_cast<unsigned>(kt + c - rlo) >= static_cast<unsigned>(rhi - rlo)) sv[c] = -INFINITY;
      }
      float m4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int c = 4; c < 64; ++c) m4[c & 3] = fmaxf(m4[c & 3], sv[c]);
      const float mc = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * qscale;
      // Move the running max only when it grows by more than 2^8 (or is
      // first set): O and l are then rescaled by alpha; otherwise weights
      // stay below 2^8 relative to the kept max.
      float alpha = 1.f;
      if (mc > m_used + kPairRescaleLog2) {
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
      if (j > 0) {  // P and the PV partial are free once PV(u, j-1) is complete
        w = mbar_wait_bounded(&sm.pv_done[u], static_cast<uint32_t>(j - 1) & 1u, abort_flag, a.status,
                              a.timeout_cycles);
        if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
        tc_fence_after();
      }
      // P -> tensor memory: p itself (read as its hi part), then p - trunc(p).
      tmem_st32(ucol + kPairColPh, sv);
      tmem_st32(ucol + kPairColPh + 32, sv + 32);
#pragma unroll
      for (int c = 0; c < 64; ++c) sv[c] = tf32_lo(sv[c]);
      tmem_st32(ucol + kPairColPl, sv);
      tmem_st32(ucol + kPairColPl + 32, sv + 32);
      if (j > 0) {
        // O = (O + PV partial of tile j-1) * alpha, both at the previous scale.
        const bool rescale = __any_sync(0xffffffffu, alpha != 1.f);
#pragma unroll
        for (int h = 0; h < 64; h += 32) {
          float t[32];
          tmem_ld32(ucol + kPairColPv + h, t);
          if (rescale) {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[h + i] = __fmul_rn(__fadd_rn(o[h + i], t[i]), alpha);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[h + i] = __fadd_rn(o[h + i], t[i]);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&sm.p_ready[u]);  // PV(u, j) may start (and overwrite the partial)
      if constexpr (TIMED) c_sm += static_cast<unsigned long long>(clock64() - c_s0);
    }
    if (ok && nu > 0) {  // the last tile's partial
      const bool w = mbar_wait_bounded(&sm.pv_done[u], static_cast<uint32_t>(nu - 1) & 1u, abort_flag, a.status,
                                       a.timeout_cycles);
      if (!__any_sync(0xffffffffu, !w)) {
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < 64; h += 32) {
          float t[32];
          tmem_ld32(ucol + kPairColPv + h, t);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[h + i] = __fadd_rn(o[h + i], t[i]);
        }
      }
    }
    // This row, normalised (+0.0f past valid_len), staged over the unit's q
    // tile (every QK of the unit is complete: its last S was read) under the
    // 128-byte swizzle, then stored by TMA: the [slices][seq][64] map clips
    // rows past the slice's end.
    {
      const float inv = (row < valid && lsum > 0.f) ? 1.0f / lsum : 0.f;
      float* stage = &sm.q[u][0][0][0][0];  // [half][128 rows][32]
#pragma unroll
      for (int c4 = 0; c4 < 16; ++c4) {
        const float4 x = row < valid ? make_float4(o[4 * c4] * inv, o[4 * c4 + 1] * inv, o[4 * c4 + 2] * inv,
                                                   o[4 * c4 + 3] * inv)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        sts128(smem_addr(stage) + chunk_offset<kBM>(r, c4), x);
      }
      fence_proxy_async_smem();
      bar_named(kPairSoftmaxBarrier + u, 128);
      if (r == 0) {
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
          for (int rb = 0; rb < 2; ++rb)
            if (r0[u] + 64 * rb < seq)  // (a box starting past the slice would be clipped whole; skip it)
              tma_store_3d(&maps.o, stage + half * kBM * 32 + rb * 64 * 32, 32 * half, r0[u] + 64 * rb,
                           static_cast<int>(bh32));
        tma_store_commit_and_wait_read();
        if constexpr (TIMED) {
          atomicAdd(&a.stage_cycles[kStageSoftmax], c_sm);
          atomicAdd(&a.stage_cycles[kStageTiles], static_cast<unsigned long long>(nu));
          atomicAdd(&a.stage_cycles[kStageTotal], static_cast<unsigned long long>(clock64() - c_start));
        }
      }
    }
  } else if (warp < 10) {
    // ---------------- split warps ----------------
    const int st = tid - kPairSplitTid0;
    unsigned long long c_split = 0;
    auto issue_k = [&](int gg) {
      fence_proxy_async_smem();
      copy_k(gg);
      last_k = gg;
    };
    auto issue_v = [&](int gg) {
      fence_proxy_async_smem();  // this stage's zeroed rows (generic proxy) before the copy overwrites them
      copy_v(gg);
      last_v = gg;
    };
    constexpr int kPer = kBN * 16 / kPairSplitThreads;  // float4s per thread per tile
    // K's lo part of union tile gg (into the one K lo stage).
    auto split_k = [&](int gg) {
      long long c_k0 = 0;
      if constexpr (TIMED) c_k0 = clock64();
      const float4* kr = reinterpret_cast<const float4*>(&sm.kraw[gg & 1][0][0][0]);
      float4* kl = reinterpret_cast<float4*>(&sm.klo[0][0][0]);
      float4 x[kPer];
#pragma unroll
      for (int i = 0; i < kPer; ++i) x[i] = kr[st + i * kPairSplitThreads];
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        kl[st + i * kPairSplitThreads] = make_float4(tf32_lo(x[i].x), tf32_lo(x[i].y), tf32_lo(x[i].z), tf32_lo(x[i].w));
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      mbar_arrive(&sm.k_ready);  // QK(gg) may start
      if constexpr (TIMED) c_split += static_cast<unsigned long long>(clock64() - c_k0);
    };
    // The K chain runs one tile ahead of the V chain: K lo(g+1) is written as
    // soon as both QK(g) are done (while the tensor core runs PV(g-1)), V lo(g)
    // once both PV(g-1) are done (while it runs QK(g+1)).
    bool w = mbar_wait_bounded(&sm.k_full[0], 0, abort_flag, a.status, a.timeout_cycles);
    if (!bar_any(kPairSplitBarrier, kPairSplitThreads, !w)) {
      split_k(0);
      for (int g = 0; g < n; ++g) {
        if (g + 1 < n) {
          // K(g+1): its raw tile, and the K lo stage (both QK(g) done).
          w = mbar_wait_bounded(&sm.k_full[(g + 1) & 1], static_cast<uint32_t>((g + 1) >> 1) & 1u, abort_flag,
                                a.status, a.timeout_cycles);
          if (w)
            w = mbar_wait_bounded(&sm.k_free, static_cast<uint32_t>(g) & 1u, abort_flag, a.status, a.timeout_cycles);
          if (bar_any(kPairSplitBarrier, kPairSplitThreads, !w)) break;
          split_k(g + 1);
          // raw K stage g % 2 held tile g, released by k_free(g)
          if (st == 0 && g + 2 < n) issue_k(g + 2);
        }
        // V(g): its raw tile, and the V lo stage (both PV(g-1) done).
        w = mbar_wait_bounded(&sm.v_full[g & 1], static_cast<uint32_t>(g >> 1) & 1u, abort_flag, a.status,
                              a.timeout_cycles);
        if (w && g > 0)
          w = mbar_wait_bounded(&sm.v_free, static_cast<uint32_t>(g - 1) & 1u, abort_flag, a.status,
                                a.timeout_cycles);
        if (bar_any(kPairSplitBarrier, kPairSplitThreads, !w)) break;
        long long c_v0 = 0;
        if constexpr (TIMED) c_v0 = clock64();
        {
          const int nv = min(kBN, valid - (g0 + g) * kBN);
          float4* vr = reinterpret_cast<float4*>(&sm.vraw[g & 1][0][0][0]);
          float4* vl = reinterpret_cast<float4*>(&sm.vlo[0][0][0]);
          float4 x[kPer];
#pragma unroll
          for (int i = 0; i < kPer; ++i) x[i] = vr[st + i * kPairSplitThreads];
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            const int f = st + i * kPairSplitThreads;
            if (((f % (kBN * 8)) >> 3) < nv) {
              vl[f] = make_float4(tf32_lo(x[i].x), tf32_lo(x[i].y), tf32_lo(x[i].z), tf32_lo(x[i].w));
            } else {  // V rows at or past valid_len become exact zeros in both parts
              vr[f] = make_float4(0.f, 0.f, 0.f, 0.f);
              vl[f] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&sm.v_ready);  // PV(g) may start
        if constexpr (TIMED) c_split += static_cast<unsigned long long>(clock64() - c_v0);
        // raw V stage (g+1) % 2 held tile g-1, released by v_free(g-1); its
        // zeroed rows (written at step g-1) are ordered by the barrier above
        if (st == 0 && g >= 1 && g + 1 < n) issue_v(g + 1);
      }
    }
    if constexpr (TIMED)
      if (st == 0) atomicAdd(&a.stage_cycles[kStageRefill], c_split);
  } else if (warp == kPairQkThread / 32) {
    // ---------------- QK^T issuer (the whole warp runs the loop; an elected lane issues) ----------------
    unsigned long long c_qk = 0, c_kw = 0;
    bool ok = true;
    for (int u = 0; u < 2 && ok; ++u)
      if (act[u]) ok = warp_wait(&sm.q_ready[u], 0);
    for (int g = 0; ok && g < n; ++g) {
      long long c_w0 = 0;
      if constexpr (TIMED) c_w0 = clock64();
      ok = warp_wait(&sm.k_ready, static_cast<uint32_t>(g) & 1u);
      if constexpr (TIMED) c_kw += static_cast<unsigned long long>(clock64() - c_w0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t khi = smem_addr(&sm.kraw[g & 1][0][0][0]);
      const uint32_t klo = smem_addr(&sm.klo[0][0][0]);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!ok || !uses(u, g)) continue;
        const int j = g0 + g - t0[u];
        if (j > 0) {  // the softmax has read S(u, j-1)
          ok = warp_wait(&sm.s_free[u], static_cast<uint32_t>(j - 1) & 1u);
          if (!ok) break;
          tc_fence_after();
        }
        long long c_i0 = 0;
        if constexpr (TIMED) c_i0 = clock64();
        const uint32_t qhi = smem_addr(&sm.q[u][0][0][0][0]), qlo = smem_addr(&sm.q[u][1][0][0][0]);
        const uint32_t d = tmem + kPairColUnit * static_cast<uint32_t>(u) + kPairColS;
        // the correction products first, then hi x hi
#pragma unroll
        for (int k = 0; k < 8; ++k) mma_tf32_ss_e(d, q_desc(qhi, k), k_desc(klo, k), kIdescQK, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 8; ++k) mma_tf32_ss_e(d, q_desc(qlo, k), k_desc(khi, k), kIdescQK, 1u);
#pragma unroll
        for (int k = 0; k < 8; ++k) mma_tf32_ss_e(d, q_desc(qhi, k), k_desc(khi, k), kIdescQK, 1u);
        commit(&sm.s_full[u], static_cast<uint32_t>(j) & 1u);
        if constexpr (TIMED) {
          ok = warp_wait(&sm.s_full[u], static_cast<uint32_t>(j) & 1u);
          c_qk += static_cast<unsigned long long>(clock64() - c_i0);
        }
      }
      if (ok && g + 1 < n) commit(&sm.k_free, static_cast<uint32_t>(g) & 1u);
    }
    if constexpr (TIMED) {
      if (tid == kPairQkThread) {
        atomicAdd(&a.stage_cycles[kStageQk], c_qk);
        atomicAdd(&a.stage_cycles[kStageKWait], c_kw);
      }
    }
  } else if (warp == kPairPvThread / 32) {
    // ---------------- PV issuer (the whole warp runs the loop; an elected lane issues) ----------------
    unsigned long long c_pv = 0, c_vw = 0;
    bool ok = true;
    for (int g = 0; ok && g < n; ++g) {
      long long c_w0 = 0;
      if constexpr (TIMED) c_w0 = clock64();
      ok = warp_wait(&sm.v_ready, static_cast<uint32_t>(g) & 1u);
      if (!ok) break;
      tc_fence_after();
      const uint32_t vhi = smem_addr(&sm.vraw[g & 1][0][0][0]);
      const uint32_t vlo = smem_addr(&sm.vlo[0][0][0]);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!ok || !uses(u, g)) continue;
        const int j = g0 + g - t0[u];
        if constexpr (TIMED) c_w0 = clock64();
        ok = warp_wait(&sm.p_ready[u], static_cast<uint32_t>(j) & 1u);
        if constexpr (TIMED) c_vw += static_cast<unsigned long long>(clock64() - c_w0);
        if (!ok) break;
        tc_fence_after();
        long long c_i0 = 0;
        if constexpr (TIMED) c_i0 = clock64();
        const uint32_t ub = tmem + kPairColUnit * static_cast<uint32_t>(u);
        const uint32_t d = ub + kPairColPv, aph = ub + kPairColPh, apl = ub + kPairColPl;
#pragma unroll
        for (int k = 0; k < 8; ++k) mma_tf32_ts_e(d, aph + 8 * k, v_desc(vlo, k), kIdescPV, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 8; ++k) mma_tf32_ts_e(d, apl + 8 * k, v_desc(vhi, k), kIdescPV, 1u);
#pragma unroll
        for (int k = 0; k < 8; ++k) mma_tf32_ts_e(d, aph + 8 * k, v_desc(vhi, k), kIdescPV, 1u);
        commit(&sm.pv_done[u], static_cast<uint32_t>(j) & 1u);
        if constexpr (TIMED) {
          ok = warp_wait(&sm.pv_done[u], static_cast<uint32_t>(j) & 1u);
          c_pv += static_cast<unsigned long long>(clock64() - c_i0);
        }
      }
      if (ok && g + 1 < n) commit(&sm.v_free, static_cast<uint32_t>(g) & 1u);
    }
    if constexpr (TIMED) {
      if (tid == kPairPvThread) {
        atomicAdd(&a.stage_cycles[kStagePv], c_pv);
        atomicAdd(&a.stage_cycles[kStageVWait], c_vw);
      }
    }
  }
  __syncwarp();

  // End (every path); after a timeout first drain this CTA's copies and MMAs
  // still in flight (bounded).
  tc_fence_before();
  __syncthreads();
  if (*abort_flag != 0) {
    const long long c0 = clock64();
    auto drain = [&](uint64_t* bar, uint32_t parity) {
      while (!mbar_try_wait(bar, parity) && clock64() - c0 < a.timeout_cycles) {
      }
    };
    if (tid == kPairSplitTid0) {  // the q copy, and the last tile issued into each raw stage
      drain(&sm.q_full, 0);
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int tk = last_k - ((last_k - s) & 1), tv = last_v - ((last_v - s) & 1);
        if (tk >= 0) drain(&sm.k_full[s], static_cast<uint32_t>(tk >> 1) & 1u);
        if (tv >= 0) drain(&sm.v_full[s], static_cast<uint32_t>(tv >> 1) & 1u);
      }
    }
    if ((tid == kPairQkThread || tid == kPairPvThread) && last_commit) drain(last_commit, last_commit_parity);
  }
  __syncthreads();
  if (warp == 10) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPipeTmemCols) : "memory");
  }
}

}  // namespace tc32
}  // namespace raya
