// tc16_ws.cuh — 3xFP16 tensor-core attention (sm_100a): every fp32 operand
// split into two fp16 halves and multiplied on tcgen05.mma kind::f16
// (M = 128, N = 64, K = 16), in a persistent warp-specialised kernel.
//
// Why fp16.  A kind::f16 MMA of M128 N64 K16 does twice the work of a
// kind::tf32 MMA of K8 in the same ~32 cycles (measured on B200: one issuing
// warp already holds the tensor core at that rate, where kind::tf32 needs
// two), so the three products of a split operand cost half the tensor time.
// fp16 has TF32's 11 significant bits; its range is the catch, and scaling
// by powers of two (exact) takes care of it:
//
//   * x -> hi + lo: hi = x with its 13 low mantissa bits cleared (exact in
//     fp16 within its normal range), lo = x - hi (exact in fp32, then
//     rounded to fp16).  A product is taken as hi*lo + lo*hi + hi*hi.  The
//     representation error is below 2^-21 of |x| (2^-10 of the truncation
//     times fp16's 2^-11), plus an absolute 2^-25 where lo or hi falls
//     below fp16's normal range.
//   * q rows are scaled by 2^eq (per row, by the softmax thread that owns
//     it), K and V tiles by 2^e (per 64-key tile, from the tile's largest
//     magnitude over its valid rows), so that the largest element lands in
//     [2^14, 2^15): no fp16 overflow, and relative precision everywhere but
//     in elements 2^28 below the largest, where the absolute floor holds.
//     The softmax removes the scales: S * 2^-(eq + ek) through the one
//     multiplier it already applies, and each tile's PV partial times 2^-ev
//     as it is summed into O.
//   * p (the softmax weights, at most 2^8 relative to the kept max) needs no
//     scale.
//
// Scores and PV partials accumulate in fp32 in tensor memory; O is summed in
// fp32 registers with round-to-nearest adds, one partial per key tile, as in
// tc32_ws.cuh (the tensor core's accumulation truncates toward zero).
//
// Persistent: CTA c runs row tiles (units) c, c + gridDim.x, ... (one unit
// per CTA when the grid covers them all).  Every ring and barrier runs on
// across units with a running key-tile counter g, so one unit's copies,
// splits and products start while the previous unit's last tiles finish.
//
// Roles (512 threads; setmaxnreg once, each role loops over the units):
//   warps 0-3   softmax: one query row per thread (TMEM lane = row): q row
//               -> scaled hi/lo in tensor memory (two buffers, by unit
//               parity); per key tile S -> mask -> online softmax -> P hi/lo
//               in tensor memory; the PV partials summed into O in
//               registers; the normalised row stored straight to global
//               memory.
//   warps 4-7   K split, warps 8-11 V split: the raw fp32 tile (TMA ring of
//               3, read only by these groups and released as soon as both
//               have loaded it) -> fp16 hi/lo operands (a ring of 3), both
//               as [key][64] rows under the 128-byte swizzle: K-major for
//               QK's B, MN-major for PV's B (no transpose).  Rows at or past
//               valid_len become exact zeros.  Each group reduces its tile's
//               largest magnitude over one named barrier and hands the scale
//               to the softmax through a ring of 8 (kfac/vfac) with its own
//               mbarriers.
//   warp 12     QK issuer: 12 MMAs per key tile into S (double-buffered).
//   warp 13     PV issuer: 12 MMAs per key tile into the PV partial.
//   warp 14     TMA producer: each unit's q tile (its own buffer) and the
//               raw K/V ring.  Warp 15 idles.
// The issuers and the producer run their loops on the whole warp and issue
// from one lane (no lane-divergent code before a warp-collective
// instruction).
//
// Tensor memory (512 columns): S0 [0,64), S1 [64,128), Q0 hi/lo [128,192),
// Q1 hi/lo [192,256), P0 hi/lo [256,320), P1 hi/lo [320,384), PV partials
// O0 [384,448), O1 [448,512).  With two PV partials the softmax releases
// P(g) before it sums the partial of tile g-1, so PV(g) overlaps that sum;
// and it prepares the next unit's Q buffer during the current unit, so the
// next unit's first QK products are ready when the current unit ends.
// (A 16-bit A operand in tensor memory packs two elements per 32-bit column,
// element 2c in the low half.)
// Every wait is bounded; after a timeout every role leaves its loop, the
// producer and the issuers drain their copies and MMAs (bounded), and
// tensor memory is freed.
#pragma once

#include "tc32_common.cuh"

namespace raya {
namespace tc16 {

using tc32::kBM;
using tc32::kBN;
using tc32::kD;

// Instruction descriptors of kind::f16: D = F32, A = B = F16, N = 64,
// M = 128; B K-major for QK^T, MN-major (transposed) for PV.
constexpr uint32_t kIdescQK = (1u << 4) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescPV = kIdescQK | (1u << 16);

constexpr int kThreads = 512;
constexpr int kGroupThreads = 128;  // one split group
constexpr int kQkWarp = 12, kPvWarp = 13, kTmaWarp = 14;
constexpr int kRawStages = 3;
constexpr int kOpStages = 3;
constexpr int kMeta = 8;  // scale ring slots: the splits run at most 5 tiles ahead of the softmax
constexpr float kRescaleLog2 = 8.0f;
// Register split (setmaxnreg): the softmax warp group holds an O row next to
// a score row; a split thread holds 32 elements; the issuer warp group walks
// the units with 64-bit coordinates.  216 + 96 + 96 + 96 = 504 <= 4 warp
// groups x the 128 registers a thread of this launch gets, so no increase
// waits on the pool.
constexpr int kSoftmaxRegs = 216, kSplitRegs = 96, kIssueRegs = 96;
static_assert(kSoftmaxRegs + 2 * kSplitRegs + kIssueRegs <= 4 * 128, "register split above the launch's allocation");
constexpr int kKBarrier = 1, kVBarrier = 3;  // named barriers of the split groups
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColQ = 128, kColP = 256, kColO = 384;
__device__ __forceinline__ uint32_t col_o(int b) { return kColO + 64u * static_cast<uint32_t>(b); }
__device__ __forceinline__ uint32_t col_s(int b) { return kColS + 64u * static_cast<uint32_t>(b); }
__device__ __forceinline__ uint32_t col_qh(int b) { return kColQ + 64u * static_cast<uint32_t>(b); }
__device__ __forceinline__ uint32_t col_ph(int b) { return kColP + 64u * static_cast<uint32_t>(b); }

constexpr int kOpElems = kBN * kD;  // one fp16 operand tile: 64 rows x 64, 8 KB
enum { kOpKh = 0, kOpKl = 1, kOpVh = 2, kOpVl = 3 };

struct Smem {
  float raw[kRawStages][2][2][kBN][32];  // [stage][K, V][column half][key][32], 128-byte swizzle of 16-byte chunks
  uint16_t op[kOpStages][4][kOpElems];   // [stage][K hi, K lo, V hi, V lo], 128-byte rows, 128-byte swizzle
  float q[2][kBM][32];                   // the unit's q tile: [column half][row][32], 128-byte swizzle
  float kfac[kMeta], vfac[kMeta];        // 2^-e of each K and V tile (slot = g % kMeta)
  uint32_t red[2][2][4];                 // [K, V][tile parity][group warp]: max |x| bits
  uint64_t raw_full[kRawStages], raw_free[kRawStages];
  uint64_t k_ready[kOpStages], v_ready[kOpStages], k_free[kOpStages], v_free[kOpStages];
  uint64_t s_full[2], s_free[2], p_ready2[2], pv_done2[2], kmeta[kMeta], vmeta[kMeta];
  uint64_t q_full, q_empty, q_ready[2], q_tfree[2], o_free[2];
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t smem_bytes() { return sizeof(Smem) + 1024; }
static_assert(smem_bytes() <= 232448, "more shared memory than one sm_100 block may hold");

// Byte offset of 16-byte chunk c (elements 8c..8c+7) of row r in a [rows][64]
// fp16 tile under the 128-byte swizzle.
__device__ __forceinline__ uint32_t op_off(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}
// K-major B operand (K: 64 rows of 128 bytes): k-step s is bytes 32s..32s+31
// of each row.
__device__ __forceinline__ uint64_t b_desc(uint32_t base, int s) { return tc32::smem_desc(base + 32 * s, 16, 1024); }
// MN-major B operand (V: [key][64], the same swizzled rows): k-step s is
// keys 16s..16s+15, two 8-row atoms 1024 bytes apart; one atom spans N.
__device__ __forceinline__ uint64_t v_desc(uint32_t base, int s) { return tc32::smem_desc(base + 2048 * s, 0, 1024); }

// e with max|x| * 2^e in [2^14, 2^15) from the bits of max|x| (0 for a zero
// or subnormal maximum), clamped so that 2^e and 2^-e are normal floats.
__device__ __forceinline__ int scale_exp(uint32_t maxbits) {
  const int E = static_cast<int>(maxbits >> 23);
  if (E == 0) return 0;
  return max(-126, min(126, 141 - E));
}
__device__ __forceinline__ float pow2(int e) { return __uint_as_float(static_cast<uint32_t>(e + 127) << 23); }

// x (already scaled) -> hi with its 13 low mantissa bits cleared, lo = x - hi.
__device__ __forceinline__ float hi_part(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }
// Two floats as fp16 (round to nearest), e0 in the low half.
__device__ __forceinline__ uint32_t pack_f16x2(float e0, float e1) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(e1), "f"(e0));
  return r;
}
// Elements (e0, e1) -> packed hi and lo words (lo = e - hi, one packed FMA).
__device__ __forceinline__ void split2(float e0, float e1, uint32_t& h, uint32_t& l) {
  const float h0 = hi_part(e0), h1 = hi_part(e1);
  h = pack_f16x2(h0, h1);
  const float2 lo = __ffma2_rn(make_float2(h0, h1), make_float2(-1.f, -1.f), make_float2(e0, e1));
  l = pack_f16x2(lo.x, lo.y);
}
// 16 consecutive fp32 columns of this thread's TMEM lane (load and wait in
// one statement).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// D (+)= A B, kind::f16, A from tensor memory, in elected-lane form (the
// whole issuing warp runs the loop, one lane issues).
template <uint32_t IDESC>
__device__ __forceinline__ void mma_f16_ts_e(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "n"(IDESC), "r"(accumulate), "r"(0u)
      : "memory");
}

// 8 packed 32-bit columns of this thread's lane; completion is awaited by
// tmem_wait_st.
__device__ __forceinline__ void tmem_st8u(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
// One 16-byte shared-memory store of four 32-bit words.
__device__ __forceinline__ void sts128u(uint32_t addr, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ bool lane_is_first(int tid) { return (tid & 31) == 0; }

// The copies of a [64 rows][32] column-half box of q (which 0), K (1) or V
// (2): head-major 2-D maps or the packed 4-D maps.
template <int LAYOUT>
__device__ __forceinline__ void load_box(void* dst, const CUtensorMap* map, int x, int head, int which, int y,
                                         uint64_t* bar) {
  if constexpr (LAYOUT == tiled64::kHeadMajor)
    tiled64::tma_load_2d(dst, map, x, y, bar);
  else
    tiled64::tma_load_4d(dst, map, x, head, which, y, bar);
}

// One unit (a 128-row tile of one (batch, head) slice): its rows, keys and
// layout coordinates.
struct Unit {
  int valid;      // valid_len of its sequence, clamped to [0, seq]
  int r0;         // first row
  int last;       // last valid row of the tile (when not padding)
  int t_begin;    // first key tile
  int ntiles;     // key tiles (0: padding only)
  int b, head;
  long long bh;        // slice
  long long row_base;  // first row of the slice (head-major) or sequence (packed) in the loads' row coordinate
};

// The unit's raw valid_len (one global load: the role loops issue it a unit
// ahead, so that its latency overlaps the current unit).
__device__ __forceinline__ int unit_valid(const AttnArgs& a, unsigned unit) {
  return a.valid_len ? a.valid_len[unit / static_cast<unsigned>(a.row_tiles) / static_cast<unsigned>(a.heads)] : a.seq;
}

template <int LAYOUT>
__device__ __forceinline__ Unit unit_of(const AttnArgs& a, unsigned unit, int vr) {
  Unit u;
  const unsigned bh32 = unit / static_cast<unsigned>(a.row_tiles);
  const int tile = static_cast<int>(unit - bh32 * static_cast<unsigned>(a.row_tiles));
  const unsigned b32 = bh32 / static_cast<unsigned>(a.heads);
  u.bh = bh32;
  u.b = static_cast<int>(b32);
  u.head = static_cast<int>(bh32 - b32 * static_cast<unsigned>(a.heads));
  u.r0 = tile * kBM;
  u.valid = vr < 0 ? 0 : (vr > a.seq ? a.seq : vr);
  u.row_base = LAYOUT == tiled64::kHeadMajor ? u.bh * a.seq : static_cast<long long>(u.b) * a.seq;
  int klo = 0, khi = 0, unused = 0;
  u.last = min(u.r0 + kBM, u.valid) - 1;
  if (u.r0 < u.valid) {
    key_range(a, u.r0, u.valid, klo, unused);
    key_range(a, u.last, u.valid, unused, khi);
  }
  u.t_begin = klo / kBN;
  u.ntiles = (u.r0 < u.valid && khi > klo) ? (khi + kBN - 1) / kBN - u.t_begin : 0;
  return u;
}

template <int LAYOUT>
__device__ __forceinline__ Unit unit_info(const AttnArgs& a, unsigned unit) {
  return unit_of<LAYOUT>(a, unit, unit_valid(a, unit));
}


// LAYOUT: tiled64::kHeadMajor (q, k, v, out as [batch*heads*seq][64]); the
// caller's packed layout runs on tc32_ws.cuh.  TIMED: the stage-timing build
// (the counterpart of the reference's StageTimes, tiled/stages.rs:1-31):
// clock64 cycles per CTA added into a.stage_cycles — [kStageQk] QK^T products
// in flight (issue to completion: in this build the QK issuer waits for each
// QK's completion), [kStageSoftmax] one softmax warp's work per tile (S read
// to P stored), [kStagePv] PV products in flight (likewise), [kStageKWait]
// the QK issuer waiting for K's split, [kStageVWait] the PV issuer waiting
// for P and V's split, [kStageRefill] one K split thread's work,
// [kStageTiles] key tiles, [kStageTotal] thread 0's cycles over the CTA's
// units.  The stages overlap in time; read them as proportions.
template <int LAYOUT, bool TIMED = false>
__global__ void __launch_bounds__(kThreads, 1)
    tc16_ws_fwd(const __grid_constant__ AttnArgs a, const __grid_constant__ tc32::PipeMaps maps) {
  static_assert(LAYOUT == tiled64::kHeadMajor, "the packed layout runs on tc32_ws.cuh");
  using namespace tc32;  // tensor-memory, barrier and TMA-store helpers
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr));

  const int tid = threadIdx.x, warp = tid >> 5;
  const int seq = a.seq;
  // 32-bit unit arithmetic (the host keeps batch * heads * row_tiles below 2^31).
  const unsigned nunits = static_cast<unsigned>(a.batch) * static_cast<unsigned>(a.heads) *
                          static_cast<unsigned>(a.row_tiles);
  const unsigned ustep = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < kRawStages; ++s) {
      mbar_init(&sm.raw_full[s], 1);
      mbar_init(&sm.raw_free[s], 2 * kGroupThreads);
    }
    for (int s = 0; s < kOpStages; ++s) {
      mbar_init(&sm.k_ready[s], kGroupThreads);
      mbar_init(&sm.v_ready[s], kGroupThreads);
      mbar_init(&sm.k_free[s], 1);
      mbar_init(&sm.v_free[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_free[s], 128);
      mbar_init(&sm.p_ready2[s], 128);
      mbar_init(&sm.pv_done2[s], 1);
      mbar_init(&sm.q_ready[s], 128);
      mbar_init(&sm.q_tfree[s], 1);
      mbar_init(&sm.o_free[s], 128);
    }
    for (int s = 0; s < kMeta; ++s) {
      mbar_init(&sm.kmeta[s], 1);
      mbar_init(&sm.vmeta[s], 1);
    }
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 128);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kQkWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&sm.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_flag = &sm.abort_flag;
  const long long t_start = TIMED ? clock64() : 0;

  // Drain bookkeeping, read after the roles: the producer's last q unit and
  // raw tile, an issuer's last commit.
  int last_q = -1, last_g = -1;
  uint64_t* last_commit = nullptr;
  uint32_t last_commit_parity = 0;
  auto commit = [&](uint64_t* bar, uint32_t parity) {  // the issuing warps: one elected lane commits
    mma_commit_e(bar);
    last_commit = bar;
    last_commit_parity = parity;
  };
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    return mbar_wait_bounded(bar, parity, abort_flag, a.status, a.timeout_cycles);
  };
  // A bounded wait whose outcome is the same on every lane of the warp.
  auto warp_wait = [&](uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, a.status, a.timeout_cycles));
  };
  // This CTA's key tiles and non-padding units (the issuers' commit guards:
  // no commit is left that nothing waits for), counted by a whole warp.
  auto totals = [&](int& tiles, int& units) {
    tiles = 0;
    units = 0;
    for (unsigned long long unit = blockIdx.x + static_cast<unsigned long long>(tid & 31) * ustep; unit < nunits;
         unit += 32ull * ustep) {
      const int n = unit_info<LAYOUT>(a, static_cast<unsigned>(unit)).ntiles;
      tiles += n;
      units += n > 0;
    }
    tiles = __reduce_add_sync(0xffffffffu, tiles);
    units = __reduce_add_sync(0xffffffffu, units);
  };

  if (warp < 4)
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
  else if (warp < 12)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kSplitRegs));
  else
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kIssueRegs));
  if (warp < 4) {
    // ---------------- softmax warpgroup ----------------
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const size_t out_stride = LAYOUT == tiled64::kHeadMajor ? kD : static_cast<size_t>(a.heads) * kD;
    unsigned long long c_a = 0, c_tiles = 0;
    auto out_row = [&](const Unit& u, int row) {
      return a.out + (LAYOUT == tiled64::kHeadMajor ? static_cast<size_t>(u.row_base) * kD
                                                    : (static_cast<size_t>(u.row_base) * a.heads + u.head) * kD) +
             static_cast<size_t>(row) * out_stride;
    };
    // The first unit at or after `unit` with keys to attend (the others'
    // rows get their exact zeros on the way).
    auto next_unit = [&](unsigned unit, Unit& u) {
      for (; unit < nunits; unit += ustep) {
        u = unit_info<LAYOUT>(a, unit);
        if (u.ntiles > 0) return unit;
        const int row = u.r0 + tid;
        if (row < seq) {
          float* o = out_row(u, row);
#pragma unroll
          for (int c4 = 0; c4 < 16; ++c4) st_stream(o + 4 * c4, make_float4(0.f, 0.f, 0.f, 0.f));
        }
      }
      return nunits;
    };
    // The q row of unit u (the CTA's uidx-th) scaled by 2^eq and split into
    // Q buffer uidx % 2; qmul = qscale * 2^-eq.  False after a timeout.  It
    // runs inside the previous unit's tile loop, next to that unit's O row,
    // so it holds 32 elements at a time: pass 1 takes the row's largest
    // magnitude, pass 2 reloads, scales, splits and stores.  Piece p is
    // elements 16p..16p+15 and 16p+32..16p+47.
    auto prepare_q = [&](const Unit& u, uint32_t uidx, float& qmul) {
      const int qb = static_cast<int>(uidx & 1u);
      const int row = u.r0 + tid;
      const bool wq = wait(&sm.q_full, uidx & 1u);
      const bool live = wq && row < u.valid;
      const uint32_t qs = smem_addr(&sm.q[0][0][0]);
      auto piece = [&](int p, float* x, float* y) {  // x: elements 16p.., y: 16p+32..
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float4 v0 = live ? lds128(qs + chunk_offset<kBM>(tid, 4 * p + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
          const float4 v1 = live ? lds128(qs + chunk_offset<kBM>(tid, 8 + 4 * p + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
          x[4 * c] = v0.x; x[4 * c + 1] = v0.y; x[4 * c + 2] = v0.z; x[4 * c + 3] = v0.w;
          y[4 * c] = v1.x; y[4 * c + 1] = v1.y; y[4 * c + 2] = v1.z; y[4 * c + 3] = v1.w;
        }
      };
      float fm = 0.f;
#pragma unroll 1
      for (int p = 0; p < 2; ++p) {
        float x[16], y[16];
        piece(p, x, y);
#pragma unroll
        for (int k = 0; k < 16; ++k) fm = fmaxf(fm, fmaxf(fabsf(x[k]), fabsf(y[k])));
      }
      const int eq = scale_exp(__float_as_uint(fm));
      const float sq = pow2(eq);
      qmul = a.qscale * pow2(-eq);
      // Q buffer qb is free once the QK products of unit uidx-2 are complete.
      bool wt = wq;
      if (uidx >= 2 && wt) wt = wait(&sm.q_tfree[qb], ((uidx - 2) >> 1) & 1u);
      if (__any_sync(0xffffffffu, !wt)) {
        mbar_arrive(&sm.q_empty);
        return false;
      }
      tc_fence_after();
      const uint32_t qh = tmem + lane_off + col_qh(qb);
#pragma unroll 1
      for (int p = 0; p < 2; ++p) {
        float x[16], y[16];
        piece(p, x, y);
        uint32_t hx[8], lx[8], hy[8], ly[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          split2(x[2 * k] * sq, x[2 * k + 1] * sq, hx[k], lx[k]);
          split2(y[2 * k] * sq, y[2 * k + 1] * sq, hy[k], ly[k]);
        }
        // column c holds elements 2c, 2c+1: x -> columns 8p..8p+7, y -> 16+8p..
        tmem_st8u(qh + 8 * p, hx);
        tmem_st8u(qh + 16 + 8 * p, hy);
        tmem_st8u(qh + 32 + 8 * p, lx);
        tmem_st8u(qh + 48 + 8 * p, ly);
      }
      mbar_arrive(&sm.q_empty);  // the producer may load the next unit's q
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&sm.q_ready[qb]);
      return true;
    };

    Unit u;
    unsigned cur = next_unit(blockIdx.x, u);
    uint32_t uidx = 0;
    int g = 0;
    float qmul = 0.f;
    bool ok = cur >= nunits || prepare_q(u, 0, qmul);
    while (ok && cur < nunits) {
      const int row = u.r0 + tid;
      int rlo = 0, rhi = 0;
      key_range(a, min(row, u.last), u.valid, rlo, rhi);
      if (a.valid_len && cur + ustep < nunits)  // the next unit's valid_len, read at `prep`
        asm volatile("prefetch.global.L1 [%0];" ::"l"(
            a.valid_len + (cur + ustep) / static_cast<unsigned>(a.row_tiles) / static_cast<unsigned>(a.heads)));
      const int prep = max(0, u.ntiles - 2);  // the tile after which the next unit's Q is prepared
      Unit nu;
      unsigned nxt = nunits;
      float qmul_next = 0.f;
      float m_used = -INFINITY, lsum = 0.f;
      float o[64];  // this row of O, summed in fp32 registers (round to nearest)
#pragma unroll
      for (int c = 0; c < 64; ++c) o[c] = 0.f;
      for (int t = 0; t < u.ntiles; ++t, ++g) {
        const int pb = g & 1;  // S, P and PV-partial buffer
        const int kt = (u.t_begin + t) * kBN;
        bool w = wait(&sm.s_full[pb], static_cast<uint32_t>(g >> 1) & 1u) &&
                 wait(&sm.kmeta[g % kMeta], static_cast<uint32_t>(g / kMeta) & 1u);
        if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
        tc_fence_after();
        long long c_s0 = 0;
        if constexpr (TIMED) c_s0 = clock64();
        // 2^-ek of this K tile; never below the smallest normal float, so that
        // a masked -inf times it stays -inf (only reached for q rows ~2^-100)
        const float mult = fmaxf(qmul * sm.kfac[g % kMeta], 1.17549435e-38f);
        const bool full = rlo <= kt && rhi >= kt + kBN;
        const uint32_t sa = tmem + lane_off + col_s(pb);
        float mraw = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {  // pass 1 over S(g), 16 columns at a time: the row max (masked keys -inf)
          float s16[16];
          tmem_ld16(sa + 16 * c, s16);
          if (!full) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (static_cast<unsigned>(kt + 16 * c + i - rlo) >= static_cast<unsigned>(rhi - rlo)) s16[i] = -INFINITY;
          }
          // Chain q takes columns q, q + 4, q + 8, q + 12.
          float m4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) m4[q] = tc32::fmax3(s16[q], s16[4 + q], fmaxf(s16[8 + q], s16[12 + q]));
          mraw = tc32::fmax3(mraw, fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        }
        const float mc = mraw * mult;
        float alpha = 1.f;
        if (mc > m_used + kRescaleLog2) {
          alpha = ex2(m_used - mc);
          m_used = mc;
        }
        const float mbase = m_used == -INFINITY ? 0.f : m_used;

        if (g >= 2) {  // P buffer pb is free once PV(g-2) is complete
          w = wait(&sm.pv_done2[pb], static_cast<uint32_t>((g - 2) >> 1) & 1u);
          if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
          tc_fence_after();
        }
        // pass 2, 16 columns at a time (a rolled loop: the code stays small
        // for the instruction cache): p = 2^(s * mult - mbase), the row sum,
        // and p's hi and lo parts into P buffer pb.
        float2 rs2 = make_float2(0.f, 0.f);
        const uint32_t ph = tmem + lane_off + col_ph(pb);
        const float2 mult2 = make_float2(mult, mult), nb2 = make_float2(-mbase, -mbase);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float s16[16];
          tmem_ld16(sa + 16 * c, s16);
          if (!full) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (static_cast<unsigned>(kt + 16 * c + i - rlo) >= static_cast<unsigned>(rhi - rlo)) s16[i] = -INFINITY;
          }
          uint32_t h[8], l[8];
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const float2 arg = __ffma2_rn(make_float2(s16[i], s16[i + 1]), mult2, nb2);
            const float p0 = ex2(arg.x), p1 = ex2(arg.y);
            rs2 = __fadd2_rn(rs2, make_float2(p0, p1));
            split2(p0, p1, h[i >> 1], l[i >> 1]);
          }
          tmem_st8u(ph + 8 * c, h);
          tmem_st8u(ph + 32 + 8 * c, l);
        }
        tc_fence_before();
        mbar_arrive(&sm.s_free[pb]);  // QK(g+2) may overwrite this S buffer
        lsum = fmaf(lsum, alpha, rs2.x + rs2.y);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&sm.p_ready2[pb]);  // PV(g) may start
        if (t > 0) {
          // O = (O + 2^-ev * PV partial of tile g-1) * alpha, both at the
          // previous max, while PV(g) runs into the other partial buffer.
          const int gp = g - 1;
          w = wait(&sm.pv_done2[gp & 1], static_cast<uint32_t>(gp >> 1) & 1u) &&
              wait(&sm.vmeta[gp % kMeta], static_cast<uint32_t>(gp / kMeta) & 1u);
          if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
          tc_fence_after();
          const float vf = sm.vfac[gp % kMeta];
          float tt[64];
          tmem_ld32(tmem + lane_off + col_o(gp & 1), tt);
          tmem_ld32(tmem + lane_off + col_o(gp & 1) + 32, tt + 32);
          tc_fence_before();
          mbar_arrive(&sm.o_free[gp & 1]);  // PV(g+1) may overwrite this partial
          const float2 vf2 = make_float2(vf, vf), al2 = make_float2(alpha, alpha);
#pragma unroll
          for (int i = 0; i < 64; i += 2) {  // (O + t) * alpha, with alpha == 1 exact when the max is kept
            const float2 r =
                __fmul2_rn(__ffma2_rn(make_float2(tt[i], tt[i + 1]), vf2, make_float2(o[i], o[i + 1])), al2);
            o[i] = r.x;
            o[i + 1] = r.y;
          }
        }
        if constexpr (TIMED) c_a += static_cast<unsigned long long>(clock64() - c_s0);
        if (t == prep) {
          nxt = next_unit(cur + ustep, nu);
          if (nxt < nunits && !prepare_q(nu, uidx + 1, qmul_next)) { ok = false; break; }
        }
      }
      if (!ok) break;
      {  // the last tile's partial
        const int gp = g - 1;
        const bool w = wait(&sm.pv_done2[gp & 1], static_cast<uint32_t>(gp >> 1) & 1u) &&
                       wait(&sm.vmeta[gp % kMeta], static_cast<uint32_t>(gp / kMeta) & 1u);
        if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
        tc_fence_after();
        const float vf = sm.vfac[gp % kMeta];
        float tt[64];
        tmem_ld32(tmem + lane_off + col_o(gp & 1), tt);
        tmem_ld32(tmem + lane_off + col_o(gp & 1) + 32, tt + 32);
        tc_fence_before();
        mbar_arrive(&sm.o_free[gp & 1]);
        const float2 vf2 = make_float2(vf, vf);
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          const float2 r = __ffma2_rn(make_float2(tt[i], tt[i + 1]), vf2, make_float2(o[i], o[i + 1]));
          o[i] = r.x;
          o[i + 1] = r.y;
        }
      }
      // This row, normalised (+0.0f past valid_len), straight to global memory.
      if (row < seq) {
        float* orow = out_row(u, row);
        const float inv = (row < u.valid && lsum > 0.f) ? 1.0f / lsum : 0.f;
#pragma unroll
        for (int c4 = 0; c4 < 16; ++c4)
          st_stream(orow + 4 * c4, row < u.valid ? make_float4(o[4 * c4] * inv, o[4 * c4 + 1] * inv,
                                                               o[4 * c4 + 2] * inv, o[4 * c4 + 3] * inv)
                                                 : make_float4(0.f, 0.f, 0.f, 0.f));
      }
      c_tiles += static_cast<unsigned long long>(u.ntiles);
      cur = nxt;
      u = nu;
      qmul = qmul_next;
      ++uidx;
    }
    if constexpr (TIMED) {
      if (tid == 0) {
        atomicAdd(&a.stage_cycles[kStageSoftmax], c_a);
        atomicAdd(&a.stage_cycles[kStageTiles], c_tiles);
        atomicAdd(&a.stage_cycles[kStageTotal], static_cast<unsigned long long>(clock64() - t_start));
      }
    }
  } else if (warp < 12) {
    // ---------------- split groups: K (warps 4-7), V (warps 8-11), one code path ----------------
    const bool is_v = warp >= 8;
    const int gt = tid - (is_v ? 256 : 128), gw = gt >> 5, lane = tid & 31;
    const int gbar = is_v ? kVBarrier : kKBarrier;
    // Four units per thread, (row r, chunk c) = elements 8c..8c+7 of row r:
    // r = gt / 8 + 16 i, c = gt % 8; the offsets of unit i are those of unit
    // 0 plus 16 rows (the swizzle depends on r % 8 only).
    const int r0s = gt >> 3, cs = gt & 7;
    // raw tile: 16-byte chunk c4 of row r at chunk_offset<kBN>(r, c4)
    // (swizzled: chunks 2c and 2c + 1 need not be adjacent)
    const uint32_t off0 = chunk_offset<kBN>(r0s, 2 * cs), off1 = chunk_offset<kBN>(r0s, 2 * cs + 1);
    const uint32_t oop = op_off(r0s, cs);
    uint64_t* const ready = is_v ? sm.v_ready : sm.k_ready;
    uint64_t* const freed = is_v ? sm.v_free : sm.k_free;
    uint64_t* const meta = is_v ? sm.vmeta : sm.kmeta;
    float* const fac = is_v ? sm.vfac : sm.kfac;
    const int op_h = is_v ? kOpVh : kOpKh;
    unsigned long long c_a = 0;
    int g = 0;
    bool ok = true;
    int vr = blockIdx.x < nunits ? unit_valid(a, blockIdx.x) : 0;
    for (unsigned unit = blockIdx.x; ok && unit < nunits; unit += ustep) {
      const Unit u = unit_of<LAYOUT>(a, unit, vr);
      vr = unit + ustep < nunits ? unit_valid(a, unit + ustep) : 0;  // in flight during this unit
      for (int t = 0; t < u.ntiles; ++t, ++g) {
        const int s = g % kRawStages, par = g & 1;
        long long c_k0 = 0;
        if constexpr (TIMED) c_k0 = clock64();
        const int kt = (u.t_begin + t) * kBN;
        const int nv = min(kBN, u.valid - kt);  // valid rows of this tile (>= 1)
        uint32_t mx = 0;
        bool w = wait(&sm.raw_full[s], static_cast<uint32_t>(g / kRawStages) & 1u);
        const uint32_t base = smem_addr(&sm.raw[s][is_v ? 1 : 0][0][0][0]);
        // unit i's 8 elements (zeros for keys at or past valid_len)
        auto unit_x = [&](int i, float* e) {
          if (r0s + 16 * i < nv) {
            const uint32_t o = static_cast<uint32_t>(i * 16 * 128);
            const float4 x0 = lds128(base + off0 + o), x1 = lds128(base + off1 + o);
            e[0] = x0.x; e[1] = x0.y; e[2] = x0.z; e[3] = x0.w; e[4] = x1.x; e[5] = x1.y; e[6] = x1.z; e[7] = x1.w;
          } else {
#pragma unroll
            for (int q = 0; q < 8; ++q) e[q] = 0.f;
          }
        };
        if (w) {  // pass 1: the largest magnitude (a NaN drops out of the max; it still propagates)
          float fm = 0.f;
#pragma unroll 1
          for (int i = 0; i < 4; ++i) {
            float e[8];
            unit_x(i, e);
#pragma unroll
            for (int q = 0; q < 8; ++q) fm = fmaxf(fm, fabsf(e[q]));
          }
          mx = __float_as_uint(fm);
        }
        // The operand stage is free once the products of tile g-3 are complete.
        if (w && g >= kOpStages) w = wait(&freed[s], static_cast<uint32_t>((g - kOpStages) / kOpStages) & 1u);
        mx = __reduce_max_sync(0xffffffffu, mx);
        if (lane == 0) sm.red[is_v][par][gw] = mx;
        if (bar_any(gbar, kGroupThreads, !w)) { ok = false; break; }  // also publishes red[][par]
        mx = max(max(sm.red[is_v][par][0], sm.red[is_v][par][1]), max(sm.red[is_v][par][2], sm.red[is_v][par][3]));
        const int e2 = scale_exp(mx);
        const float sc = pow2(e2);
        const uint32_t oh = smem_addr(&sm.op[s][op_h][0]), ol = oh + kOpElems * 2;
#pragma unroll 1
        for (int i = 0; i < 4; ++i) {  // pass 2: reload, scale, split, store
          float x[8];
          unit_x(i, x);
          uint32_t h[4], l[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) split2(x[2 * e] * sc, x[2 * e + 1] * sc, h[e], l[e]);
          const uint32_t o = static_cast<uint32_t>(i * 16 * 128);
          sts128u(oh + oop + o, h[0], h[1], h[2], h[3]);
          sts128u(ol + oop + o, l[0], l[1], l[2], l[3]);
        }
        mbar_arrive(&sm.raw_free[s]);  // this thread is done with the raw stage
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        if (gt == 0) {
          fac[g % kMeta] = pow2(-e2);
          mbar_arrive(&meta[g % kMeta]);
        }
        mbar_arrive(&ready[s]);
        if constexpr (TIMED) c_a += static_cast<unsigned long long>(clock64() - c_k0);
      }
    }
    if constexpr (TIMED)
      if (gt == 0 && !is_v) atomicAdd(&a.stage_cycles[kStageRefill], c_a);
  } else if (warp == kTmaWarp) {
    // ---------------- TMA producer: q per unit, raw K/V ring ----------------
    const bool leader = lane_is_first(tid);
    int g = 0, uidx = 0;
    bool ok = true;
    int vr = blockIdx.x < nunits ? unit_valid(a, blockIdx.x) : 0;
    for (unsigned unit = blockIdx.x; ok && unit < nunits; unit += ustep) {
      const Unit u = unit_of<LAYOUT>(a, unit, vr);
      vr = unit + ustep < nunits ? unit_valid(a, unit + ustep) : 0;  // in flight during this unit
      if (u.ntiles == 0) continue;
      // The q buffer is free once the softmax has read the previous unit's q.
      if (uidx > 0 && !warp_wait(&sm.q_empty, static_cast<uint32_t>(uidx - 1) & 1u)) { ok = false; break; }
      if (leader) {
        mbar_arrive_expect_tx(&sm.q_full, kBM * kD * 4u);
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
          for (int rb = 0; rb < 2; ++rb)
            load_box<LAYOUT>(&sm.q[half][64 * rb][0], &maps.q, 32 * half, u.head, 0,
                             static_cast<int>(u.row_base + u.r0 + 64 * rb), &sm.q_full);
      }
      last_q = uidx;
      for (int t = 0; t < u.ntiles; ++t, ++g) {
        const int s = g % kRawStages;
        // The raw stage is free once both split groups have loaded tile g-3.
        if (g >= kRawStages &&
            !warp_wait(&sm.raw_free[s], static_cast<uint32_t>((g - kRawStages) / kRawStages) & 1u)) {
          ok = false;
          break;
        }
        if (leader) {
          fence_proxy_async_smem();  // the groups' generic reads of this stage, before the async-proxy writes
          const int y = static_cast<int>(u.row_base + (u.t_begin + t) * kBN);
          mbar_arrive_expect_tx(&sm.raw_full[s], 2u * kBN * kD * 4u);
          load_box<LAYOUT>(&sm.raw[s][0][0][0][0], &maps.k, 0, u.head, 1, y, &sm.raw_full[s]);
          load_box<LAYOUT>(&sm.raw[s][0][1][0][0], &maps.k, 32, u.head, 1, y, &sm.raw_full[s]);
          load_box<LAYOUT>(&sm.raw[s][1][0][0][0], &maps.v, 0, u.head, 2, y, &sm.raw_full[s]);
          load_box<LAYOUT>(&sm.raw[s][1][1][0][0], &maps.v, 32, u.head, 2, y, &sm.raw_full[s]);
        }
        last_g = g;
        __syncwarp();
      }
      ++uidx;
    }
  } else if (warp == kQkWarp) {
    // ---------------- QK^T issuer (12 MMAs per key tile) ----------------
    int total_tiles, total_units;
    totals(total_tiles, total_units);
    unsigned long long c_a = 0, c_b = 0;
    int g = 0, uidx = 0;
    bool ok = true;
    int vr = blockIdx.x < nunits ? unit_valid(a, blockIdx.x) : 0;
    for (unsigned unit = blockIdx.x; ok && unit < nunits; unit += ustep) {
      const Unit u = unit_of<LAYOUT>(a, unit, vr);
      vr = unit + ustep < nunits ? unit_valid(a, unit + ustep) : 0;  // in flight during this unit
      if (u.ntiles == 0) continue;
      const int qb = uidx & 1;
      if (!warp_wait(&sm.q_ready[qb], static_cast<uint32_t>(uidx >> 1) & 1u)) { ok = false; break; }
      const uint32_t qh = tmem + col_qh(qb), ql = qh + 32;
      for (int t = 0; t < u.ntiles; ++t, ++g) {
        const int s = g % kOpStages, sb = g & 1;
        long long c_w0 = 0;
        if constexpr (TIMED) c_w0 = clock64();
        ok = warp_wait(&sm.k_ready[s], static_cast<uint32_t>(g / kOpStages) & 1u);
        if (ok && g >= 2)  // the softmax has read S(g-2) from this buffer
          ok = warp_wait(&sm.s_free[sb], static_cast<uint32_t>((g - 2) >> 1) & 1u);
        if constexpr (TIMED) c_b += static_cast<unsigned long long>(clock64() - c_w0);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kh = smem_addr(&sm.op[s][kOpKh][0]), kl = smem_addr(&sm.op[s][kOpKl][0]);
        const uint32_t d = tmem + col_s(sb);
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16_ts_e<kIdescQK>(d, qh + 8 * k, b_desc(kl, k), k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16_ts_e<kIdescQK>(d, ql + 8 * k, b_desc(kh, k), 1u);
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16_ts_e<kIdescQK>(d, qh + 8 * k, b_desc(kh, k), 1u);
        long long c_i0 = 0;
        if constexpr (TIMED) c_i0 = clock64();
        commit(&sm.s_full[sb], static_cast<uint32_t>(g >> 1) & 1u);
        if (g + kOpStages < total_tiles) commit(&sm.k_free[s], static_cast<uint32_t>(g / kOpStages) & 1u);
        if constexpr (TIMED) {
          ok = warp_wait(&sm.s_full[sb], static_cast<uint32_t>(g >> 1) & 1u);
          c_a += static_cast<unsigned long long>(clock64() - c_i0);
        }
      }
      if (!ok) break;
      if (uidx + 2 < total_units) commit(&sm.q_tfree[qb], static_cast<uint32_t>(uidx >> 1) & 1u);
      ++uidx;
    }
    if constexpr (TIMED) {
      if (lane_is_first(tid)) {
        atomicAdd(&a.stage_cycles[kStageQk], c_a);
        atomicAdd(&a.stage_cycles[kStageKWait], c_b);
      }
    }
  } else if (warp == kPvWarp) {
    // ---------------- PV issuer (12 MMAs per key tile) ----------------
    int total_tiles, total_units;
    totals(total_tiles, total_units);
    unsigned long long c_a = 0, c_b = 0;
    int g = 0;
    bool ok = true;
    int vr = blockIdx.x < nunits ? unit_valid(a, blockIdx.x) : 0;
    for (unsigned unit = blockIdx.x; ok && unit < nunits; unit += ustep) {
      const Unit u = unit_of<LAYOUT>(a, unit, vr);
      vr = unit + ustep < nunits ? unit_valid(a, unit + ustep) : 0;  // in flight during this unit
      for (int t = 0; t < u.ntiles; ++t, ++g) {
        const int s = g % kOpStages, pb = g & 1;
        long long c_w0 = 0;
        if constexpr (TIMED) c_w0 = clock64();
        ok = warp_wait(&sm.p_ready2[pb], static_cast<uint32_t>(g >> 1) & 1u) &&
             warp_wait(&sm.v_ready[s], static_cast<uint32_t>(g / kOpStages) & 1u);
        if (ok && g >= 2)  // the softmax has read the partial of tile g-2 from this buffer
          ok = warp_wait(&sm.o_free[pb], static_cast<uint32_t>((g - 2) >> 1) & 1u);
        if constexpr (TIMED) c_b += static_cast<unsigned long long>(clock64() - c_w0);
        if (!ok) break;
        tc_fence_after();
        const uint32_t vh = smem_addr(&sm.op[s][kOpVh][0]), vl = smem_addr(&sm.op[s][kOpVl][0]);
        const uint32_t d = tmem + col_o(pb), aph = tmem + col_ph(pb), apl = aph + 32;
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16_ts_e<kIdescPV>(d, aph + 8 * k, v_desc(vl, k), k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16_ts_e<kIdescPV>(d, apl + 8 * k, v_desc(vh, k), 1u);
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16_ts_e<kIdescPV>(d, aph + 8 * k, v_desc(vh, k), 1u);
        long long c_i0 = 0;
        if constexpr (TIMED) c_i0 = clock64();
        commit(&sm.pv_done2[pb], static_cast<uint32_t>(g >> 1) & 1u);
        if (g + kOpStages < total_tiles) commit(&sm.v_free[s], static_cast<uint32_t>(g / kOpStages) & 1u);
        if constexpr (TIMED) {
          ok = warp_wait(&sm.pv_done2[pb], static_cast<uint32_t>(g >> 1) & 1u);
          c_a += static_cast<unsigned long long>(clock64() - c_i0);
        }
      }
    }
    if constexpr (TIMED) {
      if (lane_is_first(tid)) {
        atomicAdd(&a.stage_cycles[kStagePv], c_a);
        atomicAdd(&a.stage_cycles[kStageVWait], c_b);
      }
    }
  }
  __syncwarp();

  // End (every path).  After a timeout, drain this CTA's copies and MMAs
  // still in flight (bounded) before tensor memory is freed and the CTA ends.
  tc_fence_before();
  __syncthreads();
  if (*abort_flag != 0) {
    const long long t0 = clock64();
    auto drain = [&](uint64_t* bar, uint32_t parity) {
      while (!mbar_try_wait(bar, parity) && clock64() - t0 < a.timeout_cycles) {
      }
    };
    if (tid == kTmaWarp * 32) {  // the last q copy, and the last tile copied into each raw stage
      if (last_q >= 0) drain(&sm.q_full, static_cast<uint32_t>(last_q) & 1u);
      for (int s = 0; s < kRawStages; ++s) {
        const int t = last_g - (((last_g - s) % kRawStages) + kRawStages) % kRawStages;
        if (last_g >= 0 && t >= 0) drain(&sm.raw_full[s], static_cast<uint32_t>(t / kRawStages) & 1u);
      }
    }
    if ((warp == kQkWarp || warp == kPvWarp) && lane_is_first(tid) && last_commit)
      drain(last_commit, last_commit_parity);
  }
  __syncthreads();
  if (warp == kQkWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace tc16
}  // namespace raya
