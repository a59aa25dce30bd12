// tc32_ws.cuh — 3xTF32 tensor-core attention with two MMA-issuing warps and
// the O accumulator in tensor memory (sm_100a).
//
// 3xTF32 (tc32_common.cuh: raw fp32 tiles as the hi operands, lo =
// x - trunc(x), three tcgen05.mma products per tile), warp-specialised so
// that the tensor core, the softmax and the operand split overlap, with two
// measured refinements over a single-issuer pipeline:
//
//   * Two issuing threads.  One thread issuing tcgen05.mma kind::tf32 at
//     M = 128, N = 64 sustains one instruction per ~47.5 cycles; two threads
//     in different warps sustain one per ~33.5, the tensor core's own rate
//     (about 32).  So QK^T and PV are issued by separate warps, each with
//     its own commit barriers, and the tensor core interleaves the streams.
//   * O summed in registers.  PV(j) goes into a fresh tensor-memory partial
//     (a chain of 24 products); the softmax thread adds it into its O row in
//     fp32 registers with round-to-nearest adds before PV(j+1) overwrites it.
//     The tensor core's accumulation truncates toward zero (~0.5 ulp of the
//     accumulator per MMA, measured): summing every tile's PV into one
//     tensor-memory block put 1.5e-5 (6 tiles) to 1.6e-4 (128 tiles) of
//     absolute error into outputs of size 1.  The softmax thread keeps a
//     running log2-domain max m and rescales O only when a tile raises m by
//     more than 2^8; otherwise it keeps the old m, so weights reach at most
//     256, and O and the row sum l stay on the same scale, which the final
//     O / l removes.  The softmax warp group takes 232 registers
//     (setmaxnreg) for the O row next to a score row.
//
// Roles (384 threads):
//   warps 0-3   softmax: one query row per thread (TMEM lane = row): q and
//               its lo part into tensor memory; per key tile: S row -> mask
//               -> online softmax -> (rare) O rescale -> p and its lo part
//               into tensor memory; at the end O / l to global memory.
//   warps 4-9   split: raw K/V tiles by TMA (rings of 4, the hi operands),
//               their lo parts (ring of 3), V rows at or past valid_len
//               zeroed.  K and V are released separately: K's lo part of
//               tile j waits only for QK(j-3) (k_free), V's for PV(j-3)
//               (v_free), which also frees the raw stage refilled with tile
//               j+1 (one copy for K and V).  So QK(j) never waits on a PV
//               product.  (Issuing K's copy ahead of V's, on its own barrier,
//               measured slower.)
//   warp 10     QK issuer: QK(j) into S once K's lo part is ready and S has
//               been read.
//   warp 11     PV issuer: PV(j) into O once P(j) and V's lo part are ready.
//               Both issuers run their loops on the whole warp and issue from
//               one elected lane (a chain of MMAs into one accumulator then
//               runs at ~64 cycles per MMA instead of ~120).
//
// Tensor memory (512 columns): S [0,64), Q hi [64,128), Q lo [128,192),
// P0 hi/lo [192,320), P1 hi/lo [320,448), O [448,512).  P is double-buffered
// (the softmax writes P(j) while PV(j-1) still reads P(j-1); only PV(j-2)
// must be done) and S single-buffered (QK(j+1) starts as soon as the softmax
// has read S(j), its first step, so it still overlaps the rest of softmax(j)).
// Writing P over S instead (double-buffering both, QK up to two tiles ahead)
// measured slower: QK(j+1) then waits for PV(j-1) to complete, later than
// the softmax's read of S(j).
// Every wait is bounded; every group's exit is a collective decision of that
// group; after a timeout the issuing threads drain their copies and MMAs
// (bounded) before tensor memory is freed.
#pragma once

#include "tc32_common.cuh"

namespace raya {
namespace tc32 {

constexpr int kWsThreads = 384;
constexpr int kWsSplitThreads = 192;  // warps 4-9
constexpr int kWsQkThread = 320;      // warp 10, lane 0
constexpr int kWsPvThread = 352;      // warp 11, lane 0
constexpr float kRescaleLog2 = 8.0f;  // rescale O when the running max grows by more than 2^8
// Register split (setmaxnreg): the softmax warp group holds an O row (64
// floats) next to a score row; the split and issue warp groups need few.
// 232 + 136 + 136 = 504 = 3 warp groups x the 168 registers a thread of this
// launch gets, so the increase never waits on the pool.
constexpr int kWsSoftmaxRegs = 232, kWsOtherRegs = 136;
static_assert(kWsSoftmaxRegs + 2 * kWsOtherRegs <= 3 * 168, "register split above the launch's allocation");
constexpr int kSoftmaxBarrier = 2;    // named barrier of the softmax warps
static_assert(kLoStages >= 3, "the q tile is staged in lo stage 2 before the split warps first use it");
constexpr uint32_t kWsColS = 0, kWsColQh = 64, kWsColQl = 128, kWsColP = 192, kWsColO = 448;
// P buffer b: hi at kWsColP + 128 b, lo 64 columns further.
__device__ __forceinline__ uint32_t ws_col_ph(int b) { return kWsColP + 128u * static_cast<uint32_t>(b); }

// The copies of a [64 rows][32] column-half box of q (which 0), K (1) or V
// (2): head-major 2-D maps (column, slice*seq + pos) or the packed 4-D maps
// (column, head, which, b*seq + pos).
template <int LAYOUT>
__device__ __forceinline__ void ws_load(void* dst, const CUtensorMap* map, int x, int head, int which, int y,
                                        uint64_t* bar) {
  if constexpr (LAYOUT == tiled64::kHeadMajor)
    tiled64::tma_load_2d(dst, map, x, y, bar);
  else
    tiled64::tma_load_4d(dst, map, x, head, which, y, bar);
}

// raya's rotary embedding (ops.rs:110-141, rotate-half form) of one element
// pair: (x, y) -> (x*cos - y*sin, y*cos + x*sin), unfused f32 as the
// reference computes it (the FFMA kernels' rope_rows does the same).
__device__ __forceinline__ void ws_rot(float& x, float& y, float c, float sn) {
  const float nx = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, sn));
  const float ny = __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, sn));
  x = nx;
  y = ny;
}

// LAYOUT: tiled64::kHeadMajor (q, k, v, out as [batch*heads*seq][64]) or
// tiled64::kPacked (q, k, v read in place from the packed projection
// [batch*seq][3][heads][64], the output written as the context
// [batch*seq][heads][64]: encoder.rs:34-92).  ROPE: q and k rotated first
// (packed layout only), q rows by the softmax warps before they enter tensor
// memory, K tiles by the split warps before their lo parts are taken.
// UNITS: 128-row tiles per CTA (blockIdx.x * UNITS + 0 .. UNITS-1), run one
// after the other, each exactly as a CTA of its own (empty rings, barriers
// set up again), so that only the CTA's launch, exit, tensor-memory
// allocation and valid_len loads are shared between them.
// TIMED: the stage-timing build (the counterpart of the reference's
// StageTimes, tiled/stages.rs:1-31): per unit, clock64 cycles added into
// a.stage_cycles — [kStageQk] QK^T products in flight (issue to completion,
// seen by the QK issuer, which in this build also waits for each QK's
// completion: QK(j+1) needs the softmax's read of S(j) anyway), [kStageSoftmax]
// one softmax warp's work per tile (S read to P stored), [kStagePv] PV
// products in flight (the PV issuer waits for each PV's completion before
// the next, a small perturbation), [kStageKWait] the QK issuer waiting for
// K's operand split, [kStageVWait] the PV issuer waiting for P and V's split,
// [kStageRefill] one split warp's operand preparation, [kStageTiles] key
// tiles, [kStageTotal] thread 0's cycles from the unit's start to its output
// store.  The stages overlap in time; read them as proportions.
template <int LAYOUT, bool ROPE, int UNITS, bool TIMED = false>
__global__ void __launch_bounds__(kWsThreads, 1)
    tc32_ws_fwd(const __grid_constant__ AttnArgs a, const __grid_constant__ PipeMaps maps) {
  static_assert(!ROPE || LAYOUT == tiled64::kPacked, "the rotation is fused into the packed layout only");
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  PipeSmem& sm = *reinterpret_cast<PipeSmem*>(smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr));

  const int tid = threadIdx.x, warp = tid >> 5;
  const int seq = a.seq;
  // 32-bit index math (the host keeps batch * heads * row_tiles below 2^31).
  const unsigned nunits = static_cast<unsigned>(a.batch) * static_cast<unsigned>(a.heads) *
                          static_cast<unsigned>(a.row_tiles);
  // A unit's valid_len, read one unit ahead (used after the barrier set-up).
  auto load_valid = [&](unsigned unit) {
    return unit >= nunits ? 0
           : a.valid_len ? a.valid_len[unit / static_cast<unsigned>(a.row_tiles) / static_cast<unsigned>(a.heads)]
                         : seq;
  };
  int valid_next = load_valid(blockIdx.x * UNITS);
  bool tmem_held = false;  // (uniform) tensor memory allocated by an earlier unit of this CTA
  // Stage-timing accumulators of this thread (TIMED only).
  unsigned long long c_a = 0, c_b = 0;
  long long c_t0 = 0;
#pragma unroll 1
  for (int uu = 0; uu < UNITS; ++uu) {
  const unsigned unit = blockIdx.x * UNITS + uu;
  if (unit >= nunits) break;
  const int valid_raw = valid_next;
  if (uu + 1 < UNITS) valid_next = load_valid(unit + 1);
  const unsigned bh32 = unit / static_cast<unsigned>(a.row_tiles);
  const int tile = static_cast<int>(unit - bh32 * static_cast<unsigned>(a.row_tiles));
  const unsigned b32 = bh32 / static_cast<unsigned>(a.heads);
  const long long bh = bh32;
  const int b = static_cast<int>(b32);
  const int head = static_cast<int>(bh32 - b32 * static_cast<unsigned>(a.heads));
  const int r0 = tile * kBM;
  // First row of this slice in the loads' row coordinate, and the output
  // rows (head-major: the slice's rows; packed: this head's 64 columns of
  // each context row).
  const long long row_base = LAYOUT == tiled64::kHeadMajor ? bh * seq : static_cast<long long>(b) * seq;
  const size_t out_stride = LAYOUT == tiled64::kHeadMajor ? kD : static_cast<size_t>(a.heads) * kD;
  float* __restrict__ outp =
      a.out + (LAYOUT == tiled64::kHeadMajor ? static_cast<size_t>(row_base) * kD
                                             : (static_cast<size_t>(row_base) * a.heads + head) * kD);

  if (tid == 0) {  // barrier set-up needs no valid length: it overlaps that load
    for (int s = 0; s < kRawStages; ++s) mbar_init(&sm.raw_full[s], 1);
    for (int s = 0; s < kLoStages; ++s) {
      mbar_init(&sm.k_ready[s], kWsSplitThreads);
      mbar_init(&sm.v_ready[s], kWsSplitThreads);
      mbar_init(&sm.k_free[s], 1);
      mbar_init(&sm.v_free[s], 1);
    }
    mbar_init(&sm.s_full[0], 1);
    mbar_init(&sm.s_free[0], 128);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.p_ready2[s], 128);
      mbar_init(&sm.pv_done2[s], 1);
    }
    mbar_init(&sm.q_ready, 128);
    mbar_init(&sm.q_full, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  const int valid = valid_raw < 0 ? 0 : (valid_raw > seq ? seq : valid_raw);

  int klo = 0, khi = 0, unused = 0;
  const int last = min(r0 + kBM, valid) - 1;
  if (r0 < valid) {
    key_range(a, r0, valid, klo, unused);
    key_range(a, last, valid, unused, khi);
  }
  const int t_begin = klo / kBN;
  const int ntiles = khi > klo ? (khi + kBN - 1) / kBN - t_begin : 0;

  if (r0 >= valid || ntiles <= 0) {  // padding only: exact zeros, no loads, no tensor memory
    const int rows = min(kBM, seq - r0);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int idx = tid; idx < rows * 16; idx += kWsThreads)
      st_stream(outp + static_cast<size_t>(r0 + (idx >> 4)) * out_stride + (idx & 15) * 4, zero);
    continue;
  }

  if (!tmem_held) {
    if (warp == 10) {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_addr(&sm.tmem_base)),
                   "r"(kPipeTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tmem_held = true;
  }
  if (tid == 0) {
    // A later unit's copies land where the split warps' stores went (seen
    // through the end-of-unit barrier): order those before the async proxy.
    if (UNITS > 1 && uu > 0) fence_proxy_async_smem();
    // The first copies: the q tile (into lo stage 2, which the split warps
    // first write for key tile 2; from key tile 1 on they wait for q_ready),
    // then the K/V tiles of the first four raw stages.
    float* qs = &sm.lo[2][0][0][0][0];  // [half][128 rows][32]
    mbar_arrive_expect_tx(&sm.q_full, kBM * kD * 4u);
#pragma unroll
    for (int half = 0; half < 2; ++half)
#pragma unroll
      for (int rb = 0; rb < 2; ++rb)
        ws_load<LAYOUT>(qs + half * kBM * 32 + rb * 64 * 32, &maps.q, 32 * half, head, 0,
                        static_cast<int>(row_base + r0 + 64 * rb), &sm.q_full);
  }
  // K/V tile jj of the first four (thread 0): tile 0 before the CTA-wide
  // barrier, tiles 1-3 right after it, so the other warps do not wait for
  // their issue (~55 cycles per box).
  auto first_copy = [&](int jj) {
    const int y = static_cast<int>(row_base + (t_begin + jj) * kBN);
    mbar_arrive_expect_tx(&sm.raw_full[jj], 2u * kBN * kD * 4u);
    ws_load<LAYOUT>(&sm.raw[jj][0][0][0][0], &maps.k, 0, head, 1, y, &sm.raw_full[jj]);
    ws_load<LAYOUT>(&sm.raw[jj][0][1][0][0], &maps.k, 32, head, 1, y, &sm.raw_full[jj]);
    ws_load<LAYOUT>(&sm.raw[jj][1][0][0][0], &maps.v, 0, head, 2, y, &sm.raw_full[jj]);
    ws_load<LAYOUT>(&sm.raw[jj][1][1][0][0], &maps.v, 32, head, 2, y, &sm.raw_full[jj]);
  };
  if (tid == 0) first_copy(0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0)
    for (int jj = 1; jj < kRawStages && jj < ntiles; ++jj) first_copy(jj);
  if constexpr (TIMED) {
    c_a = c_b = 0;
    c_t0 = clock64();
  }
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_flag = &sm.abort_flag;

  // Drain bookkeeping (registers of the issuing threads).
  int last_tma_tile = min(kRawStages, ntiles) - 1;  // split thread 0: last tile copied (the first four by thread 0)
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

  if (warp < 4)
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kWsSoftmaxRegs));
  else
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kWsOtherRegs));
  if (warp < 4) {
    // ---------------- softmax warpgroup ----------------
    const int row = r0 + tid;
    int rlo = 0, rhi = 0;
    key_range(a, min(row, last), valid, rlo, rhi);
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float qscale = a.qscale;
    {  // q row (staged by TMA) -> tensor memory: q itself (read as its hi part), then q - trunc(q)
      float4 qcs[ROPE ? 16 : 1];  // this row's (cos, sin) pairs, loaded while the q tile is in flight
      if constexpr (ROPE) {
        const float4* t = reinterpret_cast<const float4*>(a.rope_cs + static_cast<size_t>(min(row, seq - 1)) * 64);
#pragma unroll
        for (int i4 = 0; i4 < 16; ++i4) qcs[i4] = __ldg(t + i4);
      }
      const bool wq = mbar_wait_bounded(&sm.q_full, 0, abort_flag, a.status, a.timeout_cycles);
      float qf[64];
      const uint32_t qs = smem_addr(&sm.lo[2][0][0][0][0]);
#pragma unroll
      for (int c4 = 0; c4 < 16; ++c4) {
        const float4 x = (wq && row < valid) ? lds128(qs + chunk_offset<kBM>(tid, c4)) : make_float4(0.f, 0.f, 0.f, 0.f);
        qf[4 * c4] = x.x;
        qf[4 * c4 + 1] = x.y;
        qf[4 * c4 + 2] = x.z;
        qf[4 * c4 + 3] = x.w;
      }
      if constexpr (ROPE) {
        if (wq && row < valid) {  // element i with i + 32, (cos, sin) of this position from the table
#pragma unroll
          for (int i4 = 0; i4 < 16; ++i4) {  // pairs i = 2*i4, 2*i4 + 1
            ws_rot(qf[2 * i4], qf[2 * i4 + 32], qcs[i4].x, qcs[i4].y);
            ws_rot(qf[2 * i4 + 1], qf[2 * i4 + 33], qcs[i4].z, qcs[i4].w);
          }
        }
      }
      tmem_st32(tmem + lane_off + kWsColQh, qf);
      tmem_st32(tmem + lane_off + kWsColQh + 32, qf + 32);
#pragma unroll
      for (int i = 0; i < 64; ++i) qf[i] = tf32_lo(qf[i]);
      tmem_st32(tmem + lane_off + kWsColQl, qf);
      tmem_st32(tmem + lane_off + kWsColQl + 32, qf + 32);
      tmem_wait_st();
      tc_fence_before();
      if (tid == 0) tma_store_wait_read();  // the previous unit's output store has read lo stage 1
      mbar_arrive(&sm.q_ready);
    }

    float m_used = -INFINITY, lsum = 0.f;
    float o[64];  // this row of O, summed in fp32 registers (round to nearest)
#pragma unroll
    for (int c = 0; c < 64; ++c) o[c] = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int pb = j & 1;  // P buffer
      const int kt = (t_begin + j) * kBN;
      bool w = mbar_wait_bounded(&sm.s_full[0], static_cast<uint32_t>(j) & 1u, abort_flag, a.status,
                                 a.timeout_cycles);
      if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
      tc_fence_after();
      long long c_s0 = 0;
      if constexpr (TIMED) c_s0 = clock64();
      float sv[64];
      tmem_ld32(tmem + lane_off + kWsColS, sv);
      tmem_ld32(tmem + lane_off + kWsColS + 32, sv + 32);
      tc_fence_before();
      mbar_arrive(&sm.s_free[0]);  // QK(j+1) may overwrite S

      if (!(rlo <= kt && rhi >= kt + kBN)) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (static_cast<unsigned>(kt + c - rlo) >= static_cast<unsigned>(rhi - rlo)) sv[c] = -INFINITY;
      }
      // Four chains; chain q takes columns q, q + 4, ..., q + 60.
      float m4[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) m4[q] = fmaxf(sv[q], sv[4 + q]);
#pragma unroll
      for (int c = 8; c < 64; c += 8)
#pragma unroll
        for (int q = 0; q < 4; ++q) m4[q] = fmax3(m4[q], sv[c + q], sv[c + 4 + q]);
      const float mc = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * qscale;
      // Move the running max only when it grows by more than 2^8 (or is
      // first set): O and l are then rescaled by alpha; otherwise weights
      // stay below 2^8 relative to the kept max.
      float alpha = 1.f;
      if (mc > m_used + kRescaleLog2) {
        alpha = ex2(m_used - mc);  // 0 when m_used was -inf
        m_used = mc;
      }
      const float mbase = m_used == -INFINITY ? 0.f : m_used;
      float2 rs2 = make_float2(0.f, 0.f);
      const float2 qs2 = make_float2(qscale, qscale), nb2 = make_float2(-mbase, -mbase);
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float2 arg = __ffma2_rn(make_float2(sv[c], sv[c + 1]), qs2, nb2);
        sv[c] = ex2(arg.x);
        sv[c + 1] = ex2(arg.y);
        rs2 = __fadd2_rn(rs2, make_float2(sv[c], sv[c + 1]));
      }
      const float rs = rs2.x + rs2.y;
      lsum = fmaf(lsum, alpha, rs);

      if (j >= 2) {  // P buffer pb is free once PV(j-2) is complete
        w = mbar_wait_bounded(&sm.pv_done2[pb], static_cast<uint32_t>((j - 2) >> 1) & 1u, abort_flag, a.status,
                              a.timeout_cycles);
        if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
        tc_fence_after();
      }
      // P -> tensor memory: p itself (read as its hi part), then p - trunc(p) in place.
      const uint32_t ph = tmem + lane_off + ws_col_ph(pb);
      tmem_st32(ph, sv);
      tmem_st32(ph + 32, sv + 32);
#pragma unroll
      for (int c = 0; c < 64; c += 2) tf32_lo2(sv[c], sv[c + 1]);
      tmem_st32(ph + 64, sv);
      tmem_st32(ph + 96, sv + 32);
      if (j > 0) {
        // O = (O + PV partial of tile j-1) * alpha, both at the previous
        // scale, once PV(j-1) is complete; PV(j) then overwrites the partial.
        w = mbar_wait_bounded(&sm.pv_done2[(j - 1) & 1], static_cast<uint32_t>((j - 1) >> 1) & 1u, abort_flag,
                              a.status, a.timeout_cycles);
        if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
        tc_fence_after();
        const bool rescale = __any_sync(0xffffffffu, alpha != 1.f);
#pragma unroll
        for (int c = 0; c < 64; c += 32) {
          float t[32];
          tmem_ld32(tmem + lane_off + kWsColO + c, t);
          if (rescale) {
            const float2 al2 = make_float2(alpha, alpha);
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const float2 r = __fmul2_rn(__fadd2_rn(make_float2(o[c + i], o[c + i + 1]), make_float2(t[i], t[i + 1])), al2);
              o[c + i] = r.x;
              o[c + i + 1] = r.y;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const float2 r = __fadd2_rn(make_float2(o[c + i], o[c + i + 1]), make_float2(t[i], t[i + 1]));
              o[c + i] = r.x;
              o[c + i + 1] = r.y;
            }
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&sm.p_ready2[pb]);
      if constexpr (TIMED) c_a += static_cast<unsigned long long>(clock64() - c_s0);
    }
    if (ok) {  // the last tile's partial
      const bool w = mbar_wait_bounded(&sm.pv_done2[(ntiles - 1) & 1], static_cast<uint32_t>((ntiles - 1) >> 1) & 1u,
                                       abort_flag, a.status, a.timeout_cycles);
      if (!__any_sync(0xffffffffu, !w)) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 64; c += 32) {
          float t[32];
          tmem_ld32(tmem + lane_off + kWsColO + c, t);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c + i] = __fadd_rn(o[c + i], t[i]);
        }
      }
    }
    // This row, normalised (+0.0f past valid_len), staged in shared memory
    // (lo stage 1 is idle now: every product is complete) under the 128-byte
    // swizzle, then stored by TMA: the [slices][seq][64] map clips rows past
    // the slice's end.  Thread 0 does not wait here for the store to read
    // its source (~1.1k cycles per unit, measured by per-event clocks): it
    // waits before it releases the next unit's q (q_ready), which the split
    // warps await before they first write lo stage 1, and before the CTA
    // exits.  (Deferring the wait: c5 +1.5-2%, c2 +3%.)
    {
      const float inv = (row < valid && lsum > 0.f) ? 1.0f / lsum : 0.f;
      float* stage = &sm.lo[1][0][0][0][0];  // [half][128 rows][32]
#pragma unroll
      for (int c4 = 0; c4 < 16; ++c4) {
        const float4 x = row < valid ? make_float4(o[4 * c4] * inv, o[4 * c4 + 1] * inv, o[4 * c4 + 2] * inv,
                                                   o[4 * c4 + 3] * inv)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        sts128(smem_addr(stage) + chunk_offset<kBM>(tid, c4), x);
      }
      fence_proxy_async_smem();
      bar_named(kSoftmaxBarrier, 128);
      if (tid == 0) {
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
          for (int rb = 0; rb < 2; ++rb)
            if (r0 + 64 * rb < seq) {  // (a box starting past the slice would be clipped whole; skip it)
              if constexpr (LAYOUT == tiled64::kHeadMajor)
                tma_store_3d(&maps.o, stage + half * kBM * 32 + rb * 64 * 32, 32 * half, r0 + 64 * rb,
                             static_cast<int>(bh));
              else  // [batch][seq][heads][64]: (column, head, pos, b)
                tma_store_4d(&maps.o, stage + half * kBM * 32 + rb * 64 * 32, 32 * half, head, r0 + 64 * rb, b);
            }
        tma_store_commit();
        if constexpr (TIMED) {
          atomicAdd(&a.stage_cycles[kStageSoftmax], c_a);
          atomicAdd(&a.stage_cycles[kStageTiles], static_cast<unsigned long long>(ntiles));
          atomicAdd(&a.stage_cycles[kStageTotal], static_cast<unsigned long long>(clock64() - c_t0));
        }
      }
    }
  } else if (warp < 10) {
    // ---------------- split warps ----------------
    const int st = tid - 128;
    auto issue = [&](int jj) {  // K and V of tile jj -> raw stage jj % 4
      const int s = jj & (kRawStages - 1);
      uint64_t* bar = &sm.raw_full[s];
      const int y = static_cast<int>(row_base + (t_begin + jj) * kBN);
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(bar, 2u * kBN * kD * 4u);
      ws_load<LAYOUT>(&sm.raw[s][0][0][0][0], &maps.k, 0, head, 1, y, bar);
      ws_load<LAYOUT>(&sm.raw[s][0][1][0][0], &maps.k, 32, head, 1, y, bar);
      ws_load<LAYOUT>(&sm.raw[s][1][0][0][0], &maps.v, 0, head, 2, y, bar);
      ws_load<LAYOUT>(&sm.raw[s][1][1][0][0], &maps.v, 32, head, 2, y, bar);
      last_tma_tile = jj;
    };
    constexpr int kPer = (kBN * 16 + kWsSplitThreads - 1) / kWsSplitThreads;  // float4s per thread per tile
    // With the rotation: (cos, sin) of this thread's element pairs of the next
    // K tile, loaded one tile ahead (float4 f of a column half, f < kBN*8:
    // row f / 8, logical chunk (f % 8) ^ (row % 8)).
    constexpr int kPairs = kBN * 8;
    constexpr int kPerR = ROPE ? (kPairs + kWsSplitThreads - 1) / kWsSplitThreads : 1;
    float4 kcs0[kPerR], kcs1[kPerR];
    auto load_kcs = [&](int jj) {
      if constexpr (ROPE) {
        const int kt = (t_begin + jj) * kBN;
#pragma unroll
        for (int i = 0; i < kPerR; ++i) {
          const int f = st + i * kWsSplitThreads;
          const int r = f >> 3, c = (f & 7) ^ (r & 7), pos = kt + r;
          if (f < kPairs && pos < seq) {
            const float4* t = reinterpret_cast<const float4*>(a.rope_cs + (static_cast<size_t>(pos) * 32 + 4 * c) * 2);
            kcs0[i] = __ldg(t);  // (cos, sin) of i = 4c, 4c+1
            kcs1[i] = __ldg(t + 1);  // and 4c+2, 4c+3
          }
        }
      }
    };
    load_kcs(0);
    for (int j = 0; j < ntiles; ++j) {
      const int s3 = j % kLoStages, s4 = j & (kRawStages - 1);
      const uint32_t ph = static_cast<uint32_t>(j / kLoStages - 1) & 1u;  // phase of tile j-3's release
      // K: the raw tile and K's lo stage (QK(j-3) done).
      bool w = mbar_wait_bounded(&sm.raw_full[s4], static_cast<uint32_t>(j >> 2) & 1u, abort_flag, a.status,
                                 a.timeout_cycles);
      if (w && j >= kLoStages) w = mbar_wait_bounded(&sm.k_free[s3], ph, abort_flag, a.status, a.timeout_cycles);
      // q left lo stage 2, and the previous unit's output store has read lo stage 1
      if (w && j == 1) w = mbar_wait_bounded(&sm.q_ready, 0, abort_flag, a.status, a.timeout_cycles);
      if (bar_any(kSplitBarrier, kWsSplitThreads, !w)) break;
      long long c_k0 = 0;
      if constexpr (TIMED) c_k0 = clock64();
      const int nv = min(kBN, valid - (t_begin + j) * kBN);
      float4* kr = reinterpret_cast<float4*>(&sm.raw[s4][0][0][0][0]);
      float4* vr = reinterpret_cast<float4*>(&sm.raw[s4][1][0][0][0]);
      float4* kl = reinterpret_cast<float4*>(&sm.lo[s3][0][0][0][0]);
      float4* vl = reinterpret_cast<float4*>(&sm.lo[s3][1][0][0][0]);
      if constexpr (ROPE) {
        // Rotate K in place (it is the hi operand), then take its lo part.
        // Element i of a key row sits in column half 0 and element i + 32 in
        // half 1 at the same swizzled offset: float4 f of half 0 (row f / 8,
        // stored chunk f % 8 = logical chunk (f % 8) ^ (row % 8)) pairs with
        // float4 f of half 1.  Rows at or past valid_len stay as they are
        // (masked keys).
        const int kt = (t_begin + j) * kBN;
#pragma unroll
        for (int i = 0; i < kPerR; ++i) {
          const int f = st + i * kWsSplitThreads;
          if (f < kPairs) {
            float4 x0 = kr[f], x1 = kr[f + kPairs];
            const int r = f >> 3, pos = kt + r;
            if (pos < valid) {
              const float4 t0 = kcs0[i], t1 = kcs1[i];  // (cos, sin) of i = 4c .. 4c+3, c = (f % 8) ^ (r % 8)
              ws_rot(x0.x, x1.x, t0.x, t0.y);
              ws_rot(x0.y, x1.y, t0.z, t0.w);
              ws_rot(x0.z, x1.z, t1.x, t1.y);
              ws_rot(x0.w, x1.w, t1.z, t1.w);
              kr[f] = x0;
              kr[f + kPairs] = x1;
            }
            kl[f] = make_float4(tf32_lo(x0.x), tf32_lo(x0.y), tf32_lo(x0.z), tf32_lo(x0.w));
            kl[f + kPairs] = make_float4(tf32_lo(x1.x), tf32_lo(x1.y), tf32_lo(x1.z), tf32_lo(x1.w));
          }
        }
        if (j + 1 < ntiles) load_kcs(j + 1);
      } else {
        float4 x[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i)
          if (st + i * kWsSplitThreads < kBN * 16) x[i] = kr[st + i * kWsSplitThreads];
#pragma unroll
        for (int i = 0; i < kPer; ++i)
          if (st + i * kWsSplitThreads < kBN * 16)
            kl[st + i * kWsSplitThreads] =
                make_float4(tf32_lo(x[i].x), tf32_lo(x[i].y), tf32_lo(x[i].z), tf32_lo(x[i].w));
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      mbar_arrive(&sm.k_ready[s3]);  // QK(j) may start
      if constexpr (TIMED) c_a += static_cast<unsigned long long>(clock64() - c_k0);
      // V: V's lo stage and the raw stage of tile j-3 (PV(j-3) done).
      if (j >= kLoStages) {
        w = mbar_wait_bounded(&sm.v_free[s3], ph, abort_flag, a.status, a.timeout_cycles);
        if (w && st == 0 && j + 1 < ntiles) issue(j + 1);  // raw stage (j+1)%4 held tile j-3
      }
      if (bar_any(kSplitBarrier, kWsSplitThreads, !w)) break;
      long long c_v0 = 0;
      if constexpr (TIMED) c_v0 = clock64();
      {
        float4 x[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i)
          if (st + i * kWsSplitThreads < kBN * 16) x[i] = vr[st + i * kWsSplitThreads];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int f = st + i * kWsSplitThreads;
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
      if constexpr (TIMED) c_a += static_cast<unsigned long long>(clock64() - c_v0);
      bar_named(kSplitBarrier, kWsSplitThreads);
    }
    if constexpr (TIMED)
      if (st == 0) atomicAdd(&a.stage_cycles[kStageRefill], c_a);
  } else if (warp == kWsQkThread / 32) {
    // ---------------- QK^T issuer (the whole warp runs the loop; an elected lane issues) ----------------
    bool ok = warp_wait(&sm.q_ready, 0);
    for (int j = 0; ok && j < ntiles; ++j) {
      const int s3 = j % kLoStages;
      long long c_w0 = 0;
      if constexpr (TIMED) c_w0 = clock64();
      ok = warp_wait(&sm.k_ready[s3], static_cast<uint32_t>(j / kLoStages) & 1u);
      if constexpr (TIMED) c_b += static_cast<unsigned long long>(clock64() - c_w0);
      if (ok && j >= 1)  // the softmax has read S(j-1)
        ok = warp_wait(&sm.s_free[0], static_cast<uint32_t>(j - 1) & 1u);
      if (!ok) break;
      tc_fence_after();
      const uint32_t khi = smem_addr(&sm.raw[j & (kRawStages - 1)][0][0][0][0]);
      const uint32_t klo = smem_addr(&sm.lo[s3][0][0][0][0]);
      const uint32_t d = tmem + kWsColS;
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts_e(d, tmem + kWsColQh + 8 * k, k_desc(klo, k), kIdescQK, k > 0 ? 1u : 0u);
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts_e(d, tmem + kWsColQl + 8 * k, k_desc(khi, k), kIdescQK, 1u);
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts_e(d, tmem + kWsColQh + 8 * k, k_desc(khi, k), kIdescQK, 1u);
      long long c_i0 = 0;
      if constexpr (TIMED) c_i0 = clock64();
      commit(&sm.s_full[0], static_cast<uint32_t>(j) & 1u);
      if (j + kLoStages < ntiles) commit(&sm.k_free[s3], static_cast<uint32_t>(j / kLoStages) & 1u);
      if constexpr (TIMED) {
        ok = warp_wait(&sm.s_full[0], static_cast<uint32_t>(j) & 1u);
        c_a += static_cast<unsigned long long>(clock64() - c_i0);
      }
    }
    if constexpr (TIMED) {
      if (tid == kWsQkThread) {
        atomicAdd(&a.stage_cycles[kStageQk], c_a);
        atomicAdd(&a.stage_cycles[kStageKWait], c_b);
      }
    }
  } else if (warp == kWsPvThread / 32) {
    // ---------------- PV issuer (the whole warp runs the loop; an elected lane issues) ----------------
    bool ok = true;
    for (int j = 0; ok && j < ntiles; ++j) {
      const int s3 = j % kLoStages;
      const int pb = j & 1;
      long long c_w0 = 0;
      if constexpr (TIMED) c_w0 = clock64();
      ok = warp_wait(&sm.p_ready2[pb], static_cast<uint32_t>(j >> 1) & 1u) &&
           warp_wait(&sm.v_ready[s3], static_cast<uint32_t>(j / kLoStages) & 1u);
      if constexpr (TIMED) c_b += static_cast<unsigned long long>(clock64() - c_w0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t vh = smem_addr(&sm.raw[j & (kRawStages - 1)][1][0][0][0]);
      const uint32_t vl = smem_addr(&sm.lo[s3][1][0][0][0]);
      const uint32_t d = tmem + kWsColO, aph = tmem + ws_col_ph(pb), apl = aph + 64;
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts_e(d, aph + 8 * k, v_desc(vl, k), kIdescPV, k > 0 ? 1u : 0u);
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts_e(d, apl + 8 * k, v_desc(vh, k), kIdescPV, 1u);
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts_e(d, aph + 8 * k, v_desc(vh, k), kIdescPV, 1u);
      long long c_i0 = 0;
      if constexpr (TIMED) c_i0 = clock64();
      commit(&sm.pv_done2[pb], static_cast<uint32_t>(j >> 1) & 1u);
      if (j + kLoStages < ntiles) commit(&sm.v_free[s3], static_cast<uint32_t>(j / kLoStages) & 1u);
      if constexpr (TIMED) {
        ok = warp_wait(&sm.pv_done2[pb], static_cast<uint32_t>(j >> 1) & 1u);
        c_a += static_cast<unsigned long long>(clock64() - c_i0);
      }
    }
    if constexpr (TIMED) {
      if (tid == kWsPvThread) {
        atomicAdd(&a.stage_cycles[kStagePv], c_a);
        atomicAdd(&a.stage_cycles[kStageVWait], c_b);
      }
    }
    if constexpr (UNITS > 1) {
      // The next unit sets the barriers up again: the one commit no other
      // thread waits for (PV of tile ntiles-2) must have arrived first.
      if (ok && ntiles >= 2) warp_wait(&sm.pv_done2[(ntiles - 2) & 1], static_cast<uint32_t>((ntiles - 2) >> 1) & 1u);
    }
  }
  __syncwarp();

  // End of the unit (every path); after a timeout first drain this CTA's
  // copies and MMAs still in flight (bounded), and stop.
  tc_fence_before();
  __syncthreads();
  const bool aborted = *abort_flag != 0;
  if (aborted) {
    const long long t0 = clock64();
    auto drain = [&](uint64_t* bar, uint32_t parity) {
      while (!mbar_try_wait(bar, parity) && clock64() - t0 < a.timeout_cycles) {
      }
    };
    if (tid == 128) {  // the q copy, and the last tile issued into each raw stage
      drain(&sm.q_full, 0);
#pragma unroll
      for (int s = 0; s < kRawStages; ++s) {
        const int t = last_tma_tile - ((last_tma_tile - s) & (kRawStages - 1));
        if (t >= 0) drain(&sm.raw_full[s], static_cast<uint32_t>(t >> 2) & 1u);
      }
    }
    if ((tid == kWsQkThread || tid == kWsPvThread) && last_commit) drain(last_commit, last_commit_parity);
  }
  __syncthreads();
  if (aborted) break;
  }  // units of this CTA
  if (tid == 0) tma_store_wait_read();  // the last output store has read its source
  if (tmem_held && warp == 10) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sm.tmem_base), "r"(kPipeTmemCols)
                 : "memory");
  }
}

}  // namespace tc32
}  // namespace raya
