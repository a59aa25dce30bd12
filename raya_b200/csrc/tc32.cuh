// tc32.cuh — block-local attention on the 5th-generation tensor cores
// (tcgen05, sm_100a) in 3xTF32: fp32-level accuracy from TF32 products.
//
// Each fp32 operand x is split into hi = x rounded to TF32 (11 significant
// bits) and lo = x - hi (exact in fp32, |lo| <= 2^-11 |x|), itself rounded
// to TF32.  A product is taken as hi*hi + hi*lo + lo*hi: the rounding of lo
// and the dropped lo*lo term are both below ~2^-22 relative, near fp32's own
// 2^-24, and the accumulation in tensor memory is fp32.
//
// Structure (one CTA per (slice, 128 query rows), 4 warps, one query row per
// thread — TMEM lane r is query row r):
//   * Q tile, then per 64-key tile the K and V tiles, arrive by tensor-map
//     TMA (Q, K: 128-byte swizzle of 16-byte chunks; V: 128-byte swizzle of
//     32-byte granules, which the MN-major TF32 B operand requires); a
//     split pass rewrites each tile as hi in place plus lo in a second
//     buffer; V rows at or past valid_len are zeroed there, so padding never
//     reaches the PV product;
//   * S = Q K^T: 24 tcgen05.mma (kind::tf32, M=128, N=64, K=8) into 64 TMEM
//     columns, issued by one thread, completion through tcgen05.commit on an
//     mbarrier;
//   * each thread loads its row of S (tcgen05.ld 32x32b), masks, and runs the
//     online softmax of the FFMA kernel (running max kept pre-scaled,
//     p = 2^(s*scale*log2e - m), alpha rescale of its O row held in registers);
//     p is split into hi/lo and stored as the A operand of the next product;
//   * PV: 24 tcgen05.mma (B = V, MN-major) into another 64 TMEM columns; each
//     thread adds its row to O.
// Every mbarrier wait is bounded; TMEM is freed on every path.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "tiled64.cuh"

namespace raya {
namespace tc32 {

constexpr int kD = 64;
constexpr int kBM = 128;        // query rows per CTA (MMA M)
constexpr int kBN = 64;         // keys per tile (MMA N of QK^T, K of PV)
constexpr int kThreads = 128;
constexpr int kTmemCols = 128;  // S: columns [0, 64), PV: [64, 128)

// 128-byte-swizzled [rows][64] fp32 tiles, as two column halves of
// [rows][32] (each half 1024-byte aligned).
template <int ROWS>
struct Tile {
  float h[2][ROWS][32];
};

struct Smem {
  Tile<kBM> q, ql;    // Q hi (in place) and lo
  Tile<kBN> k, kl;    // K hi (in place) and lo
  Tile<kBN> v, vl;    // V hi (in place) and lo
  Tile<kBM> p, pl;    // P hi and lo (A operand of PV)
  uint64_t qbar, kbar, vbar, mmabar;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t smem_bytes() { return sizeof(Smem) + 1024; }

// Instruction descriptors (kind::tf32, D = F32, M = 128, N = 64): A and B
// K-major for S = Q K^T; B MN-major (V's columns contiguous) for PV.
constexpr uint32_t kIdescQK = (1u << 4) | (2u << 7) | (2u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescPV = kIdescQK | (1u << 16);

// Shared-memory matrix descriptor layouts: the 128-byte swizzle of 16-byte
// chunks (K-major operands), and the 128-byte swizzle of 32-byte granules,
// the only layout the tensor core takes for an MN-major TF32 operand.
constexpr uint64_t kSwizzle128 = 2, kSwizzle128Atom32 = 1;

// Shared-memory matrix descriptor with the Blackwell version bits: start
// address, leading and stride byte offsets (all >> 4), layout.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint64_t layout = kSwizzle128) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFF) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (layout << 61);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.  The load and its
// wait sit in one asm statement, so no use of the registers can be scheduled
// between them.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// x rounded to TF32 (11 significant bits), half away from zero: adding half
// a TF32 ulp to the magnitude bits carries into the kept bits exactly when the
// dropped 13 bits are at least half.
__device__ __forceinline__ float tf32_rn(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// x - trunc(x), where trunc(x) is the TF32 value the tensor core reads for
// the fp32 bit pattern x (its 13 low mantissa bits dropped).  Exact in fp32.
__device__ __forceinline__ float tf32_lo(float x) {
  return __fsub_rn(x, __uint_as_float(__float_as_uint(x) & 0xFFFFE000u));
}

// Split pass over a [ROWS][64] swizzled tile: hi in place, lo into `lo`.
// Rows at or past `nvalid` are zeroed in both (only asked for V).
template <int ROWS>
__device__ __forceinline__ void split_tile(Tile<ROWS>& t, Tile<ROWS>& lo, int nvalid, int tid) {
  float4* a = reinterpret_cast<float4*>(&t.h[0][0][0]);
  float4* b = reinterpret_cast<float4*>(&lo.h[0][0][0]);
  constexpr int kVec = ROWS * 16;
  for (int f = tid; f < kVec; f += kThreads) {
    const int row = (f % (ROWS * 8)) >> 3;
    float4 x = a[f];
    float4 h, l;
    if (row < nvalid) {
      h = make_float4(tf32_rn(x.x), tf32_rn(x.y), tf32_rn(x.z), tf32_rn(x.w));
      l = make_float4(tf32_rn(__fsub_rn(x.x, h.x)), tf32_rn(__fsub_rn(x.y, h.y)), tf32_rn(__fsub_rn(x.z, h.z)),
                      tf32_rn(__fsub_rn(x.w, h.w)));
    } else {
      h = l = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    a[f] = h;
    b[f] = l;
  }
}

// Byte offset of 16-byte chunk c4 (columns 4c4..4c4+3) of row r in a
// swizzled [ROWS][64] tile.
template <int ROWS>
__device__ __forceinline__ uint32_t chunk_offset(int r, int c4) {
  return static_cast<uint32_t>((c4 >> 3) * ROWS * 128 + r * 128 + ((((c4 & 7) ^ (r & 7))) << 4));
}

// 3 x 8 MMAs: D (+)= A B over K = 64 with A/B hi/lo descriptors built from
// base addresses.  Q-style A (K-major, 64 columns in two 128-byte halves of
// ROWS_A rows): k-step s is half s/4 at byte 32*(s%4).  B K-major (K^T) the
// same with 64 rows.  B MN-major (V, loaded with the 32-byte-granule
// swizzle): k-step s is key rows 8s..8s+7 (1024 bytes, two 4-row atoms 512
// bytes apart), the second 32 columns 8 KB further.
template <bool B_MN>
__device__ __forceinline__ void mma_3xtf32(uint32_t d_tmem, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi,
                                           uint32_t b_lo, uint32_t idesc) {
  constexpr uint32_t kAHalf = kBM * 128;
  constexpr uint32_t kBHalf = kBN * 128;
  auto a_at = [&](uint32_t base, int s) { return smem_desc(base + (s >> 2) * kAHalf + (s & 3) * 32, 16, 1024); };
  auto b_at = [&](uint32_t base, int s) {
    return B_MN ? smem_desc(base + s * 1024, kBHalf, 512, kSwizzle128Atom32)
                : smem_desc(base + (s >> 2) * kBHalf + (s & 3) * 32, 16, 1024);
  };
  // lo terms first (smaller), then hi*hi
#pragma unroll
  for (int s = 0; s < 8; ++s) mma_tf32(d_tmem, a_at(a_hi, s), b_at(b_lo, s), idesc, s > 0 ? 1u : 0u);
#pragma unroll
  for (int s = 0; s < 8; ++s) mma_tf32(d_tmem, a_at(a_lo, s), b_at(b_hi, s), idesc, 1u);
#pragma unroll
  for (int s = 0; s < 8; ++s) mma_tf32(d_tmem, a_at(a_hi, s), b_at(b_hi, s), idesc, 1u);
}

__global__ void __launch_bounds__(kThreads, 1)
    tc32_fwd(const __grid_constant__ AttnArgs a, const __grid_constant__ tiled64::TmaMaps maps) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));

  const int tid = threadIdx.x, warp = tid >> 5;
  const int tile = static_cast<int>(blockIdx.x % static_cast<unsigned>(a.row_tiles));
  const long long bh = blockIdx.x / static_cast<unsigned>(a.row_tiles);
  const int b = static_cast<int>(bh / a.heads);
  const int seq = a.seq;
  int valid = a.valid_len ? a.valid_len[b] : seq;
  valid = valid < 0 ? 0 : (valid > seq ? seq : valid);
  const int r0 = tile * kBM;
  const long long row_base = bh * seq;
  float* __restrict__ outp = a.out + static_cast<size_t>(row_base) * kD;

  if (r0 >= valid) {  // padding only: exact zeros, no loads, no tensor memory
    const int rows = min(kBM, seq - r0);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int idx = tid; idx < rows * 16; idx += kThreads)
      st_stream(outp + static_cast<size_t>(r0 + (idx >> 4)) * kD + (idx & 15) * 4, zero);
    return;
  }

  const int last = min(r0 + kBM, valid) - 1;
  int klo, khi, unused;
  key_range(a, r0, valid, klo, unused);
  key_range(a, last, valid, unused, khi);
  const int t_begin = klo / kBN;
  const int ntiles = (khi + kBN - 1) / kBN - t_begin;

  // This thread's query row and its key range.
  const int row = r0 + tid;
  int rlo = 0, rhi = 0;
  key_range(a, min(row, last), valid, rlo, rhi);

  if (warp == 0) {  // tensor memory: S and PV accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&sm.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(&sm.qbar, 1);
    mbar_init(&sm.kbar, 1);
    mbar_init(&sm.vbar, 1);
    mbar_init(&sm.mmabar, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t t_s = tmem, t_pv = tmem + 64;                     // column bases
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;  // this warp's TMEM lanes

  if (tid == 0) {
    tiled64::stage_tile<tiled64::kHeadMajor>(&sm.q.h[0][0][0], &sm.q.h[1][0][0], &maps.q, 0, 0,
                                             static_cast<int>(row_base + r0), kBM, &sm.qbar);
    const int y = static_cast<int>(row_base + t_begin * kBN);
    tiled64::stage_tile<tiled64::kHeadMajor>(&sm.k.h[0][0][0], &sm.k.h[1][0][0], &maps.k, 0, 1, y, kBN, &sm.kbar);
    tiled64::stage_tile<tiled64::kHeadMajor>(&sm.v.h[0][0][0], &sm.v.h[1][0][0], &maps.v, 0, 2, y, kBN, &sm.vbar);
  }

  volatile int* abort_flag = &sm.abort_flag;
  const float qscale = a.qscale;
  float o[64];
#pragma unroll
  for (int c = 0; c < 64; ++c) o[c] = 0.f;
  float msc = -INFINITY, l = 0.f;
  int kissued = 1, vissued = 1, mma_phase = 0;

  // Every exit from the key loop is a collective decision (__syncthreads_or),
  // so that no thread is ever left at a barrier the others have passed.
  bool ok = mbar_wait_bounded(&sm.qbar, 0, abort_flag, a.status, a.timeout_cycles);
  if (ok) split_tile<kBM>(sm.q, sm.ql, kBM, tid);
  ok = !__syncthreads_or(!ok);

  const uint32_t aq = smem_addr(&sm.q.h[0][0][0]), aql = smem_addr(&sm.ql.h[0][0][0]);
  const uint32_t ak = smem_addr(&sm.k.h[0][0][0]), akl = smem_addr(&sm.kl.h[0][0][0]);
  const uint32_t av = smem_addr(&sm.v.h[0][0][0]), avl = smem_addr(&sm.vl.h[0][0][0]);
  const uint32_t ap = smem_addr(&sm.p.h[0][0][0]), apl = smem_addr(&sm.pl.h[0][0][0]);

  for (int t = 0; ok && t < ntiles; ++t) {
    const uint32_t par = static_cast<uint32_t>(t) & 1u;
    const int kt = (t_begin + t) * kBN;
    const int nv = min(kBN, valid - kt);

    bool w = mbar_wait_bounded(&sm.kbar, par, abort_flag, a.status, a.timeout_cycles) &&
             mbar_wait_bounded(&sm.vbar, par, abort_flag, a.status, a.timeout_cycles);
    if (w) {
      split_tile<kBN>(sm.k, sm.kl, kBN, tid);
      split_tile<kBN>(sm.v, sm.vl, nv, tid);
    }
    fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
    tc_fence_before();
    if (__syncthreads_or(!w)) { ok = false; break; }

    // S = Q K^T (3xTF32)
    if (tid == 0) {
      tc_fence_after();
      mma_3xtf32<false>(t_s, aq, aql, ak, akl, kIdescQK);
      mma_commit(&sm.mmabar);
    }
    w = mbar_wait_bounded(&sm.mmabar, static_cast<uint32_t>(mma_phase++) & 1u, abort_flag, a.status,
                          a.timeout_cycles);
    if (__syncthreads_or(!w)) { ok = false; break; }
    tc_fence_after();
    // K is no longer read: load the next K tile behind the softmax.
    if (tid == 0 && t + 1 < ntiles) {
      tiled64::stage_tile<tiled64::kHeadMajor>(&sm.k.h[0][0][0], &sm.k.h[1][0][0], &maps.k, 0, 1,
                                               static_cast<int>(row_base + kt + kBN), kBN, &sm.kbar);
      ++kissued;
    }

    // This row of S -> online softmax -> P (hi, lo) in shared memory.
    float sv[64];
    tmem_ld32(t_s + lane_off, sv);
    tmem_ld32(t_s + lane_off + 32, sv + 32);
    const bool whole = rlo <= kt && rhi >= kt + kBN;
    if (!whole) {
#pragma unroll
      for (int c = 0; c < 64; ++c)
        if (static_cast<unsigned>(kt + c - rlo) >= static_cast<unsigned>(rhi - rlo)) sv[c] = -INFINITY;
    }
    float tmax = sv[0];
#pragma unroll
    for (int c = 1; c < 64; ++c) tmax = fmaxf(tmax, sv[c]);
    const float mnew = fmaxf(msc, tmax * qscale);
    const float mbase = mnew == -INFINITY ? 0.f : mnew;
    const float alpha = ex2(msc - mbase);
    msc = mnew;
    float rs = 0.f;
#pragma unroll
    for (int c4 = 0; c4 < 16; ++c4) {
      float4 p4;
      p4.x = ex2(fmaf(sv[4 * c4 + 0], qscale, -mbase));
      p4.y = ex2(fmaf(sv[4 * c4 + 1], qscale, -mbase));
      p4.z = ex2(fmaf(sv[4 * c4 + 2], qscale, -mbase));
      p4.w = ex2(fmaf(sv[4 * c4 + 3], qscale, -mbase));
      rs += (p4.x + p4.y) + (p4.z + p4.w);
      const float4 h = make_float4(tf32_rn(p4.x), tf32_rn(p4.y), tf32_rn(p4.z), tf32_rn(p4.w));
      const float4 lo4 = make_float4(tf32_rn(__fsub_rn(p4.x, h.x)), tf32_rn(__fsub_rn(p4.y, h.y)),
                                     tf32_rn(__fsub_rn(p4.z, h.z)), tf32_rn(__fsub_rn(p4.w, h.w)));
      const uint32_t off = chunk_offset<kBM>(tid, c4);
      sts128(ap + off, h);
      sts128(apl + off, lo4);
    }
    l = fmaf(l, alpha, rs);
#pragma unroll
    for (int c = 0; c < 64; ++c) o[c] *= alpha;
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // O += P V (3xTF32), V MN-major.
    if (tid == 0) {
      tc_fence_after();
      mma_3xtf32<true>(t_pv, ap, apl, av, avl, kIdescPV);
      mma_commit(&sm.mmabar);
    }
    w = mbar_wait_bounded(&sm.mmabar, static_cast<uint32_t>(mma_phase++) & 1u, abort_flag, a.status,
                          a.timeout_cycles);
    if (__syncthreads_or(!w)) { ok = false; break; }
    tc_fence_after();
    if (tid == 0 && t + 1 < ntiles) {
      tiled64::stage_tile<tiled64::kHeadMajor>(&sm.v.h[0][0][0], &sm.v.h[1][0][0], &maps.v, 0, 2,
                                               static_cast<int>(row_base + kt + kBN), kBN, &sm.vbar);
      ++vissued;
    }
#pragma unroll
    for (int c = 0; c < 64; c += 32) {
      float tmp[32];
      tmem_ld32(t_pv + lane_off + c, tmp);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[c + i] += tmp[i];
    }
  }

  // Epilogue: this thread's row, normalised (+0.0f past valid_len).
  if (row < seq) {
    const float inv = (row < valid && l > 0.f) ? 1.0f / l : 0.f;
    float* orow = outp + static_cast<size_t>(row) * kD;
#pragma unroll
    for (int c = 0; c < 64; c += 4) {
      const float4 x = row < valid ? make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
      st_stream(orow + c, x);
    }
  }

  // Release tensor memory (every path), after a timeout drain our copies.
  tc_fence_before();
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
    drain(&sm.kbar, kissued);
    drain(&sm.vbar, vissued);
    drain(&sm.mmabar, mma_phase);
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace tc32
}  // namespace raya
