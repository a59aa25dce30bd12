// tc32_common.cuh — building blocks of the 3xTF32 tensor-core attention
// kernels (sm_100a): tile sizes, tcgen05 instruction and shared-memory
// descriptors, tensor-memory loads and stores, the TF32 operand split, the
// TMA tile stores, and the shared-memory rings of the two-issuer kernel
// (tc32_ws.cuh).
//
// 3xTF32.  Every fp32 operand x (q, k, v and the softmax weights p) enters
// the tensor core twice: as x itself, which kind::tf32 reads with its 13 low
// mantissa bits dropped (truncation toward zero, measured on B200 with an
// operand of 1 + 2^-11 + 2^-13, which reads as exactly 1), and as
// lo = x - trunc(x), exact in fp32 and truncated in turn.  A product is taken
// as hi*lo + lo*hi + hi*hi (correction terms first, into an fp32 accumulator
// in tensor memory); the dropped lo*lo term and the truncation of lo are
// below 2^-21 relative per product, so results match fp32 FFMA arithmetic to
// ~1e-7 absolute on the parity cases.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "tiled64.cuh"

namespace raya {
namespace tc32 {

constexpr int kD = 64;
constexpr int kBM = 128;  // query rows per row tile (MMA M)
constexpr int kBN = 64;   // keys per tile (MMA N of QK^T, K of PV)

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

// 32 consecutive 32-bit columns of this thread's lane; completion is awaited
// by tmem_wait_st.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
      "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
      "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// x - trunc(x), where trunc(x) is the TF32 value the tensor core reads for
// the fp32 bit pattern x (its 13 low mantissa bits dropped).  Exact in fp32.
__device__ __forceinline__ float tf32_lo(float x) {
  return __fsub_rn(x, __uint_as_float(__float_as_uint(x) & 0xFFFFE000u));
}

// x - trunc(x) for a pair, in place (one packed FMA: x - hi is exact).
__device__ __forceinline__ void tf32_lo2(float& x, float& y) {
  const float2 hi = make_float2(__uint_as_float(__float_as_uint(x) & 0xFFFFE000u),
                                __uint_as_float(__float_as_uint(y) & 0xFFFFE000u));
  const float2 lo = __ffma2_rn(hi, make_float2(-1.f, -1.f), make_float2(x, y));
  x = lo.x;
  y = lo.y;
}

// max of three floats in one instruction.
__device__ __forceinline__ float fmax3(float x, float y, float z) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(x), "f"(y), "f"(z));
  return r;
}

// Byte offset of 16-byte chunk c4 (columns 4c4..4c4+3) of row r in a
// 128-byte-swizzled [ROWS][64] tile held as two column halves of [ROWS][32].
template <int ROWS>
__device__ __forceinline__ uint32_t chunk_offset(int r, int c4) {
  return static_cast<uint32_t>((c4 >> 3) * ROWS * 128 + r * 128 + ((((c4 & 7) ^ (r & 7))) << 4));
}

// D (+)= A B with A read from tensor memory (M = 128 rows in lanes, K = 8
// 32-bit columns) and B from a shared-memory descriptor, in elected-lane
// form: the whole issuing warp runs the issue loop (so its operands are
// warp-uniform) and one lane, picked by elect.sync, issues.
// Measured on B200 (M = 128, N = 64, K = 8, tf32): a chain of MMAs into one
// accumulator issued this way runs at ~64 cycles per MMA, against ~120 when
// a single lane issues from a divergent branch; two issuing warps with a
// chain each reach the tensor core's ~32 cycles per MMA.
__device__ __forceinline__ void mma_tf32_ts_e(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}
// tcgen05.commit from the elected lane of a warp that runs the issue loop:
// arrives once on `bar` when every MMA that lane issued is complete.
__device__ __forceinline__ void mma_commit_e(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_addr(bar))
      : "memory");
}

// K-major B (K hi/lo tile, 64 keys): k-step s is column half s/4, byte 32*(s%4).
__device__ __forceinline__ uint64_t k_desc(uint32_t base, int s) {
  return smem_desc(base + (s >> 2) * (kBN * 128) + (s & 3) * 32, 16, 1024);
}
// MN-major B (V hi/lo tile, 32-byte granules): k-step s is keys 8s..8s+7
// (1024 bytes, two 4-row atoms 512 bytes apart), the second 32 columns 8 KB
// further.
__device__ __forceinline__ uint64_t v_desc(uint32_t base, int s) {
  return smem_desc(base + s * 1024, kBN * 128, 512, kSwizzle128Atom32);
}

// Named-barrier OR over `n` threads: true when any thread passes true.
__device__ __forceinline__ bool bar_any(int id, int n, bool pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<int>(pred)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void bar_named(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// One TMA tile store from shared memory into a 3-D tensor map (rows past the
// map's bounds are clipped), tracked by the issuing thread's bulk group.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_addr(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
// The same into a 4-D tensor map (the packed layout's context tensor).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_addr(src)), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
// Commits the issuing thread's bulk stores as one group.
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the issuing thread's committed bulk stores have read their
// shared-memory sources (the global writes complete on their own).
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Tensor maps of the two-issuer kernels.
struct PipeMaps {
  CUtensorMap k;  // [rows][64] fp32, boxes [64][32 floats], 128-byte swizzle of 16-byte chunks
  CUtensorMap v;  // the same with the 128-byte swizzle of 32-byte granules
  CUtensorMap o;  // out as [slices][seq][64], boxes [1][64][32 floats], 128-byte swizzle
  CUtensorMap q;  // q as [rows][64], boxes [64][32 floats], 128-byte swizzle
};

constexpr int kSplitBarrier = 1;  // named barrier of the split warps
constexpr uint32_t kPipeTmemCols = 512;
constexpr int kRawStages = 4;
constexpr int kLoStages = 3;

// Shared memory of tc32_ws_fwd: the raw K/V ring (TMA targets, read by the
// tensor core as the hi operands) and the ring of their lo parts.
struct PipeSmem {
  float raw[kRawStages][2][2][kBN][32];  // [stage][K, V][column half][key][32]
  float lo[kLoStages][2][2][kBN][32];    // [stage][K lo, V lo][half][key][32]
  uint64_t raw_full[kRawStages], k_ready[kLoStages], v_ready[kLoStages], s_full[1], s_free[1];
  uint64_t k_free[kLoStages], v_free[kLoStages];  // K and V lo stages released separately
  uint64_t p_ready2[2], pv_done2[2];              // one per P buffer
  uint64_t q_full;                                // the q tile landed
  uint64_t q_ready;                               // q is in tensor memory
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t pipe_smem_bytes() { return sizeof(PipeSmem) + 1024; }
static_assert(pipe_smem_bytes() <= 232448, "more shared memory than one sm_100 block may hold");

}  // namespace tc32
}  // namespace raya
