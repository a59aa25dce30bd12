// common.cuh — shared definitions for the sm_100a block-local attention
// kernels: the launch argument block, the mask's key range, and the PTX
// helpers (mbarrier, TMA bulk copy, ex2) the kernels are built from.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace raya {

enum MaskKind : int { kMaskBlock = 0, kMaskWindow = 1, kMaskFull = 2 };

// Everything a kernel needs, passed by value (__grid_constant__-sized).
// Integer fields are clamped on the host so that every key-range product
// below fits in int32 (seq < 2^29, block/window/halo clamped to the sequence).
struct AttnArgs {
  const float* q;
  const float* k;
  const float* v;
  float* out;
  const int32_t* valid_len;  // device [batch] or nullptr (all = seq)
  int* status;               // device status word: bit 0 = bounded wait timed out
  int batch;
  int heads;
  int seq;
  int head_dim;
  int mask;    // MaskKind
  int block;   // BLOCK: block size (>= 1, clamped to seq)
  int halo;    // BLOCK: key blocks on each side (clamped)
  int window;  // WINDOW: half width (clamped)
  float qscale;       // softmax scale * log2(e): scores go through ex2
  int row_tiles;      // CTA row tiles per (batch, head) slice
  long long timeout_cycles;  // bound of every spin wait
  unsigned long long* stage_cycles;  // device [kStageSlots] or nullptr (timed kernels only)
  const float* rope_cs;  // device [seq][head_dim/2] of (cos, sin), rotary kernels only
};

// Stage-timing slots (the counterpart of StageTimes, tiled/stages.rs:1-31):
// cycles summed over warps, plus warp-tiles processed.
enum StageSlot : int {
  kStageQk = 0,      // QK^T register tile (and the per-element mask)
  kStageSoftmax = 1, // row max, exponentials, rescale, P to shared memory
  kStagePv = 2,      // P.V register tile
  kStageKWait = 3,   // waiting for a K tile
  kStageVWait = 4,   // waiting for a V tile
  kStageRefill = 5,  // last-warp bookkeeping and TMA issue of the next tile
  kStageTiles = 6,   // warp-tiles with work
  kStageTotal = 7,   // cycles from the first wait to the end of the key loop
  kStageSlots = 8
};

// Keys [lo, hi) that query row i may attend, clipped to valid: the rule of
// Mask::key_range (attention.rs:48-59) with BLOCK -> block, 1 -> halo and
// WINDOW -> window.  Non-decreasing in i for every mask kind.
__host__ __device__ __forceinline__ void key_range(const AttnArgs& a, int i, int valid,
                                                   int& lo, int& hi) {
  int l, h;
  if (a.mask == kMaskBlock) {
    const int b = i / a.block;
    l = (b > a.halo ? b - a.halo : 0) * a.block;
    h = (b + a.halo + 1) * a.block;
  } else if (a.mask == kMaskWindow) {
    l = i > a.window ? i - a.window : 0;
    h = i + a.window + 1;
  } else {
    l = 0;
    h = valid;
  }
  lo = l < valid ? l : valid;
  hi = h < valid ? h : valid;
}

#if defined(__CUDACC__)

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's prior generic-proxy shared-memory accesses (and those
// it has observed) before its subsequent async-proxy (TMA) operations.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// TMA bulk copy (non-tensor form) global -> this CTA's shared memory,
// completing `bytes` of transaction count on `bar`.  Both addresses must be
// 16-byte aligned and bytes a multiple of 16.
__device__ __forceinline__ void tma_load_1d(void* dst_smem, const void* src_gmem,
                                            uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 2^x on the SFU (PTX ex2.approx.ftz.f32): ex2(-inf) = +0 exactly, which is
// what gives masked keys a weight of exactly zero.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// is suspended by the hardware (until the phase completes, or for at most
// about the hint) instead of spinning, so waiting warps leave the issue
// slots of their sub-partition to the warps that have work.
constexpr uint32_t kSuspendHintNs = 100000;  // 0.1 ms
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "n"(kSuspendHintNs)
      : "memory");
  return done != 0;
}

// Bounded wait on an mbarrier phase.  Gives up after `timeout_cycles`
// (recording bit 0 in the device status word and raising the CTA's abort
// flag so that its other warps stop waiting too).  Returns false on give-up.
// Each try suspends for at most ~0.1 ms, so the bound and the abort flag are
// checked at least that often.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort_flag, int* status,
                                                  long long timeout_cycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait_suspend(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > timeout_cycles) {
      *abort_flag = 1;
      atomicOr(status, 1);
      return false;
    }
  }
}

__device__ __forceinline__ void st_stream(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }

// Explicit shared-space accesses on 32-bit shared addresses (LDS/STS).
__device__ __forceinline__ float4 lds128(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ void sts128(uint32_t addr, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ float lds32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ void sts32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v));
}

#endif  // __CUDACC__

}  // namespace raya
