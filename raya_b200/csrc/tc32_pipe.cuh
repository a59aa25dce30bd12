// tc32_pipe.cuh — the 3xTF32 tensor-core attention kernel, warp-specialised
// and pipelined (sm_100a).
//
// The 3xTF32 method of tc32_fwd (three tcgen05.mma products per tile, hi*lo +
// lo*hi + hi*hi, and the FFMA kernel's online softmax), reorganised so that
// the tensor core, the softmax and the operand preparation overlap.
//
// Operand split.  The tensor core reads an fp32 bit pattern as TF32 by
// dropping its 13 low mantissa bits (truncation toward zero, measured on
// B200 with an operand of 1 + 2^-11 + 2^-13, which reads as exactly 1).  So
// a raw fp32 tile IS its hi operand, and only lo = x - trunc(x) (exact in
// fp32; the tensor core truncates it in turn) has to be computed and stored.
// The error of the truncating split is below 2^-21 relative per product.
//
//
//   warps 0-3  (softmax): one query row per thread, TMEM lane = row.  At the
//              start each thread loads its q row from global memory and
//              stores q and its lo part into tensor memory (the A operand of
//              S = Q K^T).  Per key tile it reads its row of S, masks, runs
//              the online softmax, adds the previous tile's PV product to its
//              O row in registers, and stores p and its lo part into tensor
//              memory (the A operand of PV).
//   warps 4-6  (split):   per key tile, waits for the raw K and V tiles (TMA
//              into a ring of four stages; they are the hi operands), writes
//              their lo parts (a ring of three stages; K's first, signalled on
//              its own barrier so QK(j) can start while V's is written),
//              zeroes V rows at or past valid_len in both, and issues the TMA
//              of the next tile into the raw stage that PV(j-3) has released.
//              Three lo
//              stages let the split of tile j+1 run while the tensor core
//              works on QK(j) and PV(j-1).
//   warp 7     (MMA):     one thread issues QK(j) into S[j%2], then PV(j-1)
//              once P(j-1) is stored, so QK of the next tile runs while the
//              softmax works on this one.
//
// Tensor memory (512 columns): S0 [0,64), S1 [64,128), Q hi [128,192),
// Q lo [192,256), P hi [256,320), P lo [320,384), PV [384,448).  The tensor
// core reads A (Q, P) from tensor memory and only B (K, V) from shared
// memory.  Every wait is bounded and every group's exit is a collective
// decision of that group; after a timeout the outstanding copies and MMAs
// are drained (bounded) before tensor memory is freed.  256 threads (two
// whole warpgroups) leave the softmax rows the full register budget.
#pragma once

#include "tc32.cuh"

namespace raya {
namespace tc32 {

constexpr int kPipeThreads = 256;  // softmax 0-127, split 128-223, MMA warp 224-255
constexpr int kSplitThreads = 96;
constexpr int kSplitBarrier = 1;   // named barrier of the split warps
constexpr uint32_t kPipeTmemCols = 512;
constexpr uint32_t kColS = 0, kColQh = 128, kColQl = 192, kColPh = 256, kColPl = 320, kColPV = 384;

struct PipeMaps {
  CUtensorMap k;  // [rows][64] fp32, boxes [64][32 floats], 128-byte swizzle of 16-byte chunks
  CUtensorMap v;  // the same with the 128-byte swizzle of 32-byte granules
  CUtensorMap o;  // out as [slices][seq][64], boxes [1][64][32 floats], 128-byte swizzle (tc32_ws_fwd's stores)
  CUtensorMap q;  // q as [rows][64], boxes [64][32 floats], 128-byte swizzle (tc32_ws_fwd's q tile)
};

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
// Commits the issuing thread's bulk stores and waits until their shared-memory
// sources have been read (the global writes complete on their own).
__device__ __forceinline__ void tma_store_commit_and_wait_read() {
  asm volatile("cp.async.bulk.commit_group;\n\tcp.async.bulk.wait_group.read 0;" ::: "memory");
}

constexpr int kRawStages = 4;
constexpr int kLoStages = 3;

struct PipeSmem {
  float raw[kRawStages][2][2][kBN][32];  // [stage][K, V][column half][key][32]: TMA targets = hi operands
  float lo[kLoStages][2][2][kBN][32];    // [stage][K lo, V lo][half][key][32]
  uint64_t raw_full[kRawStages], k_ready[kLoStages], v_ready[kLoStages], kv_free[kLoStages], s_full[2], s_free[2];
  uint64_t k_free[kLoStages], v_free[kLoStages];  // tc32_ws_fwd: K and V stages released separately
  uint64_t p_ready2[2], pv_done2[2];              // tc32_ws_fwd: one per P buffer
  uint64_t q_full;                                // tc32_ws_fwd: the q tile landed
  uint64_t p_ready, pv_done, q_ready;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t pipe_smem_bytes() { return sizeof(PipeSmem) + 1024; }
static_assert(pipe_smem_bytes() <= 232448, "more shared memory than one sm_100 block may hold");

// D (+)= A B with A read from tensor memory (M = 128 rows in lanes, K = 8
// 32-bit columns) and B from a shared-memory descriptor.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
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

// K-major B (K hi/lo tile, 64 keys): k-step s is column half s/4, byte 32*(s%4).
__device__ __forceinline__ uint64_t k_desc(uint32_t base, int s) {
  return smem_desc(base + (s >> 2) * (kBN * 128) + (s & 3) * 32, 16, 1024);
}
// MN-major B (V hi/lo tile, 32-byte granules): k-step s is keys 8s..8s+7.
__device__ __forceinline__ uint64_t v_desc(uint32_t base, int s) {
  return smem_desc(base + s * 1024, kBN * 128, 512, kSwizzle128Atom32);
}

__global__ void __launch_bounds__(kPipeThreads, 1)
    tc32_pipe_fwd(const __grid_constant__ AttnArgs a, const __grid_constant__ PipeMaps maps) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  PipeSmem& sm = *reinterpret_cast<PipeSmem*>(smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr));

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
    for (int idx = tid; idx < rows * 16; idx += kPipeThreads)
      st_stream(outp + static_cast<size_t>(r0 + (idx >> 4)) * kD + (idx & 15) * 4, zero);
    return;
  }

  if (warp == 7) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&sm.tmem_base)),
                 "r"(kPipeTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < kRawStages; ++s) mbar_init(&sm.raw_full[s], 1);
    for (int s = 0; s < kLoStages; ++s) {
      mbar_init(&sm.k_ready[s], kSplitThreads);
      mbar_init(&sm.v_ready[s], kSplitThreads);
      mbar_init(&sm.kv_free[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_free[s], 128);
    }
    mbar_init(&sm.p_ready, 128);
    mbar_init(&sm.pv_done, 1);
    mbar_init(&sm.q_ready, 128);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_flag = &sm.abort_flag;

  // Drain bookkeeping (registers of the issuing threads).
  int last_tma_tile = -1;
  uint64_t* last_commit = nullptr;
  uint32_t last_commit_parity = 0;

  if (warp < 4) {
    // ---------------- softmax warpgroup ----------------
    const int row = r0 + tid;
    int rlo = 0, rhi = 0;
    key_range(a, min(row, last), valid, rlo, rhi);
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float qscale = a.qscale;
    {  // q row -> tensor memory: q itself (read as its hi part) and q - trunc(q)
      const float4* src = reinterpret_cast<const float4*>(a.q + static_cast<size_t>(row_base + row) * kD);
      float h[32], l[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 x = row < valid ? __ldg(src + half * 8 + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
          const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            h[4 * c4 + i] = xs[i];
            l[4 * c4 + i] = tf32_lo(xs[i]);
          }
        }
        tmem_st32(tmem + lane_off + kColQh + 32 * half, h);
        tmem_st32(tmem + lane_off + kColQl + 32 * half, l);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&sm.q_ready);
    }

    float o[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) o[c] = 0.f;
    float msc = -INFINITY, lsum = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int s = j & 1;
      const int kt = (t_begin + j) * kBN;
      bool w = mbar_wait_bounded(&sm.s_full[s], static_cast<uint32_t>(j >> 1) & 1u, abort_flag, a.status,
                                 a.timeout_cycles);
      if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
      tc_fence_after();
      float sv[64];
      tmem_ld32(tmem + lane_off + kColS + 64 * s, sv);
      tmem_ld32(tmem + lane_off + kColS + 64 * s + 32, sv + 32);
      tc_fence_before();
      mbar_arrive(&sm.s_free[s]);

      if (!(rlo <= kt && rhi >= kt + kBN)) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (static_cast<unsigned>(kt + c - rlo) >= static_cast<unsigned>(rhi - rlo)) sv[c] = -INFINITY;
      }
      float m4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int c = 4; c < 64; ++c) m4[c & 3] = fmaxf(m4[c & 3], sv[c]);
      const float tmax = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      const float mnew = fmaxf(msc, tmax * qscale);
      const float mbase = mnew == -INFINITY ? 0.f : mnew;
      const float alpha = ex2(msc - mbase);
      msc = mnew;
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

      if (j > 0) {  // O += the previous tile's PV; it has also released P
        w = mbar_wait_bounded(&sm.pv_done, static_cast<uint32_t>(j - 1) & 1u, abort_flag, a.status,
                              a.timeout_cycles);
        if (__any_sync(0xffffffffu, !w)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 64; c += 32) {
          float t[32];
          tmem_ld32(tmem + lane_off + kColPV + c, t);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c + i] += t[i];
        }
      }
#pragma unroll
      for (int c = 0; c < 64; ++c) o[c] *= alpha;

      // P -> tensor memory: p itself (read as its hi part), then p - trunc(p) in place.
      tmem_st32(tmem + lane_off + kColPh, sv);
      tmem_st32(tmem + lane_off + kColPh + 32, sv + 32);
#pragma unroll
      for (int c = 0; c < 64; ++c) sv[c] = tf32_lo(sv[c]);
      tmem_st32(tmem + lane_off + kColPl, sv);
      tmem_st32(tmem + lane_off + kColPl + 32, sv + 32);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&sm.p_ready);
    }
    if (ok) {
      const bool w = mbar_wait_bounded(&sm.pv_done, static_cast<uint32_t>(ntiles - 1) & 1u, abort_flag, a.status,
                                       a.timeout_cycles);
      if (__any_sync(0xffffffffu, !w)) {
        ok = false;
      } else {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 64; c += 32) {
          float t[32];
          tmem_ld32(tmem + lane_off + kColPV + c, t);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c + i] += t[i];
        }
      }
    }
    if (row < seq) {  // this row, normalised (+0.0f past valid_len)
      const float inv = (row < valid && lsum > 0.f) ? 1.0f / lsum : 0.f;
      float* orow = outp + static_cast<size_t>(row) * kD;
#pragma unroll
      for (int c = 0; c < 64; c += 4) {
        const float4 x = row < valid ? make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        st_stream(orow + c, x);
      }
    }
  } else if (warp < 7) {
    // ---------------- split warps ----------------
    const int st = tid - 128;
    auto issue = [&](int jj) {  // tile jj -> raw stage jj % 4
      const int s = jj & (kRawStages - 1);
      uint64_t* bar = &sm.raw_full[s];
      const int y = static_cast<int>(row_base + (t_begin + jj) * kBN);
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(bar, 2u * kBN * kD * 4u);
      tiled64::tma_load_2d(&sm.raw[s][0][0][0][0], &maps.k, 0, y, bar);
      tiled64::tma_load_2d(&sm.raw[s][0][1][0][0], &maps.k, 32, y, bar);
      tiled64::tma_load_2d(&sm.raw[s][1][0][0][0], &maps.v, 0, y, bar);
      tiled64::tma_load_2d(&sm.raw[s][1][1][0][0], &maps.v, 32, y, bar);
      last_tma_tile = jj;
    };
    if (st == 0)
      for (int jj = 0; jj < kRawStages && jj < ntiles; ++jj) issue(jj);
    for (int j = 0; j < ntiles; ++j) {
      const int s3 = j % kLoStages, s4 = j & (kRawStages - 1);
      bool w = true;
      if (j >= kLoStages) {  // PV(j-3) is done: lo stage s3 and raw stage (j+1)%4 are free
        w = mbar_wait_bounded(&sm.kv_free[s3], static_cast<uint32_t>(j / kLoStages - 1) & 1u, abort_flag,
                              a.status, a.timeout_cycles);
        if (w && st == 0 && j + 1 < ntiles) issue(j + 1);
      }
      w = w && mbar_wait_bounded(&sm.raw_full[s4], static_cast<uint32_t>(j >> 2) & 1u, abort_flag, a.status,
                                 a.timeout_cycles);
      if (bar_any(kSplitBarrier, kSplitThreads, !w)) break;
      const int nv = min(kBN, valid - (t_begin + j) * kBN);
      float4* kr = reinterpret_cast<float4*>(&sm.raw[s4][0][0][0][0]);
      float4* vr = reinterpret_cast<float4*>(&sm.raw[s4][1][0][0][0]);
      float4* kl = reinterpret_cast<float4*>(&sm.lo[s3][0][0][0][0]);
      float4* vl = reinterpret_cast<float4*>(&sm.lo[s3][1][0][0][0]);
#pragma unroll 4
      for (int f = st; f < kBN * 16; f += kSplitThreads) {
        const float4 x = kr[f];
        kl[f] = make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      mbar_arrive(&sm.k_ready[s3]);  // QK(j) may start; V's lo part follows
      if (nv == kBN) {
#pragma unroll 4
        for (int f = st; f < kBN * 16; f += kSplitThreads) {
          const float4 x = vr[f];
          vl[f] = make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
        }
      } else {  // the tail tile: V rows at or past valid_len become exact zeros in both parts
        for (int f = st; f < kBN * 16; f += kSplitThreads) {
          const int key = (f % (kBN * 8)) >> 3;
          if (key < nv) {
            const float4 x = vr[f];
            vl[f] = make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
          } else {
            vr[f] = make_float4(0.f, 0.f, 0.f, 0.f);
            vl[f] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&sm.v_ready[s3]);
      bar_named(kSplitBarrier, kSplitThreads);
    }
  } else if ((tid & 31) == 0) {
    // ---------------- MMA issuer (one thread) ----------------
    auto commit = [&](uint64_t* bar, uint32_t parity) {
      mma_commit(bar);
      last_commit = bar;
      last_commit_parity = parity;
    };
    auto pv = [&](int jj) {
      const int s = jj % kLoStages;
      const uint32_t vh = smem_addr(&sm.raw[jj & (kRawStages - 1)][1][0][0][0]), vl = smem_addr(&sm.lo[s][1][0][0][0]);
      const uint32_t d = tmem + kColPV;
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts(d, tmem + kColPh + 8 * k, v_desc(vl, k), kIdescPV, k > 0 ? 1u : 0u);
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts(d, tmem + kColPl + 8 * k, v_desc(vh, k), kIdescPV, 1u);
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts(d, tmem + kColPh + 8 * k, v_desc(vh, k), kIdescPV, 1u);
      commit(&sm.pv_done, static_cast<uint32_t>(jj) & 1u);
      if (jj + kLoStages < ntiles) commit(&sm.kv_free[s], static_cast<uint32_t>(jj / kLoStages) & 1u);
    };
    bool ok = mbar_wait_bounded(&sm.q_ready, 0, abort_flag, a.status, a.timeout_cycles);
    int j = 0;
    for (; ok && j < ntiles; ++j) {
      const int s = j & 1, s3 = j % kLoStages;
      ok = mbar_wait_bounded(&sm.k_ready[s3], static_cast<uint32_t>(j / kLoStages) & 1u, abort_flag, a.status,
                             a.timeout_cycles);
      if (ok && j >= 2)
        ok = mbar_wait_bounded(&sm.s_free[s], static_cast<uint32_t>((j - 2) >> 1) & 1u, abort_flag, a.status,
                               a.timeout_cycles);
      if (!ok) break;
      tc_fence_after();
      const uint32_t khi = smem_addr(&sm.raw[j & (kRawStages - 1)][0][0][0][0]), klo = smem_addr(&sm.lo[s3][0][0][0][0]);
      const uint32_t d = tmem + kColS + 64 * s;
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts(d, tmem + kColQh + 8 * k, k_desc(klo, k), kIdescQK, k > 0 ? 1u : 0u);
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts(d, tmem + kColQl + 8 * k, k_desc(khi, k), kIdescQK, 1u);
#pragma unroll
      for (int k = 0; k < 8; ++k) mma_tf32_ts(d, tmem + kColQh + 8 * k, k_desc(khi, k), kIdescQK, 1u);
      commit(&sm.s_full[s], static_cast<uint32_t>(j >> 1) & 1u);
      if (j >= 1) {
        ok = mbar_wait_bounded(&sm.p_ready, static_cast<uint32_t>(j - 1) & 1u, abort_flag, a.status,
                               a.timeout_cycles) &&
             mbar_wait_bounded(&sm.v_ready[(j - 1) % kLoStages], static_cast<uint32_t>((j - 1) / kLoStages) & 1u,
                               abort_flag, a.status, a.timeout_cycles);
        if (!ok) break;
        tc_fence_after();
        pv(j - 1);
      }
    }
    if (ok) {
      ok = mbar_wait_bounded(&sm.p_ready, static_cast<uint32_t>(ntiles - 1) & 1u, abort_flag, a.status,
                             a.timeout_cycles) &&
           mbar_wait_bounded(&sm.v_ready[(ntiles - 1) % kLoStages], static_cast<uint32_t>((ntiles - 1) / kLoStages) & 1u,
                             abort_flag, a.status, a.timeout_cycles);
      if (ok) {
        tc_fence_after();
        pv(ntiles - 1);
      }
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
    if (tid == 128) {  // the last tile issued into each raw stage
#pragma unroll
      for (int s = 0; s < kRawStages; ++s) {
        const int t = last_tma_tile - ((last_tma_tile - s) & (kRawStages - 1));
        if (t >= 0) drain(&sm.raw_full[s], static_cast<uint32_t>(t >> 2) & 1u);
      }
    }
    if (tid == 224 && last_commit) drain(last_commit, last_commit_parity);
  }
  __syncthreads();
  if (warp == 7) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPipeTmemCols) : "memory");
  }
}

}  // namespace tc32
}  // namespace raya
