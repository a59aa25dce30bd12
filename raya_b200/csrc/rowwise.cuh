// rowwise.cuh — block-local attention for any head_dim (multiple of 8, <= 256):
// one warp per query row, keys in 32-wide chunks with the same online softmax
// as the tiled kernel.  This is the kernel for shapes the head_dim-64 tiled
// kernel does not cover (the reference's tests use head_dim 8, 16, 40, 96).
//
// Per row (Naive::attend, naive.rs:22-63, in online form): the query row is
// staged in shared memory; lane j of a chunk computes s_j = q . k_j over c in
// order; the chunk max comes from warp shuffles; p_j = 2^(s_j*scale*log2e - m);
// each lane owns output columns lane + 32t and accumulates p_j * v_j[c] with
// p_j broadcast by shuffle.
#pragma once

#include "common.cuh"

namespace raya {
namespace rowwise {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxD = 256;

__global__ void __launch_bounds__(kThreads) rowwise_fwd(const __grid_constant__ AttnArgs a) {
  __shared__ __align__(16) float qs[kWarps][kMaxD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = a.head_dim;
  const long long total = static_cast<long long>(a.batch) * a.heads * a.seq;
  const float qscale = a.qscale;

  for (long long row = static_cast<long long>(blockIdx.x) * kWarps + warp; row < total;
       row += static_cast<long long>(gridDim.x) * kWarps) {
    const long long bh = row / a.seq;
    const int i = static_cast<int>(row - bh * a.seq);
    const int b = static_cast<int>(bh / a.heads);
    int valid = a.valid_len ? a.valid_len[b] : a.seq;
    valid = valid < 0 ? 0 : (valid > a.seq ? a.seq : valid);
    float* orow = a.out + static_cast<size_t>(row) * d;
    if (i >= valid) {
      for (int c = lane; c < d; c += 32) orow[c] = 0.f;
      continue;
    }
    int lo, hi;
    key_range(a, i, valid, lo, hi);
    const size_t base = static_cast<size_t>(bh) * a.seq * d;
    const float* qrow = a.q + static_cast<size_t>(row) * d;
    for (int c = lane; c < d; c += 32) qs[warp][c] = qrow[c];
    __syncwarp();

    float o[kMaxD / 32];
#pragma unroll
    for (int t = 0; t < kMaxD / 32; ++t) o[t] = 0.f;
    float msc = -INFINITY, l = 0.f;
    for (int j0 = lo; j0 < hi; j0 += 32) {
      const int j = j0 + lane;
      float s = -INFINITY;
      if (j < hi) {
        const float* krow = a.k + base + static_cast<size_t>(j) * d;
        float acc = 0.f;
        for (int c = 0; c < d; c += 8) {
          const float4 k0 = *reinterpret_cast<const float4*>(krow + c);
          const float4 k1 = *reinterpret_cast<const float4*>(krow + c + 4);
          const float4 q0 = *reinterpret_cast<const float4*>(&qs[warp][c]);
          const float4 q1 = *reinterpret_cast<const float4*>(&qs[warp][c + 4]);
          acc = fmaf(q0.x, k0.x, acc);
          acc = fmaf(q0.y, k0.y, acc);
          acc = fmaf(q0.z, k0.z, acc);
          acc = fmaf(q0.w, k0.w, acc);
          acc = fmaf(q1.x, k1.x, acc);
          acc = fmaf(q1.y, k1.y, acc);
          acc = fmaf(q1.z, k1.z, acc);
          acc = fmaf(q1.w, k1.w, acc);
        }
        s = acc;
      }
      float tmax = s;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      const float mnew = fmaxf(msc, tmax * qscale);
      const float mbase = mnew == -INFINITY ? 0.f : mnew;
      const float alpha = ex2(msc - mbase);
      msc = mnew;
      const float p = ex2(fmaf(s, qscale, -mbase));
      l = fmaf(l, alpha, p);
#pragma unroll
      for (int t = 0; t < kMaxD / 32; ++t) o[t] *= alpha;
      const int nk = min(32, hi - j0);
      for (int jj = 0; jj < nk; ++jj) {
        const float pj = __shfl_sync(0xffffffffu, p, jj);
        const float* vrow = a.v + base + static_cast<size_t>(j0 + jj) * d;
#pragma unroll
        for (int t = 0; t < kMaxD / 32; ++t) {
          const int c = lane + 32 * t;
          if (c < d) o[t] = fmaf(pj, vrow[c], o[t]);
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
    for (int t = 0; t < kMaxD / 32; ++t) {
      const int c = lane + 32 * t;
      if (c < d) orow[c] = o[t] * inv;
    }
    __syncwarp();
  }
}

}  // namespace rowwise
}  // namespace raya
