// matvec.cuh — the llama2 matmul offload's matrix-vector product
// (benchmarks/llama2/matmul_kernel.cpp:4-24 with N = 1, as every call of
// llama2/llama.cpp makes it):
//
//   C_s[r] = sum_k W_s[r, k] * x[k]      for each segment s of a batch
//
// The weights are read once from HBM and nothing else is large, so the
// kernel is bound by HBM bandwidth (4 bytes of W per multiply-add).  Layout:
//   * x (K floats) is staged once per CTA in shared memory;
//   * one warp per output row; each lane streams float4s of the row
//     (coalesced 512-byte warp loads, evict-first so the weights do not push
//     x out of L1), four loads in flight per lane;
//   * the lane partials are added with a butterfly over the warp;
//   * one wave of persistent CTAs, sized by the occupancy calculator (about
//     62 registers a thread: four CTAs, 32 warps and 64 KB of reads in flight
//     per SM).  A grid sized for more CTAs than fit ran as two waves at 0.76
//     of HBM bandwidth, against 0.84 for one wave.  Splitting each row over 2
//     to 8 warps (finer units for the last wave) measured slower.
#pragma once
#include <cuda_runtime.h>

#include "sm100.cuh"

namespace akili {

constexpr int kMatvecMaxSegs = 4;
constexpr int kMatvecThreads = 256;  // 8 warps, 8 rows in flight per CTA

struct MatvecSeg {
  const float* W;
  float* C;
  int rows;
  int row0;  // first row of the segment in the batch's row space
};

struct MatvecArgs {
  MatvecSeg seg[kMatvecMaxSegs];
  int nseg;
  int rows;  // all segments
  int K;
  const float* x;
};

// kVec: K % 4 == 0 and every W 16-byte aligned (float4 rows).
// kSmemX: x fits in shared memory (else it is read through L1).
template <bool kVec, bool kSmemX>
__global__ void __launch_bounds__(kMatvecThreads) matvec_kernel(const __grid_constant__ MatvecArgs a) {
  const KClock kclk = kclock_begin();
  // Launched as a programmatic dependent: wait for the previous kernel of the
  // stream (its outputs may be this one's x or W) before any memory access,
  // then let the next one launch while this grid runs.
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ float4 xs4[];
  float* xs = reinterpret_cast<float*>(xs4);
  const int K = a.K;
  if constexpr (kSmemX) {
    for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = a.x[i];
    __syncthreads();
  }
  const float* xv = kSmemX ? xs : a.x;
  const int lane = threadIdx.x & 31;
  const int warps = kMatvecThreads / 32;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < a.rows; row += gridDim.x * warps) {
    int s = 0;
#pragma unroll
    for (int t = 1; t < kMatvecMaxSegs; ++t)
      if (t < a.nseg && row >= a.seg[t].row0) s = t;
    const int r = row - a.seg[s].row0;
    const float* w = a.seg[s].W + static_cast<size_t>(r) * K;
    float acc = 0.0f;
    if constexpr (kVec) {
      const float4* w4 = reinterpret_cast<const float4*>(w);
      const float4* x4 = reinterpret_cast<const float4*>(xv);
      const int n4 = K >> 2;
      float p0 = 0.0f, p1 = 0.0f, p2 = 0.0f, p3 = 0.0f;
      int i = lane;
      for (; i + 96 < n4; i += 128) {
        const float4 a0 = __ldcs(w4 + i), a1 = __ldcs(w4 + i + 32), a2 = __ldcs(w4 + i + 64),
                     a3 = __ldcs(w4 + i + 96);
        const float4 b0 = x4[i], b1 = x4[i + 32], b2 = x4[i + 64], b3 = x4[i + 96];
        p0 = fmaf(a0.x, b0.x, fmaf(a0.y, b0.y, fmaf(a0.z, b0.z, fmaf(a0.w, b0.w, p0))));
        p1 = fmaf(a1.x, b1.x, fmaf(a1.y, b1.y, fmaf(a1.z, b1.z, fmaf(a1.w, b1.w, p1))));
        p2 = fmaf(a2.x, b2.x, fmaf(a2.y, b2.y, fmaf(a2.z, b2.z, fmaf(a2.w, b2.w, p2))));
        p3 = fmaf(a3.x, b3.x, fmaf(a3.y, b3.y, fmaf(a3.z, b3.z, fmaf(a3.w, b3.w, p3))));
      }
      for (; i < n4; i += 32) {
        const float4 a0 = __ldcs(w4 + i);
        const float4 b0 = x4[i];
        p0 = fmaf(a0.x, b0.x, fmaf(a0.y, b0.y, fmaf(a0.z, b0.z, fmaf(a0.w, b0.w, p0))));
      }
      acc = (p0 + p1) + (p2 + p3);
    } else {
      for (int k = lane; k < K; k += 32) acc = fmaf(__ldcs(w + k), xv[k], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) a.seg[s].C[r] = acc;
  }
  kclock_end(kclk);
}

}  // namespace akili
