// attention_unfused.cuh — the reference's unfused three-kernel attention
// (benchmarks/attention/kernel.cpp:6-68) on fp32 CUDA cores, one head:
//
//   kernel_id 0   S[N x N] = Q[N x d] . K[d x N]      (K stored d x N)
//   kernel_id 1   P = softmax(S), row by row
//   kernel_id 2   O[N x d] = P[N x N] . V[N x d]
//
// S and P are materialised in HBM between the launches, as in the
// reference.  The two products sum each output over k in order with
// separately rounded multiplies and adds, so they are bit-identical to the
// reference's loops (kernel.cpp:15-19, :59-63).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace akili {

constexpr int kAtTile = 32;  // 32 x 32 output tile per block, 32 x 8 threads, 4 rows per thread

__global__ void __launch_bounds__(256) attention_matmul_kernel(const float* __restrict__ A,
                                                               const float* __restrict__ B, float* __restrict__ C,
                                                               int M, int N, int K) {
  __shared__ float As[kAtTile][kAtTile + 1];
  __shared__ float Bs[kAtTile][kAtTile + 1];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int col = blockIdx.x * kAtTile + tx;
  const int row_base = blockIdx.y * kAtTile;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int k0 = 0; k0 < K; k0 += kAtTile) {
    for (int r = ty; r < kAtTile; r += 8) {
      const int ar = row_base + r, ak = k0 + tx;
      As[r][tx] = (ar < M && ak < K) ? A[static_cast<size_t>(ar) * K + ak] : 0.0f;
      const int bk = k0 + r;
      Bs[r][tx] = (bk < K && col < N) ? B[static_cast<size_t>(bk) * N + col] : 0.0f;
    }
    __syncthreads();
    const int kn = min(kAtTile, K - k0);
    for (int kk = 0; kk < kn; ++kk) {
      const float b = Bs[kk][tx];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(As[ty + 8 * i][kk], b));
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = row_base + ty + 8 * i;
    if (row < M && col < N) C[static_cast<size_t>(row) * N + col] = acc[i];
  }
}

// P[row] = exp(x - max) / sum exp(x - max), x = scale * S[row], one warp
// per row (kernel.cpp:25-49; the sum's order differs from the reference's
// serial loop, a difference of an ulp or so).  scale = 1 (the reference's
// attention has none) leaves x = S[row] exactly.
__global__ void attention_softmax_kernel(const float* __restrict__ S, float* __restrict__ P, int M, int N,
                                         float scale) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const float* s = S + static_cast<size_t>(row) * N;
    float mx = -INFINITY;
    for (int c = lane; c < N; c += 32) mx = fmaxf(mx, s[c] * scale);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int c = lane; c < N; c += 32) sum += expf(s[c] * scale - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    float* p = P + static_cast<size_t>(row) * N;
    for (int c = lane; c < N; c += 32) p[c] = expf(s[c] * scale - mx) / sum;
  }
}

// The fp16 form of the softmax stage for batched heads: P = softmax(scale *
// S) over each of `rows` rows of N fp16 scores (N % 8 == 0, 16-byte rows).
// One warp per row.  Pass 1 reads the row once as 16-byte vectors and keeps
// a running (max, sum) per lane in log2 units; the lanes' pairs are merged
// with a butterfly.  Pass 2 reads the row again (from L2: the rows in flight
// at once total tens of MB) and writes P.  HBM traffic is one read and one
// write of the scores.
__global__ void __launch_bounds__(256) attention_softmax_f16_kernel(const __half* __restrict__ S,
                                                                    __half* __restrict__ P, size_t rows, int N,
                                                                    float scale_log2) {
  const int lane = threadIdx.x & 31;
  const size_t warps = blockDim.x >> 5;
  const int nv = N >> 3;  // 16-byte vectors per row
  for (size_t row = blockIdx.x * warps + (threadIdx.x >> 5); row < rows; row += gridDim.x * warps) {
    const uint4* s = reinterpret_cast<const uint4*>(S + row * N);
    float m = -INFINITY, l = 0.0f;
    for (int v = lane; v < nv; v += 32) {
      const uint4 u = s[v];
      const __half2* h = reinterpret_cast<const __half2*>(&u);
      float x[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(h[e]);
        x[2 * e] = f.x * scale_log2;
        x[2 * e + 1] = f.y * scale_log2;
      }
      float vm = x[0];
#pragma unroll
      for (int e = 1; e < 8; ++e) vm = fmaxf(vm, x[e]);
      const float mn = fmaxf(m, vm);
      float add = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) add += exp2f(x[e] - mn);
      l = l * exp2f(m - mn) + add;  // exp2f(-inf) = 0 on the first vector
      m = mn;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m, o);
      const float lo = __shfl_xor_sync(0xffffffffu, l, o);
      const float mn = fmaxf(m, mo);
      l = (m == -INFINITY ? 0.0f : l * exp2f(m - mn)) + (mo == -INFINITY ? 0.0f : lo * exp2f(mo - mn));
      m = mn;
    }
    const float inv = 1.0f / l;
    uint4* p = reinterpret_cast<uint4*>(P + row * N);
    for (int v = lane; v < nv; v += 32) {
      const uint4 u = s[v];
      const __half2* h = reinterpret_cast<const __half2*>(&u);
      uint4 o;
      __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(h[e]);
        oh[e] = __floats2half2_rn(exp2f(f.x * scale_log2 - m) * inv, exp2f(f.y * scale_log2 - m) * inv);
      }
      p[v] = o;
    }
  }
}

}  // namespace akili
