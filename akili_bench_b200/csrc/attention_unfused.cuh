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
#include <cuda_runtime.h>

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

// P[row] = exp(S[row] - max) / sum exp(S[row] - max), one warp per row
// (kernel.cpp:25-49; the sum's order differs from the reference's serial
// loop, a difference of an ulp or so).
__global__ void attention_softmax_kernel(const float* __restrict__ S, float* __restrict__ P, int M, int N) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const float* s = S + static_cast<size_t>(row) * N;
    float mx = -INFINITY;
    for (int c = lane; c < N; c += 32) mx = fmaxf(mx, s[c]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int c = lane; c < N; c += 32) sum += expf(s[c] - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    float* p = P + static_cast<size_t>(row) * N;
    for (int c = lane; c < N; c += 32) p[c] = expf(s[c] - mx) / sum;
  }
}

}  // namespace akili
