// aux.cuh — the bandwidth-bound helpers around the tcgen05 GEMM:
//   * fp32 -> fp16 operand conversion (the reference kernels' f2h, done once
//     per operand instead of per tile load),
//   * the RMSNorm pre-pass of kbt_gemm_rmsnorm_swiglu (writes fp16 x_hat, the
//     operand the reference rounds at its GEMM load),
//   * finalisers that merge per-(row, column-tile) partial statistics written
//     by the GEMM epilogue: row sums, log-sum-exp + Mish, and the in-place
//     LayerNorm / softmax normalisation passes.
// All are grid-stride kernels sized to a multiple of the SM count; rows are
// handled one warp each with 16-byte vector accesses.
#pragma once
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace akili {

__global__ void cast_f32_to_f16_kernel(const float* __restrict__ src, __half* __restrict__ dst, size_t n) {
  const size_t n8 = n / 8;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n8; i += stride) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(src) + 2 * i);
    const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 2 * i + 1);
    uint4 q;
    q.x = pack_half2(a.x, a.y);
    q.y = pack_half2(a.z, a.w);
    q.z = pack_half2(b.x, b.y);
    q.w = pack_half2(b.z, b.w);
    reinterpret_cast<uint4*>(dst)[i] = q;
  }
  for (size_t i = n8 * 8 + blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
    dst[i] = __float2half_rn(src[i]);
}

// x -> (hi, lo) = (fp16(x), fp16(x - fp16(x))): hi + lo carries ~22 bits of
// x's mantissa, for the split-precision products of the fp32 flash mode.
__global__ void split_f32_to_f16x2_kernel(const float* __restrict__ src, __half* __restrict__ hi,
                                          __half* __restrict__ lo, size_t n) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    const float x = src[i];
    const __half h = __float2half_rn(x);
    hi[i] = h;
    lo[i] = __float2half_rn(x - __half2float(h));
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// x_hat[i, k] = fp16( x[i,k] * (1 / sqrtf(sum_k x^2 / K + eps)) * w[k] )
// (benchmarks/kbt_gemm_rmsnorm_swiglu/kernel.cpp:95-105, with the f2h of its
// GEMM load, kernel.cpp:48, applied at the store).  One warp per row; K % 8 == 0.
// With xlo non-null (the fp32 kb2 form, benchmarks/kb2_gemm_rmsnorm_swiglu/
// main.cpp verify loop: x_hat stays fp32) x_hat is written as fp16 hi + lo
// parts instead, hi = fp16(x_hat), lo = fp16(x_hat - hi).
template <typename InT>
__global__ void rmsnorm_prepass_kernel(const InT* __restrict__ x, const float* __restrict__ w,
                                       __half* __restrict__ xhat, __half* __restrict__ xlo, int M, int K,
                                       float eps) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const InT* xr = x + static_cast<size_t>(row) * K;
    float ss = 0.0f;
    for (int k = lane * 8; k < K; k += 256) {
      float f[8];
      if constexpr (sizeof(InT) == 2) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(xr + k));
        const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 t = __half22float2(h[i]);
          f[2 * i] = t.x;
          f[2 * i + 1] = t.y;
        }
      } else {
        const float4 a = __ldg(reinterpret_cast<const float4*>(xr + k));
        const float4 b = __ldg(reinterpret_cast<const float4*>(xr + k) + 1);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
    }
    ss = warp_sum(ss);
    const float inv_rms = 1.0f / sqrtf(ss / static_cast<float>(K) + eps);
    __half* out = xhat + static_cast<size_t>(row) * K;
    for (int k = lane * 8; k < K; k += 256) {
      float f[8];
      if constexpr (sizeof(InT) == 2) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(xr + k));
        const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 t = __half22float2(h[i]);
          f[2 * i] = t.x;
          f[2 * i + 1] = t.y;
        }
      } else {
        const float4 a = __ldg(reinterpret_cast<const float4*>(xr + k));
        const float4 b = __ldg(reinterpret_cast<const float4*>(xr + k) + 1);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
      }
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + k));
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + k) + 1);
      const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float h[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = f[i] * inv_rms * ww[i];
      uint4 q;
      q.x = pack_half2(h[0], h[1]);
      q.y = pack_half2(h[2], h[3]);
      q.z = pack_half2(h[4], h[5]);
      q.w = pack_half2(h[6], h[7]);
      *reinterpret_cast<uint4*>(out + k) = q;
      if (xlo != nullptr) {
        const __half2* hh = reinterpret_cast<const __half2*>(&q);
        float r[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 t = __half22float2(hh[i]);
          r[2 * i] = h[2 * i] - t.x;
          r[2 * i + 1] = h[2 * i + 1] - t.y;
        }
        uint4 lq;
        lq.x = pack_half2(r[0], r[1]);
        lq.y = pack_half2(r[2], r[3]);
        lq.z = pack_half2(r[4], r[5]);
        lq.w = pack_half2(r[6], r[7]);
        *reinterpret_cast<uint4*>(xlo + static_cast<size_t>(row) * K + k) = lq;
      }
    }
  }
}

template <typename OutT>
__device__ __forceinline__ void store_scalar(OutT* p, float v) {
  if constexpr (sizeof(OutT) == 2) *p = __float2half_rn(v);
  else *p = v;
}

// out[i] = scale * sum_t ws[t][i]   (tiles summed in a fixed order: deterministic)
template <typename OutT>
__global__ void finalize_rowsum_kernel(const float* __restrict__ ws, OutT* __restrict__ out, int M, int ntiles,
                                       float scale) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < M; i += gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int t = 0; t < ntiles; ++t) s += ws[static_cast<size_t>(t) * M + i];
    store_scalar(out + i, s * scale);
  }
}

// Merge per-tile (max, sumexp) partials — kept in the log2 domain by the GEMM
// epilogue — into the row's natural log-sum-exp and apply
// out = lse * (lse * tanh(log(1 + exp(lse))))
// (benchmarks/kbt_matmul_scale_residadd_clamp/main.cpp:145-151 semantics).
template <typename OutT>
__global__ void finalize_lse_mish_kernel(const float* __restrict__ ws, OutT* __restrict__ out, int M,
                                         int ntiles) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < M; i += gridDim.x * blockDim.x) {
    float m = -INFINITY;
    for (int t = 0; t < ntiles; ++t) m = fmaxf(m, ws[static_cast<size_t>(t) * M + i]);
    float l = 0.0f;
    const float* lt = ws + static_cast<size_t>(ntiles) * M;
    for (int t = 0; t < ntiles; ++t) {
      const float mt = ws[static_cast<size_t>(t) * M + i];
      if (mt != -INFINITY) l += lt[static_cast<size_t>(t) * M + i] * exp2f(mt - m);
    }
    const float lse = (m + log2f(l)) * 0.6931471805599453f;
    const float mish = lse * tanhf(logf(1.0f + expf(lse)));
    store_scalar(out + i, lse * mish);
  }
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
  if constexpr (sizeof(T) == 2) {
    const uint4 q = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&f)[8]) {
  if constexpr (sizeof(T) == 2) {
    uint4 q;
    q.x = pack_half2(f[0], f[1]);
    q.y = pack_half2(f[2], f[3]);
    q.z = pack_half2(f[4], f[5]);
    q.w = pack_half2(f[6], f[7]);
    *reinterpret_cast<uint4*>(p) = q;
  } else {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
    *(reinterpret_cast<float4*>(p) + 1) = make_float4(f[4], f[5], f[6], f[7]);
  }
}

// Warp-wide merge of per-tile LayerNorm partials (count, mean, M2) with Chan
// et al.'s pairwise formula: lane t merges tiles t, t+32, ... then a
// butterfly combines the lanes, so the partial loads are issued in parallel.
__device__ __forceinline__ void chan_merge(float& n, float& mean, float& m2, float nb, float mb, float m2b) {
  const float ntot = n + nb;
  if (nb == 0.0f) return;
  if (n == 0.0f) {
    n = nb;
    mean = mb;
    m2 = m2b;
    return;
  }
  const float delta = mb - mean;
  mean += delta * (nb / ntot);
  m2 += m2b + delta * delta * (n * nb / ntot);
  n = ntot;
}

// The in-place LayerNorm finaliser is run by CTAs that each own
// kFinRows rows x kFinCols columns of the output (grid: row blocks x column
// blocks).  The CTA's warps first merge its rows' statistics into shared
// memory; then each thread owns 8 columns and streams the rows, 16-byte
// accesses that a warp makes contiguous.  Each pass keeps 8 rows (fp16) or 4
// rows (fp32) of loads in flight per thread, held raw, so that four CTAs
// (fp16; three for fp32) fit per SM and about 128 KB per SM is in flight.
#ifndef AKILI_FIN_ROWS
#define AKILI_FIN_ROWS 16
#endif
constexpr int kFinRows = AKILI_FIN_ROWS;
constexpr int kFinThreads = 256;
constexpr int kFinCols = kFinThreads * 8;  // columns per CTA
template <typename T>
constexpr int fin_rows_in_flight() { return sizeof(T) == 2 ? 8 : 4; }
static_assert(kFinRows % 8 == 0, "whole passes");

// Eight consecutive values of T, as loaded (16 or 32 bytes).
template <typename T>
struct Raw8 {
  uint4 v[sizeof(T) / 2];
};
template <typename T>
__device__ __forceinline__ void load_raw8(const T* p, Raw8<T>& r) {
#pragma unroll
  for (int k = 0; k < static_cast<int>(sizeof(T) / 2); ++k) r.v[k] = reinterpret_cast<const uint4*>(p)[k];
}
template <typename T>
__device__ __forceinline__ void raw8_to_float(const Raw8<T>& r, float (&f)[8]) {
  if constexpr (sizeof(T) == 2) {
    const __half2* h = reinterpret_cast<const __half2*>(&r.v[0]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  } else {
    const float* x = reinterpret_cast<const float*>(&r.v[0]);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = x[i];
  }
}

// Rows [row0, row0 + nrows) x columns [j, j + 8) of c, in place: f = op(r, f)
// with r the row within the block.
template <typename T, typename Op>
__device__ __forceinline__ void stream_block_rows(T* __restrict__ c, int N, int row0, int nrows, int j, Op op) {
  constexpr int kR = fin_rows_in_flight<T>();
  for (int r0 = 0; r0 < nrows; r0 += kR) {
    Raw8<T> raw[kR];
#pragma unroll
    for (int q = 0; q < kR; ++q)
      if (r0 + q < nrows) load_raw8(c + static_cast<size_t>(row0 + r0 + q) * N + j, raw[q]);
#pragma unroll
    for (int q = 0; q < kR; ++q) {
      if (r0 + q < nrows) {
        float f[8];
        raw8_to_float(raw[q], f);
        op(r0 + q, f);
        store8(c + static_cast<size_t>(row0 + r0 + q) * N + j, f);
      }
    }
  }
}

// In-place LayerNorm of the pre-normalised rows y = x.W + b written by the
// GEMM epilogue.  Per-tile (mean, M2) partials over `tile_n` columns are
// (half tiles; a slot past the row's end is empty) merged with Chan et al.'s
// pairwise formula (a warp per row, a lane per partial, a butterfly);
// var = M2 / N (biased, as benchmarks/kbt_gemm_layernorm/main.cpp:159-166);
// inv_std = 1/sqrtf(var+eps).  Gamma and beta of a thread's 8 columns stay in
// registers.
template <typename T>
__global__ void __launch_bounds__(kFinThreads, sizeof(T) == 2 ? 4 : 3)
    layernorm_finalize_kernel(T* __restrict__ c, const float* __restrict__ ws, const float* __restrict__ ln_w,
                              const float* __restrict__ ln_b, int M, int N, int ntiles, int tile_n, float eps) {
  __shared__ float s_mean[kFinRows], s_inv[kFinRows];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kFinRows;
  for (int r = warp; r < kFinRows; r += kFinThreads / 32) {
    const int row = min(row0 + r, M - 1);
    float n = 0.0f, mu = 0.0f, m2 = 0.0f;
    for (int t = lane; t < ntiles; t += 32)
      chan_merge(n, mu, m2, static_cast<float>(max(0, min(tile_n, N - t * tile_n))),
                 ws[static_cast<size_t>(t) * M + row], ws[static_cast<size_t>(ntiles + t) * M + row]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float nb = __shfl_xor_sync(0xffffffffu, n, o);
      const float mb = __shfl_xor_sync(0xffffffffu, mu, o);
      const float m2b = __shfl_xor_sync(0xffffffffu, m2, o);
      chan_merge(n, mu, m2, nb, mb, m2b);
    }
    if (lane == 0) {
      s_mean[r] = mu;
      s_inv[r] = 1.0f / sqrtf(m2 / static_cast<float>(N) + eps);
    }
  }
  __syncthreads();
  const int j = blockIdx.y * kFinCols + threadIdx.x * 8;
  if (j >= N) return;  // N % 8 == 0: a thread's 8 columns are all in or all out
  const float4 g0 = __ldg(reinterpret_cast<const float4*>(ln_w + j));
  const float4 g1 = __ldg(reinterpret_cast<const float4*>(ln_w + j) + 1);
  const float4 b0 = __ldg(reinterpret_cast<const float4*>(ln_b + j));
  const float4 b1 = __ldg(reinterpret_cast<const float4*>(ln_b + j) + 1);
  const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
  const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
  stream_block_rows(c, N, row0, min(kFinRows, M - row0), j, [&](int r, float (&f)[8]) {
    const float mean = s_mean[r], inv_std = s_inv[r];
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = ((f[i] - mean) * inv_std) * g[i] + b[i];
  });
}

// Merge of (max, sum of exp2) partials in the log2 domain; -inf max = empty.
__device__ __forceinline__ void lse2_merge(float& m, float& l, float mb, float lb) {
  if (mb == -INFINITY) return;
  if (m == -INFINITY) {
    m = mb;
    l = lb;
    return;
  }
  const float mn = fmaxf(m, mb);
  l = l * exp2f(m - mn) + lb * exp2f(mb - mn);
  m = mn;
}

// Warp-wide merge of a row's per-tile (max, sumexp) partials.
__device__ __forceinline__ void row_lse2(const float* __restrict__ ws, int M, int ntiles, int row, int lane, float& m,
                                         float& l) {
  m = -INFINITY;
  l = 0.0f;
  for (int t = lane; t < ntiles; t += 32)
    lse2_merge(m, l, ws[static_cast<size_t>(t) * M + row], ws[static_cast<size_t>(ntiles + t) * M + row]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float mb = __shfl_xor_sync(0xffffffffu, m, o);
    const float lb = __shfl_xor_sync(0xffffffffu, l, o);
    lse2_merge(m, l, mb, lb);
  }
}

// In-place softmax of the rows y written by the GEMM epilogue, from the
// per-tile (max, sumexp) partials in the log2 domain:
// out = exp2(y * log2 e - m2) * (1 / l).  One warp per row.  (The
// column-owning form of the LayerNorm finaliser measured 2% slower here: with
// no per-column operands the row walk is not L1-bound.)
template <typename T>
__global__ void softmax_finalize_kernel(T* __restrict__ c, const float* __restrict__ ws, int M, int N,
                                        int ntiles) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    float m, l;
    row_lse2(ws, M, ntiles, row, lane, m, l);
    const float inv = 1.0f / l;
    constexpr float kLog2e = 1.4426950408889634f;
    T* cr = c + static_cast<size_t>(row) * N;
#pragma unroll 4
    for (int j = lane * 8; j < N; j += 256) {
      float f[8];
      load8(cr + j, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = exp2f(fmaf(f[i], kLog2e, -m)) * inv;
      store8(cr + j, f);
    }
  }
}

}  // namespace akili
