// gemm.cuh — persistent, warp-specialised tcgen05 GEMM with fused epilogues,
// the engine behind every kbt_* op.
//
//   C-tile[128 x BN] = A[128 x K] . B[K x BN]   (fp16 operands, fp32 in TMEM)
//
// Roles (192 threads, one CTA per SM, grid = min(#tiles, #SMs)):
//   warp 0      TMA producer: A tile (K-major, 128B swizzle) and B tile
//               (W[K x N] row-major = MN-major B, or K-major B for Q.K^T)
//               into a kStages-deep shared-memory ring (full/empty mbarriers).
//   warp 1      allocates 512 TMEM columns (two 256-column accumulators) and
//               issues tcgen05.mma (M=128, N=256 or 2 x N=128 for the dual
//               GEMMs, K=16 per instruction) from the whole warp, converged,
//               one elected lane issuing; tcgen05.commit frees ring slots and
//               publishes finished accumulators.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time (one thread per
//               output row), apply the op, and either stage the tile through
//               swizzled shared memory for a TMA store (which also clips the
//               M/N edges) or reduce it to per-row partial statistics.
// The double-buffered accumulator lets the epilogue of tile i overlap the
// main loop of tile i+1.  Tiles are visited in groups of 16 row-blocks so
// the A and B panels in flight stay L2-resident.
#pragma once
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace akili {

constexpr int kBM = 128;          // rows per tile (UMMA M)
constexpr int kBK = 64;           // K per ring slot: 64 fp16 = one 128-byte swizzle row
constexpr int kStages = 4;        // ring depth
constexpr int kGemmThreads = 192; // 6 warps
constexpr int kATileBytes = kBM * kBK * 2;       // 16 KB
constexpr int kBTileBytes = 256 * kBK * 2;       // 32 KB (256 columns, or 2 x 128 for dual)
constexpr int kStageBytes = kATileBytes + kBTileBytes;
constexpr int kAccCols = 256;     // TMEM columns per accumulator buffer
constexpr int kTmemCols = 512;
#ifndef AKILI_GROUP_M
#define AKILI_GROUP_M 16
#endif
constexpr int kGroupM = AKILI_GROUP_M;  // tile raster: row-blocks per group

enum class Epi : int {
  kPlain = 0,        // C = acc                                   (kbt_sgemm)
  kBiasRelu,         // C = max(acc + b, 0)                       (kbt_gemm_add_relu)
  kBiasMulLeaky,     // v=(acc+b)*s0; C = v>=0 ? v : v*s1         (kbt_gemm_mul_leakyrelu)
  kRowSumHalf,       // partial: sum_j acc*0.5                    (kbt_gemm_div_sum_scale)
  kRowSumBias,       // partial: sum_j (acc + b)                  (kbt_matmul_sum_max_avgpool)
  kLnPre,            // C = y = acc + b; partial (mean, M2)       (kbt_gemm_layernorm)
  kSoftmaxPre,       // C = y = acc*s0; partial (max, sumexp), log2 domain   (kbt_attention_score, kbt_matmul_softmax)
  kLseClamp,         // t=clamp(2*(acc*s0)); partial (max, sumexp), log2 domain (kbt_matmul_scale_residadd_clamp)
  kSiluMulBias,      // dual: g=acc0+b0, u=acc1+b1, C=silu(g)*u   (kbt_gemm_silu_mul)
  kSwiglu,           // dual: C = silu(acc0)*acc1                 (kbt_gemm_rmsnorm_swiglu)
};

__host__ __device__ constexpr bool epi_dual(Epi e) { return e == Epi::kSiluMulBias || e == Epi::kSwiglu; }
__host__ __device__ constexpr bool epi_stores(Epi e) {
  return !(e == Epi::kRowSumHalf || e == Epi::kRowSumBias || e == Epi::kLseClamp);
}
__host__ __device__ constexpr int epi_stats(Epi e) {
  return (e == Epi::kRowSumHalf || e == Epi::kRowSumBias) ? 1
         : (e == Epi::kLnPre || e == Epi::kSoftmaxPre || e == Epi::kLseClamp) ? 2
                                                                              : 0;
}
// Output columns per tile.
__host__ __device__ constexpr int epi_bn(Epi e) { return epi_dual(e) ? 128 : 256; }

struct EpiArgs {
  const float* vec0;  // per-column vector (bias / ba)
  const float* vec1;  // per-column vector (bb)
  float s0, s1, s2, s3;
  float* row_ws;      // partial stats: [stat][n_tile][M]
  int M, N, K;
  int num_n_tiles;
  // Row-fused LayerNorm / softmax (CTA-pair kernel): one arrival counter per
  // 128-row block, zeroed before the launch; nullptr = the two-pass form
  // (statistics here, a finaliser kernel afterwards).
  unsigned int* row_sync;
  const float* ln_w;  // LayerNorm gamma / beta and eps (row-fused kLnPre)
  const float* ln_b;
  float eps;
  // CTA-pair tile order: 1 = row-block-major (every column tile of a row
  // block in turn; the B panels stay in L2 when B fits there), 0 = groups of
  // kGroupM row blocks walked row-block-fastest.
  int row_major;
};

// Epilogues that normalise whole rows (longer than one tile).
__host__ __device__ constexpr bool epi_rownorm(Epi e) { return e == Epi::kLnPre || e == Epi::kSoftmaxPre; }

// Split mode (fp32 operands as fp16 hi + lo parts, the kb2_* family): a
// stage holds [A_hi][B_hi][A_lo][B_lo], twice the bytes, so the ring is two deep.
__host__ __device__ constexpr int gemm_stages(bool split) { return split ? 2 : kStages; }
__host__ __device__ constexpr int gemm_stage_bytes(bool split) { return split ? 2 * kStageBytes : kStageBytes; }

__host__ __device__ inline int gemm_smem_bytes(bool stores, int out_bytes, bool split = false) {
  int s = gemm_stages(split) * gemm_stage_bytes(split);
  if (stores) s += 2 * kBM * 32 * out_bytes;
  s += 256;   // barriers + TMEM address
  s += 1024;  // alignment slack
  return s;
}

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& m_blk, int& n_blk) {
  const int per_group = kGroupM * num_n;
  const int group = tile / per_group;
  const int first_m = group * kGroupM;
  const int gm = min(kGroupM, num_m - first_m);
  const int idx = tile - group * per_group;
  m_blk = first_m + idx % gm;
  n_blk = idx / gm;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

template <typename OutT>
__device__ __forceinline__ float round_out(float x) {
  if constexpr (sizeof(OutT) == 2) return __half2float(__float2half_rn(x));
  return x;
}

// Reductions of a 32-value chunk with 4 independent accumulators (no 32-long
// dependency chain in the epilogue's single warp per sub-partition).
__device__ __forceinline__ float sum4(const float (&a)[4]) { return (a[0] + a[1]) + (a[2] + a[3]); }
__device__ __forceinline__ float max4(const float (&a)[4]) { return fmaxf(fmaxf(a[0], a[1]), fmaxf(a[2], a[3])); }

// Per-row running statistics of one tile.
struct RowState {
  float a, b, n;
};

// Epilogues that read the per-column vectors vec0 (bias, ba) / vec1 (bb).
__host__ __device__ constexpr bool epi_vec0(Epi e) {
  return e == Epi::kBiasRelu || e == Epi::kBiasMulLeaky || e == Epi::kRowSumBias || e == Epi::kLnPre ||
         e == Epi::kLseClamp || e == Epi::kSiluMulBias;
}
__host__ __device__ constexpr bool epi_vec1(Epi e) { return e == Epi::kSiluMulBias; }

// This lane's share of a per-column vector for up to four 32-column chunks of
// a tile: lane l holds vec[n0 + (c_begin + i) * 32 + l] (0 past c_end, past N
// or without a vector).  Loaded once per tile with one coalesced load per
// chunk; the epilogue broadcasts column j of chunk i with a warp shuffle
// (lane_pick + __shfl_sync) instead of 32 dependent scalar loads per chunk.
struct LaneVec {
  float v[4];
};
__device__ __forceinline__ LaneVec lane_vec(const float* vec, int n0, int c_begin, int c_end, int N) {
  LaneVec r;
  const int lane = static_cast<int>(threadIdx.x & 31);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int col = n0 + (c_begin + i) * 32 + lane;
    r.v[i] = (vec != nullptr && c_begin + i < c_end && col < N) ? __ldg(vec + col) : 0.0f;
  }
  return r;
}
__device__ __forceinline__ float lane_pick(const LaneVec& lv, int i) {
  return i == 0 ? lv.v[0] : (i == 1 ? lv.v[1] : (i == 2 ? lv.v[2] : lv.v[3]));
}
__device__ __forceinline__ float col_of(float lane_val, int j) { return __shfl_sync(0xffffffffu, lane_val, j); }

// One 32-column chunk of the epilogue: b0 / b1 are this lane's values of
// vec0 / vec1 for the chunk (lane_vec), column j is col_of(b0, j).
// kFastExp: the clamp's log-sum-exp statistics take the hardware exp2
// (ex2.approx, relative error near 2^-22); the kernels set it for fp16
// operands, not for the fp32 (split) mode, which keeps exp2f.
template <Epi E, typename OutT, bool kFastExp = false>
__device__ __forceinline__ void epi_chunk(const EpiArgs& ea, int col0, int nvalid, float (&v)[32],
                                          const float (&u)[32], RowState& st, float b0 = 0.0f, float b1 = 0.0f) {
  (void)col0;
  if constexpr (E == Epi::kPlain) {
    (void)u;
  } else if constexpr (E == Epi::kBiasRelu) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float b = col_of(b0, j);
      const float s = v[j] + b;
      v[j] = s > 0.0f ? s : 0.0f;
    }
  } else if constexpr (E == Epi::kBiasMulLeaky) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float b = col_of(b0, j);
      const float val = (v[j] + b) * ea.s0;
      v[j] = val >= 0.0f ? val : val * ea.s1;
    }
  } else if constexpr (E == Epi::kRowSumHalf) {
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 32; ++j) s[j & 3] += (j < nvalid) ? v[j] * 0.5f : 0.0f;
    st.a += sum4(s);
  } else if constexpr (E == Epi::kRowSumBias) {
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float b = col_of(b0, j);
      s[j & 3] += (j < nvalid) ? (v[j] + b) : 0.0f;
    }
    st.a += sum4(s);
  } else if constexpr (E == Epi::kLnPre) {
    // y = acc + b, rounded to the stored precision; chunk mean/M2 merged into
    // the running (n, mean, M2) with Chan et al.'s pairwise update.
    float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float b = col_of(b0, j);
      v[j] = round_out<OutT>(v[j] + b);
      sum[j & 3] += (j < nvalid) ? v[j] : 0.0f;
    }
    if (nvalid > 0) {
      const float nc = static_cast<float>(nvalid);
      const float mc = sum4(sum) / nc;
      float m2a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float d = v[j] - mc;
        m2a[j & 3] += (j < nvalid) ? d * d : 0.0f;
      }
      const float m2 = sum4(m2a);
      const float ntot = st.n + nc;
      const float delta = mc - st.a;
      st.a += delta * (nc / ntot);
      st.b += m2 + delta * delta * (st.n * nc / ntot);
      st.n = ntot;
    }
  } else if constexpr (E == Epi::kSoftmaxPre || E == Epi::kLseClamp) {
    // Running (max, sum of exp) kept in the log2 domain: m2 = max(y*log2 e),
    // l = sum exp2(y*log2 e - m2), so each element costs one FMA + one ex2.
    constexpr float kLog2e = 1.4426950408889634f;
    float cm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float y;
      if constexpr (E == Epi::kSoftmaxPre) {
        y = round_out<OutT>(v[j] * ea.s0);
      } else {
        // kb2_matmul_scale_residadd_clamp adds a bias first (vec0); kbt has none
        const float b = col_of(b0, j);
        const float scaled = (v[j] + b) * ea.s0;
        float t = scaled + scaled;
        if (t < ea.s1) t = ea.s1;
        if (t > ea.s2) t = ea.s2;
        y = t;
      }
      v[j] = y;
      if (j < nvalid) cm[j & 3] = fmaxf(cm[j & 3], y);
    }
    if (nvalid > 0) {
      const float mnew = fmaxf(st.a, max4(cm) * kLog2e);
      float la[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      // fp16-output softmax and the fp16-operand clamp: the hardware exp2
      // (ex2.approx, relative error near 2^-22) is far inside what the
      // outputs resolve; otherwise exp2f.
      constexpr bool kApprox = (E == Epi::kSoftmaxPre && sizeof(OutT) == 2) || (E == Epi::kLseClamp && kFastExp);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float x = fmaf(v[j], kLog2e, -mnew);
        la[j & 3] += (j < nvalid) ? (kApprox ? ex2_mufu(x) : exp2f(x)) : 0.0f;
      }
      st.b = ((st.a == -INFINITY) ? 0.0f : st.b * exp2f(st.a - mnew)) + sum4(la);
      st.a = mnew;
    }
  } else if constexpr (E == Epi::kSiluMulBias) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float g = v[j] + col_of(b0, j);
      const float uu = u[j] + col_of(b1, j);
      v[j] = silu(g) * uu;
    }
  } else if constexpr (E == Epi::kSwiglu) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = silu(v[j]) * u[j];
  }
}

// Write this thread's 32 values (row r of the 128-row staging tile) in the
// swizzle the TMA store map uses: 64-byte rows (fp16) with the 64B pattern,
// 128-byte rows (fp32) with the 128B pattern.
template <typename OutT>
__device__ __forceinline__ void stage_row(uint8_t* stage, int r, const float (&v)[32]) {
  if constexpr (sizeof(OutT) == 2) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 q;
      q.x = pack_half2(v[8 * c + 0], v[8 * c + 1]);
      q.y = pack_half2(v[8 * c + 2], v[8 * c + 3]);
      q.z = pack_half2(v[8 * c + 4], v[8 * c + 5]);
      q.w = pack_half2(v[8 * c + 6], v[8 * c + 7]);
      const int phys = c ^ ((r >> 1) & 3);
      *reinterpret_cast<uint4*>(stage + r * 64 + phys * 16) = q;
    }
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float4 q = make_float4(v[4 * c + 0], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
      const int phys = c ^ (r & 7);
      *reinterpret_cast<float4*>(stage + r * 128 + phys * 16) = q;
    }
  }
}

// Epilogue of one half of a tile's output columns: 32-column chunks
// [c_begin, c_end) read from TMEM by 128 threads (one per accumulator row,
// TMEM base `tbase` already offset to this warp's lane quarter), the op
// applied, and the result either staged through `staging` (two ping-pong
// buffers) for TMA stores issued by `issuer`, or reduced to the row's
// statistics, which are returned.  `bar_id` is the named barrier of these
// 128 threads.
template <Epi E, typename OutT, bool kFastExp = false>
__device__ __forceinline__ RowState epilogue_half(const EpiArgs& ea, const CUtensorMap* tmC, uint32_t tbase, int n0,
                                                  int mrow0, int r, int c_begin, int c_end, uint8_t* staging,
                                                  uint32_t bar_id, bool issuer, int& chunk_ctr) {
  constexpr bool kDual = epi_dual(E);
  constexpr bool kStore = epi_stores(E);
  constexpr int kStats = epi_stats(E);
  constexpr int kStageOut = kBM * 32 * sizeof(OutT);
  RowState st;
  st.a = (kStats == 2 && E != Epi::kLnPre) ? -INFINITY : 0.0f;
  st.b = 0.0f;
  st.n = 0.0f;
  float v2[64];
  float u2[kDual ? 64 : 1];
  const LaneVec lv0 = lane_vec(epi_vec0(E) ? ea.vec0 : nullptr, n0, c_begin, c_end, ea.N);
  const LaneVec lv1 = lane_vec(epi_vec1(E) ? ea.vec1 : nullptr, n0, c_begin, c_end, ea.N);
  for (int c = c_begin; c < c_end; ++c) {
    const bool odd = ((c - c_begin) & 1) != 0;
    // TMEM is read 64 columns at a time: one load + wait per chunk pair.
    if (!odd) {
      tmem_ld64(tbase + c * 32, v2);
      if constexpr (kDual) tmem_ld64(tbase + 128 + c * 32, reinterpret_cast<float(&)[64]>(u2));
    }
    float v[32];
    float u[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      v[i] = odd ? v2[32 + i] : v2[i];
      if constexpr (kDual) u[i] = odd ? u2[32 + i] : u2[i];
    }
    const int col0 = n0 + c * 32;
    const int nvalid = min(32, ea.N - col0);
    epi_chunk<E, OutT, kFastExp>(ea, col0, nvalid, v, u, st, lane_pick(lv0, c - c_begin),
                                 lane_pick(lv1, c - c_begin));
    if constexpr (kStore) {
      uint8_t* stg = staging + (chunk_ctr & 1) * kStageOut;
      if (issuer) bulk_wait_read<1>();
      named_bar_sync(bar_id, 128);
      stage_row<OutT>(stg, r, v);
      fence_async_shared();
      named_bar_sync(bar_id, 128);
      if (issuer) {
        tma_store_2d(tmC, stg, col0, mrow0);
        bulk_commit();
      }
      ++chunk_ctr;
    }
  }
  return st;
}

// ---- row-fused LayerNorm / softmax (the CTA-pair kernel with ea.row_sync) ----
// Pass 1 reads a half tile's accumulator columns and returns the row's
// statistics of the unrounded values y (LayerNorm: y = acc + b, (mean, M2)
// merged chunk by chunk with Chan et al.'s update; softmax: y = acc * s0,
// (max, sum of exp2) in the log2 domain).  Nothing is stored.
template <Epi E>
__device__ __forceinline__ RowState rowstats_half(const EpiArgs& ea, uint32_t tbase, int n0, int c_begin,
                                                  int c_end) {
  RowState st;
  st.a = (E == Epi::kLnPre) ? 0.0f : -INFINITY;
  st.b = 0.0f;
  st.n = 0.0f;
  float v2[64];
  float u[32];
  const LaneVec lv0 = lane_vec(epi_vec0(E) ? ea.vec0 : nullptr, n0, c_begin, c_end, ea.N);
  for (int c = c_begin; c < c_end; ++c) {
    const bool odd = ((c - c_begin) & 1) != 0;
    if (!odd) tmem_ld64(tbase + c * 32, v2);
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = odd ? v2[32 + i] : v2[i];
    const int col0 = n0 + c * 32;
    epi_chunk<E, float>(ea, col0, min(32, ea.N - col0), v, u, st, lane_pick(lv0, c - c_begin));
  }
  return st;
}

// A row's statistics merged over all its half-tile slots (written by the
// CTAs of every tile of this row block): LayerNorm -> (mean, 1/sqrt(var +
// eps)) with var = M2 / N; softmax -> (m2, 1/l) in the log2 domain.  The slots are read
// through L2 (other SMs wrote them during this launch).
template <Epi E>
__device__ __forceinline__ void rowstats_merge(const EpiArgs& ea, int row, float& s0, float& s1) {
  const int nslots = ea.num_n_tiles;
  const size_t plane = static_cast<size_t>(nslots) * ea.M;
  const int rr = min(row, ea.M - 1);
  float a = (E == Epi::kLnPre) ? 0.0f : -INFINITY, b = 0.0f, n = 0.0f;
  for (int t0 = 0; t0 < nslots; t0 += 8) {
    float pa[8], pb[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int t = t0 + q;
      pa[q] = t < nslots ? __ldcg(ea.row_ws + static_cast<size_t>(t) * ea.M + rr) : 0.0f;
      pb[q] = t < nslots ? __ldcg(ea.row_ws + plane + static_cast<size_t>(t) * ea.M + rr) : 0.0f;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int t = t0 + q;
      if (t >= nslots) break;
      if constexpr (E == Epi::kLnPre) {
        const float nb = static_cast<float>(max(0, min(kAccCols / 2, ea.N - t * (kAccCols / 2))));
        if (nb > 0.0f) {
          if (n == 0.0f) {
            a = pa[q];
            b = pb[q];
            n = nb;
          } else {
            const float ntot = n + nb;
            const float delta = pa[q] - a;
            a += delta * (nb / ntot);
            b += pb[q] + delta * delta * (n * nb / ntot);
            n = ntot;
          }
        }
      } else {
        if (pa[q] != -INFINITY) {
          if (a == -INFINITY) {
            a = pa[q];
            b = pb[q];
          } else {
            const float mn = fmaxf(a, pa[q]);
            b = b * exp2f(a - mn) + pb[q] * exp2f(pa[q] - mn);
            a = mn;
          }
        }
      }
    }
  }
  if constexpr (E == Epi::kLnPre) {
    s0 = a;
    s1 = 1.0f / sqrtf(b / static_cast<float>(ea.N) + ea.eps);
  } else {
    s0 = a;
    s1 = 1.0f / b;
  }
}

// Pass 2: the same half tile read again from TMEM, normalised with the row's
// merged statistics (LayerNorm: ((y - mean) * inv_std) * gamma + beta;
// softmax: exp2(y * log2 e - m2) * (1 / l)) and written once through the
// staging buffers and TMA stores of the ordinary epilogue.
template <Epi E, typename OutT>
__device__ __forceinline__ void rownorm_half(const EpiArgs& ea, const CUtensorMap* tmC, uint32_t tbase, int n0,
                                             int mrow0, int r, int c_begin, int c_end, uint8_t* staging,
                                             uint32_t bar_id, bool issuer, int& chunk_ctr, float s0, float s1) {
  constexpr int kStageOut = kBM * 32 * sizeof(OutT);
  constexpr float kLog2e = 1.4426950408889634f;
  float v2[64];
  const bool ln = E == Epi::kLnPre;
  const LaneVec lb = lane_vec(ln ? ea.vec0 : nullptr, n0, c_begin, c_end, ea.N);
  const LaneVec lg = lane_vec(ln ? ea.ln_w : nullptr, n0, c_begin, c_end, ea.N);
  const LaneVec lbeta = lane_vec(ln ? ea.ln_b : nullptr, n0, c_begin, c_end, ea.N);
  for (int c = c_begin; c < c_end; ++c) {
    const bool odd = ((c - c_begin) & 1) != 0;
    if (!odd) tmem_ld64(tbase + c * 32, v2);
    const int col0 = n0 + c * 32;
    const float pb = lane_pick(lb, c - c_begin), pg = lane_pick(lg, c - c_begin), pbeta = lane_pick(lbeta, c - c_begin);
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float acc = odd ? v2[32 + j] : v2[j];
      if constexpr (E == Epi::kLnPre) {
        const float y = acc + col_of(pb, j);
        v[j] = ((y - s0) * s1) * col_of(pg, j) + col_of(pbeta, j);
      } else {
        v[j] = exp2f(fmaf(acc * ea.s0, kLog2e, -s0)) * s1;
      }
    }
    uint8_t* stg = staging + (chunk_ctr & 1) * kStageOut;
    if (issuer) bulk_wait_read<1>();
    named_bar_sync(bar_id, 128);
    stage_row<OutT>(stg, r, v);
    fence_async_shared();
    named_bar_sync(bar_id, 128);
    if (issuer) {
      tma_store_2d(tmC, stg, col0, mrow0);
      bulk_commit();
    }
    ++chunk_ctr;
  }
}

// Row-fused epilogues with fp16 output keep their tile in registers between
// the passes.  Pass 1 rounds y to fp16, the stored precision, as the
// two-pass form stores it, folds the rounded values into the row statistics
// and keeps them as fp16 pairs: a warp's 32 rows x 32 * kChunks columns in
// 16 * kChunks registers.  The accumulator is then free before the row-block
// wait, and pass 2 normalises from registers.
template <Epi E, int kChunks>
__device__ __forceinline__ RowState rowstats_keep(const EpiArgs& ea, uint32_t tbase, int n0, int c_begin,
                                                  int c_end, uint32_t (&yh)[kChunks][16]) {
  RowState st;
  st.a = (E == Epi::kLnPre) ? 0.0f : -INFINITY;
  st.b = 0.0f;
  st.n = 0.0f;
  float u[32];
  const LaneVec lv0 = lane_vec(epi_vec0(E) ? ea.vec0 : nullptr, n0, c_begin, c_end, ea.N);
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = c_begin + i;
    if (c < c_end) {
      float v[32];
      tmem_ld32(tbase + c * 32, v);
      const int col0 = n0 + c * 32;
      epi_chunk<E, __half>(ea, col0, min(32, ea.N - col0), v, u, st, lane_pick(lv0, i));
#pragma unroll
      for (int j = 0; j < 16; ++j) yh[i][j] = pack_half2(v[2 * j], v[2 * j + 1]);
    }
  }
  return st;
}

// Pass 2 of rowstats_keep's tile: normalise the kept fp16 y (LayerNorm:
// (y - mean) * rstd * gamma + beta; softmax: exp2(y log2 e - max) / sum),
// stage and TMA-store it as rownorm_half does.  gamma and beta come as
// 16-byte loads at one address for the whole warp (four columns each).
template <Epi E, int kChunks>
__device__ __forceinline__ void rownorm_regs(const EpiArgs& ea, const CUtensorMap* tmC,
                                             const uint32_t (&yh)[kChunks][16], int n0, int mrow0, int r,
                                             int c_begin, int c_end, uint8_t* staging, uint32_t bar_id, bool issuer,
                                             int& chunk_ctr, float s0, float s1) {
  constexpr int kStageOut = kBM * 32 * 2;
  constexpr float kLog2e = 1.4426950408889634f;
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = c_begin + i;
    if (c >= c_end) break;  // uniform over the 128 threads of the half
    const int col0 = n0 + c * 32;
    float v[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float y[4];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const __half2 h = *reinterpret_cast<const __half2*>(&yh[i][2 * q + e]);
        const float2 f = __half22float2(h);
        y[2 * e] = f.x;
        y[2 * e + 1] = f.y;
      }
      if constexpr (E == Epi::kLnPre) {
        const int col = col0 + 4 * q;
        float4 g = make_float4(0.f, 0.f, 0.f, 0.f), be = make_float4(0.f, 0.f, 0.f, 0.f);
        if (col < ea.N) {  // N is a multiple of 8: four columns are all in or all out
          g = __ldg(reinterpret_cast<const float4*>(ea.ln_w + col));
          be = __ldg(reinterpret_cast<const float4*>(ea.ln_b + col));
        }
        v[4 * q + 0] = ((y[0] - s0) * s1) * g.x + be.x;
        v[4 * q + 1] = ((y[1] - s0) * s1) * g.y + be.y;
        v[4 * q + 2] = ((y[2] - s0) * s1) * g.z + be.z;
        v[4 * q + 3] = ((y[3] - s0) * s1) * g.w + be.w;
      } else {
        // fp16 output: the hardware exp2 suffices (see epi_chunk)
#pragma unroll
        for (int e = 0; e < 4; ++e) v[4 * q + e] = ex2_mufu(fmaf(y[e], kLog2e, -s0)) * s1;
      }
    }
    uint8_t* stg = staging + (chunk_ctr & 1) * kStageOut;
    if (issuer) bulk_wait_read<1>();
    named_bar_sync(bar_id, 128);
    stage_row<__half>(stg, r, v);
    fence_async_shared();
    named_bar_sync(bar_id, 128);
    if (issuer) {
      tma_store_2d(tmC, stg, col0, mrow0);
      bulk_commit();
    }
    ++chunk_ctr;
  }
}

// Per-row partial statistics of one half tile go to slot `slot` of the
// [stat][slot][M] workspace (two slots per BN-column tile).
template <Epi E>
__device__ __forceinline__ void write_stats(const EpiArgs& ea, int slot, int row, const RowState& st) {
  constexpr int kStats = epi_stats(E);
  if constexpr (kStats > 0) {
    if (row < ea.M) {
      const size_t plane = static_cast<size_t>(ea.num_n_tiles) * ea.M;
      ea.row_ws[static_cast<size_t>(slot) * ea.M + row] = st.a;
      if constexpr (kStats == 2) ea.row_ws[plane + static_cast<size_t>(slot) * ea.M + row] = st.b;
    }
  }
}

// kSplit: A and B arrive as fp16 hi and lo parts (tmAlo, tmB0lo, tmB1lo;
// unused otherwise) and every K-step issues A_hi.B_hi + A_hi.B_lo + A_lo.B_hi
// into the fp32 accumulator: fp32 operands at about 2^-21 relative error.
template <Epi E, typename OutT, bool kBKMajor, bool kSplit = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmC,
                const __grid_constant__ CUtensorMap tmAlo, const __grid_constant__ CUtensorMap tmB0lo,
                const __grid_constant__ CUtensorMap tmB1lo, const EpiArgs ea) {
  constexpr int kSt = gemm_stages(kSplit);
  constexpr int kSB = gemm_stage_bytes(kSplit);
  constexpr bool kDual = epi_dual(E);
  constexpr bool kStore = epi_stores(E);
  constexpr int kStats = epi_stats(E);
  constexpr int BN = epi_bn(E);
  constexpr int kOutBytes = sizeof(OutT);
  constexpr int kStageOut = kBM * 32 * kOutBytes;

  const KClock kclk = kclock_begin();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* staging = ring + kSt * kSB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + (kStore ? 2 * kStageOut : 0));
  uint64_t* full = bars;
  uint64_t* empty = bars + kSt;
  uint64_t* acc_full = bars + 2 * kSt;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int M = ea.M, N = ea.N, K = ea.K;
  const int num_m = (M + kBM - 1) / kBM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + kBK - 1) / kBK;
  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSt; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);  // one arrive per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB0);
    if constexpr (kDual) tma_prefetch_desc(&tmB1);
    if constexpr (kStore) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int m_blk, n_blk;
      tile_coords(tile, num_m, num_n, m_blk, n_blk);
      for (int kb = 0; kb < num_kb; ++kb) {
        if (lane == 0) {
          ok = mbar_wait(&empty[stage], phase ^ 1, kSiteProducerEmpty);
          if (ok) {
            uint8_t* sa = ring + stage * kSB;
            mbar_expect_tx(&full[stage], kSB);
#pragma unroll
            for (int part = 0; part < (kSplit ? 2 : 1); ++part) {
              // part 0: hi parts (or the fp16 operands), part 1: lo parts
              uint8_t* pa = sa + part * kStageBytes;
              uint8_t* sb = pa + kATileBytes;
              const CUtensorMap* mA = part ? &tmAlo : &tmA;
              const CUtensorMap* mB0 = part ? &tmB0lo : &tmB0;
              const CUtensorMap* mB1 = part ? &tmB1lo : &tmB1;
              tma_load_2d(pa, mA, &full[stage], kb * kBK, m_blk * kBM);
              if constexpr (kBKMajor) {
                tma_load_2d(sb, mB0, &full[stage], kb * kBK, n_blk * BN);
              } else if constexpr (kDual) {
                tma_load_2d(sb, mB0, &full[stage], n_blk * BN, kb * kBK);
                tma_load_2d(sb + 8192, mB0, &full[stage], n_blk * BN + 64, kb * kBK);
                tma_load_2d(sb + 16384, mB1, &full[stage], n_blk * BN, kb * kBK);
                tma_load_2d(sb + 24576, mB1, &full[stage], n_blk * BN + 64, kb * kBK);
              } else {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                  tma_load_2d(sb + q * 8192, mB0, &full[stage], n_blk * BN + q * 64, kb * kBK);
              }
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (++stage == kSt) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    constexpr uint32_t idesc = kDual ? make_idesc_f16(kBM, 128, false, !kBKMajor)
                                     : make_idesc_f16(kBM, 256, false, !kBKMajor);
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      // The whole warp issues, converged: each wait's outcome is made
      // warp-uniform and one elected lane (lane 0) issues each MMA and commit.
      ok = __all_sync(0xffffffffu, mbar_wait(&acc_empty[acc], acc_phase ^ 1, kSiteMmaAccEmpty));
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * kAccCols;
      for (int kb = 0; kb < num_kb; ++kb) {
        ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase, kSiteMmaFull));
        if (!ok) break;
        tc_fence_after();
        {
          const uint32_t sa = smem_u32(ring + stage * kSB);
          const uint32_t sb = sa + kATileBytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = make_sdesc(sa + k * 32, 16, 1024, kSw128);
            const uint32_t accum = (kb | k) != 0;
            // B descriptors of the hi part at byte offset `o` from sb (the lo
            // part sits kStageBytes further on, as does A's)
            auto bdesc = [&](uint32_t o) -> uint64_t {
              return kBKMajor ? make_sdesc(sb + o + k * 32, 16, 1024, kSw128)
                              : make_sdesc(sb + o + k * 2048, 8192, 1024, kSw128);
            };
            constexpr int kOps = kDual ? 2 : 1;
#pragma unroll
            for (int op = 0; op < kOps; ++op) {
              const uint32_t d = d_tmem + op * 128;
              const uint64_t bd = bdesc(op * 16384);
              umma_f16_ss_warp(d, ad, bd, idesc, accum);
              if constexpr (kSplit) {
                umma_f16_ss_warp(d, ad, bdesc(kStageBytes + op * 16384), idesc, 1);
                umma_f16_ss_warp(d, make_sdesc(sa + kStageBytes + k * 32, 16, 1024, kSw128), bd, idesc, 1);
              }
            }
          }
          umma_commit_warp(&empty[stage]);
        }
        if (++stage == kSt) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      umma_commit_warp(&acc_full[acc]);
    }
    // Drain: every issued MMA has completed before TMEM is released.
    umma_commit_warp(drain);
    mbar_wait(drain, 0, kSiteDrain);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int ep_tid = threadIdx.x - 64;          // 0..127
    const int wq = static_cast<int>(warp & 3);    // TMEM lane quarter this warp may access
    const int r = wq * 32 + static_cast<int>(lane);
    int it = 0;
    int chunk_ctr = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      int m_blk, n_blk;
      tile_coords(tile, num_m, num_n, m_blk, n_blk);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&acc_full[acc], acc_phase, kSiteEpiAccFull)) *abort_flag = 1;
      named_bar_sync(1, 128);
      if (*abort_flag) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + acc * kAccCols;
      const int n0 = n_blk * BN;
      const int row = m_blk * kBM + r;
      const int nchunks = min(BN / 32, (N - n0 + 31) / 32);
      constexpr int HC = BN / 64;  // chunks per half tile
      RowState st[2];
#pragma unroll
      for (int h = 0; h < 2; ++h)
        st[h] = epilogue_half<E, OutT, !kSplit>(ea, &tmC, tbase, n0, m_blk * kBM, r, h * HC,
                                                min((h + 1) * HC, nchunks), staging, 1, ep_tid == 0, chunk_ctr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      write_stats<E>(ea, 2 * n_blk, row, st[0]);
      write_stats<E>(ea, 2 * n_blk + 1, row, st[1]);
    }
    if constexpr (kStore) {
      if (ep_tid == 0) bulk_wait<0>();
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  kclock_end(kclk);
}

}  // namespace akili

namespace akili {

// ---------------------------------------------------------------------------
// gemm_pair_kernel — the same GEMM on a CTA pair (cluster of 2): one
// tcgen05.mma.cta_group::2 (M = 256) per K-step covers a 256 x BN tile.  Each
// CTA loads its own 128 rows of A and its half of the tile's B columns (no
// TMA multicast), so the B operand bytes each SM pulls from L2/shared memory
// per tensor-core cycle are halved against the single-CTA kernel, and the
// ring can be 6 stages deep.  The even CTA issues the MMAs; its TMA-full
// barriers count both CTAs' loads (the odd CTA's loads signal them through
// the cluster address); one multicast tcgen05.commit frees both CTAs' ring
// slots and publishes both CTAs' accumulators; the odd CTA's epilogue warps
// release an accumulator with a remote arrive on the even CTA's barrier.
// Each CTA's epilogue handles its own 128 rows exactly as in gemm_kernel.
// ---------------------------------------------------------------------------
constexpr int kPairThreads = 320;  // TMA, MMA, 8 epilogue warps (two per TMEM lane quarter)
constexpr int kPairStageBytes = kATileBytes + kBTileBytes / 2;  // 16 KB A + 16 KB half of B
// Split mode (fp32 operands as fp16 hi + lo) stages [A_hi][B_hi][A_lo][B_lo].
__host__ __device__ constexpr int pair_stage_bytes(bool split) { return split ? 2 * kPairStageBytes : kPairStageBytes; }
// Ring depth: 6 slots, 5 when the two epilogue groups stage fp32 output;
// split mode 3 (2 with fp32 staging).
__host__ __device__ constexpr int pair_stages(bool stores, int out_bytes, bool split = false) {
  return split ? (stores && out_bytes == 4 ? 2 : 3) : (stores && out_bytes == 4 ? 5 : 6);
}

__host__ __device__ inline int gemm_pair_smem_bytes(bool stores, int out_bytes, bool split = false) {
  int s = pair_stages(stores, out_bytes, split) * pair_stage_bytes(split);
  if (stores) s += 2 * 2 * kBM * 32 * out_bytes;
  s += 256 + 1024;
  return s;
}

// Tile order of the CTA-pair kernel: the grouped raster, or row-block-major
// (every column tile of a row block in turn) for the row-fused epilogues.
__device__ __forceinline__ void pair_tile_coords(int tile, int num_m, int num_n, bool row_major, int& m_blk,
                                                 int& n_blk) {
  if (row_major) {
    m_blk = tile / num_n;
    n_blk = tile - m_blk * num_n;
  } else {
    tile_coords(tile, num_m, num_n, m_blk, n_blk);
  }
}

template <Epi E, typename OutT, bool kBKMajor, bool kSplit = false>
__global__ void __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                     const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmC,
                     const __grid_constant__ CUtensorMap tmAlo, const __grid_constant__ CUtensorMap tmB0lo,
                     const __grid_constant__ CUtensorMap tmB1lo, const EpiArgs ea) {
  constexpr bool kDual = epi_dual(E);
  constexpr bool kStore = epi_stores(E);
  constexpr int kStats = epi_stats(E);
  constexpr int BN = epi_bn(E);   // output columns per tile
  constexpr int BNH = BN / 2;     // B columns this CTA loads (dual: BN columns of its operand)
  constexpr int kOutBytes = sizeof(OutT);
  constexpr int kStageOut = kBM * 32 * kOutBytes;
  constexpr int kPairStages = pair_stages(kStore, kOutBytes, kSplit);
  constexpr int kSB = pair_stage_bytes(kSplit);

  const KClock kclk = kclock_begin();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* staging = ring + kPairStages * kSB;  // [group][2 ping-pong buffers]
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + (kStore ? 2 * 2 * kStageOut : 0));
  uint64_t* full = bars;                       // [stages], used in the even CTA
  uint64_t* empty = bars + kPairStages;        // [stages]
  uint64_t* acc_full = bars + 2 * kPairStages; // [2]
  uint64_t* acc_empty = acc_full + 2;          // [2], used in the even CTA
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);  // one per epilogue group

  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int M = ea.M, N = ea.N, K = ea.K;
  const int num_m = (M + 2 * kBM - 1) / (2 * kBM);
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + kBK - 1) / kBK;
  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  // Row-fused LayerNorm / softmax: tiles in row-block-major order, so the
  // tiles of one row block run in the same wave (see the epilogue).
  const bool rowfused = epi_rownorm(E) && ea.row_sync != nullptr;
  const bool row_major = rowfused || ea.row_major != 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 16);  // one arrive per epilogue warp (8 per CTA) of both CTAs
    }
    mbar_init(drain, 1);
    abort_flag[0] = 0;
    abort_flag[1] = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB0);
    if constexpr (kDual) tma_prefetch_desc(&tmB1);
    if constexpr (kStore) tma_prefetch_desc(&tmC);
  }
  cluster_sync();  // barriers initialised before the peer signals them
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kTmemCols);
    tmem_relinquish_pair();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t full_c = mapa_shared(smem_u32(full), 0);  // the even CTA's full barriers
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        int m_blk, n_blk;
        pair_tile_coords(tile, num_m, num_n, row_major, m_blk, n_blk);
        const int row0 = m_blk * 2 * kBM + static_cast<int>(rank) * kBM;
        const int col0 = n_blk * BN + static_cast<int>(rank) * BNH;
        for (int kb = 0; kb < num_kb && ok; ++kb) {
          ok = mbar_wait_cluster(&empty[stage], phase ^ 1, kSiteProducerEmpty);
          if (!ok) break;
          uint8_t* sa = ring + stage * kSB;
          uint8_t* sb = sa + kATileBytes;
          const uint32_t fb = full_c + stage * 8;
          if (leader) mbar_expect_tx(&full[stage], 2 * kSB);
          tma_load_2d_pair(sa, &tmA, fb, kb * kBK, row0);
          if constexpr (kBKMajor) {
            tma_load_2d_pair(sb, &tmB0, fb, kb * kBK, col0);
          } else if constexpr (kDual) {
            // the even CTA supplies the tile's 128 columns of B0, the odd CTA
            // the same columns of B1: one N = 256 pair MMA then writes
            // A.B0 to accumulator columns 0..127 and A.B1 to 128..255
            const CUtensorMap* tb = leader ? &tmB0 : &tmB1;
            tma_load_2d_pair(sb, tb, fb, n_blk * BN, kb * kBK);
            tma_load_2d_pair(sb + 8192, tb, fb, n_blk * BN + 64, kb * kBK);
          } else {
            tma_load_2d_pair(sb, &tmB0, fb, col0, kb * kBK);
            tma_load_2d_pair(sb + 8192, &tmB0, fb, col0 + 64, kb * kBK);
          }
          if constexpr (kSplit) {  // the lo parts, same boxes, behind the hi parts
            uint8_t* sal = sa + kPairStageBytes;
            uint8_t* sbl = sal + kATileBytes;
            tma_load_2d_pair(sal, &tmAlo, fb, kb * kBK, row0);
            if constexpr (kBKMajor) {
              tma_load_2d_pair(sbl, &tmB0lo, fb, kb * kBK, col0);
            } else if constexpr (kDual) {
              const CUtensorMap* tbl = leader ? &tmB0lo : &tmB1lo;
              tma_load_2d_pair(sbl, tbl, fb, n_blk * BN, kb * kBK);
              tma_load_2d_pair(sbl + 8192, tbl, fb, n_blk * BN + 64, kb * kBK);
            } else {
              tma_load_2d_pair(sbl, &tmB0lo, fb, col0, kb * kBK);
              tma_load_2d_pair(sbl + 8192, &tmB0lo, fb, col0 + 64, kb * kBK);
            }
          }
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA (even CTA)
    // Dual GEMMs too are one N = 256 MMA per K-step (B0 | B1, see the
    // producer).  Two N = 128 pair MMAs (64 columns per CTA) kept the tensor
    // pipe 62% busy; MMAs of 64 columns run at 48 cycles for 32 of work.
    constexpr uint32_t idesc = make_idesc_f16(2 * kBM, 256, false, !kBKMajor);
    // The whole warp issues, converged: each wait's outcome is made
    // warp-uniform and one elected lane (lane 0) issues each MMA and commit.
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        ok = __all_sync(0xffffffffu, mbar_wait_cluster(&acc_empty[acc], acc_phase ^ 1, kSiteMmaAccEmpty));
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccCols;
        for (int kb = 0; kb < num_kb; ++kb) {
          ok = __all_sync(0xffffffffu, mbar_wait_cluster(&full[stage], phase, kSiteMmaFull));
          if (!ok) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(ring + stage * kSB);
          const uint32_t sb = sa + kATileBytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = make_sdesc(sa + k * 32, 16, 1024, kSw128);
            const uint32_t accum = (kb | k) != 0;
            const uint64_t bd = kBKMajor ? make_sdesc(sb + k * 32, 16, 1024, kSw128)
                                         : make_sdesc(sb + k * 2048, 8192, 1024, kSw128);
            umma_f16_ss_pair_warp(d_tmem, ad, bd, idesc, accum);
            if constexpr (kSplit) {  // + A_hi.B_lo + A_lo.B_hi (lo parts kPairStageBytes behind)
              constexpr uint64_t lo = kPairStageBytes >> 4;
              umma_f16_ss_pair_warp(d_tmem, ad, bd + lo, idesc, 1);
              umma_f16_ss_pair_warp(d_tmem, ad + lo, bd, idesc, 1);
            }
          }
          umma_commit_pair_warp(&empty[stage], 0x3);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair_warp(&acc_full[acc], 0x3);
      }
      // Drain: every issued MMA has completed before either CTA frees TMEM.
      umma_commit_pair_warp(drain, 0x1);
      mbar_wait(drain, 0, kSiteDrain);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // Two groups of four warps: group h takes output columns of half h of
    // each tile, for all 128 rows (warp w reads TMEM lanes 32*(w%4)..).
    const int grp = (static_cast<int>(warp) - 2) >> 2;
    const int gtid = threadIdx.x - 64 - 128 * grp;
    const int wq = static_cast<int>(warp & 3);
    const int r = wq * 32 + static_cast<int>(lane);
    const uint32_t bar_id = 1 + grp;
    uint8_t* gstaging = staging + grp * 2 * kStageOut;
    const uint32_t acc_empty_c = mapa_shared(smem_u32(acc_empty), 0);
    constexpr int HC = BN / 64;  // chunks per half tile
    int it = 0;
    int chunk_ctr = 0;
    if (rowfused) {
      // Row-fused LayerNorm / softmax.  Per tile: pass 1 reads this CTA's
      // accumulator and publishes each row's statistics of its half tile;
      // the CTA then arrives on its 128-row block's counter and waits until
      // the CTAs of all num_n tiles of the block have arrived; pass 2 merges
      // the row's statistics, reads the accumulator again, normalises and
      // stores the result once.  Both epilogue groups share one barrier (3)
      // and one abort flag so that they leave together.
      //
      // Progress: tiles run row-block-major and num_n <= npairs, so the tile
      // a pair handles before tile t of row block R (t - npairs) lies in an
      // earlier row block, as does the tile whose accumulator tile t reuses
      // (t - 2 npairs).  Pass 1 of every tile of R therefore depends only on
      // earlier row blocks, and the wait in tile t ends once they are done.
      // All pairs are resident at once (cooperative launch).
      for (int tile = pair; tile < num_tiles; tile += npairs, ++it) {
        int m_blk, n_blk;
        pair_tile_coords(tile, num_m, num_n, true, m_blk, n_blk);
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait_cluster(&acc_full[acc], acc_phase, kSiteEpiAccFull)) abort_flag[0] = 1;
        named_bar_sync(3, 256);
        if (abort_flag[0]) break;
        tc_fence_after();
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + acc * kAccCols;
        const int n0 = n_blk * BN;
        const int mrow0 = m_blk * 2 * kBM + static_cast<int>(rank) * kBM;
        const int nchunks = min(BN / 32, (N - n0 + 31) / 32);
        const int c0 = grp * HC, c1 = min((grp + 1) * HC, nchunks);
        constexpr bool kKeep = sizeof(OutT) == 2;  // fp16 out: the tile stays in registers
        uint32_t yh[kKeep ? HC : 1][16];
        RowState st;
        if constexpr (kKeep) {
          st = rowstats_keep<E, HC>(ea, tbase, n0, c0, c1, yh);
          // pass 2 reads registers: release the accumulator before the wait
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (leader) mbar_arrive(&acc_empty[acc]);
            else mbar_arrive_cluster(acc_empty_c + acc * 8);
          }
        } else {
          st = rowstats_half<E>(ea, tbase, n0, c0, c1);
        }
        write_stats<E>(ea, 2 * n_blk + grp, mrow0 + r, st);
        __threadfence();
        named_bar_sync(3, 256);
        if (threadIdx.x == 64) {
          unsigned int* cnt = ea.row_sync + mrow0 / kBM;
          atomicAdd(cnt, 1u);
          if (!counter_wait_geq(cnt, static_cast<unsigned int>(num_n), kSiteRowSync)) abort_flag[0] = 1;
        }
        named_bar_sync(3, 256);
        if (abort_flag[0]) break;
        __threadfence();
        float s0, s1;
        rowstats_merge<E>(ea, mrow0 + r, s0, s1);
        if constexpr (kKeep) {
          rownorm_regs<E, HC>(ea, &tmC, yh, n0, mrow0, r, c0, c1, gstaging, bar_id, gtid == 0, chunk_ctr, s0, s1);
        } else {
          rownorm_half<E, OutT>(ea, &tmC, tbase, n0, mrow0, r, c0, c1, gstaging, bar_id, gtid == 0, chunk_ctr, s0,
                                s1);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (leader) mbar_arrive(&acc_empty[acc]);
            else mbar_arrive_cluster(acc_empty_c + acc * 8);
          }
        }
      }
    } else {
      for (int tile = pair; tile < num_tiles; tile += npairs, ++it) {
        int m_blk, n_blk;
        pair_tile_coords(tile, num_m, num_n, row_major, m_blk, n_blk);
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        // Each group reads only its own flag, after its own barrier, so all of
        // its threads leave together.
        if (!mbar_wait_cluster(&acc_full[acc], acc_phase, kSiteEpiAccFull)) abort_flag[grp] = 1;
        named_bar_sync(bar_id, 128);
        if (abort_flag[grp]) break;
        tc_fence_after();
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + acc * kAccCols;
        const int n0 = n_blk * BN;
        const int mrow0 = m_blk * 2 * kBM + static_cast<int>(rank) * kBM;
        const int nchunks = min(BN / 32, (N - n0 + 31) / 32);
        const RowState st = epilogue_half<E, OutT, !kSplit>(ea, &tmC, tbase, n0, mrow0, r, grp * HC,
                                                   min((grp + 1) * HC, nchunks), gstaging, bar_id, gtid == 0,
                                                   chunk_ctr);
        // This warp has read its TMEM rows: release the accumulator to the even CTA's MMA.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive(&acc_empty[acc]);
          else mbar_arrive_cluster(acc_empty_c + acc * 8);
        }
        write_stats<E>(ea, 2 * n_blk + grp, mrow0 + r, st);
      }
    }
    if constexpr (kStore) {
      if (gtid == 0) bulk_wait<0>();
    }
  }

  __syncthreads();
  cluster_sync();  // neither CTA frees TMEM or exits while the pair still uses it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  kclock_end(kclk);
}

}  // namespace akili
