// softmax_rows.cuh — row softmax of a short-K product, fused end to end:
//
//   C[m, :] = softmax_n( s * A[m, :] . B[:, n] )        K <= 256
//
// (kbt_attention_score: A = Q [M x D], B = K [N x D] K-major, s = 1/sqrt(D);
//  kbt_matmul_softmax at short K: B = W [K x N] row-major, s = 1.)
//
// With K this short the product costs less than writing C, so each CTA owns
// a 128-row block, keeps its A rows resident in shared memory, and runs the
// MMA over all N tiles twice:
//   sweep 1  the epilogue folds each tile into running per-row statistics
//            (max, sum of exp2) in the log2 domain; nothing is stored;
//   sweep 2  the same tiles are recomputed and written once, normalised:
//            C = exp2(acc * s * log2 e - (max + log2 sum)).
// C touches HBM exactly once (the unfused pipeline writes it, reads it back
// and writes it again).
//
// Roles (640 threads, one CTA per SM, persistent over row blocks):
//   warp 0       TMA: the block's A rows (K/64 chunks, once per block), then
//                B tiles (256 columns x 64 K, 32 KB) through a ring.
//   warp 1       TMEM owner (two 256-column accumulators) and MMA issuer
//                (tcgen05.mma M=128, N=256, K=16).
//   warps 2..17  four epilogue groups of four warps (four warps on each SM
//                sub-partition, to hide the latency of the exponential
//                chains); group g takes columns [64g, 64g + 64) of every
//                tile, thread = row.  Each warp reads its 32 rows x 64
//                columns with one tcgen05.ld, frees the accumulator, then
//                works from registers; in sweep 2 it stages 32-row x
//                128-byte boxes in its own swizzled buffer and issues its own
//                TMA stores (no barrier across warps).  After sweep 1 the
//                groups exchange their row statistics through shared memory
//                (an mbarrier with a bounded wait) and merge them.
//   warps 18, 19 idle: they make every sub-partition hold five warps, so the
//                register budget (96 per thread) is uniform.
#pragma once
#include <cuda_fp16.h>

#include "gemm.cuh"

namespace akili {

constexpr int kSmThreads = 640;
constexpr int kSmGroups = 4;          // epilogue column groups
constexpr int kSmGroupCols = 64;      // columns of a tile per group
constexpr int kSmEpiWarps = 4 * kSmGroups;
constexpr int kSmMaxK = 256;
constexpr int kSmBTileBytes = 256 * kBK * 2;  // one 64-K chunk of a 256-column B tile
constexpr int kSmMaxStages = 6;
constexpr int kSmWarpStage = 32 * 128;  // one staged store box: 32 rows x 128 bytes

// Shared-memory carve-up (offsets from the 1024-aligned base).
struct SmLayout {
  int a_off, ring_off, stg_off, xchg_off, bar_off, total, stages;
};

inline SmLayout softmax_rows_layout(int K, int out_bytes, int smem_limit) {
  SmLayout L;
  const int kb = (K + kBK - 1) / kBK;
  (void)out_bytes;
  const int stg = kSmEpiWarps * kSmWarpStage;        // [epilogue warp] 32 rows x 128 B
  const int xchg = 2 * kSmGroups * kBM * 2 * 4;       // [parity][group][row](max, sum)
  L.a_off = 0;
  L.ring_off = kb * kATileBytes;
  const int fixed = L.ring_off + stg + xchg + 256 + 1024;
  int stages = (smem_limit - fixed) / kSmBTileBytes;
  L.stages = stages > kSmMaxStages ? kSmMaxStages : stages;
  L.stg_off = L.ring_off + L.stages * kSmBTileBytes;
  L.xchg_off = L.stg_off + stg;
  L.bar_off = L.xchg_off + xchg;
  L.total = L.bar_off + 256 + 1024;
  return L;
}

struct SoftmaxRowsArgs {
  int M, N, K;
  float c;  // s * log2(e), > 0
  SmLayout L;
};

// Exponentials of sweep 1: of each kSmFmaEvery consecutive columns the last
// goes to the FMA pipe (exp2_fma), the rest to the MUFU; 0 keeps all on the MUFU.
#ifndef AKILI_SM_FMA_EVERY
#define AKILI_SM_FMA_EVERY 0
#endif
constexpr int kSmFmaEvery = AKILI_SM_FMA_EVERY;
// fp16 output of sweep 2: exponentials as fp16x2 pairs (one MUFU op per two
// outputs) when 1, fp32 exponentials rounded to fp16 when 0.
#ifndef AKILI_SM_EXP_H2
#define AKILI_SM_EXP_H2 0
#endif
constexpr bool kSmExpH2 = AKILI_SM_EXP_H2 != 0;

// exp2 of element j of a fully unrolled loop: every kSmFmaEvery-th on the
// FMA pipe, the rest on the MUFU (the condition folds at compile time).
__device__ __forceinline__ float sm_exp2(int j, float x) {
  if (kSmFmaEvery > 0 && (j % (kSmFmaEvery > 0 ? kSmFmaEvery : 1)) == kSmFmaEvery - 1) return exp2_fma(x);
  return ex2_mufu(x);
}

// Sweep 1 by pairs: of each kSmFmaPairs consecutive column pairs the last
// goes to the FMA pipe as one packed cubic (exp2_fma3_pair, relative error
// 7.5e-5, below the rounding of an fp16 output), the rest to the MUFU; 0
// keeps all on the MUFU (then kSmFmaEvery applies).  At the 16384 x 4096 x
// 128 attention score, with the packed fp32x2 fold, one pair in 6 / 4 / 3
// measured 306 / 304 / 308 TFLOP/s against 296 for none (scalar fold: 301
// with one in 6, 284 with none).  The same offload in sweep 2 (the fp16
// stores) gained nothing.
#ifndef AKILI_SM_FMA_PAIRS
#define AKILI_SM_FMA_PAIRS 6
#endif
constexpr int kSmFmaPairs = AKILI_SM_FMA_PAIRS;

// Two passes over 64 accumulator columns (the first `nvalid` of which
// exist): the block maximum first, then sum exp2(x - max); merged into the
// row's running (m, l), m = max of x = acc * c, l = sum exp2(x - m).
// kPairs: the FMA-pipe share of kSmFmaPairs applies (fp16 outputs, whose
// rounding hides the cubic's 7.5e-5; fp32 outputs keep every exponential on
// the MUFU).
template <bool kPairs>
__device__ __forceinline__ void softmax_fold64(const float (&v)[64], int nvalid, float c, float& m, float& l) {
  float cm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  float la[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (nvalid >= 64) {
    if constexpr (kPairs) {
      // Packed: per score pair one 3-input max, one fp32x2 FMA (x * c - m),
      // two exponentials and one fp32x2 add into the row sum.
#pragma unroll
      for (int jp = 0; jp < 32; ++jp) cm[jp & 3] = fmax3(cm[jp & 3], v[2 * jp], v[2 * jp + 1]);
      const float mnew = fmaxf(m, max4(cm) * c);
      const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(-mnew, -mnew);
      uint64_t la2[2] = {0ull, 0ull};
#pragma unroll
      for (int jp = 0; jp < 32; ++jp) {
        float x0, x1, p0, p1;
        f2_unpack(f2_fma(f2_pack(v[2 * jp], v[2 * jp + 1]), c2, nm2), x0, x1);
        if (kSmFmaPairs > 0 && jp % (kSmFmaPairs > 0 ? kSmFmaPairs : 1) == kSmFmaPairs - 1) {
          exp2_fma3_pair(x0, x1, p0, p1);
        } else {
          p0 = ex2_mufu(x0);
          p1 = ex2_mufu(x1);
        }
        la2[jp & 1] = f2_add(la2[jp & 1], f2_pack(p0, p1));
      }
      float s0, s1, s2, s3;
      f2_unpack(la2[0], s0, s1);
      f2_unpack(la2[1], s2, s3);
      l = l * ex2_mufu(m - mnew) + ((s0 + s1) + (s2 + s3));
      m = mnew;
      return;
    }
#pragma unroll
    for (int j = 0; j < 64; ++j) cm[j & 3] = fmaxf(cm[j & 3], v[j]);
    const float mnew = fmaxf(m, max4(cm) * c);
    {
#pragma unroll
      for (int j = 0; j < 64; ++j) la[j & 3] += sm_exp2(j, fmaf(v[j], c, -mnew));
    }
    l = l * ex2_mufu(m - mnew) + sum4(la);
    m = mnew;
  } else {
#pragma unroll
    for (int j = 0; j < 64; ++j)
      if (j < nvalid) cm[j & 3] = fmaxf(cm[j & 3], v[j]);
    const float mnew = fmaxf(m, max4(cm) * c);
#pragma unroll
    for (int j = 0; j < 64; ++j) la[j & 3] += (j < nvalid) ? ex2_mufu(fmaf(v[j], c, -mnew)) : 0.0f;
    l = l * ex2_mufu(m - mnew) + sum4(la);
    m = mnew;
  }
}

// Row `lane` of a 32-row x 128-byte store box (128B swizzle: 16-byte unit u
// of row r sits at unit u ^ (r & 7)): exp2(v[j0 + j] * c - mm) for the
// 128 / sizeof(OutT) columns of the box.
template <typename OutT>
__device__ __forceinline__ void stage_box_exp(uint8_t* box, int lane, const float (&v)[64], int j0, float c,
                                              float mm) {
  uint8_t* row = box + lane * 128;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    uint4 q;
    if constexpr (sizeof(OutT) == 2) {
      const int j = j0 + 8 * u;
      if constexpr (kSmExpH2) {
        q.x = ex2_h2(pack_half2(fmaf(v[j + 0], c, -mm), fmaf(v[j + 1], c, -mm)));
        q.y = ex2_h2(pack_half2(fmaf(v[j + 2], c, -mm), fmaf(v[j + 3], c, -mm)));
        q.z = ex2_h2(pack_half2(fmaf(v[j + 4], c, -mm), fmaf(v[j + 5], c, -mm)));
        q.w = ex2_h2(pack_half2(fmaf(v[j + 6], c, -mm), fmaf(v[j + 7], c, -mm)));
      } else {
        // one fp32x2 FMA (x * c - mm) per pair, then two exponentials
        const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(-mm, -mm);
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(v[j + 2 * e], v[j + 2 * e + 1]), c2, nm2), x0, x1);
          w[e] = pack_half2(ex2_mufu(x0), ex2_mufu(x1));
        }
        q = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
      const int j = j0 + 4 * u;
      q.x = __float_as_uint(ex2_mufu(fmaf(v[j + 0], c, -mm)));
      q.y = __float_as_uint(ex2_mufu(fmaf(v[j + 1], c, -mm)));
      q.z = __float_as_uint(ex2_mufu(fmaf(v[j + 2], c, -mm)));
      q.w = __float_as_uint(ex2_mufu(fmaf(v[j + 3], c, -mm)));
    }
    *reinterpret_cast<uint4*>(row + ((u ^ (lane & 7)) << 4)) = q;
  }
}

template <typename OutT, bool kBKMajor>
__global__ void __launch_bounds__(kSmThreads, 1)
    softmax_rows_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const SoftmaxRowsArgs p) {
  const KClock kclk = kclock_begin();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_smem = smem + p.L.a_off;
  uint8_t* ring = smem + p.L.ring_off;
  uint8_t* staging = smem + p.L.stg_off;
  float* xchg = reinterpret_cast<float*>(smem + p.L.xchg_off);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.L.bar_off);
  uint64_t* full = bars;                      // [kSmMaxStages]
  uint64_t* empty = bars + kSmMaxStages;      // [kSmMaxStages]
  uint64_t* acc_full = bars + 2 * kSmMaxStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* a_full = acc_empty + 2;
  uint64_t* a_empty = a_full + 1;
  uint64_t* xbar = a_empty + 1;
  uint64_t* drain = xbar + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int S = p.L.stages;
  const int M = p.M, N = p.N;
  const int num_rb = (M + kBM - 1) / kBM;
  const int T = (N + 255) / 256;
  const int KB = (p.K + kBK - 1) / kBK;
  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kSmEpiWarps);  // one arrive per epilogue warp
    }
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    mbar_init(xbar, 32 * kSmEpiWarps);  // every epilogue thread
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
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
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int rbi = 0;
      bool ok = true;
      for (int rb = blockIdx.x; rb < num_rb && ok; rb += gridDim.x, ++rbi) {
        ok = mbar_wait(a_empty, (rbi & 1) ^ 1, kSiteProducerEmpty);
        if (!ok) break;
        mbar_expect_tx(a_full, KB * kATileBytes);
        for (int kb = 0; kb < KB; ++kb) tma_load_2d(a_smem + kb * kATileBytes, &tmA, a_full, kb * kBK, rb * kBM);
        for (int i = 0; i < 2 * T && ok; ++i) {
          const int n0 = (i < T ? i : i - T) * 256;
          for (int kb = 0; kb < KB; ++kb) {
            ok = mbar_wait(&empty[stage], phase ^ 1, kSiteProducerEmpty);
            if (!ok) break;
            uint8_t* sb = ring + stage * kSmBTileBytes;
            mbar_expect_tx(&full[stage], kSmBTileBytes);
            if constexpr (kBKMajor) {
              tma_load_2d(sb, &tmB, &full[stage], kb * kBK, n0);
            } else {
#pragma unroll
              for (int q = 0; q < 4; ++q) tma_load_2d(sb + q * 8192, &tmB, &full[stage], n0 + q * 64, kb * kBK);
            }
            if (++stage == S) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    constexpr uint32_t idesc = make_idesc_f16(kBM, 256, false, !kBKMajor);
    // The whole warp issues, converged: each wait's outcome is made
    // warp-uniform and one elected lane (lane 0) issues each MMA and commit.
    {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      int rbi = 0;
      bool ok = true;
      const uint32_t sa0 = smem_u32(a_smem);
      for (int rb = blockIdx.x; rb < num_rb && ok; rb += gridDim.x, ++rbi) {
        ok = __all_sync(0xffffffffu, mbar_wait(a_full, rbi & 1, kSiteMmaFull));
        if (!ok) break;
        tc_fence_after();
        for (int i = 0; i < 2 * T && ok; ++i, ++it) {
          const int acc = it & 1;
          const uint32_t acc_phase = (it >> 1) & 1;
          ok = __all_sync(0xffffffffu, mbar_wait(&acc_empty[acc], acc_phase ^ 1, kSiteMmaAccEmpty));
          if (!ok) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * kAccCols;
          for (int kb = 0; kb < KB; ++kb) {
            ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase, kSiteMmaFull));
            if (!ok) break;
            tc_fence_after();
            const uint32_t sa = sa0 + kb * kATileBytes;
            const uint32_t sb = smem_u32(ring + stage * kSmBTileBytes);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              const uint64_t ad = make_sdesc(sa + k * 32, 16, 1024, kSw128);
              const uint32_t accum = (kb | k) != 0;
              if constexpr (kBKMajor)
                umma_f16_ss_warp(d_tmem, ad, make_sdesc(sb + k * 32, 16, 1024, kSw128), idesc, accum);
              else
                umma_f16_ss_warp(d_tmem, ad, make_sdesc(sb + k * 2048, 8192, 1024, kSw128), idesc,
                                 accum);
            }
            umma_commit_warp(&empty[stage]);
            if (++stage == S) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          umma_commit_warp(&acc_full[acc]);
        }
        if (!ok) break;
        umma_commit_warp(a_empty);  // the A rows are free once this block's MMAs complete
      }
      // Drain: every issued MMA has completed before TMEM is released.
      umma_commit_warp(drain);
      mbar_wait(drain, 0, kSiteDrain);
    }
    __syncwarp();
  } else if (warp < 2 + kSmEpiWarps) {
    // ------------------------------------------------------------ epilogue
    // Warps decide alone: a wait that gives up ends this warp's loop (the
    // others then give up on their own bounded waits).
    const int grp = (static_cast<int>(warp) - 2) >> 2;
    const int wq = static_cast<int>(warp & 3);  // TMEM lane quarter this warp may access
    const int r = wq * 32 + static_cast<int>(lane);
    uint8_t* box = staging + (static_cast<int>(warp) - 2) * kSmWarpStage;
    const float c = p.c;
    int it = 0;
    int rbi = 0;
    bool ok = true;
    for (int rb = blockIdx.x; rb < num_rb && ok; rb += gridDim.x, ++rbi) {
      float m = -INFINITY, l = 0.0f, mm = 0.0f;
      for (int i = 0; i < 2 * T; ++i, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_phase, kSiteEpiAccFull));
        if (!ok) break;
        tc_fence_after();
        const uint32_t tbase =
            tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + acc * kAccCols + grp * kSmGroupCols;
        float v[64];
        tmem_ld64(tbase, v);
        // this warp's columns are in registers: release the accumulator
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        const int cb = (i < T ? i : i - T) * 256 + grp * kSmGroupCols;  // first column of this warp's 64
        if (i < T) {
          if (cb < N) softmax_fold64<sizeof(OutT) == 2>(v, N - cb, c, m, l);
          if (i == T - 1) {
            // Merge the groups' statistics of each row (double-buffered by
            // row-block parity; the mbarrier wait is bounded).
            float* xs = xchg + (rbi & 1) * (kSmGroups * kBM * 2);
            xs[grp * (kBM * 2) + 2 * r] = m;
            xs[grp * (kBM * 2) + 2 * r + 1] = l;
            mbar_arrive(xbar);
            ok = __all_sync(0xffffffffu, mbar_wait(xbar, rbi & 1, kSiteExchange));
            if (!ok) break;
            float mg[kSmGroups], lg[kSmGroups];
            float mx = -INFINITY;
#pragma unroll
            for (int g = 0; g < kSmGroups; ++g) {
              mg[g] = xs[g * (kBM * 2) + 2 * r];
              lg[g] = xs[g * (kBM * 2) + 2 * r + 1];
              mx = fmaxf(mx, mg[g]);
            }
            float lt = 0.0f;
#pragma unroll
            for (int g = 0; g < kSmGroups; ++g) lt += lg[g] * ex2_mufu(mg[g] - mx);
            mm = mx + log2f(lt);
          }
        } else {
          constexpr int kBoxCols = 128 / static_cast<int>(sizeof(OutT));  // output columns per store box
#pragma unroll
          for (int q = 0; q < kSmGroupCols / kBoxCols; ++q) {
            const int col0 = cb + q * kBoxCols;
            if (col0 < N) {  // uniform over the warp
              if (lane == 0) bulk_wait_read<0>();  // the previous store from this buffer has read it
              __syncwarp();
              stage_box_exp<OutT>(box, static_cast<int>(lane), v, q * kBoxCols, c, mm);
              fence_async_shared();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmC, box, col0, rb * kBM + wq * 32);
                bulk_commit();
              }
            }
          }
        }
      }
    }
    if (lane == 0) bulk_wait<0>();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  kclock_end(kclk);
}

}  // namespace akili
