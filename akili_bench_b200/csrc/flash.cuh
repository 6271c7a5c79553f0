// flash.cuh — flash-attention forward on tcgen05 (the TCU flash of
// benchmarks/flash/kernel.cpp:138-342, re-designed for sm_100a):
//
//   O[bh, i, :] = sum_j softmax_j(scale * Q[bh,i,:].K[bh,j,:]) V[bh, j, :]
//
// One CTA per (256 queries = two 128-row Q tiles, batch*head), 576 threads:
//   warp 0       TMA: both Q tiles once, then K_j and V_j (128 keys each)
//                into two-deep K and V rings.
//   warp 1       TMEM owner and MMA issuer.  Per key block j and Q tile t:
//                  O_t += P_t,j-1 . V_j-1   (A = P from TMEM, B = V, MN-major)
//                  S_t,j  = Q_t . K_j^T     (into the columns P_t,j-1 occupied)
//                Issued in that order by one elected lane of the converged
//                warp, the MMAs run in order, so S may overwrite P once the
//                P.V that reads it is ahead of it.
//   warps 2..9   softmax of Q tile 0, warps 10..17 of Q tile 1: two threads
//                per query row, each taking 64 of the block's 128 scores.
//                While one tile's softmax runs, the tensor core works on the
//                other tile.  Per block: read the half's 64 scores of S_t,j
//                from TMEM (scores never leave the chip), swap the halves'
//                maxima through shared memory (one barrier per tile), rescale
//                O_t in TMEM only when the running max grows by more than 2^8
//                (the stale max cancels in O / l), then write
//                P = exp2(scale*log2e*s - m) as packed fp16 over the first 64
//                columns of S_t in parts (four at head dim 128, two at 64),
//                announcing each: the P.V K-steps over the first parts' keys
//                start while the later parts are computed.  S_t,j being complete implies
//                O_t += P_t,j-1 V_j-1 is complete, and the next P.V waits for
//                the first part, so the rescale never races the accumulation.
// Finally the halves add their row sums, and each divides its O columns by l,
// stages them through swizzled shared memory (the drained K/V rings) and
// TMA-stores them.  Head dims up to 64 use a 64-column tile, up to 128 a
// 128-column tile; TMA zero-fills the padding and the key tail; keys >=
// seq_len (and, causal, after the query) are masked to -inf.
#pragma once
#include <cuda_fp16.h>

#include "../../include/akili.h"
#include "gemm.cuh"
#include "sm100.cuh"

namespace akili {

constexpr int kFlashBM = 128;  // query rows per Q tile (two tiles per CTA)
constexpr int kFlashBN = 128;  // keys per block
constexpr int kFlashQTiles = 2;
// Two threads per query row: each softmax warp takes 64 of a block's 128
// scores for 32 rows, so a Q tile has 8 softmax warps (two halves of 4).
constexpr int kFlashThreads = 64 + 256 * kFlashQTiles;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Of each group of kExpGroup consecutive score pairs, the last is exponentiated
// on the FMA pipe (exp2_fma3_pair), the others by the MUFU's exp2; 0 keeps every
// exponential on the MUFU, which measured fastest once the softmax loop used
// packed fp32x2 arithmetic (C5: 0.587 TFLOP/s per MHz against 0.559, 0.564
// and 0.537 with one pair in 4, 3 and 2 on the FMA pipe).
#ifndef AKILI_FLASH_EXP_GROUP
#define AKILI_FLASH_EXP_GROUP 0
#endif
constexpr int kExpGroup = AKILI_FLASH_EXP_GROUP;

// The softmax writes each block's P in parts and announces each one, so the
// P.V MMAs over the keys of the first parts run while the later parts'
// exponentials are computed.  Each half of a row holds 64 keys, four P.V
// K-steps of 16 keys (8 packed P columns each); part p covers K-steps
// [p * steps, (p + 1) * steps) of both halves.  At B8 H32 S4096 d128, two
// parts measured +4% over one and four parts +1% over two; two uneven
// parts (1 + 3 or 3 + 1 K-steps) gained less.  Head dims up to 64 keep two
// parts (four spill there).  AKILI_FLASH_P_PARTS (1, 2 or 4) overrides both.
#ifndef AKILI_FLASH_P_PARTS
#define AKILI_FLASH_P_PARTS 0
#endif
__host__ __device__ constexpr int flash_p_parts(int dp) {
  return AKILI_FLASH_P_PARTS > 0 ? AKILI_FLASH_P_PARTS : (dp >= 128 ? 4 : 2);
}
static_assert(flash_p_parts(64) == 1 || flash_p_parts(64) == 2 || flash_p_parts(64) == 4,
              "P is announced in 1, 2 or 4 parts");
static_assert(flash_p_parts(128) == 1 || flash_p_parts(128) == 2 || flash_p_parts(128) == 4,
              "P is announced in 1, 2 or 4 parts");

// Store one part's n packed P columns (8, 16 or 32); waits for it.
template <int n>
__device__ __forceinline__ void tmem_st_p(uint32_t taddr, const uint32_t (&v)[n]) {
  if constexpr (n == 32) {
    float f[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
    tmem_st32(taddr, f);
  } else if constexpr (n == 16) {
    tmem_st16(taddr, v);
  } else {
    tmem_st8(taddr, v);
  }
}

struct FlashArgs {
  int seq_len;
  int head_dim;
  float scale_log2;  // softmax scale * log2(e)
  int causal;        // 1: query i sees keys j <= i only
  float* m_out;      // optional [bh][seq_len]: row max of the scaled scores
  float* l_out;      // optional [bh][seq_len]: sum_j exp(score_j - m)
};

// kSplit: Q and K also carry their fp16 low parts (x - fp16(x)), doubling
// their tiles; S is then Q_hi.K_hi + Q_hi.K_lo + Q_lo.K_hi in fp32.
template <int DP, bool kSplit = false>
struct FlashSmem {
  static constexpr int kQ = kFlashBM * DP * 2;   // one Q tile (one part)
  static constexpr int kKV = kFlashBN * DP * 2;  // one K or V block (one part)
  static constexpr int kParts = kSplit ? 2 : 1;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kFlashQTiles * kQ * kParts;
  static constexpr int kVOff = kKOff + 2 * kKV * kParts;
  static constexpr int kBarOff = kVOff + 2 * kKV;
  // row-statistics exchange between the two halves of a row:
  // [parity][tile][half][128 rows] floats
  static constexpr int kXOff = kBarOff + 256;
  static constexpr int kBytes = kXOff + 2 * kFlashQTiles * 2 * kFlashBM * 4 + 1024;
  // the output staging of both softmax groups reuses the drained K/V rings
  static_assert(2 * kFlashQTiles * (DP / 64) * kFlashBM * 32 * 4 <= 4 * kKV, "staging must fit in the K/V rings");
};

// 18 warps put five on two of the SM sub-partitions, whose 16384 registers
// then allow at most 102 per thread.
template <int DP, typename OutT, bool kSplit>
__global__ void __maxnreg__(96)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                     const __grid_constant__ CUtensorMap tmQlo, const __grid_constant__ CUtensorMap tmKlo,
                     const FlashArgs fa) {
  using L = FlashSmem<DP, kSplit>;
  constexpr int kChunks = DP / 64;  // 64-column swizzle chunks of Q/K/V
  constexpr int kPParts = flash_p_parts(DP);
  constexpr int kPSteps = 4 / kPParts;  // P.V K-steps per part and half
  constexpr int kPPairs = 8 * kPSteps;  // packed P columns (score pairs) per part and half
  constexpr int kStageOut = kFlashBM * 32 * sizeof(OutT);
  constexpr uint32_t kColO = 256;   // O_t at 256 + 128 t; S_t / P_t at 128 t

  const KClock kclk = kclock_begin();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* rel = bars + 5;       // [2] end of key-block iteration j -> rel[j & 1]
  uint64_t* s_full = bars + 9;    // [2] per Q tile
  uint64_t* p_full = bars + 11;   // [2] per Q tile
  uint64_t* o_done = bars + 13;   // [2] per Q tile
  uint64_t* drain = bars + 15;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 16);
  // [tile][parity]: a wait that gave up in block j sets slot j & 1, read by
  // the whole tile after block j's barrier (the next block's slot is apart)
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 17);
  uint64_t* p_part = bars + 19;   // [kPParts - 1][2]: parts before the last of P_t
  // the barrier that announces part p of tile t's P (the last is p_full)
  auto p_bar = [&](int p, int t) { return p == kPParts - 1 ? &p_full[t] : &p_part[2 * p + t]; };

  const int N = fa.seq_len;
  // Causal: the CTA of query tile pair x visits 2x + 2 key blocks, so the
  // pairs are handed out last first (the longest CTAs start earliest).
  const int pair = fa.causal ? static_cast<int>(gridDim.x - 1 - blockIdx.x) : static_cast<int>(blockIdx.x);
  const int m0 = pair * (kFlashBM * kFlashQTiles);
  // Causal: this CTA's queries end at m0 + 255, so key blocks past that are
  // never visited (benchmarks/cupbop_dao_flash/dao_flash_cupbop.cu:64-71 skips
  // them the same way); keys after a row's own index are masked per row.
  const int nkv_all = (N + kFlashBN - 1) / kFlashBN;
  const int nkv = fa.causal ? min(nkv_all, (m0 + kFlashBM * kFlashQTiles + kFlashBN - 1) / kFlashBN) : nkv_all;
  // Under causal masking Q tile 0 (rows m0 .. m0 + 127) sees no key past
  // m0 + 127, so unless the sequence end cuts the range its last key block is
  // fully masked.  That block is skipped for tile 0: no S or P.V MMAs and no
  // softmax pass (its P would be all zeros, so the result is unchanged).
  const int nkv_t0 = fa.causal ? min(nkv_all, (m0 + kFlashBM + kFlashBN - 1) / kFlashBN) : nkv_all;
  static_assert(kFlashQTiles == 2, "two Q tiles per CTA");
  const int bh = blockIdx.y;
  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&rel[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 8);  // one arrive per softmax warp of the tile
      for (int p = 0; p + 1 < kPParts; ++p) mbar_init(&p_part[2 * p + s], 8);
      mbar_init(&o_done[s], 1);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 2 * kFlashQTiles; ++i) abort_flag[i] = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ loads
    if (lane == 0) {
      mbar_expect_tx(q_full, kFlashQTiles * L::kQ * L::kParts);
      for (int t = 0; t < kFlashQTiles; ++t)
        for (int q = 0; q < kChunks; ++q) {
          tma_load_3d(sQ + t * L::kQ + q * 16384, &tmQ, q_full, q * 64, m0 + t * kFlashBM, bh);
          if constexpr (kSplit)
            tma_load_3d(sQ + (kFlashQTiles + t) * L::kQ + q * 16384, &tmQlo, q_full, q * 64, m0 + t * kFlashBM, bh);
        }
      for (int j = 0; j < nkv; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        // K_j reuses the slot of K_j-2, free once iteration j-2 of the MMA
        // loop has completed; V_j the slot of V_j-2, read in iteration j-1.
        if (j >= 2 && !mbar_wait(&rel[st], ph ^ 1, kSiteFlashFree)) break;
        mbar_expect_tx(&k_full[st], L::kKV * L::kParts);
        for (int q = 0; q < kChunks; ++q) {
          tma_load_3d(sK + st * L::kKV + q * 16384, &tmK, &k_full[st], q * 64, j * kFlashBN, bh);
          if constexpr (kSplit)
            tma_load_3d(sK + (2 + st) * L::kKV + q * 16384, &tmKlo, &k_full[st], q * 64, j * kFlashBN, bh);
        }
        if (j >= 2 && !mbar_wait(&rel[(j - 1) & 1], ((j - 1) >> 1) & 1, kSiteFlashFree)) break;
        mbar_expect_tx(&v_full[st], L::kKV);
        for (int q = 0; q < kChunks; ++q)
          tma_load_3d(sV + st * L::kKV + q * 16384, &tmV, &v_full[st], q * 64, j * kFlashBN, bh);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    constexpr uint32_t idesc_s = make_idesc_f16(kFlashBM, kFlashBN, false, false);  // K-major K
    constexpr uint32_t idesc_o = make_idesc_f16(kFlashBM, DP, false, true);         // MN-major V
    // The whole warp runs the issue loop, converged: every lane waits, each
    // wait's outcome is made warp-uniform, and one elected lane (lane 0, so
    // the commits track its MMAs) issues each MMA and commit.  One MMA here
    // is only 64 tensor cycles; issued from a single diverged lane the loop
    // fell behind the tensor pipe (at most 0.80 TFLOP/s per MHz even with no
    // softmax at all).  Shared-memory descriptors are built once; the
    // start-address field is (address >> 4) in the low bits, so an operand at
    // byte offset `off` from a base is base descriptor + (off >> 4).
    bool ok = __all_sync(0xffffffffu, mbar_wait(q_full, 0, kSiteFlashQ));
    {
      const uint64_t qd0 = make_sdesc(smem_u32(sQ), 16, 1024, kSw128);
      const uint64_t kd0 = make_sdesc(smem_u32(sK), 16, 1024, kSw128);
      const uint64_t vd0 = make_sdesc(smem_u32(sV), 16384, 1024, kSw128);
      for (int j = 0; j <= nkv && ok; ++j) {
        const int st = j & 1;
        const int jj = j - 1;  // the block whose P.V this iteration issues
        // K_j, V_j-1 and the first part of P_0,j-1 in one wait; every other
        // part of P just before the P.V K-steps that read it.
        ok = __all_sync(0xffffffffu,
                        mbar_wait3(j < nkv ? &k_full[st] : nullptr, (j >> 1) & 1, j >= 1 ? &v_full[jj & 1] : nullptr,
                                   (jj >> 1) & 1, (j >= 1 && j <= nkv_t0) ? p_bar(0, 0) : nullptr, jj & 1,
                                   kSiteFlashKV));
        const uint64_t kd = kd0 + static_cast<uint64_t>((st * L::kKV) >> 4);
        const uint64_t vd = vd0 + static_cast<uint64_t>(((jj & 1) * L::kKV) >> 4);
#pragma unroll
        for (int t = 0; t < kFlashQTiles; ++t) {
          if (!ok) break;
          const int nkv_t = t == 0 ? nkv_t0 : nkv;
          if (j >= 1 && j <= nkv_t) {
            // O_t += P_t,j-1 . V_j-1, part by part as the softmax announces P.
            // K-step 0 goes first, so it alone starts a fresh accumulator.
            const uint32_t o_tmem = tmem + kColO + t * 128;
            const uint32_t p_tmem = tmem + t * 128;
#pragma unroll
            for (int p = 0; p < kPParts; ++p) {
              if (t > 0 || p > 0) ok = __all_sync(0xffffffffu, mbar_wait(p_bar(p, t), jj & 1, kSiteFlashP));
              if (!ok) break;
              tc_fence_after();
#pragma unroll
              for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int q = 0; q < kPSteps; ++q) {
                  const int k = 4 * h + p * kPSteps + q;
                  umma_f16_ts_warp(o_tmem, p_tmem + k * 8, vd + static_cast<uint64_t>((k * 2048) >> 4), idesc_o,
                                   (jj | k) != 0);
                }
            }
            if (!ok) break;
          }
          // O_t is final once every MMA issued so far completes; both tiles
          // commit in the last iteration, when the K/V rings that the output
          // staging reuses are drained.
          if (j == nkv) umma_commit_warp(&o_done[t]);
          if (j < nkv_t) {
            // S_t,j = Q_t . K_j^T
            tc_fence_after();
            const uint64_t qd = qd0 + static_cast<uint64_t>((t * L::kQ) >> 4);
            const uint32_t s_tmem = tmem + t * 128;
#pragma unroll
            for (int k = 0; k < DP / 16; ++k) {
              const uint64_t off = static_cast<uint64_t>(((k >> 2) * 16384 + (k & 3) * 32) >> 4);
              const uint64_t qh = qd + off;
              const uint64_t kh = kd + off;
              umma_f16_ss_warp(s_tmem, qh, kh, idesc_s, k != 0);
              if constexpr (kSplit) {
                umma_f16_ss_warp(s_tmem, qh, kh + static_cast<uint64_t>((2 * L::kKV) >> 4), idesc_s, 1);
                umma_f16_ss_warp(s_tmem, qh + static_cast<uint64_t>((kFlashQTiles * L::kQ) >> 4), kh, idesc_s,
                                 1);
              }
            }
            umma_commit_warp(&s_full[t]);
          }
        }
        if (!ok) break;
        // K_j (read by S_t,j) and V_j-1 (read by P_t,j-1 . V_j-1) are free once
        // this iteration's MMAs complete.
        umma_commit_warp(&rel[st]);
      }
      umma_commit_warp(drain);
      mbar_wait(drain, 0, kSiteDrain);
    }
    __syncwarp();
  } else {
    // --------------------------------------------------- softmax / output
    // Warps 2 + 8t .. 9 + 8t serve Q tile t: half h = ((warp - 2) >> 2) & 1
    // takes scores [64h, 64h + 64) of each block and O columns
    // [h * DP/2, (h + 1) * DP/2) of its rows (thread = row within the TMEM
    // lane quarter warp & 3).  The halves of a row swap their block maxima
    // through shared memory behind one 256-thread barrier per block, which
    // also orders every S load of the tile before any P store.
    const int grp = (static_cast<int>(warp) - 2) >> 3;  // Q tile
    const int half = ((static_cast<int>(warp) - 2) >> 2) & 1;
    const int wq = static_cast<int>(warp & 3);          // TMEM lane quarter
    const int r = wq * 32 + static_cast<int>(lane);
    const int gtid = threadIdx.x - 64 - 256 * grp - 128 * half;  // 0..127 within (tile, half)
    const uint32_t tile_bar = 1 + grp;                  // 256 threads
    const uint32_t half_bar = 3 + 2 * grp + half;       // 128 threads
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + grp * 128 + half * 64;   // this half's 64 scores
    const uint32_t tP = tmem + lane_off + grp * 128 + half * 32;   // its 32 packed P columns
    const uint32_t tO = tmem + lane_off + kColO + grp * 128 + half * (DP / 2);
    float* xchg = reinterpret_cast<float*>(smem + L::kXOff);
    const float sl = fa.scale_log2;
    float m_use = -INFINITY;
    float m_true = -INFINITY;  // the row's exact running max (m_use may lag it by the rescale threshold)
    float l = 0.0f;            // this half's share of the row sum
    const int qrow = m0 + grp * kFlashBM + r;
    const int nkv_my = grp == 0 ? nkv_t0 : nkv;  // this tile's key blocks
    bool ok = true;
    for (int j = 0; j < nkv_my; ++j) {
      if (!mbar_wait(&s_full[grp], j & 1, kSiteFlashS)) abort_flag[2 * grp + (j & 1)] = 1;
      tc_fence_after();
      const int kv0 = j * kFlashBN + half * 64;
      float s[64];
      tmem_ld64(tS, s);
      // keys of this half the row may see: all but those past the end and,
      // when causal, those after the row's own index (may be <= 0)
      const int nvalid = fa.causal ? min(N - kv0, qrow - kv0 + 1) : N - kv0;
      // Max of the raw scores (the scale is positive, so it commutes with
      // max); masked keys exist only in a tail or diagonal block.
      float mx[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) mx[a] = -INFINITY;
      if (nvalid >= 64) {
#pragma unroll
        for (int i = 0; i < 32; ++i) mx[i & 7] = fmax3(mx[i & 7], s[2 * i], s[2 * i + 1]);
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          if (i >= nvalid) s[i] = -INFINITY;
          mx[i & 7] = fmaxf(mx[i & 7], s[i]);
        }
      }
      const float pmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      float* xs = xchg + ((j & 1) * kFlashQTiles + grp) * (2 * kFlashBM);
      xs[half * kFlashBM + r] = pmax;
      tc_fence_before();
      named_bar_sync(tile_bar, 256);
      tc_fence_after();
      if (abort_flag[2 * grp + (j & 1)]) {
        ok = false;
        break;
      }
      const float rmax = sl * fmaxf(pmax, xs[(half ^ 1) * kFlashBM + r]);
      m_true = fmaxf(m_true, rmax);
      const bool grow = rmax > m_use + kRescaleThreshold;
      const float m_new = grow ? rmax : m_use;
      const float alpha = grow ? exp2f(m_use - m_new) : 1.0f;  // 0 on the first block
      // Rescale this half's O columns when the running max grew (rare after
      // the first blocks), before any part of P is announced: S_t,j being
      // complete implies O_t += P_t,j-1 V_j-1 is, and the next P.V waits for
      // this warp's first arrive below.
      // The scores are live here, so O goes through in 8-column chunks.
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll 1
        for (int c = 0; c < DP / 16; ++c) {
          uint32_t o[8];
          tmem_ld8(tO + c * 8, o);
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st8(tO + c * 8, o);
        }
      }
      // P = exp2(s * sl - m) as packed fp16: per score pair one packed FFMA,
      // two exponentials (MUFU, or the FMA pipe for one pair in kExpGroup),
      // one packed add into the row sum and one pack.  Each part is one TMEM
      // store and one arrive per warp (the store has completed when it returns).
      const uint64_t sl2 = f2_pack(sl, sl);
      const uint64_t nm2 = f2_pack(-m_new, -m_new);
      uint64_t sm2[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) sm2[a] = 0ull;
#pragma unroll
      for (int p = 0; p < kPParts; ++p) {
        uint32_t pk[kPPairs];
#pragma unroll
        for (int ii = 0; ii < kPPairs; ++ii) {
          const int i = p * kPPairs + ii;
          const bool fma_pipe = kExpGroup > 0 && (i % (kExpGroup > 0 ? kExpGroup : 1)) == kExpGroup - 1;
          float x0, x1, p0, p1;
          f2_unpack(f2_fma(f2_pack(s[2 * i], s[2 * i + 1]), sl2, nm2), x0, x1);
          if (fma_pipe) {
            exp2_fma3_pair(x0, x1, p0, p1);
          } else {
            p0 = ex2_mufu(x0);
            p1 = ex2_mufu(x1);
          }
          sm2[i & 3] = f2_add(sm2[i & 3], f2_pack(p0, p1));
          pk[ii] = pack_half2(p0, p1);
        }
        tmem_st_p(tP + p * kPPairs, pk);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_bar(p, grp));
      }
      float sv[8];
#pragma unroll
      for (int a = 0; a < 4; ++a) f2_unpack(sm2[a], sv[2 * a], sv[2 * a + 1]);
      const float rsum = ((sv[0] + sv[1]) + (sv[2] + sv[3])) + ((sv[4] + sv[5]) + (sv[6] + sv[7]));
      l = l * alpha + rsum;
      m_use = m_new;
    }
    if (ok && nkv_my >= 1) {
      // The row sum: the two halves' shares (slot of parity nkv_my, last read
      // two blocks ago).
      float* xs = xchg + ((nkv_my & 1) * kFlashQTiles + grp) * (2 * kFlashBM);
      xs[half * kFlashBM + r] = l;
      named_bar_sync(tile_bar, 256);
      const float lt = l + xs[(half ^ 1) * kFlashBM + r];
      if (fa.m_out != nullptr && half == 0 && qrow < N) {
        // softmax statistics in the reference's natural-log form
        const size_t o = static_cast<size_t>(bh) * N + qrow;
        fa.m_out[o] = m_true * 0.6931471805599453f;
        fa.l_out[o] = lt * exp2f(m_use - m_true);
      }
      if (!mbar_wait(&o_done[grp], 0, kSiteFlashPV)) abort_flag[2 * grp + (nkv_my & 1)] = 1;
      named_bar_sync(tile_bar, 256);
      if (!abort_flag[2 * grp + (nkv_my & 1)]) {
        tc_fence_after();
        const float inv_l = 1.0f / lt;
        // Staging: each (tile, half) takes its own span of the drained K/V
        // rings, one or two 128 x 32 buffers.
        constexpr int kNBuf = DP / 64;  // 32-column chunks per half (1 or 2)
        uint8_t* stg_base = sK + (2 * grp + half) * kNBuf * kStageOut;
        const int c_lo = half * (DP / 2);
        const int ncols = max(0, min(DP / 2, fa.head_dim - c_lo) + 31) / 32;
        for (int c = 0; c < ncols; ++c) {
          float o[32];
          tmem_ld32(tO + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= inv_l;
          uint8_t* stg = stg_base + (c % kNBuf) * kStageOut;
          if (gtid == 0) bulk_wait_read<kNBuf - 1>();
          named_bar_sync(half_bar, 128);
          stage_row<OutT>(stg, r, o);
          fence_async_shared();
          named_bar_sync(half_bar, 128);
          if (gtid == 0) {
            tma_store_3d(&tmO, stg, c_lo + c * 32, m0 + grp * kFlashBM, bh);
            bulk_commit();
          }
        }
        if (gtid == 0) bulk_wait<0>();
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  kclock_end(kclk);
}

template <int DP, bool kSplit>
int launch_flash(dim3 grid, bool out_f32, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                 const CUtensorMap& to, const CUtensorMap& tqlo, const CUtensorMap& tklo, const FlashArgs& fa,
                 cudaStream_t st) {
  const int smem = FlashSmem<DP, kSplit>::kBytes;
  auto k32 = flash_fwd_kernel<DP, float, kSplit>;
  auto k16 = flash_fwd_kernel<DP, __half, kSplit>;
  auto kern = out_f32 ? k32 : k16;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    cudaGetLastError();
    return AKILI_E_LAUNCH;
  }
  kern<<<grid, kFlashThreads, smem, st>>>(tq, tk, tv, to, tqlo, tklo, fa);
  return cudaGetLastError() == cudaSuccess ? AKILI_OK : AKILI_E_LAUNCH;
}

}  // namespace akili
