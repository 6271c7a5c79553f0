// flash.cuh — flash-attention forward on tcgen05 (the TCU flash of
// benchmarks/flash/kernel.cpp:138-342, re-designed for sm_100a):
//
//   O[bh, i, :] = sum_j softmax_j(scale * Q[bh,i,:].K[bh,j,:]) V[bh, j, :]
//
// One CTA per (128-query tile, batch*head).  192 threads:
//   warp 0      TMA: the Q tile once, then K_j / V_j tiles (128 keys) into a
//               two-deep ring.
//   warp 1      TMEM owner and MMA issuer:  S_j = Q.K_j^T into one of two
//               128-column TMEM buffers, then O += P_j.V_j into a TMEM
//               accumulator (S_{j+1} is issued before O += P_j.V_j so the
//               tensor core works on the next scores while softmax runs).
//   warps 2..5  one thread per query row: read S_j from TMEM, online softmax
//               in base 2 (exp2 of scale*log2(e)*s - m), write P_j as fp16 to
//               a 128B-swizzled shared tile (the A operand of the P.V MMA),
//               and rescale the O row in TMEM only when its running max
//               grows by more than 2^8 (the stale max cancels in O / l).
//               Finally O / l is staged in shared memory and TMA-stored.
// The score matrix never touches HBM.  Head dims up to 64 use a 64-column
// padded tile, up to 128 a 128-column tile; TMA zero-fills the padding and
// the key tail, and keys >= seq_len are masked to -inf.
#pragma once
#include <cuda_fp16.h>

#include "../../include/akili.h"
#include "gemm.cuh"
#include "sm100.cuh"

namespace akili {

constexpr int kFlashBM = 128;  // query rows per CTA
constexpr int kFlashBN = 128;  // keys per step
constexpr int kFlashThreads = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct FlashArgs {
  int seq_len;
  int head_dim;
  float scale_log2;  // softmax scale * log2(e)
};

template <int DP>
struct FlashSmem {
  static constexpr int kQ = kFlashBM * DP * 2;
  static constexpr int kKV = kFlashBN * DP * 2;
  static constexpr int kP = kFlashBM * kFlashBN * 2;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQ;
  static constexpr int kVOff = kKOff + 2 * kKV;
  static constexpr int kPOff = kVOff + 2 * kKV;
  static constexpr int kBarOff = kPOff + kP;
  static constexpr int kBytes = kBarOff + 256 + 1024;
};

template <int DP, typename OutT>
__global__ void __launch_bounds__(kFlashThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                     const FlashArgs fa) {
  using L = FlashSmem<DP>;
  constexpr int kChunks = DP / 64;              // 64-column swizzle chunks of Q/K/V
  constexpr int kOutBytes = sizeof(OutT);
  constexpr int kStageOut = kFlashBM * 32 * kOutBytes;
  constexpr uint32_t kColS0 = 0, kColO = 256;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint8_t* sP = smem + L::kPOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* kv_empty = bars + 5;  // [2]
  uint64_t* s_full = bars + 7;    // [2]
  uint64_t* s_free = bars + 9;    // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* pv_done = bars + 12;
  uint64_t* drain = bars + 13;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 15);

  const int N = fa.seq_len;
  const int nkv = (N + kFlashBN - 1) / kFlashBN;
  const int m0 = blockIdx.x * kFlashBM;
  const int bh = blockIdx.y;
  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
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
      mbar_expect_tx(q_full, L::kQ);
      for (int q = 0; q < kChunks; ++q) tma_load_3d(sQ + q * 16384, &tmQ, q_full, q * 64, m0, bh);
      for (int j = 0; j < nkv; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, kSiteFlashFree)) break;
        mbar_expect_tx(&k_full[st], L::kKV);
        for (int q = 0; q < kChunks; ++q)
          tma_load_3d(sK + st * L::kKV + q * 16384, &tmK, &k_full[st], q * 64, j * kFlashBN, bh);
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
    bool ok = true;
    if (lane == 0) ok = mbar_wait(q_full, 0, kSiteFlashQ);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    const uint32_t q_addr = smem_u32(sQ);
    const uint32_t p_addr = smem_u32(sP);
    auto issue_pv = [&](int jj) -> bool {
      const int st = jj & 1;
      bool good = true;
      if (lane == 0) {
        good = mbar_wait(p_full, jj & 1, kSiteFlashP) && mbar_wait(&v_full[st], (jj >> 1) & 1, kSiteFlashKV);
        if (good) {
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sV + st * L::kKV);
#pragma unroll
          for (int k = 0; k < kFlashBN / 16; ++k) {
            const uint64_t ad = make_sdesc(p_addr + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024, kSw128);
            const uint64_t bd = make_sdesc(v_addr + k * 2048, 16384, 1024, kSw128);
            umma_f16_ss(tmem + kColO, ad, bd, idesc_o, (jj | k) != 0);
          }
          umma_commit(pv_done);
          umma_commit(&kv_empty[st]);
        }
      }
      return __shfl_sync(0xffffffffu, good, 0);
    };
    for (int j = 0; j < nkv && ok; ++j) {
      const int st = j & 1;
      if (lane == 0) {
        ok = mbar_wait(&k_full[st], (j >> 1) & 1, kSiteFlashKV) &&
             mbar_wait(&s_free[st], ((j >> 1) & 1) ^ 1, kSiteFlashS);
        if (ok) {
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + st * L::kKV);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k) {
            const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
            umma_f16_ss(tmem + kColS0 + st * kFlashBN, make_sdesc(q_addr + off, 16, 1024, kSw128),
                        make_sdesc(k_addr + off, 16, 1024, kSw128), idesc_s, k != 0);
          }
          umma_commit(&s_full[st]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (ok && j >= 1) ok = issue_pv(j - 1);
    }
    if (ok && nkv >= 1) issue_pv(nkv - 1);
    if (lane == 0) {
      umma_commit(drain);
      mbar_wait(drain, 0, kSiteDrain);
    }
    __syncwarp();
  } else {
    // --------------------------------------------------- softmax / output
    const int ep_tid = threadIdx.x - 64;
    const int wq = static_cast<int>(warp & 3);
    const int r = wq * 32 + static_cast<int>(lane);
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    float m_use = -INFINITY;  // max used for exponentiation (log2 domain)
    float l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&s_full[sb], (j >> 1) & 1, kSiteFlashS)) *abort_flag = 1;
      named_bar_sync(1, 128);
      if (*abort_flag) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t[32];
        tmem_ld32(tmem + lane_off + kColS0 + sb * kFlashBN + c * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = t[i];
      }
      tc_fence_before();
      mbar_arrive(&s_free[sb]);
      // scale into the log2 domain and mask keys past the end
      const int kv0 = j * kFlashBN;
      float rmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        s[i] = (kv0 + i < N) ? s[i] * fa.scale_log2 : -INFINITY;
        rmax = fmaxf(rmax, s[i]);
      }
      const bool grow = rmax > m_use + kRescaleThreshold;
      const float m_new = grow ? rmax : m_use;
      const float alpha = grow ? exp2f(m_use - m_new) : 1.0f;  // exp2(-inf) = 0 on the first block
      float rsum = 0.0f;
      uint32_t pk[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float p0 = exp2f(s[2 * i] - m_new);
        const float p1 = exp2f(s[2 * i + 1] - m_new);
        rsum += p0 + p1;
        pk[i] = pack_half2(p0, p1);
      }
      // PV_{j-1} must be done: the P tile is reused and O is about to be rescaled.
      if (j >= 1) {
        if (!mbar_wait(pv_done, (j - 1) & 1, kSiteFlashPV)) *abort_flag = 1;
        named_bar_sync(1, 128);
        if (*abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll 1
          for (int c = 0; c < DP / 32; ++c) {
            float o[32];
            tmem_ld32(tmem + lane_off + kColO + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tmem + lane_off + kColO + c * 32, o);
          }
        }
      }
      // P_j -> shared memory, K-major with the 128B swizzle (two 64-key chunks)
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int chunk = u >> 3, unit = u & 7;
        uint4 q;
        q.x = pk[4 * u + 0];
        q.y = pk[4 * u + 1];
        q.z = pk[4 * u + 2];
        q.w = pk[4 * u + 3];
        *reinterpret_cast<uint4*>(sP + chunk * 16384 + r * 128 + ((unit ^ (r & 7)) * 16)) = q;
      }
      fence_async_shared();
      tc_fence_before();
      mbar_arrive(p_full);
      l = l * alpha + rsum;
      m_use = m_new;
    }
    if (ok && nkv >= 1) {
      if (!mbar_wait(pv_done, (nkv - 1) & 1, kSiteFlashPV)) *abort_flag = 1;
      named_bar_sync(1, 128);
      if (!*abort_flag) {
        tc_fence_after();
        const float inv_l = 1.0f / l;
        const int ncols = (fa.head_dim + 31) / 32;
        for (int c = 0; c < ncols; ++c) {
          float o[32];
          tmem_ld32(tmem + lane_off + kColO + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= inv_l;
          uint8_t* stg = sP + (c & 1) * kStageOut;
          if (ep_tid == 0) bulk_wait_read<1>();
          named_bar_sync(1, 128);
          stage_row<OutT>(stg, r, o);
          fence_async_shared();
          named_bar_sync(1, 128);
          if (ep_tid == 0) {
            tma_store_3d(&tmO, stg, c * 32, m0, bh);
            bulk_commit();
          }
        }
        if (ep_tid == 0) bulk_wait<0>();
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int DP>
int launch_flash(dim3 grid, bool out_f32, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                 const CUtensorMap& to, const FlashArgs& fa, cudaStream_t st) {
  const int smem = FlashSmem<DP>::kBytes;
  auto k32 = flash_fwd_kernel<DP, float>;
  auto k16 = flash_fwd_kernel<DP, __half>;
  auto kern = out_f32 ? k32 : k16;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    cudaGetLastError();
    return AKILI_E_LAUNCH;
  }
  kern<<<grid, kFlashThreads, smem, st>>>(tq, tk, tv, to, fa);
  return cudaGetLastError() == cudaSuccess ? AKILI_OK : AKILI_E_LAUNCH;
}

}  // namespace akili
