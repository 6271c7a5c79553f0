/*
 * dao_flash_ref.cu — TEST INFRASTRUCTURE: builds akili-bench's CuPBoP
 * causal flash benchmark (benchmarks/cupbop_dao_flash/dao_flash_cupbop.cu),
 * unchanged and read in place through the include path that
 * oracle/build_oracle.py passes, into oracle/_ref/libdao_flash_ref.so, and
 * gives its two computations C entry points for the oracle pins:
 *
 *   akili_ref_attention_cpu  the reference's CPU gold attention_cpu
 *                            (dao_flash_cupbop.cu:134-169): scale 1/sqrt(d),
 *                            causal mask j > i -> -1e30f, [B][nh][N][d]
 *                            layout, N <= 64 (its scores[64] array).
 *   akili_ref_dao_flash_fwd  the reference's CUDA kernel dao_flash_fwd
 *                            (dao_flash_cupbop.cu:32-132) run on the current
 *                            GPU from host arrays, returning O and the
 *                            kernel's own m / l row statistics.
 *
 * The reference file's main() is renamed by -Dmain=akili_ref_dao_main so it
 * links as a library; akili_ref_dao_selftest runs it (the reference's eight
 * tests of its kernel against its CPU gold) on the current GPU.
 */
#include <cuda_runtime.h>

#include "dao_flash_cupbop.cu"

extern "C" int akili_ref_attention_cpu(const float* q, const float* k, const float* v, float* o, int B, int nh,
                                       int N, int d, int causal) {
  if (N < 1 || N > 64 || d < 1 || B < 1 || nh < 1) return -1;  // scores[64] bounds the reference loop
  attention_cpu(q, k, v, o, B, nh, N, d, causal);
  return 0;
}

/* One block per (batch, head) with Bc threads; every thread owns one query
 * row of a Br-row tile, so the kernel needs Br == Bc and N a multiple of Bc
 * (the last K/V tile is read whole: dao_flash_cupbop.cu:55-58).  Those
 * conditions are checked here before any device call. */
extern "C" int akili_ref_dao_flash_fwd(const float* q, const float* k, const float* v, float* o, float* m,
                                       float* l, int B, int nh, int N, int d, int Bc, float softmax_scale,
                                       int causal) {
  if (B < 1 || nh < 1 || N < 1 || d < 1 || Bc < 1 || Bc > 1024 || N % Bc != 0) return -1;
  const int Br = Bc, Tc = N / Bc, Tr = N / Br;
  const size_t nqkv = (size_t)B * nh * N * d, nlm = (size_t)B * nh * N;
  const int sram = (3 * Bc * d + Bc * Br) * (int)sizeof(float);
  if (sram > 48 * 1024) return -1;
  float *dq = nullptr, *dk = nullptr, *dv = nullptr, *dO = nullptr, *dm = nullptr, *dl = nullptr;
  int rc = 0;
  if (cudaMalloc(&dq, nqkv * 4) || cudaMalloc(&dk, nqkv * 4) || cudaMalloc(&dv, nqkv * 4) ||
      cudaMalloc(&dO, nqkv * 4) || cudaMalloc(&dm, nlm * 4) || cudaMalloc(&dl, nlm * 4)) {
    rc = -2;
  } else {
    /* the reference harness's initial state: O = 0, l = 0, m = -1e30f (dao_flash_cupbop.cu:196-197) */
    float* m0 = (float*)malloc(nlm * 4);
    for (size_t i = 0; i < nlm; ++i) m0[i] = -1e30f;
    cudaMemcpy(dq, q, nqkv * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dk, k, nqkv * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dv, v, nqkv * 4, cudaMemcpyHostToDevice);
    cudaMemset(dO, 0, nqkv * 4);
    cudaMemset(dl, 0, nlm * 4);
    cudaMemcpy(dm, m0, nlm * 4, cudaMemcpyHostToDevice);
    free(m0);
    dao_flash_fwd<<<dim3(B, nh), dim3(Bc), sram>>>(dq, dk, dv, N, d, Tc, Tr, Bc, Br, softmax_scale, causal, dl,
                                                   dm, dO);
    if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) rc = -3;
    if (!rc) {
      cudaMemcpy(o, dO, nqkv * 4, cudaMemcpyDeviceToHost);
      cudaMemcpy(m, dm, nlm * 4, cudaMemcpyDeviceToHost);
      cudaMemcpy(l, dl, nlm * 4, cudaMemcpyDeviceToHost);
    }
  }
  cudaFree(dq);
  cudaFree(dk);
  cudaFree(dv);
  cudaFree(dO);
  cudaFree(dm);
  cudaFree(dl);
  return rc;
}

extern "C" int akili_ref_dao_selftest(void) { return akili_ref_dao_main(); }
