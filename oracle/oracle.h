/*
 * oracle.h — CPU oracle for the akili-bench kbt_* / flash hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the host gold
 * loops of akili-bench (benchmarks/<bench>/main.cpp verify blocks and
 * benchmarks/flash/main.cpp attention_cpu), in the reference's loop order
 * and fp32 arithmetic.  It is the checker for the CUDA path: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.  The
 * product library never links it.
 *
 * Parity pin: oracle/build_oracle.py compiles each reference main.cpp unchanged
 * against a host-memory Vortex runtime whose "device" runs these functions
 * and a probe that turns the reference's own verify loop into an
 * exact-equality check; the binaries print PASSED! only when every output of
 * this oracle is bit-identical to the reference gold.  The same recipe
 * captured the golden vectors under tests/golden/.
 *
 * Every function computes output rows [row0, row1) and leaves other rows
 * untouched, so callers can evaluate a subset of rows or split rows over
 * threads.  Matrices are row-major fp32; W/B are [K x N], K of attention
 * score is [N x D].
 */
#ifndef AKILI_ORACLE_H_
#define AKILI_ORACLE_H_
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void oracle_kbt_sgemm(const float* a, const float* b, float* c,
                      uint32_t M, uint32_t N, uint32_t K, uint32_t row0, uint32_t row1);
void oracle_kbt_gemm_add_relu(const float* a, const float* w, const float* bias, float* c,
                              uint32_t M, uint32_t N, uint32_t K, uint32_t row0, uint32_t row1);
void oracle_kbt_gemm_mul_leakyrelu(const float* a, const float* w, const float* bias, float* c,
                                   uint32_t M, uint32_t N, uint32_t K, float multiplier,
                                   float negative_slope, uint32_t row0, uint32_t row1);
void oracle_kbt_gemm_div_sum_scale(const float* a, const float* w, float* c, uint32_t M,
                                   uint32_t N, uint32_t K, float scaling_factor, uint32_t row0,
                                   uint32_t row1);
void oracle_kbt_gemm_layernorm(const float* a, const float* w, const float* bias,
                               const float* ln_w, const float* ln_b, float* c, uint32_t M,
                               uint32_t N, uint32_t K, float eps, uint32_t row0, uint32_t row1);
void oracle_kbt_attention_score(const float* q, const float* k, float* c, uint32_t M,
                                uint32_t N, uint32_t D, uint32_t row0, uint32_t row1);
void oracle_kbt_matmul_softmax(const float* a, const float* b, float* c, uint32_t M, uint32_t N,
                               uint32_t K, uint32_t row0, uint32_t row1);
void oracle_kbt_matmul_scale_residadd_clamp(const float* a, const float* b, float* c, uint32_t M,
                                            uint32_t N, uint32_t K, float scale_factor,
                                            float clamp_min, float clamp_max, uint32_t row0,
                                            uint32_t row1);
void oracle_kbt_matmul_sum_max_avgpool(const float* a, const float* w, const float* bias,
                                       float* c, uint32_t M, uint32_t N, uint32_t K,
                                       uint32_t row0, uint32_t row1);
void oracle_kbt_gemm_rmsnorm_swiglu(const float* x, const float* rms_w, const float* wg,
                                    const float* wu, float* c, uint32_t M, uint32_t N,
                                    uint32_t K, float eps, uint32_t row0, uint32_t row1);
void oracle_kbt_gemm_silu_mul(const float* a, const float* wa, const float* ba, const float* wb,
                              const float* bb, float* c, uint32_t M, uint32_t N, uint32_t K,
                              uint32_t row0, uint32_t row1);
/* One head: Q/K/V/O [seq_len x d].  `scale` multiplies each Q.K^T dot
 * product; 1.0f reproduces the reference (which has no scale). */
void oracle_flash(float* out, const float* q, const float* k, const float* v, uint32_t seq_len,
                  uint32_t d, float scale, uint32_t row0, uint32_t row1);
void oracle_flash_causal(float* out, float* m_out, float* l_out, const float* q, const float* k, const float* v,
                         uint32_t seq_len, uint32_t d, float scale, uint32_t causal, uint32_t row0, uint32_t row1);
void oracle_attention_matmul(float* out, const float* A, const float* B, uint32_t M, uint32_t N, uint32_t K,
                             uint32_t row0, uint32_t row1);
void oracle_attention_softmax(float* out, const float* A, uint32_t M, uint32_t N, uint32_t row0, uint32_t row1);
/* llama2 matmul offload: C[M x N] = A[M x K] . B[K x N], summed over k in order. */
void oracle_llama2_matmul(float* C, const float* A, const float* B, uint32_t M, uint32_t N, uint32_t K,
                          uint32_t row0, uint32_t row1);
void oracle_kb2_gemm_add_relu(const float* a, const float* w, const float* bias, float* c, uint32_t M,
                              uint32_t N, uint32_t K, uint32_t row0, uint32_t row1);
void oracle_kb2_gemm_mul_leakyrelu(const float* a, const float* w, const float* bias, float* c, uint32_t M,
                                   uint32_t N, uint32_t K, float multiplier, float negative_slope, uint32_t row0,
                                   uint32_t row1);
void oracle_kb2_gemm_div_sum_scale(const float* a, const float* w, float* c, uint32_t M, uint32_t N, uint32_t K,
                                   float scaling_factor, uint32_t row0, uint32_t row1);
void oracle_kb2_gemm_layernorm(const float* a, const float* w, const float* bias, const float* ln_w,
                               const float* ln_b, float* c, uint32_t M, uint32_t N, uint32_t K, float eps,
                               uint32_t row0, uint32_t row1);
void oracle_kb2_attention_score(const float* q, const float* k, float* c, uint32_t M, uint32_t N, uint32_t D,
                                uint32_t row0, uint32_t row1);
void oracle_kb2_matmul_softmax(const float* a, const float* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                               uint32_t row0, uint32_t row1);
void oracle_kb2_matmul_scale_residadd_clamp(const float* a, const float* w, const float* bias, float* c,
                                            uint32_t M, uint32_t N, uint32_t K, float scale_factor,
                                            float clamp_min, float clamp_max, uint32_t row0, uint32_t row1);
void oracle_kb2_matmul_sum_max_avgpool(const float* a, const float* w, const float* bias, float* c, uint32_t M,
                                       uint32_t N, uint32_t K, uint32_t row0, uint32_t row1);
void oracle_kb2_gemm_rmsnorm_swiglu(const float* x, const float* rms_w, const float* wg, const float* wu, float* c,
                                    uint32_t M, uint32_t N, uint32_t K, float eps, uint32_t row0, uint32_t row1);
void oracle_kb2_gemm_silu_mul(const float* a, const float* wa, const float* ba, const float* wb, const float* bb,
                              float* c, uint32_t M, uint32_t N, uint32_t K, uint32_t row0, uint32_t row1);

/* Helpers used by tests to reproduce the device's operand rounding. */
float oracle_round_f16(float x);                 /* fp32 -> nearest-even fp16 -> fp32 */
void oracle_round_f16_array(float* x, uint64_t n);

#ifdef __cplusplus
}
#endif
#endif
