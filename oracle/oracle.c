/*
 * oracle.c — CPU oracle (TEST INFRASTRUCTURE, never linked by the product).
 *
 * Plain-C restatement of akili-bench's host gold loops; each function cites
 * the verify block it restates.  Loop order, accumulation order, the point
 * where each scalar is applied and the libm calls (expf, logf, tanhf, sqrtf)
 * follow the reference so that, compiled with the reference's host flags
 * (-O2, no fast-math, no FMA ISA), the outputs are bit-identical to it.
 * oracle/build_oracle.py builds the reference harnesses that prove that
 * per op at several sizes.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* benchmarks/kbt_sgemm/main.cpp:117-131 */
void oracle_kbt_sgemm(const float* a, const float* b, float* c, uint32_t M, uint32_t N,
                      uint32_t K, uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i)
    for (uint32_t j = 0; j < N; ++j) {
      float expected = 0;
      for (uint32_t k = 0; k < K; ++k) expected += a[(uint64_t)i * K + k] * b[(uint64_t)k * N + j];
      c[(uint64_t)i * N + j] = expected;
    }
}

/* benchmarks/kbt_gemm_add_relu/main.cpp:124-129 */
void oracle_kbt_gemm_add_relu(const float* a, const float* w, const float* bias, float* c,
                              uint32_t M, uint32_t N, uint32_t K, uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i)
    for (uint32_t j = 0; j < N; ++j) {
      float sum = bias[j];
      for (uint32_t k = 0; k < K; ++k) sum += a[(uint64_t)i * K + k] * w[(uint64_t)k * N + j];
      c[(uint64_t)i * N + j] = (sum > 0.0f) ? sum : 0.0f;
    }
}

/* benchmarks/kbt_gemm_mul_leakyrelu/main.cpp:130-136 */
void oracle_kbt_gemm_mul_leakyrelu(const float* a, const float* w, const float* bias, float* c,
                                   uint32_t M, uint32_t N, uint32_t K, float multiplier,
                                   float negative_slope, uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i)
    for (uint32_t j = 0; j < N; ++j) {
      float sum = bias[j];
      for (uint32_t k = 0; k < K; ++k) sum += a[(uint64_t)i * K + k] * w[(uint64_t)k * N + j];
      float val = sum * multiplier;
      c[(uint64_t)i * N + j] = (val >= 0.0f) ? val : val * negative_slope;
    }
}

/* benchmarks/kbt_gemm_div_sum_scale/main.cpp:120-128 */
void oracle_kbt_gemm_div_sum_scale(const float* a, const float* w, float* c, uint32_t M,
                                   uint32_t N, uint32_t K, float scaling_factor, uint32_t row0,
                                   uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i) {
    float row_sum = 0.0f;
    for (uint32_t j = 0; j < N; ++j) {
      float gemm_val = 0.0f;
      for (uint32_t k = 0; k < K; ++k)
        gemm_val += a[(uint64_t)i * K + k] * w[(uint64_t)k * N + j];
      row_sum += gemm_val * 0.5f;
    }
    c[i] = row_sum * scaling_factor;
  }
}

/* benchmarks/kbt_gemm_layernorm/main.cpp:145-170 (GEMM+bias :146-152, LayerNorm :154-170) */
void oracle_kbt_gemm_layernorm(const float* a, const float* w, const float* bias,
                               const float* ln_w, const float* ln_b, float* c, uint32_t M,
                               uint32_t N, uint32_t K, float eps, uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i) {
    float* ref = c + (uint64_t)i * N;
    for (uint32_t j = 0; j < N; ++j) {
      float sum = 0;
      for (uint32_t k = 0; k < K; ++k) sum += a[(uint64_t)i * K + k] * w[(uint64_t)k * N + j];
      ref[j] = sum + bias[j];
    }
    float mean = 0;
    for (uint32_t j = 0; j < N; ++j) mean += ref[j];
    mean /= (float)N;
    float var = 0;
    for (uint32_t j = 0; j < N; ++j) {
      float d = ref[j] - mean;
      var += d * d;
    }
    var /= (float)N;
    float inv_std = 1.0f / sqrtf(var + eps);
    for (uint32_t j = 0; j < N; ++j) {
      float norm = (ref[j] - mean) * inv_std;
      ref[j] = norm * ln_w[j] + ln_b[j];
    }
  }
}

/* Row-wise softmax shared by attention_score and matmul_softmax:
 * benchmarks/kbt_attention_score/main.cpp:132-142 and
 * benchmarks/kbt_matmul_softmax/main.cpp:127-137. */
static void softmax_row(float* ref, uint32_t N) {
  float row_max = -INFINITY;
  for (uint32_t j = 0; j < N; ++j)
    if (ref[j] > row_max) row_max = ref[j];
  float sum = 0;
  for (uint32_t j = 0; j < N; ++j) {
    ref[j] = expf(ref[j] - row_max);
    sum += ref[j];
  }
  float inv = 1.0f / sum;
  for (uint32_t j = 0; j < N; ++j) ref[j] *= inv;
}

/* benchmarks/kbt_attention_score/main.cpp:117-142: Q.K^T (accumulated in the
 * output cell), a separate scaling pass by 1/sqrtf(D), then softmax. */
void oracle_kbt_attention_score(const float* q, const float* k, float* c, uint32_t M,
                                uint32_t N, uint32_t D, uint32_t row0, uint32_t row1) {
  (void)M;
  float inv_sqrt_d = 1.0f / sqrtf((float)D);
  for (uint32_t i = row0; i < row1; ++i) {
    float* ref = c + (uint64_t)i * N;
    for (uint32_t j = 0; j < N; ++j) {
      ref[j] = 0;
      for (uint32_t d = 0; d < D; ++d) ref[j] += q[(uint64_t)i * D + d] * k[(uint64_t)j * D + d];
    }
    for (uint32_t j = 0; j < N; ++j) ref[j] *= inv_sqrt_d;
    softmax_row(ref, N);
  }
}

/* benchmarks/kbt_matmul_softmax/main.cpp:117-137 */
void oracle_kbt_matmul_softmax(const float* a, const float* b, float* c, uint32_t M, uint32_t N,
                               uint32_t K, uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i) {
    float* ref = c + (uint64_t)i * N;
    for (uint32_t j = 0; j < N; ++j) {
      ref[j] = 0;
      for (uint32_t k = 0; k < K; ++k) ref[j] += a[(uint64_t)i * K + k] * b[(uint64_t)k * N + j];
    }
    softmax_row(ref, N);
  }
}

/* benchmarks/kbt_matmul_scale_residadd_clamp/main.cpp:129-153.  The output
 * is one scalar per row; the row of clamped values (`row_vals`) is heap
 * scratch because N can be large. */
void oracle_kbt_matmul_scale_residadd_clamp(const float* a, const float* b, float* c, uint32_t M,
                                            uint32_t N, uint32_t K, float scale_factor,
                                            float clamp_min, float clamp_max, uint32_t row0,
                                            uint32_t row1) {
  (void)M;
  float* row_vals = (float*)malloc(sizeof(float) * (N ? N : 1));
  for (uint32_t i = row0; i < row1; ++i) {
    for (uint32_t j = 0; j < N; ++j) {
      float dot = 0.0f;
      for (uint32_t k = 0; k < K; ++k) dot += a[(uint64_t)i * K + k] * b[(uint64_t)k * N + j];
      float scaled = dot * scale_factor;
      float res = scaled + scaled;
      float clamped = res;
      if (clamped < clamp_min) clamped = clamp_min;
      if (clamped > clamp_max) clamped = clamp_max;
      row_vals[j] = clamped;
    }
    float max_val = row_vals[0];
    for (uint32_t j = 1; j < N; ++j)
      if (row_vals[j] > max_val) max_val = row_vals[j];
    float sum_exp = 0.0f;
    for (uint32_t j = 0; j < N; ++j) sum_exp += expf(row_vals[j] - max_val);
    float lse = max_val + logf(sum_exp);
    float mish_lse = lse * tanhf(logf(1.0f + expf(lse)));
    c[i] = lse * mish_lse;
  }
  free(row_vals);
}

/* benchmarks/kbt_matmul_sum_max_avgpool/main.cpp:124-132 */
void oracle_kbt_matmul_sum_max_avgpool(const float* a, const float* w, const float* bias,
                                       float* c, uint32_t M, uint32_t N, uint32_t K,
                                       uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i) {
    float total = 0.0f;
    for (uint32_t j = 0; j < N; ++j) {
      float dot = bias[j];
      for (uint32_t k = 0; k < K; ++k) dot += a[(uint64_t)i * K + k] * w[(uint64_t)k * N + j];
      total += dot;
    }
    c[i] = total;
  }
}

/* benchmarks/kbt_gemm_rmsnorm_swiglu/main.cpp:146-172: RMSNorm row (:147-156),
 * dual GEMM from the fp32 normalised row (:158-168), SiLU(g)*u (:170-175). */
void oracle_kbt_gemm_rmsnorm_swiglu(const float* x, const float* rms_w, const float* wg,
                                    const float* wu, float* c, uint32_t M, uint32_t N,
                                    uint32_t K, float eps, uint32_t row0, uint32_t row1) {
  (void)M;
  float* norm = (float*)malloc(sizeof(float) * (K ? K : 1));
  for (uint32_t i = row0; i < row1; ++i) {
    const float* xr = x + (uint64_t)i * K;
    float ss = 0;
    for (uint32_t k = 0; k < K; ++k) {
      float v = xr[k];
      ss += v * v;
    }
    float inv_rms = 1.0f / sqrtf(ss / (float)K + eps);
    for (uint32_t k = 0; k < K; ++k) norm[k] = xr[k] * inv_rms * rms_w[k];
    for (uint32_t j = 0; j < N; ++j) {
      float sum_g = 0, sum_u = 0;
      for (uint32_t k = 0; k < K; ++k) {
        sum_g += norm[k] * wg[(uint64_t)k * N + j];
        sum_u += norm[k] * wu[(uint64_t)k * N + j];
      }
      float silu_g = sum_g / (1.0f + expf(-sum_g));
      c[(uint64_t)i * N + j] = silu_g * sum_u;
    }
  }
  free(norm);
}

/* benchmarks/kbt_gemm_silu_mul/main.cpp:145-162 */
void oracle_kbt_gemm_silu_mul(const float* a, const float* wa, const float* ba, const float* wb,
                              const float* bb, float* c, uint32_t M, uint32_t N, uint32_t K,
                              uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i)
    for (uint32_t j = 0; j < N; ++j) {
      float sum_a = 0, sum_b = 0;
      for (uint32_t k = 0; k < K; ++k) {
        sum_a += a[(uint64_t)i * K + k] * wa[(uint64_t)k * N + j];
        sum_b += a[(uint64_t)i * K + k] * wb[(uint64_t)k * N + j];
      }
      float g = sum_a + ba[j];
      float u = sum_b + bb[j];
      float silu_g = g / (1.0f + expf(-g));
      c[(uint64_t)i * N + j] = silu_g * u;
    }
}

/* benchmarks/flash/main.cpp:52-85 (attention_cpu), per query row, plus a
 * scale on each dot product (1.0f is exact, so scale=1 is the reference). */
void oracle_flash(float* out, const float* q, const float* k, const float* v, uint32_t seq_len,
                  uint32_t d, float scale, uint32_t row0, uint32_t row1) {
  uint32_t N = seq_len;
  float* scores = (float*)malloc(sizeof(float) * (N ? N : 1));
  float* probs = (float*)malloc(sizeof(float) * (N ? N : 1));
  for (uint32_t i = row0; i < row1; ++i) {
    for (uint32_t j = 0; j < N; ++j) {
      float sum = 0.0f;
      for (uint32_t kk = 0; kk < d; ++kk) sum += q[(uint64_t)i * d + kk] * k[(uint64_t)j * d + kk];
      scores[j] = sum * scale;
    }
    float mx = scores[0];
    for (uint32_t j = 1; j < N; ++j) mx = (mx < scores[j]) ? scores[j] : mx; /* std::max */
    float exp_sum = 0.0f;
    for (uint32_t j = 0; j < N; ++j) {
      float e = expf(scores[j] - mx);
      probs[j] = e;
      exp_sum += e;
    }
    for (uint32_t j = 0; j < N; ++j) probs[j] /= exp_sum;
    for (uint32_t kk = 0; kk < d; ++kk) {
      float sum = 0.0f;
      for (uint32_t j = 0; j < N; ++j) sum += probs[j] * v[(uint64_t)j * d + kk];
      out[(uint64_t)i * d + kk] = sum;
    }
  }
  free(scores);
  free(probs);
}

/* benchmarks/cupbop_dao_flash/dao_flash_cupbop.cu:135-168 (attention_cpu
 * with its causal mask: key j > query i scores -1e30f), per query row, with
 * the scale as a parameter.  When m_out / l_out are non-null the row's
 * softmax statistics are written as the reference kernel keeps them
 * (dao_flash_cupbop.cu:111-125, fmha_cupbop.cu:115-116): m = the row maximum
 * of the scaled scores, l = sum_j exp(score_j - m) (masked keys add 0). */
void oracle_flash_causal(float* out, float* m_out, float* l_out, const float* q, const float* k, const float* v,
                         uint32_t seq_len, uint32_t d, float scale, uint32_t causal, uint32_t row0, uint32_t row1) {
  uint32_t N = seq_len;
  float* scores = (float*)malloc(sizeof(float) * (N ? N : 1));
  for (uint32_t i = row0; i < row1; ++i) {
    float max_s = -1e30f;
    for (uint32_t j = 0; j < N; ++j) {
      if (causal && j > i) {
        scores[j] = -1e30f;
      } else {
        float sum = 0.0f;
        for (uint32_t kk = 0; kk < d; ++kk) sum += q[(uint64_t)i * d + kk] * k[(uint64_t)j * d + kk];
        scores[j] = sum * scale;
      }
      if (scores[j] > max_s) max_s = scores[j];
    }
    float sum_exp = 0.0f;
    for (uint32_t j = 0; j < N; ++j) {
      scores[j] = expf(scores[j] - max_s);
      sum_exp += scores[j];
    }
    if (m_out) m_out[i] = max_s;
    if (l_out) l_out[i] = sum_exp;
    for (uint32_t j = 0; j < N; ++j) scores[j] /= sum_exp;
    for (uint32_t kk = 0; kk < d; ++kk) {
      float val = 0.0f;
      for (uint32_t j = 0; j < N; ++j) val += scores[j] * v[(uint64_t)j * d + kk];
      out[(uint64_t)i * d + kk] = val;
    }
  }
  free(scores);
}

/* ---- the kb2_* family: fp32 gold loops of benchmarks/kb2_<bench>/main.cpp,
 * restated in their loop order (the bias starts the dot product). ---- */

/* kb2_gemm_add_relu/main.cpp:113-121 (verify loop) */
void oracle_kb2_gemm_add_relu(const float* a, const float* w, const float* bias, float* c, uint32_t M,
                              uint32_t N, uint32_t K, uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i)
    for (uint32_t j = 0; j < N; ++j) {
      float sum = bias[j];
      for (uint32_t k = 0; k < K; ++k) sum += a[(uint64_t)i * K + k] * w[(uint64_t)k * N + j];
      c[(uint64_t)i * N + j] = (sum > 0.0f) ? sum : 0.0f;
    }
}

/* kb2_gemm_mul_leakyrelu/main.cpp (verify loop) */
void oracle_kb2_gemm_mul_leakyrelu(const float* a, const float* w, const float* bias, float* c, uint32_t M,
                                   uint32_t N, uint32_t K, float multiplier, float negative_slope, uint32_t row0,
                                   uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i)
    for (uint32_t j = 0; j < N; ++j) {
      float sum = bias[j];
      for (uint32_t k = 0; k < K; ++k) sum += a[(uint64_t)i * K + k] * w[(uint64_t)k * N + j];
      sum *= multiplier;
      c[(uint64_t)i * N + j] = (sum >= 0.0f) ? sum : sum * negative_slope;
    }
}

/* kb2_gemm_div_sum_scale/main.cpp (verify loop): out[i] = scaling * sum_j (dot * 0.5) */
void oracle_kb2_gemm_div_sum_scale(const float* a, const float* w, float* c, uint32_t M, uint32_t N, uint32_t K,
                                   float scaling_factor, uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i) {
    float total = 0.0f;
    for (uint32_t j = 0; j < N; ++j) {
      float dot = 0.0f;
      for (uint32_t k = 0; k < K; ++k) dot += a[(uint64_t)i * K + k] * w[(uint64_t)k * N + j];
      total += dot * 0.5f;
    }
    c[i] = total * scaling_factor;
  }
}

/* kb2_gemm_layernorm/main.cpp (verify loop): bias-first dot, then the
 * two-pass biased LayerNorm of the row */
void oracle_kb2_gemm_layernorm(const float* a, const float* w, const float* bias, const float* ln_w,
                               const float* ln_b, float* c, uint32_t M, uint32_t N, uint32_t K, float eps,
                               uint32_t row0, uint32_t row1) {
  (void)M;
  float* vals = (float*)malloc(sizeof(float) * (N ? N : 1));
  for (uint32_t i = row0; i < row1; ++i) {
    for (uint32_t j = 0; j < N; ++j) {
      float dot = bias[j];
      for (uint32_t k = 0; k < K; ++k) dot += a[(uint64_t)i * K + k] * w[(uint64_t)k * N + j];
      vals[j] = dot;
    }
    float sum = 0.0f;
    for (uint32_t j = 0; j < N; ++j) sum += vals[j];
    float mean = sum / (float)N;
    float var = 0.0f;
    for (uint32_t j = 0; j < N; ++j) {
      float diff = vals[j] - mean;
      var += diff * diff;
    }
    var /= (float)N;
    float inv_std = 1.0f / sqrtf(var + eps);
    for (uint32_t j = 0; j < N; ++j) {
      float normalized = (vals[j] - mean) * inv_std;
      c[(uint64_t)i * N + j] = normalized * ln_w[j] + ln_b[j];
    }
  }
  free(vals);
}

/* softmax of one row as the kb2 verify loops compute it: max from element 0,
 * sum of expf(x - max), then expf(x - max) / sum recomputed per element */
static void kb2_softmax_row(const float* x, float* out, uint32_t N) {
  float max_val = x[0];
  for (uint32_t j = 1; j < N; ++j)
    if (x[j] > max_val) max_val = x[j];
  float sum_exp = 0.0f;
  for (uint32_t j = 0; j < N; ++j) sum_exp += expf(x[j] - max_val);
  for (uint32_t j = 0; j < N; ++j) out[j] = expf(x[j] - max_val) / sum_exp;
}

/* kb2_attention_score/main.cpp (verify loop): softmax_j(Q_i . K_j * (1/sqrt(D))) */
void oracle_kb2_attention_score(const float* q, const float* k, float* c, uint32_t M, uint32_t N, uint32_t D,
                                uint32_t row0, uint32_t row1) {
  (void)M;
  float inv_sqrt_d = 1.0f / sqrtf((float)D);
  float* scores = (float*)malloc(sizeof(float) * (N ? N : 1));
  for (uint32_t i = row0; i < row1; ++i) {
    for (uint32_t j = 0; j < N; ++j) {
      float dot = 0.0f;
      for (uint32_t d = 0; d < D; ++d) dot += q[(uint64_t)i * D + d] * k[(uint64_t)j * D + d];
      scores[j] = dot * inv_sqrt_d;
    }
    kb2_softmax_row(scores, c + (uint64_t)i * N, N);
  }
  free(scores);
}

/* kb2_matmul_softmax/main.cpp (verify loop): softmax_j(A_i . B_:j), no scale */
void oracle_kb2_matmul_softmax(const float* a, const float* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                               uint32_t row0, uint32_t row1) {
  (void)M;
  float* vals = (float*)malloc(sizeof(float) * (N ? N : 1));
  for (uint32_t i = row0; i < row1; ++i) {
    for (uint32_t j = 0; j < N; ++j) {
      float dot = 0.0f;
      for (uint32_t k = 0; k < K; ++k) dot += a[(uint64_t)i * K + k] * b[(uint64_t)k * N + j];
      vals[j] = dot;
    }
    kb2_softmax_row(vals, c + (uint64_t)i * N, N);
  }
  free(vals);
}

/* kb2_matmul_scale_residadd_clamp/main.cpp (verify loop): t = clamp(2 *
 * (bias + dot) * scale); lse = max + logf(sum expf(t - max)); out = lse *
 * (lse * tanhf(logf(1 + expf(lse)))) */
void oracle_kb2_matmul_scale_residadd_clamp(const float* a, const float* w, const float* bias, float* c,
                                            uint32_t M, uint32_t N, uint32_t K, float scale_factor,
                                            float clamp_min, float clamp_max, uint32_t row0, uint32_t row1) {
  (void)M;
  float* vals = (float*)malloc(sizeof(float) * (N ? N : 1));
  for (uint32_t i = row0; i < row1; ++i) {
    for (uint32_t j = 0; j < N; ++j) {
      float dot = bias[j];
      for (uint32_t k = 0; k < K; ++k) dot += a[(uint64_t)i * K + k] * w[(uint64_t)k * N + j];
      dot *= scale_factor;
      dot += dot;
      if (dot < clamp_min) dot = clamp_min;
      if (dot > clamp_max) dot = clamp_max;
      vals[j] = dot;
    }
    float max_val = vals[0];
    for (uint32_t j = 1; j < N; ++j)
      if (vals[j] > max_val) max_val = vals[j];
    float sum_exp = 0.0f;
    for (uint32_t j = 0; j < N; ++j) sum_exp += expf(vals[j] - max_val);
    float lse = max_val + logf(sum_exp);
    float mish_lse = lse * tanhf(logf(1.0f + expf(lse)));
    c[i] = lse * mish_lse;
  }
  free(vals);
}

/* kb2_matmul_sum_max_avgpool/main.cpp (verify loop): out[i] = sum_j (bias + dot) */
void oracle_kb2_matmul_sum_max_avgpool(const float* a, const float* w, const float* bias, float* c, uint32_t M,
                                       uint32_t N, uint32_t K, uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i) {
    float total = 0.0f;
    for (uint32_t j = 0; j < N; ++j) {
      float dot = bias[j];
      for (uint32_t k = 0; k < K; ++k) dot += a[(uint64_t)i * K + k] * w[(uint64_t)k * N + j];
      total += dot;
    }
    c[i] = total;
  }
}

/* kb2_gemm_rmsnorm_swiglu/main.cpp (verify loop): r = 1/sqrtf(sum x^2 / K +
 * eps); h_k = x_k * r * w_k in fp32; gate, up = h . Wg, h . Wu; out =
 * gate / (1 + expf(-gate)) * up */
void oracle_kb2_gemm_rmsnorm_swiglu(const float* x, const float* rms_w, const float* wg, const float* wu, float* c,
                                    uint32_t M, uint32_t N, uint32_t K, float eps, uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i) {
    float ss = 0.0f;
    for (uint32_t k = 0; k < K; ++k) {
      float v = x[(uint64_t)i * K + k];
      ss += v * v;
    }
    float inv_rms = 1.0f / sqrtf(ss / (float)K + eps);
    for (uint32_t j = 0; j < N; ++j) {
      float gate = 0.0f, up = 0.0f;
      for (uint32_t k = 0; k < K; ++k) {
        float h = x[(uint64_t)i * K + k] * inv_rms * rms_w[k];
        gate += h * wg[(uint64_t)k * N + j];
        up += h * wu[(uint64_t)k * N + j];
      }
      float silu_gate = gate / (1.0f + expf(-gate));
      c[(uint64_t)i * N + j] = silu_gate * up;
    }
  }
}

/* kb2_gemm_silu_mul/main.cpp (verify loop): gate = ba + a.Wa, up = bb + a.Wb
 * (bias first); out = gate / (1 + expf(-gate)) * up */
void oracle_kb2_gemm_silu_mul(const float* a, const float* wa, const float* ba, const float* wb, const float* bb,
                              float* c, uint32_t M, uint32_t N, uint32_t K, uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t i = row0; i < row1; ++i)
    for (uint32_t j = 0; j < N; ++j) {
      float gate = ba[j];
      for (uint32_t k = 0; k < K; ++k) gate += a[(uint64_t)i * K + k] * wa[(uint64_t)k * N + j];
      float up = bb[j];
      for (uint32_t k = 0; k < K; ++k) up += a[(uint64_t)i * K + k] * wb[(uint64_t)k * N + j];
      float silu_gate = gate / (1.0f + expf(-gate));
      c[(uint64_t)i * N + j] = silu_gate * up;
    }
}

/* ---- benchmarks/attention: the unfused three-kernel attention (fp32) ---- */

/* attention/main.cpp:55-65 (matmul_cpu): out[M x N] = A[M x K] . B[K x N],
 * each element summed over k in order. */
void oracle_attention_matmul(float* out, const float* A, const float* B, uint32_t M, uint32_t N, uint32_t K,
                             uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t row = row0; row < row1; ++row)
    for (uint32_t col = 0; col < N; ++col) {
      float sum = 0.0f;
      for (uint32_t e = 0; e < K; ++e) sum += A[(uint64_t)row * K + e] * B[(uint64_t)e * N + col];
      out[(uint64_t)row * N + col] = sum;
    }
}

/* attention/main.cpp:67-81 (softmax_cpu): per row, max from element 0
 * (std::max), out = expf(x - max), then out /= sum in order. */
void oracle_attention_softmax(float* out, const float* A, uint32_t M, uint32_t N, uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t row = row0; row < row1; ++row) {
    const float* a = A + (uint64_t)row * N;
    float* o = out + (uint64_t)row * N;
    float max_val = a[0];
    for (uint32_t col = 1; col < N; ++col) max_val = (max_val < a[col]) ? a[col] : max_val;
    float exp_sum = 0.0f;
    for (uint32_t col = 0; col < N; ++col) {
      o[col] = expf(a[col] - max_val);
      exp_sum += o[col];
    }
    for (uint32_t col = 0; col < N; ++col) o[col] /= exp_sum;
  }
}

/* IEEE binary16 round-to-nearest-even, as the reference's f2h (`(__fp16)x`,
 * benchmarks/kbt_sgemm/kernel.cpp:13-18) and CUDA's __float2half_rn do.
 * Written from the format definition: 1 sign, 5 exponent (bias 15),
 * 10 fraction bits; subnormals below 2^-14; overflow to infinity. */
float oracle_round_f16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  uint32_t sign = u & 0x80000000u;
  uint32_t absu = u & 0x7fffffffu;
  float r;
  if (absu >= 0x7f800000u) return x; /* inf / nan unchanged */
  float ax;
  memcpy(&ax, &absu, 4);
  if (ax >= 65520.0f) { /* rounds to inf */
    uint32_t inf = sign | 0x7f800000u;
    memcpy(&r, &inf, 4);
    return r;
  }
  if (ax < 6.103515625e-05f) { /* subnormal range: quantum 2^-24 */
    const float q = 5.9604644775390625e-08f;
    float t = ax / q;                 /* exact: power-of-two divide */
    float n = nearbyintf(t);          /* ties-to-even under the default mode */
    r = n * q;
  } else {
    /* keep 10 fraction bits: round the low 13 bits, ties to even */
    uint32_t low = absu & 0x1fffu;
    uint32_t base = absu & ~0x1fffu;
    if (low > 0x1000u || (low == 0x1000u && (base & 0x2000u))) base += 0x2000u;
    memcpy(&r, &base, 4);
  }
  uint32_t ru;
  memcpy(&ru, &r, 4);
  ru |= sign;
  memcpy(&r, &ru, 4);
  return r;
}

void oracle_round_f16_array(float* x, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i) x[i] = oracle_round_f16(x[i]);
}

/* ---- benchmarks/llama2: the matmul offload (fp32) ---- */

/* llama2/matmul_kernel.cpp:15-22, one thread per output: C[row, col] =
 * sum over k in order of A[row, k] * B[k, col]; with N = 1 this is the
 * CPU matmul of llama2/llama.cpp:236-243 (val += w[i*n + j] * x[j]). */
void oracle_llama2_matmul(float* C, const float* A, const float* B, uint32_t M, uint32_t N, uint32_t K,
                          uint32_t row0, uint32_t row1) {
  (void)M;
  for (uint32_t row = row0; row < row1; ++row)
    for (uint32_t col = 0; col < N; ++col) {
      float sum = 0.0f;
      for (uint32_t k = 0; k < K; ++k) sum += A[(uint64_t)row * K + k] * B[(uint64_t)k * N + col];
      C[(uint64_t)row * N + col] = sum;
    }
}
