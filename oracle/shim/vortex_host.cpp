/*
 * vortex_host.cpp — a host-memory stand-in for the Vortex runtime, used only
 * to build akili-bench's own harnesses (benchmarks/<bench>/main.cpp) into the
 * oracle pin and golden-capture binaries under oracle/_ref/.  TEST
 * INFRASTRUCTURE: nothing in the product links it.
 *
 * "Device" buffers are host allocations (zero-filled), their "device
 * addresses" are the host pointers, and vx_start runs, for the op named by
 * the executable's file name (or AKILI_OP), either
 *   AKILI_HOST_DEVICE=oracle (default)  the oracle of oracle/oracle.c over
 *                                       all rows, or
 *   AKILI_HOST_DEVICE=zero              nothing (outputs stay 0).
 * With AKILI_CAPTURE_DIR set, the argument block and every host->device
 * upload are written there (arg.bin, in_0.bin, in_1.bin, ... in upload
 * order) for the golden-vector script tests/golden/make_golden.py.
 * The fabs probe of probe.h is defined here.
 */
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/akili.h"
#include "../../include/vortex.h"
#include "../oracle.h"

extern "C" char* program_invocation_short_name;

namespace {

struct HostBuf {
  std::vector<unsigned char> bytes;
};

std::string g_op;
std::vector<unsigned char> g_args;
int g_uploads = 0;

std::string op_name() {
  if (const char* e = std::getenv("AKILI_OP")) return e;
  return program_invocation_short_name ? program_invocation_short_name : "";
}

void capture(const char* name, const void* p, size_t n) {
  const char* dir = std::getenv("AKILI_CAPTURE_DIR");
  if (!dir) return;
  std::string path = std::string(dir) + "/" + name;
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) return;
  std::fwrite(p, 1, n, f);
  std::fclose(f);
}

template <class T>
const T* as(const std::vector<unsigned char>& v) {
  return reinterpret_cast<const T*>(v.data());
}
inline float* fp(uint64_t a) { return reinterpret_cast<float*>(a); }

int run_oracle() {
  const std::string& op = g_op;
  if (op == "kbt_sgemm") {
    auto a = as<kbt_sgemm_arg_t>(g_args);
    oracle_kbt_sgemm(fp(a->a_addr), fp(a->b_addr), fp(a->c_addr), a->M, a->N, a->K, 0, a->M);
  } else if (op == "kbt_gemm_add_relu") {
    auto a = as<kbt_gemm_add_relu_arg_t>(g_args);
    oracle_kbt_gemm_add_relu(fp(a->a_addr), fp(a->w_addr), fp(a->bias_addr), fp(a->c_addr), a->M,
                             a->N, a->K, 0, a->M);
  } else if (op == "kbt_gemm_mul_leakyrelu") {
    auto a = as<kbt_gemm_mul_leakyrelu_arg_t>(g_args);
    oracle_kbt_gemm_mul_leakyrelu(fp(a->a_addr), fp(a->w_addr), fp(a->bias_addr), fp(a->c_addr),
                                  a->M, a->N, a->K, a->multiplier, a->negative_slope, 0, a->M);
  } else if (op == "kbt_gemm_div_sum_scale") {
    auto a = as<kbt_gemm_div_sum_scale_arg_t>(g_args);
    oracle_kbt_gemm_div_sum_scale(fp(a->a_addr), fp(a->w_addr), fp(a->c_addr), a->M, a->N, a->K,
                                  a->scaling_factor, 0, a->M);
  } else if (op == "kbt_gemm_layernorm") {
    auto a = as<kbt_gemm_layernorm_arg_t>(g_args);
    oracle_kbt_gemm_layernorm(fp(a->a_addr), fp(a->w_addr), fp(a->bias_addr), fp(a->ln_w_addr),
                              fp(a->ln_b_addr), fp(a->c_addr), a->M, a->N, a->K, a->eps, 0, a->M);
  } else if (op == "kbt_attention_score") {
    auto a = as<kbt_attention_score_arg_t>(g_args);
    oracle_kbt_attention_score(fp(a->q_addr), fp(a->k_addr), fp(a->c_addr), a->M, a->N, a->D, 0,
                               a->M);
  } else if (op == "kbt_matmul_softmax") {
    auto a = as<kbt_matmul_softmax_arg_t>(g_args);
    oracle_kbt_matmul_softmax(fp(a->a_addr), fp(a->b_addr), fp(a->c_addr), a->M, a->N, a->K, 0,
                              a->M);
  } else if (op == "kbt_matmul_scale_residadd_clamp") {
    auto a = as<kbt_matmul_scale_residadd_clamp_arg_t>(g_args);
    oracle_kbt_matmul_scale_residadd_clamp(fp(a->a_addr), fp(a->b_addr), fp(a->c_addr), a->M,
                                           a->N, a->K, a->scale_factor, a->clamp_min,
                                           a->clamp_max, 0, a->M);
  } else if (op == "kbt_matmul_sum_max_avgpool") {
    auto a = as<kbt_matmul_sum_max_avgpool_arg_t>(g_args);
    oracle_kbt_matmul_sum_max_avgpool(fp(a->a_addr), fp(a->w_addr), fp(a->bias_addr),
                                      fp(a->c_addr), a->M, a->N, a->K, 0, a->M);
  } else if (op == "kbt_gemm_rmsnorm_swiglu") {
    auto a = as<kbt_gemm_rmsnorm_swiglu_arg_t>(g_args);
    oracle_kbt_gemm_rmsnorm_swiglu(fp(a->x_addr), fp(a->rms_w_addr), fp(a->wg_addr),
                                   fp(a->wu_addr), fp(a->c_addr), a->M, a->N, a->K, a->eps, 0,
                                   a->M);
  } else if (op == "kbt_gemm_silu_mul") {
    auto a = as<kbt_gemm_silu_mul_arg_t>(g_args);
    oracle_kbt_gemm_silu_mul(fp(a->a_addr), fp(a->wa_addr), fp(a->ba_addr), fp(a->wb_addr),
                             fp(a->bb_addr), fp(a->c_addr), a->M, a->N, a->K, 0, a->M);
  } else if (op == "kb2_gemm_add_relu") {
    auto a = as<kb2_gemm_add_relu_arg_t>(g_args);
    oracle_kb2_gemm_add_relu(fp(a->a_addr), fp(a->w_addr), fp(a->bias_addr), fp(a->c_addr), a->M, a->N, a->K, 0,
                             a->M);
  } else if (op == "kb2_gemm_mul_leakyrelu") {
    auto a = as<kb2_gemm_mul_leakyrelu_arg_t>(g_args);
    oracle_kb2_gemm_mul_leakyrelu(fp(a->a_addr), fp(a->w_addr), fp(a->bias_addr), fp(a->c_addr), a->M, a->N, a->K,
                                  a->multiplier, a->negative_slope, 0, a->M);
  } else if (op == "kb2_gemm_div_sum_scale") {
    auto a = as<kb2_gemm_div_sum_scale_arg_t>(g_args);
    oracle_kb2_gemm_div_sum_scale(fp(a->a_addr), fp(a->w_addr), fp(a->c_addr), a->M, a->N, a->K,
                                  a->scaling_factor, 0, a->M);
  } else if (op == "kb2_gemm_layernorm") {
    auto a = as<kb2_gemm_layernorm_arg_t>(g_args);
    oracle_kb2_gemm_layernorm(fp(a->a_addr), fp(a->w_addr), fp(a->bias_addr), fp(a->ln_w_addr), fp(a->ln_b_addr),
                              fp(a->c_addr), a->M, a->N, a->K, a->eps, 0, a->M);
  } else if (op == "kb2_attention_score") {
    auto a = as<kb2_attention_score_arg_t>(g_args);
    oracle_kb2_attention_score(fp(a->q_addr), fp(a->k_addr), fp(a->c_addr), a->M, a->N, a->D, 0, a->M);
  } else if (op == "kb2_matmul_softmax") {
    auto a = as<kb2_matmul_softmax_arg_t>(g_args);
    oracle_kb2_matmul_softmax(fp(a->a_addr), fp(a->b_addr), fp(a->c_addr), a->M, a->N, a->K, 0, a->M);
  } else if (op == "kb2_matmul_scale_residadd_clamp") {
    auto a = as<kb2_matmul_scale_residadd_clamp_arg_t>(g_args);
    oracle_kb2_matmul_scale_residadd_clamp(fp(a->a_addr), fp(a->w_addr), fp(a->bias_addr), fp(a->c_addr), a->M,
                                           a->N, a->K, a->scale_factor, a->clamp_min, a->clamp_max, 0, a->M);
  } else if (op == "kb2_matmul_sum_max_avgpool") {
    auto a = as<kb2_matmul_sum_max_avgpool_arg_t>(g_args);
    oracle_kb2_matmul_sum_max_avgpool(fp(a->a_addr), fp(a->w_addr), fp(a->bias_addr), fp(a->c_addr), a->M, a->N,
                                      a->K, 0, a->M);
  } else if (op == "kb2_gemm_rmsnorm_swiglu") {
    auto a = as<kb2_gemm_rmsnorm_swiglu_arg_t>(g_args);
    oracle_kb2_gemm_rmsnorm_swiglu(fp(a->x_addr), fp(a->rms_w_addr), fp(a->wg_addr), fp(a->wu_addr),
                                   fp(a->c_addr), a->M, a->N, a->K, a->eps, 0, a->M);
  } else if (op == "kb2_gemm_silu_mul") {
    auto a = as<kb2_gemm_silu_mul_arg_t>(g_args);
    oracle_kb2_gemm_silu_mul(fp(a->a_addr), fp(a->wa_addr), fp(a->ba_addr), fp(a->wb_addr), fp(a->bb_addr),
                             fp(a->c_addr), a->M, a->N, a->K, 0, a->M);
  } else if (op == "attention") {
    auto a = as<attention_arg_t>(g_args);
    if (a->kernel_id == 0)
      oracle_attention_matmul(fp(a->S_addr), fp(a->Q_addr), fp(a->K_addr), a->N, a->N, a->d, 0, a->N);
    else if (a->kernel_id == 1)
      oracle_attention_softmax(fp(a->P_addr), fp(a->S_addr), a->N, a->N, 0, a->N);
    else
      oracle_attention_matmul(fp(a->O_addr), fp(a->P_addr), fp(a->V_addr), a->N, a->d, a->N, 0, a->N);
  } else if (op == "llama" || op == "llama2_matmul") {
    auto a = as<matmul_kernel_args_t>(g_args);
    oracle_llama2_matmul(fp(a->C_addr), fp(a->A_addr), fp(a->B_addr), a->M, a->N, a->K, 0, a->M);
  } else if (op == "flash") {
    auto a = as<flash_arg_t>(g_args);
    oracle_flash(fp(a->O_addr), fp(a->Q_addr), fp(a->K_addr), fp(a->V_addr), a->seq_len,
                 a->head_dim, 1.0f, 0, a->seq_len);
  } else {
    std::fprintf(stderr, "vortex_host: unknown op '%s'\n", op.c_str());
    return -1;
  }
  return 0;
}

}  // namespace

/* ---- fabs probe (see probe.h) ------------------------------------------- */
extern "C++" float akili_probe_fabsf(float x) {
  static int mode = -1;
  static FILE* rec = nullptr;
  if (mode < 0) {
    const char* m = std::getenv("AKILI_PROBE");
    mode = !m ? 0 : (std::strcmp(m, "exact") == 0 ? 1 : (std::strcmp(m, "record") == 0 ? 2 : 0));
    if (mode == 2) {
      const char* f = std::getenv("AKILI_PROBE_FILE");
      rec = f ? std::fopen(f, "wb") : nullptr;
    }
  }
  if (mode == 1) return (x == 0.0f) ? 0.0f : 1e30f;
  if (mode == 2 && rec) {
    std::fwrite(&x, 4, 1, rec);
    std::fflush(rec);
  }
  return __builtin_fabsf(x);
}

/* Integer abs of the kb2 harnesses' ulp check, std::abs(actual_bits -
 * expected_bits) (see probe.h): exact mode reports any non-zero difference as
 * far beyond every tolerance; record mode appends the argument (as int32) to
 * the same file as the fabs probe. */
extern "C++" int akili_probe_iabs(int x) {
  static int mode = -1;
  static FILE* rec = nullptr;
  if (mode < 0) {
    const char* m = std::getenv("AKILI_PROBE");
    mode = !m ? 0 : (std::strcmp(m, "exact") == 0 ? 1 : (std::strcmp(m, "record") == 0 ? 2 : 0));
    if (mode == 2) {
      const char* f = std::getenv("AKILI_PROBE_FILE");
      rec = f ? std::fopen(f, "ab") : nullptr;
    }
  }
  if (mode == 1) return x == 0 ? 0 : 0x7fffffff;
  if (mode == 2 && rec) {
    std::fwrite(&x, 4, 1, rec);
    std::fflush(rec);
  }
  return x < 0 ? -x : x;
}

/* ---- runtime API ------------------------------------------------------- */
extern "C" {

int vx_dev_open(vx_device_h* hdevice) {
  static int dev;
  *hdevice = &dev;
  return 0;
}
int vx_dev_close(vx_device_h) { return 0; }

int vx_dev_caps(vx_device_h, uint32_t caps_id, uint64_t* value) {
  /* The configuration the reference's results were recorded on
   * (README.md:349-368): 1 core, 4 warps, 8 threads, 16 KB local memory. */
  switch (caps_id) {
    case VX_CAPS_NUM_THREADS: *value = 8; return 0;
    case VX_CAPS_NUM_WARPS: *value = 4; return 0;
    case VX_CAPS_NUM_CORES: *value = 1; return 0;
    case VX_CAPS_LOCAL_MEM_SIZE: *value = 16384; return 0;
    default: *value = 0; return 0;
  }
}

int vx_mem_alloc(vx_device_h, uint64_t size, int, vx_buffer_h* hbuffer) {
  auto* b = new HostBuf;
  b->bytes.assign(size ? size : 1, 0);
  *hbuffer = b;
  return 0;
}
int vx_mem_free(vx_buffer_h hbuffer) {
  delete static_cast<HostBuf*>(hbuffer);
  return 0;
}
int vx_mem_address(vx_buffer_h hbuffer, uint64_t* address) {
  *address = reinterpret_cast<uint64_t>(static_cast<HostBuf*>(hbuffer)->bytes.data());
  return 0;
}
int vx_copy_to_dev(vx_buffer_h hbuffer, const void* host_ptr, uint64_t off, uint64_t size) {
  auto* b = static_cast<HostBuf*>(hbuffer);
  if (off + size > b->bytes.size()) return -1;
  std::memcpy(b->bytes.data() + off, host_ptr, size);
  char name[32];
  std::snprintf(name, sizeof name, "in_%d.bin", g_uploads++);
  capture(name, host_ptr, size);
  return 0;
}
int vx_copy_from_dev(void* host_ptr, vx_buffer_h hbuffer, uint64_t off, uint64_t size) {
  auto* b = static_cast<HostBuf*>(hbuffer);
  if (off + size > b->bytes.size()) return -1;
  std::memcpy(host_ptr, b->bytes.data() + off, size);
  return 0;
}
int vx_upload_kernel_file(vx_device_h, const char*, vx_buffer_h* hbuffer) {
  g_op = op_name();
  *hbuffer = new HostBuf; /* released by the harness with vx_mem_free */
  return 0;
}
int vx_upload_bytes(vx_device_h, const void* content, uint64_t size, vx_buffer_h* hbuffer) {
  g_args.assign(static_cast<const unsigned char*>(content),
                static_cast<const unsigned char*>(content) + size);
  capture("arg.bin", content, size);
  auto* b = new HostBuf; /* released by the harness with vx_mem_free */
  b->bytes = g_args;
  *hbuffer = b;
  return 0;
}
int vx_start(vx_device_h, vx_buffer_h, vx_buffer_h harguments) {
  /* the argument block is the buffer's bytes, whether it came from
   * vx_upload_bytes (the kbt harnesses) or from vx_mem_alloc +
   * vx_copy_to_dev (llama2/vxmath.cpp:127-135) */
  if (harguments) g_args = static_cast<HostBuf*>(harguments)->bytes;
  const char* m = std::getenv("AKILI_HOST_DEVICE");
  if (m && std::strcmp(m, "zero") == 0) return 0;
  int rc = run_oracle();
  if (rc == 0 && m && std::strcmp(m, "oracle_ulp") == 0) {
    /* negative control: move the first output element by one ulp */
    uint64_t out;
    if (g_op == "flash") {
      out = as<flash_arg_t>(g_args)->O_addr;
    } else if (g_op == "attention") {
      auto a = as<attention_arg_t>(g_args);
      out = a->kernel_id == 0 ? a->S_addr : (a->kernel_id == 1 ? a->P_addr : a->O_addr);
    } else if (g_op == "llama" || g_op == "llama2_matmul") {
      out = as<matmul_kernel_args_t>(g_args)->C_addr;
    } else {
      out = *reinterpret_cast<const uint64_t*>(g_args.data() + g_args.size() -
                                               8 * (g_op == "kbt_matmul_scale_residadd_clamp" ? 2 : 1));
    }
    float* c = fp(out);
    c[0] = std::nextafter(c[0], INFINITY);
  }
  return rc;
}
int vx_ready_wait(vx_device_h, uint64_t) { return 0; }
int vx_check_occupancy(vx_device_h, uint32_t, uint32_t* max_localmem) {
  *max_localmem = 16384;
  return 0;
}

int vx_dump_perf(vx_device_h, FILE*) { return 0; }

}  // extern "C"
