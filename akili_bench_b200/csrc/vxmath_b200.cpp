// vxmath_b200.cpp — the llama2 matmul offload API (benchmarks/llama2/vxmath.h)
// on a B200, for the unchanged llama2/llama.cpp.
//
// The reference (llama2/vxmath.cpp:82-221) uploads the weight matrix on every
// call and, for the batched QKV and FFN products, first concatenates the
// weight matrices on the host.  Here:
//   * a weight matrix that lives in read-only host memory (llama.cpp maps
//     the checkpoint PROT_READ, llama2/llama.cpp:166) cannot change, so it is
//     uploaded once and stays resident in HBM, keyed by its host address
//     and checked on every call against a fingerprint of its host bytes
//     (a mapping can be replaced by another at the same address);
//     any other operand is copied for each call, as the reference does;
//   * vx_matmul with N = 1 is one matrix-vector launch
//     (akili_llama2_matmul), other N the library's GEMM paths;
//   * vx_matmul_qkv_batch / vx_matmul_ffn_batch are ONE launch over the
//     resident Wq/Wk/Wv (W1/W3) with no concatenation
//     (akili_llama2_matvec_batch), then one device-to-host copy per output.
// Errors print and exit(-1), as the reference's RT_CHECK does
// (llama2/vxmath.cpp:15-23).  Single-threaded, like its caller.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <unordered_map>
#include <utility>
#include <vector>

#include "akili.h"

namespace {

struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
};

// A read-only mapping cannot change while it is mapped, but it can be unmapped
// and another mapping (another checkpoint, or writable memory) placed at the
// same address.  A resident matrix therefore keeps kSamples 32-bit words of
// its host bytes, at fixed offsets from the first to the last; every call
// compares them, and a mismatch drops the entry and decides afresh.
constexpr int kSamples = 16;
struct Resident {
  DevBuf buf;
  uint32_t sample[kSamples];
};

void fingerprint(const float* host, size_t bytes, uint32_t (&out)[kSamples]) {
  const size_t words = bytes / 4;
  const uint32_t* w = reinterpret_cast<const uint32_t*>(host);
  for (int i = 0; i < kSamples; ++i) out[i] = words ? w[(words - 1) * i / (kSamples - 1)] : 0u;
}

struct State {
  bool open = false;
  std::unordered_map<const float*, Resident> resident;  // read-only host matrices
  std::vector<std::pair<uintptr_t, uintptr_t>> ro_ranges;  // read-only mappings seen so far
  DevBuf x, y, a;  // per-call operand, result and non-resident matrix buffers
};

State g;

#define VXM_CHECK(expr)                                                        \
  do {                                                                         \
    const long _r = static_cast<long>(expr);                                   \
    if (_r != 0) {                                                             \
      std::printf("Error: '%s' returned %ld!\n", #expr, _r);                   \
      std::exit(-1);                                                           \
    }                                                                          \
  } while (false)

void grow(DevBuf& b, size_t bytes) {
  if (b.bytes >= bytes) return;
  if (b.ptr) VXM_CHECK(cudaFree(b.ptr));
  b.ptr = nullptr;
  VXM_CHECK(cudaMalloc(&b.ptr, bytes));
  b.bytes = bytes;
}

// Whether [p, p + bytes) lies in one read-only mapping of this process.
bool read_only(const void* p, size_t bytes) {
  const uintptr_t lo = reinterpret_cast<uintptr_t>(p), hi = lo + bytes;
  for (const auto& r : g.ro_ranges)
    if (lo >= r.first && hi <= r.second) return true;
  FILE* f = std::fopen("/proc/self/maps", "r");
  if (!f) return false;
  char line[512];
  bool found = false;
  while (std::fgets(line, sizeof(line), f)) {
    unsigned long a = 0, b = 0;
    char perms[8] = {0};
    if (std::sscanf(line, "%lx-%lx %7s", &a, &b, perms) != 3) continue;
    if (perms[0] == 'r' && perms[1] != 'w' && lo >= a && hi <= b) {
      g.ro_ranges.emplace_back(a, b);
      found = true;
      break;
    }
  }
  std::fclose(f);
  return found;
}

// Device copy of a host matrix: resident if the host memory is read-only,
// else copied into the per-call buffer `scratch`.
const float* matrix_on_device(const float* host, size_t bytes, DevBuf& scratch) {
  auto it = g.resident.find(host);
  if (it != g.resident.end()) {
    uint32_t now[kSamples];
    fingerprint(host, bytes, now);
    if (it->second.buf.bytes >= bytes && std::memcmp(now, it->second.sample, sizeof(now)) == 0)
      return static_cast<const float*>(it->second.buf.ptr);
    // another size or other bytes at this address: the mapping may have
    // changed, so forget the entry and the read-only ranges that cover it
    VXM_CHECK(cudaFree(it->second.buf.ptr));
    g.resident.erase(it);
    const uintptr_t lo = reinterpret_cast<uintptr_t>(host);
    std::vector<std::pair<uintptr_t, uintptr_t>> keep;
    for (const auto& r : g.ro_ranges)
      if (!(lo >= r.first && lo < r.second)) keep.push_back(r);
    g.ro_ranges.swap(keep);
  }
  if (read_only(host, bytes)) {
    Resident e;
    VXM_CHECK(cudaMalloc(&e.buf.ptr, bytes));
    e.buf.bytes = bytes;
    VXM_CHECK(cudaMemcpy(e.buf.ptr, host, bytes, cudaMemcpyHostToDevice));
    fingerprint(host, bytes, e.sample);
    g.resident.emplace(host, e);
    return static_cast<const float*>(e.buf.ptr);
  }
  grow(scratch, bytes);
  VXM_CHECK(cudaMemcpyAsync(scratch.ptr, host, bytes, cudaMemcpyHostToDevice, nullptr));
  return static_cast<const float*>(scratch.ptr);
}

uint64_t u64(const void* p) { return static_cast<uint64_t>(reinterpret_cast<uintptr_t>(p)); }

void ensure_open() {
  if (g.open) return;
  int n = 0;
  VXM_CHECK(cudaGetDeviceCount(&n) != cudaSuccess || n == 0);
  g.open = true;
}

// out_s <- W_s . input for up to three segments, one launch.
void batched(int nseg, float* const* outs, const float* const* ws, const int* rows, const float* input, int K) {
  ensure_open();
  size_t total = 0;
  for (int i = 0; i < nseg; ++i) total += static_cast<size_t>(rows[i]);
  grow(g.x, static_cast<size_t>(K) * 4 + 16);
  grow(g.y, total * 4 + 16);
  VXM_CHECK(cudaMemcpyAsync(g.x.ptr, input, static_cast<size_t>(K) * 4, cudaMemcpyHostToDevice, nullptr));
  akili_matvec_seg_t segs[4];
  std::vector<DevBuf> tmp(nseg);
  size_t off = 0;
  for (int i = 0; i < nseg; ++i) {
    segs[i].W_addr = u64(matrix_on_device(ws[i], static_cast<size_t>(rows[i]) * K * 4, tmp[i]));
    segs[i].C_addr = u64(static_cast<float*>(g.y.ptr) + off);
    segs[i].rows = rows[i];
    segs[i].reserved = 0;
    off += static_cast<size_t>(rows[i]);
  }
  VXM_CHECK(akili_llama2_matvec_batch(segs, nseg, u64(g.x.ptr), K, nullptr));
  off = 0;
  for (int i = 0; i < nseg; ++i) {
    VXM_CHECK(cudaMemcpyAsync(outs[i], static_cast<float*>(g.y.ptr) + off, static_cast<size_t>(rows[i]) * 4,
                              cudaMemcpyDeviceToHost, nullptr));
    off += static_cast<size_t>(rows[i]);
  }
  VXM_CHECK(cudaStreamSynchronize(nullptr));
  for (auto& b : tmp)
    if (b.ptr) VXM_CHECK(cudaFree(b.ptr));
}

}  // namespace

// llama2/vxmath.cpp:27-34
void vx_init() {
  std::printf("open device connection\n");
  ensure_open();
}

// llama2/vxmath.cpp:82-145: C[M x N] = A[M x K] . B[K x N]
void vx_matmul(float* C, float* A, float* B, int M, int N, int K) {
  ensure_open();
  const size_t a_bytes = static_cast<size_t>(M) * K * 4, b_bytes = static_cast<size_t>(K) * N * 4,
               c_bytes = static_cast<size_t>(M) * N * 4;
  const float* dA = matrix_on_device(A, a_bytes, g.a);
  grow(g.x, b_bytes + 16);
  grow(g.y, c_bytes + 16);
  VXM_CHECK(cudaMemcpyAsync(g.x.ptr, B, b_bytes, cudaMemcpyHostToDevice, nullptr));
  matmul_kernel_args_t arg{};
  // the reference's launch hints (llama2/vxmath.cpp:91-95); the kernels ignore them
  arg.block_dim[0] = 4;
  arg.block_dim[1] = N == 1 ? 1 : 4;
  arg.grid_dim[0] = (M + 3) / 4;
  arg.grid_dim[1] = (N + arg.block_dim[1] - 1) / arg.block_dim[1];
  arg.A_addr = u64(dA);
  arg.B_addr = u64(g.x.ptr);
  arg.C_addr = u64(g.y.ptr);
  arg.M = M;
  arg.N = N;
  arg.K = K;
  VXM_CHECK(akili_llama2_matmul(&arg, nullptr));
  VXM_CHECK(cudaMemcpyAsync(C, g.y.ptr, c_bytes, cudaMemcpyDeviceToHost, nullptr));
  VXM_CHECK(cudaStreamSynchronize(nullptr));
}

// llama2/vxmath.cpp:36-55
void matmul_cleanup() {
  if (!g.open) return;
  for (auto& kv : g.resident) cudaFree(kv.second.buf.ptr);
  g.resident.clear();
  g.ro_ranges.clear();
  for (DevBuf* b : {&g.x, &g.y, &g.a}) {
    if (b->ptr) cudaFree(b->ptr);
    *b = DevBuf{};
  }
  g.open = false;
}

// llama2/vxmath.cpp:147-183: Q = Wq.x, K = Wk.x, V = Wv.x
void vx_matmul_qkv_batch(float* Q, float* K, float* V, float* input, float* Wq, float* Wk, float* Wv, int dim,
                         int kv_dim) {
  float* outs[3] = {Q, K, V};
  const float* ws[3] = {Wq, Wk, Wv};
  const int rows[3] = {dim, kv_dim, kv_dim};
  batched(3, outs, ws, rows, input, dim);
}

// llama2/vxmath.cpp:186-221: out1 = W1.x, out2 = W3.x
void vx_matmul_ffn_batch(float* out1, float* out2, float* input, float* W1, float* W3, int input_dim,
                         int hidden_dim) {
  float* outs[2] = {out1, out2};
  const float* ws[2] = {W1, W3};
  const int rows[2] = {hidden_dim, hidden_dim};
  batched(2, outs, ws, rows, input, input_dim);
}
