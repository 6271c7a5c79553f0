// akili.cu — the C ABI of include/akili.h: argument validation, scratch,
// tensor-map construction and kernel launches for every kbt_* op and flash.
//
// Each akili_<bench>() replaces the Vortex launch of benchmarks/<bench>/
// kernel.cpp (the vx_upload_bytes + vx_start + vx_ready_wait sequence of its
// main.cpp).  The plain form keeps the reference semantics (fp32 buffers,
// operands rounded to fp16 on the device, fp32 outputs); the _ex form takes
// an akili_ex_t (fp16 I/O, flash batch/heads/scale, caller workspace).
// Validation runs before any CUDA call, so a bad argument block is rejected
// even where no GPU is present.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <mutex>
#include <thread>
#include <tuple>
#include <utility>

#include "../../include/akili.h"
#include "attention_unfused.cuh"
#include "aux.cuh"
#include "flash.cuh"
#include "gemm.cuh"
#include "matvec.cuh"
#include "softmax_rows.cuh"

using namespace akili;

namespace {

std::atomic<uint64_t> g_launches{0};

// ------------------------------------------------------------ arguments --
struct Mode {
  bool in_f32 = true;
  bool out_f32 = true;
  uint32_t batch = 1, heads = 1;
  float scale = 1.0f;
  bool causal = false;  // flash only
  void* workspace = nullptr;
  uint64_t workspace_bytes = 0;
};

int parse_ex(const akili_ex_t* ex, Mode* md) {
  *md = Mode{};
  if (!ex) return AKILI_OK;
  if (ex->abi_version != AKILI_ABI_VERSION) return AKILI_E_ABI;
  if (ex->in_dtype > AKILI_DTYPE_F16 || ex->out_dtype > AKILI_DTYPE_F16) return AKILI_E_DTYPE;
  if (ex->causal > 1 || ex->flags != 0) return AKILI_E_UNSUPPORTED;
  md->causal = ex->causal == 1;
  md->in_f32 = ex->in_dtype == AKILI_DTYPE_F32;
  md->out_f32 = ex->out_dtype == AKILI_DTYPE_F32;
  md->batch = ex->batch ? ex->batch : 1;
  md->heads = ex->heads ? ex->heads : 1;
  if (ex->softmax_scale < 0.0f || ex->softmax_scale != ex->softmax_scale) return AKILI_E_UNSUPPORTED;
  md->scale = ex->softmax_scale != 0.0f ? ex->softmax_scale : 1.0f;
  md->workspace = reinterpret_cast<void*>(ex->workspace);
  md->workspace_bytes = ex->workspace ? ex->workspace_bytes : 0;
  return AKILI_OK;
}

int check_dims(uint32_t N, uint32_t K) {
  if (N == 0 || K == 0 || (N % 8) || (K % 8)) return AKILI_E_SHAPE;
  return AKILI_OK;
}
int check_m(uint32_t M) { return (M % 8) ? AKILI_E_SHAPE : AKILI_OK; }

int check_ptrs(std::initializer_list<uint64_t> ps) {
  for (uint64_t p : ps)
    if (p == 0) return AKILI_E_NULL_ARG;
  for (uint64_t p : ps)
    if (p % 16) return AKILI_E_ALIGN;
  return AKILI_OK;
}
int check_opt_ptr(uint64_t p) { return (p % 16) ? AKILI_E_ALIGN : AKILI_OK; }

// --------------------------------------------------------------- device --
struct DevInfo {
  int sms = 0;
  bool sm100 = false;
};

int device_info(DevInfo* out) {
  static std::mutex mu;
  static std::map<int, DevInfo> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return AKILI_E_NO_DEVICE;
  }
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(dev);
  if (it == cache.end()) {
    DevInfo d;
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      return AKILI_E_NO_DEVICE;
    }
    d.sm100 = (major == 10 && minor == 0);
    it = cache.emplace(dev, d).first;
  }
  *out = it->second;
  return out->sm100 ? AKILI_OK : AKILI_E_NO_DEVICE;
}

// ----------------------------------------------------------- tensor maps --
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    cudaGetLastError();
  });
  return fn;
}

// Row-major [outer x inner] tensor, tile [box_outer x box_inner].
bool map2d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
           uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [d2][d1][d0] tensor with contiguous d0.
bool map3d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, uint64_t d0, uint64_t d1, uint64_t d2,
           uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw, uint32_t elem_bytes) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * elem_bytes, d0 * d1 * elem_bytes};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, dt, 3, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ------------------------------------------------------------- contexts --
// Identity of the calling thread's current CUDA context: the current
// device's primary context under the runtime API.  A device reset destroys
// that context and every device address it handed out; the next runtime call
// creates a new one with a new identity.  Caches of device addresses are keyed
// by it, so none outlives its context.  Without the driver entry points (a
// driver older than CUDA 12.0) the device ordinal stands in.
int current_context_id(unsigned long long* id) {
  using GetCurrentFn = CUresult (*)(CUcontext*);
  using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetIdFn>(p);
    cudaGetLastError();
  });
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return AKILI_E_NO_DEVICE;
  }
  constexpr unsigned long long kOrdinalTag = 1ull << 63;  // context ids count up from 1
  if (!get_current || !get_id) {
    *id = kOrdinalTag | static_cast<unsigned long long>(dev);
    return AKILI_OK;
  }
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
    // no context current on this thread yet: cudaSetDevice makes the
    // device's primary context current, creating it if need be
    if (cudaSetDevice(dev) != cudaSuccess || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
      cudaGetLastError();
      return AKILI_E_NO_DEVICE;
    }
  }
  if (get_id(ctx, id) != CUDA_SUCCESS) return AKILI_E_NO_DEVICE;
  return AKILI_OK;
}

// --------------------------------------------------------------- scratch --
// Internal scratch, one grow-only buffer per (context, stream): calls on one
// stream are ordered, so they can share it.  Used when the caller gives no
// akili_ex_t workspace.  Growing it frees the old buffer (a device sync).
// cudaStreamPerThread names a different stream in every host thread, so for
// it the calling thread is part of the key.
struct Pool {
  void* ptr = nullptr;
  size_t bytes = 0;
};

int pool_get(cudaStream_t st, size_t bytes, void** out) {
  static std::mutex mu;
  static std::map<std::tuple<unsigned long long, cudaStream_t, std::thread::id>, Pool> pools;
  unsigned long long ctx = 0;
  int rc = current_context_id(&ctx);
  if (rc) return rc;
  const std::thread::id owner = st == cudaStreamPerThread ? std::this_thread::get_id() : std::thread::id();
  std::lock_guard<std::mutex> g(mu);
  Pool& p = pools[{ctx, st, owner}];
  if (p.bytes < bytes) {
    if (p.ptr) cudaFree(p.ptr);
    p.ptr = nullptr;
    p.bytes = 0;
    size_t want = bytes + bytes / 4 + (1u << 20);
    if (cudaMalloc(&p.ptr, want) != cudaSuccess) {
      cudaGetLastError();
      return AKILI_E_ALLOC;
    }
    p.bytes = want;
  }
  *out = p.ptr;
  return AKILI_OK;
}

struct Carve {
  char* base = nullptr;
  size_t off = 0;
  size_t need(size_t n) {  // sizing pass when base == nullptr
    size_t o = off;
    off += (n + 255) & ~size_t(255);
    return o;
  }
  void* take(size_t n) { return base + need(n); }
};

int acquire_scratch(const Mode& md, size_t bytes, cudaStream_t st, char** out) {
  *out = nullptr;
  if (bytes == 0) return AKILI_OK;
  if (md.workspace) {
    if (md.workspace_bytes < bytes) return AKILI_E_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(md.workspace) % 256) return AKILI_E_ALIGN;
    *out = static_cast<char*>(md.workspace);
    return AKILI_OK;
  }
  void* p = nullptr;
  int rc = pool_get(st, bytes, &p);
  *out = static_cast<char*>(p);
  return rc;
}

int launch_status() {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AKILI_OK : AKILI_E_LAUNCH;
}

int grid_for(const DevInfo& di, size_t work_items, int per_block, int waves = 4) {
  size_t blocks = (work_items + per_block - 1) / per_block;
  size_t cap = static_cast<size_t>(di.sms) * waves;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : static_cast<int>(blocks);
}

int cast_to_f16(const DevInfo& di, const float* src, __half* dst, size_t n, cudaStream_t st) {
  cast_f32_to_f16_kernel<<<grid_for(di, n / 8 + 1, 256, 8), 256, 0, st>>>(src, dst, n);
  return launch_status();
}

// x = hi + lo with hi = fp16(x), lo = fp16(x - hi) (the split operands).
int split_to_f16x2(const DevInfo& di, const float* src, __half* hi, __half* lo, size_t n, cudaStream_t st) {
  split_f32_to_f16x2_kernel<<<grid_for(di, n, 256, 8), 256, 0, st>>>(src, hi, lo, n);
  return launch_status();
}

// ------------------------------------------------------------ GEMM jobs --
struct GemmJob {
  Epi epi = Epi::kPlain;
  bool b_kmajor = false;
  bool split = false;  // fp32 operands as fp16 hi + lo parts (the kb2_* family)
  uint32_t M = 0, N = 0, K = 0;
  const void* A = nullptr;   // [M x K] (in dtype)
  const void* B0 = nullptr;  // [K x N] or, when b_kmajor, [N x K]
  const void* B1 = nullptr;  // second weight of the dual GEMMs
  const float* vec0 = nullptr;
  const float* vec1 = nullptr;
  float s0 = 0, s1 = 0, s2 = 0;
  void* C = nullptr;                 // [M x N] or [M]
  void* stats_hint = nullptr;        // caller scratch usable for partial stats
  size_t stats_hint_bytes = 0;
  // RMSNorm pre-pass (A = x_hat computed from X)
  bool rmsnorm = false;
  const float* rms_w = nullptr;
  void* xhat_hint = nullptr;         // caller scratch for x_hat (norm_addr)
  // finalisers
  float final_scale = 1.0f;
  float eps = 0.0f;
  const float* ln_w = nullptr;
  const float* ln_b = nullptr;
};

// Row softmax of a short-K product runs fused end to end (softmax_rows_kernel):
// no partial statistics, no finaliser.
bool softmax_fused(const GemmJob& j) {
  return j.epi == Epi::kSoftmaxPre && !j.split && j.K <= static_cast<uint32_t>(kSmMaxK);
}

// Partial statistics: two slots (half tiles of BN/2 columns) per BN-column tile.
size_t stats_bytes(const GemmJob& j) {
  if (softmax_fused(j)) return 0;
  const int bn = epi_bn(j.epi);
  const size_t nt = 2 * ((j.N + bn - 1) / bn);
  return static_cast<size_t>(epi_stats(j.epi)) * nt * j.M * sizeof(float);
}

// Sizing and carving share one routine so they cannot disagree.
struct JobBuffers {
  const __half* A = nullptr;
  const __half* B0 = nullptr;
  const __half* B1 = nullptr;
  __half* castA = nullptr;
  __half* castB0 = nullptr;
  __half* castB1 = nullptr;
  // split mode: the lo parts
  __half* Alo = nullptr;
  __half* B0lo = nullptr;
  __half* B1lo = nullptr;
  float* stats = nullptr;
  unsigned int* row_sync = nullptr;  // row-fused LayerNorm / softmax: one counter per 128-row block
};

// Row-fused LayerNorm / softmax candidates: the CTA-pair kernel (M > 128)
// with a row-normalising epilogue.  Whether a launch fuses is decided at
// launch (launch_gemm_pair); the counters are laid out either way.
bool rownorm_candidate(const GemmJob& j) {
  return epi_rownorm(j.epi) && !softmax_fused(j) && j.M > static_cast<uint32_t>(kBM);
}
size_t row_sync_count(const GemmJob& j) { return 2 * ((static_cast<size_t>(j.M) + 2 * kBM - 1) / (2 * kBM)); }

size_t layout_job(const GemmJob& j, const Mode& md, Carve& cv, JobBuffers* jb) {
  const bool dual = epi_dual(j.epi);
  const size_t nA = static_cast<size_t>(j.M) * j.K;
  const size_t nB = static_cast<size_t>(j.K) * j.N;
  auto grab = [&](size_t bytes) -> void* { return cv.base ? cv.take(bytes) : (cv.need(bytes), nullptr); };
  if (j.rmsnorm) {
    if (j.xhat_hint) jb->castA = static_cast<__half*>(j.xhat_hint);
    else jb->castA = static_cast<__half*>(grab(nA * 2));
    jb->A = jb->castA;
    if (j.split) jb->Alo = static_cast<__half*>(grab(nA * 2));
  } else if (md.in_f32) {
    jb->castA = static_cast<__half*>(grab(nA * 2));
    jb->A = jb->castA;
    if (j.split) jb->Alo = static_cast<__half*>(grab(nA * 2));
  } else {
    jb->A = static_cast<const __half*>(j.A);
  }
  if (md.in_f32) {
    jb->castB0 = static_cast<__half*>(grab(nB * 2));
    jb->B0 = jb->castB0;
    if (j.split) jb->B0lo = static_cast<__half*>(grab(nB * 2));
    if (dual) {
      jb->castB1 = static_cast<__half*>(grab(nB * 2));
      jb->B1 = jb->castB1;
      if (j.split) jb->B1lo = static_cast<__half*>(grab(nB * 2));
    }
  } else {
    jb->B0 = static_cast<const __half*>(j.B0);
    jb->B1 = static_cast<const __half*>(j.B1);
  }
  const size_t sb = stats_bytes(j);
  if (sb) {
    if (j.stats_hint && j.stats_hint_bytes >= sb) jb->stats = static_cast<float*>(j.stats_hint);
    else jb->stats = static_cast<float*>(grab(sb));
  }
  if (rownorm_candidate(j)) jb->row_sync = static_cast<unsigned int*>(grab(row_sync_count(j) * sizeof(unsigned int)));
  return cv.off;
}

// Row-fused LayerNorm / softmax switch: AKILI_ROWNORM=0 in the environment
// selects the two-pass form (statistics, then a finaliser kernel).
// AKILI_COOP=0 launches the row-fused kernel without the cooperative
// attribute, for profilers that cannot replay cooperative cluster launches.
bool rownorm_enabled() {
  const char* e = std::getenv("AKILI_ROWNORM");
  return !(e && e[0] == '0');
}
// Tile order of the CTA-pair kernel: row-block-major when the B operand
// (K x N fp16, both weights for the dual GEMMs) fits well inside L2, so each
// A row block is read from HBM once while B stays resident (C2: 115 against
// 167 MB of DRAM reads per launch, same time); groups of row blocks otherwise
// (C4's 172 MB of weights: row-major re-reads them and ran 26% slower).
// AKILI_RASTER=row / group in the environment forces one.
constexpr uint64_t kRowMajorMaxB = 48ull << 20;
bool raster_row_major(uint64_t b_bytes) {
  const char* e = std::getenv("AKILI_RASTER");
  if (e && e[0] == 'r') return true;
  if (e && e[0] == 'g') return false;
  return b_bytes <= kRowMajorMaxB;
}

bool coop_enabled() {
  const char* e = std::getenv("AKILI_COOP");
  return !(e && e[0] == '0');
}

// Persistent launch of the CTA-pair kernel: clusters of 2, as many pairs as
// can be resident at once (cudaOccupancyMaxActiveClusters), at most one per tile.
// With ea.row_sync set (a row-normalising epilogue) the launch is row-fused
// when every column tile of a row block fits in one wave (num_n <= pairs):
// the counters are zeroed on the stream and the kernel goes out as a
// cooperative launch, so all its pairs are resident together.  Otherwise, or
// if the cooperative launch is refused, it runs in the two-pass form and
// *fused is false (the caller runs the finaliser).
template <Epi E, typename OutT, bool BK, bool kSplit = false>
int launch_gemm_pair(const DevInfo& di, const CUtensorMap& tmA, const CUtensorMap& tmB0, const CUtensorMap& tmB1,
                     const CUtensorMap& tmC, const CUtensorMap& tmAlo, const CUtensorMap& tmB0lo,
                     const CUtensorMap& tmB1lo, EpiArgs ea, cudaStream_t st, bool* fused) {
  constexpr int BN = epi_bn(E);
  const int smem = gemm_pair_smem_bytes(epi_stores(E), sizeof(OutT), kSplit);
  auto kern = gemm_pair_kernel<E, OutT, BK, kSplit>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kPairThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static std::mutex mu;
  static std::map<int, int> max_pairs;
  int dev = 0;
  cudaGetDevice(&dev);
  int pairs_cap = 0;
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = max_pairs.find(dev);
    if (it == max_pairs.end()) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return AKILI_E_LAUNCH;
      }
      cfg.gridDim = dim3(di.sms & ~1);
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters < 1) {
        cudaGetLastError();
        clusters = di.sms / 2;
      }
      it = max_pairs.emplace(dev, clusters).first;
    }
    pairs_cap = it->second;
  }
  const int num_n = (ea.N + BN - 1) / BN;
  const int tiles = ((ea.M + 2 * kBM - 1) / (2 * kBM)) * num_n;
  const int pairs = tiles < pairs_cap ? tiles : pairs_cap;
  cfg.gridDim = dim3(2 * pairs);
  if (fused) *fused = false;
  if constexpr (epi_rownorm(E)) {
    if (ea.row_sync && fused && num_n <= pairs && rownorm_enabled()) {
      const size_t nsync = 2 * static_cast<size_t>((ea.M + 2 * kBM - 1) / (2 * kBM));
      if (cudaMemsetAsync(ea.row_sync, 0, nsync * sizeof(unsigned int), st) != cudaSuccess) {
        cudaGetLastError();
        return AKILI_E_LAUNCH;
      }
      attr[1].id = cudaLaunchAttributeCooperative;
      attr[1].val.cooperative = 1;
      cfg.numAttrs = coop_enabled() ? 2 : 1;
      if (cudaLaunchKernelEx(&cfg, kern, tmA, tmB0, tmB1, tmC, tmAlo, tmB0lo, tmB1lo, ea) == cudaSuccess) {
        *fused = true;
        return launch_status();
      }
      cudaGetLastError();  // refused: fall back to the two-pass form below
      cfg.numAttrs = 1;
    }
  }
  ea.row_sync = nullptr;
  if (cudaLaunchKernelEx(&cfg, kern, tmA, tmB0, tmB1, tmC, tmAlo, tmB0lo, tmB1lo, ea) != cudaSuccess) {
    cudaGetLastError();
    return AKILI_E_LAUNCH;
  }
  return launch_status();
}

template <Epi E, typename OutT, bool BK, bool kSplit = false>
int launch_gemm(const DevInfo& di, const GemmJob& j, const JobBuffers& jb, cudaStream_t st, bool* fused) {
  constexpr bool kStore = epi_stores(E);
  constexpr int BN = epi_bn(E);
  CUtensorMap tmA, tmB0, tmB1, tmC;
  const uint64_t M = j.M, N = j.N, K = j.K;
  bool ok = map2d(&tmA, jb.A, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, K, M, K * 2, 64, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  // CTA pairs (two SMs per 256-row tile) whenever M fills more than one 128-row
  // block, in the split (fp32) mode too.
  const bool pair = M > static_cast<uint64_t>(kBM);
  if (BK) {
    ok = ok && map2d(&tmB0, jb.B0, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, K, N, K * 2, 64, pair ? BN / 2 : BN,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    ok = ok && map2d(&tmB0, jb.B0, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, K, N * 2, 64, 64,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (epi_dual(E)) {
    ok = ok && map2d(&tmB1, jb.B1, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, K, N * 2, 64, 64,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    tmB1 = tmB0;
  }
  if (kStore) {
    if (sizeof(OutT) == 2)
      ok = ok && map2d(&tmC, j.C, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, M, N * 2, 32, kBM, CU_TENSOR_MAP_SWIZZLE_64B);
    else
      ok = ok && map2d(&tmC, j.C, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, N, M, N * 4, 32, kBM,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    tmC = tmA;
  }
  if (!ok) return AKILI_E_LAUNCH;

  EpiArgs ea;
  ea.vec0 = j.vec0;
  ea.vec1 = j.vec1;
  ea.s0 = j.s0;
  ea.s1 = j.s1;
  ea.s2 = j.s2;
  ea.s3 = 0.0f;
  ea.row_ws = jb.stats;
  ea.M = static_cast<int>(M);
  ea.N = static_cast<int>(N);
  ea.K = static_cast<int>(K);
  ea.num_n_tiles = static_cast<int>(2 * ((N + BN - 1) / BN));  // statistics slots: two per tile
  ea.row_sync = jb.row_sync;
  ea.ln_w = j.ln_w;
  ea.ln_b = j.ln_b;
  ea.eps = j.eps;
  ea.row_major = raster_row_major(K * N * 2 * (epi_dual(E) ? 2 : 1) * (kSplit ? 2 : 1)) ? 1 : 0;

  // the lo parts of the split mode: the same boxes over the lo copies
  CUtensorMap tmAlo = tmA, tmB0lo = tmB0, tmB1lo = tmB1;
  if constexpr (kSplit) {
    constexpr auto kF16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    constexpr auto kSw = CU_TENSOR_MAP_SWIZZLE_128B;
    ok = map2d(&tmAlo, jb.Alo, kF16, K, M, K * 2, 64, kBM, kSw);
    if (BK) ok = ok && map2d(&tmB0lo, jb.B0lo, kF16, K, N, K * 2, 64, pair ? BN / 2 : BN, kSw);
    else ok = ok && map2d(&tmB0lo, jb.B0lo, kF16, N, K, N * 2, 64, 64, kSw);
    if (epi_dual(E)) ok = ok && map2d(&tmB1lo, jb.B1lo, kF16, N, K, N * 2, 64, 64, kSw);
    if (!ok) return AKILI_E_LAUNCH;
  }
  if (pair)
    return launch_gemm_pair<E, OutT, BK, kSplit>(di, tmA, tmB0, tmB1, tmC, tmAlo, tmB0lo, tmB1lo, ea, st, fused);
  if (fused) *fused = false;
  const int smem = gemm_smem_bytes(kStore, sizeof(OutT), kSplit);
  static std::mutex mu;
  static std::map<int, bool> attr_done;
  {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (!attr_done[dev]) {
      if (cudaFuncSetAttribute(gemm_kernel<E, OutT, BK, kSplit>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
          cudaSuccess) {
        cudaGetLastError();
        return AKILI_E_LAUNCH;
      }
      attr_done[dev] = true;
    }
  }
  const int tiles = static_cast<int>(((M + kBM - 1) / kBM) * ((N + BN - 1) / BN));
  const int grid = tiles < di.sms ? tiles : di.sms;
  gemm_kernel<E, OutT, BK, kSplit><<<grid, kGemmThreads, smem, st>>>(tmA, tmB0, tmB1, tmC, tmAlo, tmB0lo, tmB1lo,
                                                                     ea);
  return launch_status();
}

constexpr int kSmemOptin = 232448;  // 227 KB of dynamic shared memory per CTA (sm_100)

template <typename OutT, bool BK>
int launch_softmax_rows(const DevInfo& di, const GemmJob& j, const JobBuffers& jb, cudaStream_t st) {
  CUtensorMap tmA, tmB, tmC;
  const uint64_t M = j.M, N = j.N, K = j.K;
  bool ok = map2d(&tmA, jb.A, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, K, M, K * 2, 64, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (BK)
    ok = ok && map2d(&tmB, jb.B0, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, K, N, K * 2, 64, 256, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    ok = ok && map2d(&tmB, jb.B0, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, K, N * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  // store boxes: 32 rows x 128 bytes (64 fp16 or 32 fp32 columns), one per warp
  if (sizeof(OutT) == 2)
    ok = ok && map2d(&tmC, j.C, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, M, N * 2, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    ok = ok && map2d(&tmC, j.C, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, N, M, N * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok) return AKILI_E_LAUNCH;
  SoftmaxRowsArgs p;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.c = j.s0 * 1.4426950408889634f;
  p.L = softmax_rows_layout(p.K, sizeof(OutT), kSmemOptin);
  if (p.L.stages < 2) return AKILI_E_UNSUPPORTED;
  auto kern = softmax_rows_kernel<OutT, BK>;
  static std::mutex mu;
  static std::map<int, bool> attr_done;
  {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (!attr_done[dev]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemOptin) != cudaSuccess) {
        cudaGetLastError();
        return AKILI_E_LAUNCH;
      }
      attr_done[dev] = true;
    }
  }
  const int blocks = static_cast<int>((M + kBM - 1) / kBM);
  const int grid = blocks < di.sms ? blocks : di.sms;
  kern<<<grid, kSmThreads, p.L.total, st>>>(tmA, tmB, tmC, p);
  return launch_status();
}

template <Epi E, bool BK = false>
int launch_gemm_out(const DevInfo& di, const GemmJob& j, const JobBuffers& jb, bool out_f32, cudaStream_t st,
                    bool* fused = nullptr) {
  if (j.split) return launch_gemm<E, float, BK, true>(di, j, jb, st, fused);  // the kb2_* family: fp32 out
  if constexpr (!epi_stores(E)) {
    return launch_gemm<E, float, BK>(di, j, jb, st, fused);
  } else {
    return out_f32 ? launch_gemm<E, float, BK>(di, j, jb, st, fused)
                   : launch_gemm<E, __half, BK>(di, j, jb, st, fused);
  }
}

int run_job(const GemmJob& j, const Mode& md, cudaStream_t st) {
  if (j.M == 0) return AKILI_OK;
  DevInfo di;
  int rc = device_info(&di);
  if (rc) return rc;

  JobBuffers jb;
  Carve sizing;
  const size_t bytes = layout_job(j, md, sizing, &jb);
  char* base = nullptr;
  rc = acquire_scratch(md, bytes, st, &base);
  if (rc) return rc;
  Carve cv;
  cv.base = base;
  jb = JobBuffers{};
  layout_job(j, md, cv, &jb);

  const size_t nA = static_cast<size_t>(j.M) * j.K;
  const size_t nB = static_cast<size_t>(j.K) * j.N;
  // 1. operand preparation
  if (j.rmsnorm) {
    const int rows_per_block = 8;
    const int grid = grid_for(di, j.M, rows_per_block, 8);
    if (md.in_f32)
      rmsnorm_prepass_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(j.A), j.rms_w, jb.castA,
                                                          jb.Alo, static_cast<int>(j.M), static_cast<int>(j.K),
                                                          j.eps);
    else
      rmsnorm_prepass_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(j.A), j.rms_w, jb.castA,
                                                           nullptr, static_cast<int>(j.M), static_cast<int>(j.K),
                                                           j.eps);
    if ((rc = launch_status())) return rc;
  } else if (md.in_f32) {
    if (j.split) rc = split_to_f16x2(di, static_cast<const float*>(j.A), jb.castA, jb.Alo, nA, st);
    else rc = cast_to_f16(di, static_cast<const float*>(j.A), jb.castA, nA, st);
    if (rc) return rc;
  }
  if (md.in_f32) {
    if (j.split) rc = split_to_f16x2(di, static_cast<const float*>(j.B0), jb.castB0, jb.B0lo, nB, st);
    else rc = cast_to_f16(di, static_cast<const float*>(j.B0), jb.castB0, nB, st);
    if (rc) return rc;
    if (epi_dual(j.epi)) {
      if (j.split) rc = split_to_f16x2(di, static_cast<const float*>(j.B1), jb.castB1, jb.B1lo, nB, st);
      else rc = cast_to_f16(di, static_cast<const float*>(j.B1), jb.castB1, nB, st);
      if (rc) return rc;
    }
  }
  // 2. the fused GEMM
  if (softmax_fused(j)) {
    if (md.out_f32)
      return j.b_kmajor ? launch_softmax_rows<float, true>(di, j, jb, st)
                        : launch_softmax_rows<float, false>(di, j, jb, st);
    return j.b_kmajor ? launch_softmax_rows<__half, true>(di, j, jb, st)
                      : launch_softmax_rows<__half, false>(di, j, jb, st);
  }
  bool rowfused = false;  // the row-normalising epilogue finished the rows in the GEMM kernel
  switch (j.epi) {
    case Epi::kPlain: rc = launch_gemm_out<Epi::kPlain>(di, j, jb, md.out_f32, st); break;
    case Epi::kBiasRelu: rc = launch_gemm_out<Epi::kBiasRelu>(di, j, jb, md.out_f32, st); break;
    case Epi::kBiasMulLeaky: rc = launch_gemm_out<Epi::kBiasMulLeaky>(di, j, jb, md.out_f32, st); break;
    case Epi::kRowSumHalf: rc = launch_gemm_out<Epi::kRowSumHalf>(di, j, jb, md.out_f32, st); break;
    case Epi::kRowSumBias: rc = launch_gemm_out<Epi::kRowSumBias>(di, j, jb, md.out_f32, st); break;
    case Epi::kLnPre: rc = launch_gemm_out<Epi::kLnPre>(di, j, jb, md.out_f32, st, &rowfused); break;
    case Epi::kSoftmaxPre:
      rc = j.b_kmajor ? launch_gemm_out<Epi::kSoftmaxPre, true>(di, j, jb, md.out_f32, st, &rowfused)
                      : launch_gemm_out<Epi::kSoftmaxPre, false>(di, j, jb, md.out_f32, st, &rowfused);
      break;
    case Epi::kLseClamp: rc = launch_gemm_out<Epi::kLseClamp>(di, j, jb, md.out_f32, st); break;
    case Epi::kSiluMulBias: rc = launch_gemm_out<Epi::kSiluMulBias>(di, j, jb, md.out_f32, st); break;
    case Epi::kSwiglu: rc = launch_gemm_out<Epi::kSwiglu>(di, j, jb, md.out_f32, st); break;
  }
  if (rc) return rc;
  if (rowfused) return AKILI_OK;
  // 3. finalisers
  const int M = static_cast<int>(j.M), N = static_cast<int>(j.N);
  const int nt = 2 * ((N + epi_bn(j.epi) - 1) / epi_bn(j.epi));  // statistics slots (half tiles)
  const dim3 fin_grid((M + kFinRows - 1) / kFinRows, (N + kFinCols - 1) / kFinCols);  // LayerNorm finaliser
  switch (j.epi) {
    case Epi::kRowSumHalf:
    case Epi::kRowSumBias:
      if (md.out_f32)
        finalize_rowsum_kernel<float><<<grid_for(di, M, 256), 256, 0, st>>>(jb.stats, static_cast<float*>(j.C),
                                                                            M, nt, j.final_scale);
      else
        finalize_rowsum_kernel<__half><<<grid_for(di, M, 256), 256, 0, st>>>(jb.stats, static_cast<__half*>(j.C),
                                                                             M, nt, j.final_scale);
      return launch_status();
    case Epi::kLseClamp:
      if (md.out_f32)
        finalize_lse_mish_kernel<float><<<grid_for(di, M, 256), 256, 0, st>>>(jb.stats, static_cast<float*>(j.C),
                                                                              M, nt);
      else
        finalize_lse_mish_kernel<__half><<<grid_for(di, M, 256), 256, 0, st>>>(
            jb.stats, static_cast<__half*>(j.C), M, nt);
      return launch_status();
    case Epi::kLnPre:
      if (md.out_f32)
        layernorm_finalize_kernel<float><<<fin_grid, kFinThreads, 0, st>>>(
            static_cast<float*>(j.C), jb.stats, j.ln_w, j.ln_b, M, N, nt, epi_bn(j.epi) / 2, j.eps);
      else
        layernorm_finalize_kernel<__half><<<fin_grid, kFinThreads, 0, st>>>(
            static_cast<__half*>(j.C), jb.stats, j.ln_w, j.ln_b, M, N, nt, epi_bn(j.epi) / 2, j.eps);
      return launch_status();
    case Epi::kSoftmaxPre:
      if (md.out_f32)
        softmax_finalize_kernel<float><<<grid_for(di, M, 8, 8), 256, 0, st>>>(static_cast<float*>(j.C), jb.stats,
                                                                              M, N, nt);
      else
        softmax_finalize_kernel<__half><<<grid_for(di, M, 8, 8), 256, 0, st>>>(static_cast<__half*>(j.C),
                                                                               jb.stats, M, N, nt);
      return launch_status();
    default:
      return AKILI_OK;
  }
}

size_t job_scratch_bytes(const GemmJob& j, const Mode& md) {
  if (j.M == 0) return 0;
  Carve c;
  JobBuffers jb;
  return layout_job(j, md, c, &jb);
}

template <class T>
const void* P(T v) {
  return reinterpret_cast<const void*>(static_cast<uintptr_t>(v));
}
template <class T>
void* W(T v) {
  return reinterpret_cast<void*>(static_cast<uintptr_t>(v));
}
const float* F(uint64_t v) { return reinterpret_cast<const float*>(static_cast<uintptr_t>(v)); }

// ---------------------------------------------------------- job builders --
// Each returns 0 and fills `j`, or an AKILI_E_* code.  No CUDA calls.

int job_sgemm(const kbt_sgemm_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->b_addr, a->c_addr}))) return rc;
  j.epi = Epi::kPlain;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->b_addr); j.C = W(a->c_addr);
  return AKILI_OK;
}

int job_add_relu(const kbt_gemm_add_relu_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->w_addr, a->bias_addr, a->c_addr}))) return rc;
  j.epi = Epi::kBiasRelu;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->w_addr); j.vec0 = F(a->bias_addr); j.C = W(a->c_addr);
  return AKILI_OK;
}

int job_mul_leakyrelu(const kbt_gemm_mul_leakyrelu_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->w_addr, a->bias_addr, a->c_addr}))) return rc;
  j.epi = Epi::kBiasMulLeaky;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->w_addr); j.vec0 = F(a->bias_addr); j.C = W(a->c_addr);
  j.s0 = a->multiplier; j.s1 = a->negative_slope;
  return AKILI_OK;
}

int job_div_sum_scale(const kbt_gemm_div_sum_scale_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->w_addr, a->c_addr}))) return rc;
  j.epi = Epi::kRowSumHalf;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->w_addr); j.C = W(a->c_addr);
  j.final_scale = a->scaling_factor;
  return AKILI_OK;
}

int job_layernorm(const kbt_gemm_layernorm_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->w_addr, a->bias_addr, a->ln_w_addr, a->ln_b_addr, a->c_addr}))) return rc;
  j.epi = Epi::kLnPre;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->w_addr); j.vec0 = F(a->bias_addr); j.C = W(a->c_addr);
  j.ln_w = F(a->ln_w_addr); j.ln_b = F(a->ln_b_addr); j.eps = a->eps;
  return AKILI_OK;
}

int job_attention_score(const kbt_attention_score_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->D))) return rc;
  if (chk && (rc = check_ptrs({a->q_addr, a->k_addr, a->c_addr}))) return rc;
  j.epi = Epi::kSoftmaxPre;
  j.b_kmajor = true;
  j.M = a->M; j.N = a->N; j.K = a->D;
  j.A = P(a->q_addr); j.B0 = P(a->k_addr); j.C = W(a->c_addr);
  j.s0 = 1.0f / sqrtf(static_cast<float>(a->D));  // kbt_attention_score/main.cpp:117
  return AKILI_OK;
}

int job_matmul_softmax(const kbt_matmul_softmax_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->b_addr, a->c_addr}))) return rc;
  j.epi = Epi::kSoftmaxPre;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->b_addr); j.C = W(a->c_addr);
  j.s0 = 1.0f;
  return AKILI_OK;
}

int job_clamp(const kbt_matmul_scale_residadd_clamp_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && ((rc = check_ptrs({a->a_addr, a->b_addr, a->c_addr})) || (rc = check_opt_ptr(a->temp_addr)))) return rc;
  j.epi = Epi::kLseClamp;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->b_addr); j.C = W(a->c_addr);
  j.s0 = a->scale_factor; j.s1 = a->clamp_min; j.s2 = a->clamp_max;
  // temp_addr is the reference's [M x N] fp32 scratch; it holds the partials.
  j.stats_hint = W(a->temp_addr);
  j.stats_hint_bytes = a->temp_addr ? static_cast<size_t>(a->M) * a->N * sizeof(float) : 0;
  return AKILI_OK;
}

int job_sum_max_avgpool(const kbt_matmul_sum_max_avgpool_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->w_addr, a->bias_addr, a->c_addr}))) return rc;
  j.epi = Epi::kRowSumBias;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->w_addr); j.vec0 = F(a->bias_addr); j.C = W(a->c_addr);
  j.final_scale = 1.0f;
  return AKILI_OK;
}

int job_rmsnorm_swiglu(const kbt_gemm_rmsnorm_swiglu_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->x_addr, a->rms_w_addr, a->wg_addr, a->wu_addr, a->c_addr})) ||
      (chk && ((rc = check_opt_ptr(a->norm_addr)) || (rc = check_opt_ptr(a->gate_addr)))))
    return rc;
  j.epi = Epi::kSwiglu;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->x_addr); j.B0 = P(a->wg_addr); j.B1 = P(a->wu_addr); j.C = W(a->c_addr);
  j.rmsnorm = true; j.rms_w = F(a->rms_w_addr); j.eps = a->eps;
  j.xhat_hint = W(a->norm_addr);  // the reference's [M x K] normalised-x scratch
  return AKILI_OK;
}

int job_silu_mul(const kbt_gemm_silu_mul_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->wa_addr, a->ba_addr, a->wb_addr, a->bb_addr, a->c_addr})) ||
      (chk && (rc = check_opt_ptr(a->gate_addr))))
    return rc;
  j.epi = Epi::kSiluMulBias;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->wa_addr); j.B1 = P(a->wb_addr); j.C = W(a->c_addr);
  j.vec0 = F(a->ba_addr); j.vec1 = F(a->bb_addr);
  return AKILI_OK;
}

// ----------------------------------------------------- kb2_* job builders --
// The fp32 SIMT family (benchmarks/kb2_<bench>/kernel.cpp): the same fused
// ops with fp32 operands kept to fp32 accuracy through the split mode.
int job_kb2_add_relu(const kb2_gemm_add_relu_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->w_addr, a->bias_addr, a->c_addr}))) return rc;
  j.epi = Epi::kBiasRelu; j.split = true;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->w_addr); j.vec0 = F(a->bias_addr); j.C = W(a->c_addr);
  return AKILI_OK;
}

int job_kb2_mul_leakyrelu(const kb2_gemm_mul_leakyrelu_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->w_addr, a->bias_addr, a->c_addr}))) return rc;
  j.epi = Epi::kBiasMulLeaky; j.split = true;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->w_addr); j.vec0 = F(a->bias_addr); j.C = W(a->c_addr);
  j.s0 = a->multiplier; j.s1 = a->negative_slope;
  return AKILI_OK;
}

int job_kb2_div_sum_scale(const kb2_gemm_div_sum_scale_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->w_addr, a->c_addr}))) return rc;
  j.epi = Epi::kRowSumHalf; j.split = true;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->w_addr); j.C = W(a->c_addr);
  j.final_scale = a->scaling_factor;
  return AKILI_OK;
}

int job_kb2_layernorm(const kb2_gemm_layernorm_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->w_addr, a->bias_addr, a->ln_w_addr, a->ln_b_addr, a->c_addr}))) return rc;
  j.epi = Epi::kLnPre; j.split = true;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->w_addr); j.vec0 = F(a->bias_addr); j.C = W(a->c_addr);
  j.ln_w = F(a->ln_w_addr); j.ln_b = F(a->ln_b_addr); j.eps = a->eps;
  return AKILI_OK;
}

int job_kb2_attention_score(const kb2_attention_score_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->D))) return rc;
  if (chk && (rc = check_ptrs({a->q_addr, a->k_addr, a->c_addr}))) return rc;
  j.epi = Epi::kSoftmaxPre; j.split = true;
  j.b_kmajor = true;
  j.M = a->M; j.N = a->N; j.K = a->D;
  j.A = P(a->q_addr); j.B0 = P(a->k_addr); j.C = W(a->c_addr);
  j.s0 = 1.0f / sqrtf(static_cast<float>(a->D));  // kb2_attention_score/main.cpp verify loop
  return AKILI_OK;
}

int job_kb2_matmul_softmax(const kb2_matmul_softmax_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->b_addr, a->c_addr}))) return rc;
  j.epi = Epi::kSoftmaxPre; j.split = true;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->b_addr); j.C = W(a->c_addr);
  j.s0 = 1.0f;
  return AKILI_OK;
}

int job_kb2_clamp(const kb2_matmul_scale_residadd_clamp_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->w_addr, a->bias_addr, a->c_addr}))) return rc;
  j.epi = Epi::kLseClamp; j.split = true;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->w_addr); j.vec0 = F(a->bias_addr); j.C = W(a->c_addr);
  j.s0 = a->scale_factor; j.s1 = a->clamp_min; j.s2 = a->clamp_max;
  return AKILI_OK;
}

int job_kb2_sum_max_avgpool(const kb2_matmul_sum_max_avgpool_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->w_addr, a->bias_addr, a->c_addr}))) return rc;
  j.epi = Epi::kRowSumBias; j.split = true;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->w_addr); j.vec0 = F(a->bias_addr); j.C = W(a->c_addr);
  j.final_scale = 1.0f;
  return AKILI_OK;
}

int job_kb2_rmsnorm_swiglu(const kb2_gemm_rmsnorm_swiglu_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->x_addr, a->rms_w_addr, a->wg_addr, a->wu_addr, a->c_addr}))) return rc;
  j.epi = Epi::kSwiglu; j.split = true;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->x_addr); j.B0 = P(a->wg_addr); j.B1 = P(a->wu_addr); j.C = W(a->c_addr);
  j.rmsnorm = true; j.rms_w = F(a->rms_w_addr); j.eps = a->eps;
  return AKILI_OK;
}

int job_kb2_silu_mul(const kb2_gemm_silu_mul_arg_t* a, GemmJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  int rc;
  if ((rc = check_m(a->M)) || (rc = check_dims(a->N, a->K))) return rc;
  if (chk && (rc = check_ptrs({a->a_addr, a->wa_addr, a->ba_addr, a->wb_addr, a->bb_addr, a->c_addr}))) return rc;
  j.epi = Epi::kSiluMulBias; j.split = true;
  j.M = a->M; j.N = a->N; j.K = a->K;
  j.A = P(a->a_addr); j.B0 = P(a->wa_addr); j.B1 = P(a->wb_addr); j.C = W(a->c_addr);
  j.vec0 = F(a->ba_addr); j.vec1 = F(a->bb_addr);
  return AKILI_OK;
}

// -------------------------------------------------------------- flash --
struct FlashJob {
  uint32_t seq_len = 0, head_dim = 0;
  uint32_t kernel_type = 1;  // 0: the reference's fp32 SIMT flash, 1: its fp16 tensor-core flash
  const void *Q = nullptr, *K = nullptr, *V = nullptr;
  void* O = nullptr;
  float* m_out = nullptr;  // optional row statistics (akili_flash_ml_ex)
  float* l_out = nullptr;
};

// fp32 operands with the reference's SIMT kernel type (fp32 arithmetic,
// benchmarks/flash/kernel.cpp:27-135) compute S in split precision, so
// scores of the unscaled reference inputs keep fp32-level accuracy; head
// dims up to 64 (the reference's SIMT path allows 16).
bool flash_split(const FlashJob& j, const Mode& md) {
  return md.in_f32 && j.kernel_type == 0 && j.head_dim <= 64;
}

int job_flash(const flash_arg_t* a, FlashJob& j, bool chk = true) {
  if (!a) return AKILI_E_NULL_ARG;
  if (a->seq_len == 0 || a->head_dim == 0 || (a->head_dim % 8)) return AKILI_E_SHAPE;
  if (a->head_dim > 128) return AKILI_E_UNSUPPORTED;
  int rc;
  if (chk && (rc = check_ptrs({a->Q_addr, a->K_addr, a->V_addr, a->O_addr}))) return rc;
  j.seq_len = a->seq_len; j.head_dim = a->head_dim; j.kernel_type = a->kernel_type;
  j.Q = P(a->Q_addr); j.K = P(a->K_addr); j.V = P(a->V_addr); j.O = W(a->O_addr);
  return AKILI_OK;
}

size_t flash_scratch_bytes(const FlashJob& j, const Mode& md) {
  if (!md.in_f32) return 0;
  const size_t n = static_cast<size_t>(md.batch) * md.heads * j.seq_len * j.head_dim;
  Carve c;
  for (int i = 0; i < (flash_split(j, md) ? 5 : 3); ++i) c.need(n * 2);
  return c.off;
}

int run_flash(const FlashJob& j, const Mode& md, cudaStream_t st) {
  DevInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const size_t n = static_cast<size_t>(md.batch) * md.heads * j.seq_len * j.head_dim;
  const __half *q = static_cast<const __half*>(j.Q), *k = static_cast<const __half*>(j.K),
               *v = static_cast<const __half*>(j.V);
  const __half *qlo = nullptr, *klo = nullptr;
  const bool split = flash_split(j, md);
  if (md.in_f32) {
    char* base = nullptr;
    if ((rc = acquire_scratch(md, flash_scratch_bytes(j, md), st, &base))) return rc;
    Carve cv;
    cv.base = base;
    __half* cq = static_cast<__half*>(cv.take(n * 2));
    __half* ck = static_cast<__half*>(cv.take(n * 2));
    __half* cvv = static_cast<__half*>(cv.take(n * 2));
    if (split) {
      __half* cql = static_cast<__half*>(cv.take(n * 2));
      __half* ckl = static_cast<__half*>(cv.take(n * 2));
      const int g = grid_for(di, n, 256, 8);
      split_f32_to_f16x2_kernel<<<g, 256, 0, st>>>(static_cast<const float*>(j.Q), cq, cql, n);
      if ((rc = launch_status())) return rc;
      split_f32_to_f16x2_kernel<<<g, 256, 0, st>>>(static_cast<const float*>(j.K), ck, ckl, n);
      if ((rc = launch_status())) return rc;
      qlo = cql; klo = ckl;
    } else {
      if ((rc = cast_to_f16(di, static_cast<const float*>(j.Q), cq, n, st))) return rc;
      if ((rc = cast_to_f16(di, static_cast<const float*>(j.K), ck, n, st))) return rc;
    }
    if ((rc = cast_to_f16(di, static_cast<const float*>(j.V), cvv, n, st))) return rc;
    q = cq; k = ck; v = cvv;
  }
  const uint32_t bh = md.batch * md.heads;
  const uint32_t D = j.head_dim;
  const uint32_t dpad = D <= 64 ? 64 : 128;
  CUtensorMap tq, tk, tv, to;
  bool ok = map3d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, D, j.seq_len, bh, 64, kFlashBM,
                  CU_TENSOR_MAP_SWIZZLE_128B, 2) &&
            map3d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, D, j.seq_len, bh, 64, kFlashBN,
                  CU_TENSOR_MAP_SWIZZLE_128B, 2) &&
            map3d(&tv, v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, D, j.seq_len, bh, 64, kFlashBN,
                  CU_TENSOR_MAP_SWIZZLE_128B, 2);
  if (md.out_f32)
    ok = ok && map3d(&to, j.O, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, D, j.seq_len, bh, 32, kFlashBM,
                     CU_TENSOR_MAP_SWIZZLE_128B, 4);
  else
    ok = ok && map3d(&to, j.O, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, D, j.seq_len, bh, 32, kFlashBM,
                     CU_TENSOR_MAP_SWIZZLE_64B, 2);
  CUtensorMap tql = tq, tkl = tk;
  if (split)
    ok = ok && map3d(&tql, qlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, D, j.seq_len, bh, 64, kFlashBM,
                     CU_TENSOR_MAP_SWIZZLE_128B, 2) &&
         map3d(&tkl, klo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, D, j.seq_len, bh, 64, kFlashBN,
               CU_TENSOR_MAP_SWIZZLE_128B, 2);
  if (!ok) return AKILI_E_LAUNCH;
  FlashArgs fa;
  fa.seq_len = static_cast<int>(j.seq_len);
  fa.head_dim = static_cast<int>(D);
  fa.scale_log2 = md.scale * 1.4426950408889634f;
  fa.causal = md.causal ? 1 : 0;
  fa.m_out = j.m_out;
  fa.l_out = j.l_out;
  dim3 grid((j.seq_len + kFlashBM * kFlashQTiles - 1) / (kFlashBM * kFlashQTiles), bh);
  if (split) rc = launch_flash<64, true>(grid, md.out_f32, tq, tk, tv, to, tql, tkl, fa, st);
  else if (dpad == 64) rc = launch_flash<64, false>(grid, md.out_f32, tq, tk, tv, to, tql, tkl, fa, st);
  else rc = launch_flash<128, false>(grid, md.out_f32, tq, tk, tv, to, tql, tkl, fa, st);
  if (rc == AKILI_OK) g_launches.fetch_add(1, std::memory_order_relaxed);
  return rc;
}

cudaStream_t S(akili_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// ------------------------------------------------- no-alloc LayerNorm scratch --
// Fixed device scratch of akili_kbt_gemm_layernorm_noalloc: the per-(row,
// 128-column half tile) (mean, M2) partials its GEMM epilogue writes and its
// row merge (or finaliser) reads, and the row-fused epilogue's arrival
// counters.  Every statistics slot read is written earlier in the same call;
// the counters are zeroed on the stream before each GEMM.  Concurrent calls race.
static __device__ __align__(256) unsigned char g_noalloc_scratch[AKILI_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch for the current device.  In host code
// the array's name is only a host-side stand-in; the kernel must be given the
// address cudaGetSymbolAddress returns, looked up once per device (per
// context: a device reset reloads the module at a new address).
int noalloc_scratch_ptr(void** out) {
  static std::mutex mu;
  static std::map<unsigned long long, void*> addr;
  unsigned long long dev = 0;
  int rc = current_context_id(&dev);
  if (rc) return rc;
  std::lock_guard<std::mutex> g(mu);
  auto it = addr.find(dev);
  if (it == addr.end()) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return AKILI_E_LAUNCH;
    }
    it = addr.emplace(dev, p).first;
  }
  *out = it->second;
  return AKILI_OK;
}

template <class Arg, int (*Build)(const Arg*, GemmJob&, bool)>
int entry(const Arg* a, const akili_ex_t* ex, akili_stream_t s) {
  Mode md;
  int rc = parse_ex(ex, &md);
  if (rc) return rc;
  if (md.causal) return AKILI_E_UNSUPPORTED;  // a mask has no meaning for the GEMM ops
  if (!a) return AKILI_E_NULL_ARG;
  GemmJob j;
  // An empty batch (M == 0) is a no-op; its buffers may legitimately be null.
  if ((rc = Build(a, j, a->M != 0))) return rc;
  return run_job(j, md, S(s));
}

static_assert((0x1000u | kSiteSelfTest) == AKILI_STATUS_SELFTEST, "status code of the self-test wait");

// One CTA waits on an mbarrier that nothing arrives at, bounded by limit_ns:
// the wait gives up, records kSiteSelfTest and the kernel returns.
__global__ void selftest_wait_kernel(uint64_t limit_ns) {
  __shared__ alignas(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_for(&bar, 0, kSiteSelfTest, limit_ns);
  __syncthreads();
}

// kb2_* entries: fp32 in, fp32 out; an akili_ex_t may only add a workspace.
template <class Arg, int (*Build)(const Arg*, GemmJob&, bool)>
int entry_kb2(const Arg* a, const akili_ex_t* ex, akili_stream_t s) {
  Mode md;
  int rc = parse_ex(ex, &md);
  if (rc) return rc;
  if (!md.in_f32 || !md.out_f32) return AKILI_E_DTYPE;
  if (md.causal || md.batch != 1 || md.heads != 1) return AKILI_E_UNSUPPORTED;
  if (!a) return AKILI_E_NULL_ARG;
  GemmJob j;
  if ((rc = Build(a, j, a->M != 0))) return rc;
  return run_job(j, md, S(s));
}

// ------------------------------------------------------ llama2 offload --
// x is staged in shared memory up to this size (the largest llama2 K is the
// FFN hidden size, 11008 for 7B: 44 KB).
constexpr size_t kMatvecSmemMax = 200 * 1024;

// AKILI_PDL=0 launches the matrix-vector kernels without the programmatic
// dependent launch attribute (for A/B measurements).
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("AKILI_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <bool kVec, bool kSmemX>
int launch_matvec_t(const DevInfo& di, const MatvecArgs& a, cudaStream_t st) {
  auto kern = matvec_kernel<kVec, kSmemX>;
  const size_t smem = kSmemX ? ((static_cast<size_t>(a.K) * 4 + 15) & ~size_t(15)) : 0;
  static std::atomic<size_t> opted{48 * 1024};
  if (smem > opted.load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kMatvecSmemMax)) !=
        cudaSuccess) {
      cudaGetLastError();
      return AKILI_E_LAUNCH;
    }
    opted.store(kMatvecSmemMax, std::memory_order_relaxed);
  }
  // One wave of persistent CTAs (as many as are resident at once, from the
  // occupancy calculator), never more than one row group per CTA.
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kMatvecThreads, smem) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  const int warps = kMatvecThreads / 32;
  const int need = (a.rows + warps - 1) / warps;
  const int blocks = std::max(1, std::min(need, di.sms * per_sm));
  // A programmatic dependent launch: a decode step is tens of these launches
  // back to back, and each may be dispatched while the previous one drains
  // (the kernel waits for it before touching memory).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(kMatvecThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, a) != cudaSuccess) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaGetLastError();
    return AKILI_E_LAUNCH;
  }
  return launch_status();
}

int launch_matvec(const DevInfo& di, const MatvecArgs& a, bool vec, cudaStream_t st) {
  const bool smem = static_cast<size_t>(a.K) * 4 <= kMatvecSmemMax;
  // without staging, x is read as float4s in place
  if (!smem && reinterpret_cast<uintptr_t>(a.x) % 16) vec = false;
  if (vec) return smem ? launch_matvec_t<true, true>(di, a, st) : launch_matvec_t<true, false>(di, a, st);
  return smem ? launch_matvec_t<false, true>(di, a, st) : launch_matvec_t<false, false>(di, a, st);
}

int check_f32_ptr(uint64_t p) {
  if (p == 0) return AKILI_E_NULL_ARG;
  return (p % 4) ? AKILI_E_ALIGN : AKILI_OK;
}

// ----------------------------------------------- unfused attention --
// Per-head GEMMs of one launch stage run on kAttnStreams streams forked from
// and joined back to the caller's stream (events; a CUDA graph captures them
// as parallel branches): one head's P.V product (N = head_dim) fills only a
// few CTA pairs.
constexpr int kAttnStreams = 4;
struct AttnStreams {
  std::mutex mu;
  bool ready = false;
  cudaStream_t s[kAttnStreams] = {};
  cudaEvent_t fork = nullptr, join[kAttnStreams] = {};
};

int attn_streams(AttnStreams** out) {
  static AttnStreams per_dev[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return AKILI_E_NO_DEVICE;
  }
  AttnStreams& a = per_dev[dev];
  std::lock_guard<std::mutex> lk(a.mu);
  if (!a.ready) {
    bool ok = cudaEventCreateWithFlags(&a.fork, cudaEventDisableTiming) == cudaSuccess;
    for (int i = 0; i < kAttnStreams && ok; ++i)
      ok = cudaStreamCreateWithFlags(&a.s[i], cudaStreamNonBlocking) == cudaSuccess &&
           cudaEventCreateWithFlags(&a.join[i], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
      cudaGetLastError();
      return AKILI_E_LAUNCH;
    }
    a.ready = true;
  }
  *out = &a;
  return AKILI_OK;
}

// One of the three launches of benchmarks/attention (kernel_id 0: S = Q.K
// with K stored d x N, 1: P = softmax(scale * S) by rows, 2: O = P.V) for
// each of batch*heads heads stored one after another.  fp32 buffers run the
// reference's exact fp32 CUDA-core kernels head by head; fp16 buffers run
// the two products on the tensor-core GEMM and the softmax as one HBM pass
// over all heads' rows, with S and P materialised in between.
int attention_run(const attention_arg_t* a, const Mode& md, cudaStream_t st) {
  if (!a) return AKILI_E_NULL_ARG;
  if (a->N == 0 || a->d == 0) return AKILI_E_SHAPE;
  if (a->kernel_id > 2) return AKILI_E_UNSUPPORTED;
  if (md.causal) return AKILI_E_UNSUPPORTED;
  if (md.in_f32 != md.out_f32) return AKILI_E_DTYPE;
  int rc;
  if (a->kernel_id == 0) rc = check_ptrs({a->Q_addr, a->K_addr, a->S_addr});
  else if (a->kernel_id == 1) rc = check_ptrs({a->S_addr, a->P_addr});
  else rc = check_ptrs({a->P_addr, a->V_addr, a->O_addr});
  if (rc) return rc;
  DevInfo di;
  if ((rc = device_info(&di))) return rc;
  const int N = static_cast<int>(a->N), d = static_cast<int>(a->d);
  const size_t heads = static_cast<size_t>(md.batch) * md.heads;
  const size_t nd = static_cast<size_t>(N) * d, nn = static_cast<size_t>(N) * N;
  const size_t esz = md.in_f32 ? 4 : 2;
  auto at = [&](uint64_t base, size_t elems) { return reinterpret_cast<char*>(static_cast<uintptr_t>(base)) + elems * esz; };
  if (md.in_f32) {
    for (size_t h = 0; h < heads; ++h) {
      if (a->kernel_id == 1) {
        attention_softmax_kernel<<<grid_for(di, N, 8, 8), 256, 0, st>>>(
            reinterpret_cast<const float*>(at(a->S_addr, h * nn)), reinterpret_cast<float*>(at(a->P_addr, h * nn)),
            N, N, md.scale);
      } else {
        const int M = N, Nc = a->kernel_id == 0 ? N : d, K = a->kernel_id == 0 ? d : N;
        const float* A = reinterpret_cast<const float*>(a->kernel_id == 0 ? at(a->Q_addr, h * nd)
                                                                          : at(a->P_addr, h * nn));
        const float* B = reinterpret_cast<const float*>(a->kernel_id == 0 ? at(a->K_addr, h * nd)
                                                                          : at(a->V_addr, h * nd));
        float* C = reinterpret_cast<float*>(a->kernel_id == 0 ? at(a->S_addr, h * nn) : at(a->O_addr, h * nd));
        dim3 grid((Nc + kAtTile - 1) / kAtTile, (M + kAtTile - 1) / kAtTile);
        if (grid.y > 65535u) return AKILI_E_SHAPE;
        attention_matmul_kernel<<<grid, dim3(kAtTile, 8), 0, st>>>(A, B, C, M, Nc, K);
      }
      if ((rc = launch_status())) return rc;
    }
    return AKILI_OK;
  }
  // fp16: the tensor-core GEMM needs 16-byte rows
  if (N % 8 || d % 8) return AKILI_E_SHAPE;
  if (a->kernel_id == 1) {
    const size_t rows = heads * N;
    attention_softmax_f16_kernel<<<grid_for(di, rows, 8, 16), 256, 0, st>>>(
        reinterpret_cast<const __half*>(at(a->S_addr, 0)), reinterpret_cast<__half*>(at(a->P_addr, 0)), rows, N,
        md.scale * 1.4426950408889634f);
    return launch_status();
  }
  Mode gm;
  gm.in_f32 = gm.out_f32 = false;
  gm.workspace = md.workspace;
  gm.workspace_bytes = md.workspace_bytes;
  AttnStreams* ax = nullptr;
  if ((rc = attn_streams(&ax))) return rc;
  std::lock_guard<std::mutex> lk(ax->mu);
  const int nst = heads > 1 ? kAttnStreams : 0;
  if (nst) {
    bool ok = cudaEventRecord(ax->fork, st) == cudaSuccess;
    for (int i = 0; i < nst && ok; ++i) ok = cudaStreamWaitEvent(ax->s[i], ax->fork, 0) == cudaSuccess;
    if (!ok) {
      cudaGetLastError();
      return AKILI_E_LAUNCH;
    }
  }
  for (size_t h = 0; h < heads && rc == AKILI_OK; ++h) {
    GemmJob j;
    j.epi = Epi::kPlain;
    if (a->kernel_id == 0) {  // S_h[N x N] = Q_h[N x d] . K_h[d x N]
      j.M = N; j.N = N; j.K = d;
      j.A = at(a->Q_addr, h * nd); j.B0 = at(a->K_addr, h * nd); j.C = at(a->S_addr, h * nn);
    } else {                  // O_h[N x d] = P_h[N x N] . V_h[N x d]
      j.M = N; j.N = d; j.K = N;
      j.A = at(a->P_addr, h * nn); j.B0 = at(a->V_addr, h * nd); j.C = at(a->O_addr, h * nd);
    }
    rc = run_job(j, gm, nst ? ax->s[h % nst] : st);
  }
  // join every branch back, also after an error, so the caller's stream (or
  // capture) is left consistent
  for (int i = 0; i < nst; ++i)
    if (cudaEventRecord(ax->join[i], ax->s[i]) != cudaSuccess || cudaStreamWaitEvent(st, ax->join[i], 0) != cudaSuccess) {
      cudaGetLastError();
      if (rc == AKILI_OK) rc = AKILI_E_LAUNCH;
    }
  return rc;
}

// ------------------------------------------------------------ host calls --
// One GEMM-family op on HOST buffers (the harness's copy-in / run / copy-out
// as one pipelined call).  The whole operands (W, bias and affine vectors)
// are copied once; then the rows go through in chunks on three streams:
// host->device copy of chunk c+1, the fused GEMM of chunk c and the
// device->host copy of chunk c-1 overlap, so the two copy engines and the
// SMs work at once.  Row chunks are independent for every op here: each
// output row (or row value) depends on its own input row only.
constexpr int kHostSlots = 3;  // chunk buffers in flight

struct HostPipe {
  std::mutex mu;
  bool ready = false;
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t loaded[kHostSlots] = {}, computed[kHostSlots] = {}, stored[kHostSlots] = {};
  void* whole = nullptr;  // W, B1 and the per-column vectors
  size_t whole_bytes = 0;
  void* rows = nullptr;   // kHostSlots x (A chunk + C chunk)
  size_t rows_bytes = 0;
};

int host_pipe(HostPipe** out) {
  static HostPipe per_dev[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return AKILI_E_NO_DEVICE;
  }
  HostPipe& h = per_dev[dev];
  *out = &h;
  return AKILI_OK;
}

int grow_buffer(void** p, size_t* have, size_t need) {
  if (*have >= need) return AKILI_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *have = 0;
  if (cudaMalloc(p, need) != cudaSuccess) {
    cudaGetLastError();
    *p = nullptr;
    return AKILI_E_ALLOC;
  }
  *have = need;
  return AKILI_OK;
}

// Streams and events of the pipeline, created on first use (call with hp->mu held).
int host_pipe_ready(HostPipe* hp) {
  if (hp->ready) return AKILI_OK;
  bool ok = cudaStreamCreateWithFlags(&hp->h2d, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&hp->d2h, cudaStreamNonBlocking) == cudaSuccess;
  for (int i = 0; i < kHostSlots && ok; ++i)
    ok = cudaEventCreateWithFlags(&hp->loaded[i], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&hp->computed[i], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&hp->stored[i], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    return AKILI_E_LAUNCH;
  }
  hp->ready = true;
  return AKILI_OK;
}

bool epi_vector_out(Epi e) { return e == Epi::kRowSumHalf || e == Epi::kRowSumBias || e == Epi::kLseClamp; }

int run_host_job(GemmJob j, const Mode& md, cudaStream_t st) {
  if (j.M == 0) return AKILI_OK;
  const bool dual = epi_dual(j.epi);
  const bool bias = j.epi == Epi::kBiasRelu || j.epi == Epi::kBiasMulLeaky || j.epi == Epi::kRowSumBias ||
                    j.epi == Epi::kLnPre || j.epi == Epi::kSiluMulBias;
  if (!j.A || !j.B0 || !j.C || (dual && !j.B1) || (bias && !j.vec0) ||
      (j.epi == Epi::kSiluMulBias && !j.vec1) || (j.epi == Epi::kLnPre && (!j.ln_w || !j.ln_b)) ||
      (j.rmsnorm && !j.rms_w))
    return AKILI_E_NULL_ARG;
  HostPipe* hp = nullptr;
  int rc = host_pipe(&hp);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(hp->mu);
  if ((rc = host_pipe_ready(hp))) return rc;
  const size_t ein = md.in_f32 ? 4 : 2, eout = md.out_f32 ? 4 : 2;
  const size_t M = j.M, N = j.N, K = j.K;
  const size_t a_row = K * ein, c_row = (epi_vector_out(j.epi) ? 1 : N) * eout;
  // the whole operands, 256-byte aligned pieces
  auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
  struct Piece { const void* host; size_t bytes; const void** dev; };
  Piece pieces[8];
  int np = 0;
  pieces[np++] = {j.B0, K * N * ein, &j.B0};
  if (dual) pieces[np++] = {j.B1, K * N * ein, &j.B1};
  const void* v0 = j.vec0; const void* v1 = j.vec1; const void* lw = j.ln_w; const void* lb = j.ln_b;
  const void* rw = j.rms_w;
  if (v0) pieces[np++] = {v0, N * 4, &v0};
  if (v1) pieces[np++] = {v1, N * 4, &v1};
  if (lw) pieces[np++] = {lw, N * 4, &lw};
  if (lb) pieces[np++] = {lb, N * 4, &lb};
  if (rw) pieces[np++] = {rw, K * 4, &rw};
  size_t whole = 0;
  for (int i = 0; i < np; ++i) whole += up(pieces[i].bytes);
  // chunks of a multiple of 128 rows, about 8 of them
  size_t chunk = ((M + 7) / 8 + 127) / 128 * 128;
  if (chunk > M) chunk = M;
  const size_t slot_bytes = up(chunk * a_row) + up(chunk * c_row);
  if ((rc = grow_buffer(&hp->whole, &hp->whole_bytes, whole)) ||
      (rc = grow_buffer(&hp->rows, &hp->rows_bytes, slot_bytes * kHostSlots)))
    return rc;
  bool ok = true;
  size_t off = 0;
  for (int i = 0; i < np && ok; ++i) {
    char* d = static_cast<char*>(hp->whole) + off;
    ok = cudaMemcpyAsync(d, pieces[i].host, pieces[i].bytes, cudaMemcpyHostToDevice, hp->h2d) == cudaSuccess;
    *pieces[i].dev = d;
    off += up(pieces[i].bytes);
  }
  j.vec0 = static_cast<const float*>(v0); j.vec1 = static_cast<const float*>(v1);
  j.ln_w = static_cast<const float*>(lw); j.ln_b = static_cast<const float*>(lb);
  j.rms_w = static_cast<const float*>(rw);
  j.stats_hint = nullptr; j.stats_hint_bytes = 0; j.xhat_hint = nullptr;  // scratch from the pool
  const char* hA = static_cast<const char*>(j.A);
  char* hC = static_cast<char*>(j.C);
  const size_t nchunks = (M + chunk - 1) / chunk;
  for (size_t c = 0; c < nchunks && ok && rc == AKILI_OK; ++c) {
    const int sl = static_cast<int>(c % kHostSlots);
    const size_t r0 = c * chunk, rows = std::min(chunk, M - r0);
    char* dA = static_cast<char*>(hp->rows) + sl * slot_bytes;
    char* dC = dA + up(chunk * a_row);
    // the slot is free once chunk c - kHostSlots has been copied out
    if (c >= static_cast<size_t>(kHostSlots)) ok = cudaStreamWaitEvent(hp->h2d, hp->stored[sl], 0) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(dA, hA + r0 * a_row, rows * a_row, cudaMemcpyHostToDevice, hp->h2d) == cudaSuccess &&
         cudaEventRecord(hp->loaded[sl], hp->h2d) == cudaSuccess &&
         cudaStreamWaitEvent(st, hp->loaded[sl], 0) == cudaSuccess;
    if (!ok) break;
    GemmJob jc = j;
    jc.M = static_cast<uint32_t>(rows);
    jc.A = dA;
    jc.C = dC;
    rc = run_job(jc, md, st);
    ok = rc == AKILI_OK && cudaEventRecord(hp->computed[sl], st) == cudaSuccess &&
         cudaStreamWaitEvent(hp->d2h, hp->computed[sl], 0) == cudaSuccess &&
         cudaMemcpyAsync(hC + r0 * c_row, dC, rows * c_row, cudaMemcpyDeviceToHost, hp->d2h) == cudaSuccess &&
         cudaEventRecord(hp->stored[sl], hp->d2h) == cudaSuccess;
  }
  // the call returns with the outputs in host memory (and every stream idle)
  const bool synced = cudaStreamSynchronize(hp->h2d) == cudaSuccess && cudaStreamSynchronize(st) == cudaSuccess &&
                      cudaStreamSynchronize(hp->d2h) == cudaSuccess;
  if (rc) return rc;
  if (!ok || !synced) {
    cudaGetLastError();
    return AKILI_E_LAUNCH;
  }
  return AKILI_OK;
}

// Flash on HOST buffers: the batch*heads heads go through in about 8
// chunks, the host->device copy of Q, K, V of chunk c+1, the flash kernel
// of chunk c and the device->host copy of O of chunk c-1 overlapped, as in
// run_host_job (heads are independent).
int run_host_flash(const FlashJob& j, const Mode& md, cudaStream_t st) {
  if (!j.Q || !j.K || !j.V || !j.O) return AKILI_E_NULL_ARG;
  HostPipe* hp = nullptr;
  int rc = host_pipe(&hp);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(hp->mu);
  if ((rc = host_pipe_ready(hp))) return rc;
  const size_t heads = static_cast<size_t>(md.batch) * md.heads;
  const size_t ein = md.in_f32 ? 4 : 2, eout = md.out_f32 ? 4 : 2;
  const size_t elems = static_cast<size_t>(j.seq_len) * j.head_dim;  // per head
  const size_t hin = elems * ein, hout = elems * eout;
  const size_t chunk = std::max<size_t>(1, (heads + 7) / 8);
  auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t slot_bytes = 3 * up(chunk * hin) + up(chunk * hout);
  if ((rc = grow_buffer(&hp->rows, &hp->rows_bytes, slot_bytes * kHostSlots))) return rc;
  const char* hq = static_cast<const char*>(j.Q);
  const char* hk = static_cast<const char*>(j.K);
  const char* hv = static_cast<const char*>(j.V);
  char* ho = static_cast<char*>(j.O);
  const size_t nchunks = (heads + chunk - 1) / chunk;
  bool ok = true;
  for (size_t c = 0; c < nchunks && ok && rc == AKILI_OK; ++c) {
    const int sl = static_cast<int>(c % kHostSlots);
    const size_t h0 = c * chunk, nh = std::min(chunk, heads - h0);
    char* dq = static_cast<char*>(hp->rows) + sl * slot_bytes;
    char* dk = dq + up(chunk * hin);
    char* dv = dk + up(chunk * hin);
    char* d_o = dv + up(chunk * hin);
    if (c >= static_cast<size_t>(kHostSlots)) ok = cudaStreamWaitEvent(hp->h2d, hp->stored[sl], 0) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(dq, hq + h0 * hin, nh * hin, cudaMemcpyHostToDevice, hp->h2d) == cudaSuccess &&
         cudaMemcpyAsync(dk, hk + h0 * hin, nh * hin, cudaMemcpyHostToDevice, hp->h2d) == cudaSuccess &&
         cudaMemcpyAsync(dv, hv + h0 * hin, nh * hin, cudaMemcpyHostToDevice, hp->h2d) == cudaSuccess &&
         cudaEventRecord(hp->loaded[sl], hp->h2d) == cudaSuccess &&
         cudaStreamWaitEvent(st, hp->loaded[sl], 0) == cudaSuccess;
    if (!ok) break;
    FlashJob jc = j;
    jc.Q = dq; jc.K = dk; jc.V = dv; jc.O = d_o;
    jc.m_out = nullptr; jc.l_out = nullptr;
    Mode mc = md;
    mc.batch = 1;
    mc.heads = static_cast<uint32_t>(nh);
    rc = run_flash(jc, mc, st);
    ok = rc == AKILI_OK && cudaEventRecord(hp->computed[sl], st) == cudaSuccess &&
         cudaStreamWaitEvent(hp->d2h, hp->computed[sl], 0) == cudaSuccess &&
         cudaMemcpyAsync(ho + h0 * hout, d_o, nh * hout, cudaMemcpyDeviceToHost, hp->d2h) == cudaSuccess &&
         cudaEventRecord(hp->stored[sl], hp->d2h) == cudaSuccess;
  }
  const bool synced = cudaStreamSynchronize(hp->h2d) == cudaSuccess && cudaStreamSynchronize(st) == cudaSuccess &&
                      cudaStreamSynchronize(hp->d2h) == cudaSuccess;
  if (rc) return rc;
  if (!ok || !synced) {
    cudaGetLastError();
    return AKILI_E_LAUNCH;
  }
  return AKILI_OK;
}

}  // namespace

// ===================================================================== ABI ==
extern "C" {

#define AKILI_GEMM_ENTRY(name, T, build)                                                       \
  int akili_##name(const T* a, akili_stream_t s) { return entry<T, build>(a, nullptr, s); }   \
  int akili_##name##_ex(const T* a, const akili_ex_t* ex, akili_stream_t s) {                 \
    if (!ex) return AKILI_E_NULL_ARG;                                                          \
    return entry<T, build>(a, ex, s);                                                          \
  }

AKILI_GEMM_ENTRY(kbt_sgemm, kbt_sgemm_arg_t, job_sgemm)
AKILI_GEMM_ENTRY(kbt_gemm_add_relu, kbt_gemm_add_relu_arg_t, job_add_relu)
AKILI_GEMM_ENTRY(kbt_gemm_mul_leakyrelu, kbt_gemm_mul_leakyrelu_arg_t, job_mul_leakyrelu)
AKILI_GEMM_ENTRY(kbt_gemm_div_sum_scale, kbt_gemm_div_sum_scale_arg_t, job_div_sum_scale)
AKILI_GEMM_ENTRY(kbt_gemm_layernorm, kbt_gemm_layernorm_arg_t, job_layernorm)
AKILI_GEMM_ENTRY(kbt_attention_score, kbt_attention_score_arg_t, job_attention_score)
AKILI_GEMM_ENTRY(kbt_matmul_softmax, kbt_matmul_softmax_arg_t, job_matmul_softmax)
AKILI_GEMM_ENTRY(kbt_matmul_scale_residadd_clamp, kbt_matmul_scale_residadd_clamp_arg_t, job_clamp)
AKILI_GEMM_ENTRY(kbt_matmul_sum_max_avgpool, kbt_matmul_sum_max_avgpool_arg_t, job_sum_max_avgpool)
AKILI_GEMM_ENTRY(kbt_gemm_rmsnorm_swiglu, kbt_gemm_rmsnorm_swiglu_arg_t, job_rmsnorm_swiglu)
AKILI_GEMM_ENTRY(kbt_gemm_silu_mul, kbt_gemm_silu_mul_arg_t, job_silu_mul)
#undef AKILI_GEMM_ENTRY

#define AKILI_KB2_ENTRY(name, build)                                                                \
  int akili_##name(const name##_arg_t* a, akili_stream_t s) { return entry_kb2<name##_arg_t, build>(a, nullptr, s); } \
  int akili_##name##_ex(const name##_arg_t* a, const akili_ex_t* ex, akili_stream_t s) {          \
    if (!ex) return AKILI_E_NULL_ARG;                                                              \
    return entry_kb2<name##_arg_t, build>(a, ex, s);                                               \
  }
AKILI_KB2_ENTRY(kb2_gemm_add_relu, job_kb2_add_relu)
AKILI_KB2_ENTRY(kb2_gemm_mul_leakyrelu, job_kb2_mul_leakyrelu)
AKILI_KB2_ENTRY(kb2_gemm_div_sum_scale, job_kb2_div_sum_scale)
AKILI_KB2_ENTRY(kb2_gemm_layernorm, job_kb2_layernorm)
AKILI_KB2_ENTRY(kb2_attention_score, job_kb2_attention_score)
AKILI_KB2_ENTRY(kb2_matmul_softmax, job_kb2_matmul_softmax)
AKILI_KB2_ENTRY(kb2_matmul_scale_residadd_clamp, job_kb2_clamp)
AKILI_KB2_ENTRY(kb2_matmul_sum_max_avgpool, job_kb2_sum_max_avgpool)
AKILI_KB2_ENTRY(kb2_gemm_rmsnorm_swiglu, job_kb2_rmsnorm_swiglu)
AKILI_KB2_ENTRY(kb2_gemm_silu_mul, job_kb2_silu_mul)
#undef AKILI_KB2_ENTRY

// kbt_gemm_layernorm with its scratch in g_noalloc_scratch: no cudaMalloc,
// cudaFree or other device allocation on any path (fp16 operands need no
// converted copies; the caller-workspace and internal-pool paths are unused).
int akili_kbt_gemm_layernorm_noalloc(const kbt_gemm_layernorm_arg_t* a, const akili_ex_t* ex,
                                     akili_stream_t s) {
  if (!ex) return AKILI_E_NULL_ARG;
  Mode md;
  int rc = parse_ex(ex, &md);
  if (rc) return rc;
  if (md.in_f32) return AKILI_E_DTYPE;
  if (md.workspace || md.causal) return AKILI_E_UNSUPPORTED;
  if (!a) return AKILI_E_NULL_ARG;
  GemmJob j;
  if ((rc = job_layernorm(a, j, a->M != 0))) return rc;
  if (j.M == 0) return AKILI_OK;
  if (job_scratch_bytes(j, md) > AKILI_NOALLOC_SCRATCH_BYTES) return AKILI_E_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if ((rc = noalloc_scratch_ptr(&scratch))) return rc;
  md.workspace = scratch;
  md.workspace_bytes = AKILI_NOALLOC_SCRATCH_BYTES;
  return run_job(j, md, S(s));
}

int akili_flash_ex(const flash_arg_t* a, const akili_ex_t* ex, akili_stream_t s) {
  Mode md;
  int rc = parse_ex(ex, &md);
  if (rc) return rc;
  FlashJob j;
  if ((rc = job_flash(a, j))) return rc;
  return run_flash(j, md, S(s));
}
int akili_flash(const flash_arg_t* a, akili_stream_t s) { return akili_flash_ex(a, nullptr, s); }

int akili_attention(const attention_arg_t* a, akili_stream_t s) { return attention_run(a, Mode{}, S(s)); }

int akili_attention_ex(const attention_arg_t* a, const akili_ex_t* ex, akili_stream_t s) {
  if (!ex) return AKILI_E_NULL_ARG;
  Mode md;
  const int rc = parse_ex(ex, &md);
  if (rc) return rc;
  return attention_run(a, md, S(s));
}

int akili_llama2_matmul(const matmul_kernel_args_t* a, akili_stream_t s) {
  if (!a) return AKILI_E_NULL_ARG;
  if (a->M < 0 || a->N < 0 || a->K < 0) return AKILI_E_SHAPE;
  if (a->M == 0 || a->N == 0) return AKILI_OK;
  int rc;
  if ((rc = check_f32_ptr(a->C_addr))) return rc;
  if (a->K > 0 && ((rc = check_f32_ptr(a->A_addr)) || (rc = check_f32_ptr(a->B_addr)))) return rc;
  DevInfo di;
  if ((rc = device_info(&di))) return rc;
  cudaStream_t st = S(s);
  const int M = a->M, N = a->N, K = a->K;
  float* C = reinterpret_cast<float*>(static_cast<uintptr_t>(a->C_addr));
  if (K == 0) {  // an empty sum: the reference kernel stores 0.0f
    if (cudaMemsetAsync(C, 0, static_cast<size_t>(M) * N * 4, st) != cudaSuccess) {
      cudaGetLastError();
      return AKILI_E_LAUNCH;
    }
    return AKILI_OK;
  }
  if (N == 1) {
    MatvecArgs m{};
    m.seg[0] = MatvecSeg{F(a->A_addr), C, M, 0};
    m.nseg = 1;
    m.rows = M;
    m.K = K;
    m.x = F(a->B_addr);
    return launch_matvec(di, m, K % 4 == 0 && a->A_addr % 16 == 0, st);
  }
  if (M % 8 == 0 && N % 8 == 0 && K % 8 == 0 && a->A_addr % 16 == 0 && a->B_addr % 16 == 0 && a->C_addr % 16 == 0) {
    GemmJob j;
    j.epi = Epi::kPlain;
    j.split = true;
    j.M = M; j.N = N; j.K = K;
    j.A = P(a->A_addr); j.B0 = P(a->B_addr); j.C = W(a->C_addr);
    Mode md;
    return run_job(j, md, st);
  }
  const dim3 grid((N + kAtTile - 1) / kAtTile, (M + kAtTile - 1) / kAtTile);
  if (grid.y > 65535u) return AKILI_E_SHAPE;
  attention_matmul_kernel<<<grid, dim3(kAtTile, 8), 0, st>>>(F(a->A_addr), F(a->B_addr), C, M, N, K);
  return launch_status();
}

int akili_llama2_matvec_batch(const akili_matvec_seg_t* segs, int nseg, uint64_t x_addr, int32_t K,
                              akili_stream_t s) {
  if (!segs) return AKILI_E_NULL_ARG;
  if (nseg < 1 || nseg > kMatvecMaxSegs) return AKILI_E_UNSUPPORTED;
  if (K < 0) return AKILI_E_SHAPE;
  int rc;
  MatvecArgs m{};
  int64_t rows = 0;
  bool vec = K % 4 == 0;
  for (int i = 0; i < nseg; ++i) {
    if (segs[i].rows < 0) return AKILI_E_SHAPE;
    if (segs[i].rows == 0) continue;
    if ((rc = check_f32_ptr(segs[i].C_addr)) || (K > 0 && (rc = check_f32_ptr(segs[i].W_addr)))) return rc;
    vec = vec && segs[i].W_addr % 16 == 0;
    m.seg[m.nseg++] = MatvecSeg{F(segs[i].W_addr), reinterpret_cast<float*>(static_cast<uintptr_t>(segs[i].C_addr)),
                                segs[i].rows, static_cast<int>(rows)};
    rows += segs[i].rows;
  }
  if (rows > INT32_MAX) return AKILI_E_SHAPE;
  if (rows == 0) return AKILI_OK;
  if (K > 0 && (rc = check_f32_ptr(x_addr))) return rc;
  DevInfo di;
  if ((rc = device_info(&di))) return rc;
  cudaStream_t st = S(s);
  if (K == 0) {
    for (int i = 0; i < m.nseg; ++i)
      if (cudaMemsetAsync(m.seg[i].C, 0, static_cast<size_t>(m.seg[i].rows) * 4, st) != cudaSuccess) {
        cudaGetLastError();
        return AKILI_E_LAUNCH;
      }
    return AKILI_OK;
  }
  m.rows = static_cast<int>(rows);
  m.K = K;
  m.x = F(x_addr);
  return launch_matvec(di, m, vec, st);
}

int akili_flash_ml_ex(const flash_arg_t* a, const akili_ex_t* ex, uint64_t m_addr, uint64_t l_addr,
                      akili_stream_t s) {
  Mode md;
  int rc = parse_ex(ex, &md);
  if (rc) return rc;
  FlashJob j;
  if ((rc = job_flash(a, j))) return rc;
  if (!m_addr || !l_addr) return AKILI_E_NULL_ARG;
  if ((m_addr | l_addr) % 4) return AKILI_E_ALIGN;
  j.m_out = reinterpret_cast<float*>(static_cast<uintptr_t>(m_addr));
  j.l_out = reinterpret_cast<float*>(static_cast<uintptr_t>(l_addr));
  return run_flash(j, md, S(s));
}

const char* akili_strerror(int code) {
  switch (code) {
    case AKILI_OK: return "ok";
    case AKILI_E_NULL_ARG: return "null argument block or buffer address";
    case AKILI_E_SHAPE: return "invalid shape (sizes must be non-zero multiples of 8; M may be 0)";
    case AKILI_E_ALIGN: return "buffer address not 16-byte aligned";
    case AKILI_E_DTYPE: return "unsupported dtype";
    case AKILI_E_UNSUPPORTED: return "unsupported option";
    case AKILI_E_NO_DEVICE: return "no sm_100 CUDA device is current";
    case AKILI_E_ALLOC: return "scratch allocation failed";
    case AKILI_E_LAUNCH: return "kernel launch or tensor-map encode failed";
    case AKILI_E_DEVICE_TIMEOUT: return "a device-side wait timed out";
    case AKILI_E_ABI: return "akili_ex_t.abi_version mismatch";
    case AKILI_E_WORKSPACE: return "workspace smaller than required";
    case AKILI_E_SCRATCH_LIMIT: return "problem exceeds the fixed no-alloc scratch (AKILI_NOALLOC_SCRATCH_BYTES)";
    default: return "unknown error";
  }
}

int akili_workspace_bytes(const char* op, const void* arg, const akili_ex_t* ex, uint64_t* bytes) {
  if (!op || !arg || !bytes) return AKILI_E_NULL_ARG;
  Mode md;
  int rc = parse_ex(ex, &md);
  if (rc) return rc;
  md.workspace = nullptr;
  GemmJob j;
  const std::string name(op);
#define AKILI_WS(nm, T, build) \
  if (name == #nm) {           \
    rc = build(static_cast<const T*>(arg), j, false); \
    if (rc) return rc;         \
    *bytes = job_scratch_bytes(j, md); \
    return AKILI_OK;           \
  }
  AKILI_WS(kbt_sgemm, kbt_sgemm_arg_t, job_sgemm)
  AKILI_WS(kb2_gemm_add_relu, kb2_gemm_add_relu_arg_t, job_kb2_add_relu)
  AKILI_WS(kb2_gemm_mul_leakyrelu, kb2_gemm_mul_leakyrelu_arg_t, job_kb2_mul_leakyrelu)
  AKILI_WS(kb2_gemm_div_sum_scale, kb2_gemm_div_sum_scale_arg_t, job_kb2_div_sum_scale)
  AKILI_WS(kb2_gemm_layernorm, kb2_gemm_layernorm_arg_t, job_kb2_layernorm)
  AKILI_WS(kb2_attention_score, kb2_attention_score_arg_t, job_kb2_attention_score)
  AKILI_WS(kb2_matmul_softmax, kb2_matmul_softmax_arg_t, job_kb2_matmul_softmax)
  AKILI_WS(kb2_matmul_scale_residadd_clamp, kb2_matmul_scale_residadd_clamp_arg_t, job_kb2_clamp)
  AKILI_WS(kb2_matmul_sum_max_avgpool, kb2_matmul_sum_max_avgpool_arg_t, job_kb2_sum_max_avgpool)
  AKILI_WS(kb2_gemm_rmsnorm_swiglu, kb2_gemm_rmsnorm_swiglu_arg_t, job_kb2_rmsnorm_swiglu)
  AKILI_WS(kb2_gemm_silu_mul, kb2_gemm_silu_mul_arg_t, job_kb2_silu_mul)
  AKILI_WS(kbt_gemm_add_relu, kbt_gemm_add_relu_arg_t, job_add_relu)
  AKILI_WS(kbt_gemm_mul_leakyrelu, kbt_gemm_mul_leakyrelu_arg_t, job_mul_leakyrelu)
  AKILI_WS(kbt_gemm_div_sum_scale, kbt_gemm_div_sum_scale_arg_t, job_div_sum_scale)
  AKILI_WS(kbt_gemm_layernorm, kbt_gemm_layernorm_arg_t, job_layernorm)
  AKILI_WS(kbt_attention_score, kbt_attention_score_arg_t, job_attention_score)
  AKILI_WS(kbt_matmul_softmax, kbt_matmul_softmax_arg_t, job_matmul_softmax)
  AKILI_WS(kbt_matmul_scale_residadd_clamp, kbt_matmul_scale_residadd_clamp_arg_t, job_clamp)
  AKILI_WS(kbt_matmul_sum_max_avgpool, kbt_matmul_sum_max_avgpool_arg_t, job_sum_max_avgpool)
  AKILI_WS(kbt_gemm_rmsnorm_swiglu, kbt_gemm_rmsnorm_swiglu_arg_t, job_rmsnorm_swiglu)
  AKILI_WS(kbt_gemm_silu_mul, kbt_gemm_silu_mul_arg_t, job_silu_mul)
#undef AKILI_WS
  if (name == "flash") {
    FlashJob fj;
    if ((rc = job_flash(static_cast<const flash_arg_t*>(arg), fj, false))) return rc;
    *bytes = flash_scratch_bytes(fj, md);
    return AKILI_OK;
  }
  return AKILI_E_UNSUPPORTED;
}

int akili_host_call(const char* op, const void* arg, const akili_ex_t* ex, akili_stream_t s) {
  if (!op || !arg) return AKILI_E_NULL_ARG;
  Mode md;
  int rc = parse_ex(ex, &md);
  if (rc) return rc;
  const std::string name(op);
  if (name == "flash") {
    FlashJob fj;
    if ((rc = job_flash(static_cast<const flash_arg_t*>(arg), fj, false))) return rc;
    return run_host_flash(fj, md, S(s));
  }
  if (md.causal || md.batch != 1 || md.heads != 1) return AKILI_E_UNSUPPORTED;
  GemmJob j;
  const bool kb2 = name.rfind("kb2_", 0) == 0;
  if (kb2 && (!md.in_f32 || !md.out_f32)) return AKILI_E_DTYPE;
#define AKILI_HC(nm, T, build)                                          \
  if (name == #nm) {                                                    \
    if ((rc = build(static_cast<const T*>(arg), j, false))) return rc; \
    return run_host_job(j, md, S(s));                                   \
  }
  AKILI_HC(kbt_sgemm, kbt_sgemm_arg_t, job_sgemm)
  AKILI_HC(kbt_gemm_add_relu, kbt_gemm_add_relu_arg_t, job_add_relu)
  AKILI_HC(kbt_gemm_mul_leakyrelu, kbt_gemm_mul_leakyrelu_arg_t, job_mul_leakyrelu)
  AKILI_HC(kbt_gemm_div_sum_scale, kbt_gemm_div_sum_scale_arg_t, job_div_sum_scale)
  AKILI_HC(kbt_gemm_layernorm, kbt_gemm_layernorm_arg_t, job_layernorm)
  AKILI_HC(kbt_attention_score, kbt_attention_score_arg_t, job_attention_score)
  AKILI_HC(kbt_matmul_softmax, kbt_matmul_softmax_arg_t, job_matmul_softmax)
  AKILI_HC(kbt_matmul_scale_residadd_clamp, kbt_matmul_scale_residadd_clamp_arg_t, job_clamp)
  AKILI_HC(kbt_matmul_sum_max_avgpool, kbt_matmul_sum_max_avgpool_arg_t, job_sum_max_avgpool)
  AKILI_HC(kbt_gemm_rmsnorm_swiglu, kbt_gemm_rmsnorm_swiglu_arg_t, job_rmsnorm_swiglu)
  AKILI_HC(kbt_gemm_silu_mul, kbt_gemm_silu_mul_arg_t, job_silu_mul)
  AKILI_HC(kb2_gemm_add_relu, kb2_gemm_add_relu_arg_t, job_kb2_add_relu)
  AKILI_HC(kb2_gemm_mul_leakyrelu, kb2_gemm_mul_leakyrelu_arg_t, job_kb2_mul_leakyrelu)
  AKILI_HC(kb2_gemm_div_sum_scale, kb2_gemm_div_sum_scale_arg_t, job_kb2_div_sum_scale)
  AKILI_HC(kb2_gemm_layernorm, kb2_gemm_layernorm_arg_t, job_kb2_layernorm)
  AKILI_HC(kb2_attention_score, kb2_attention_score_arg_t, job_kb2_attention_score)
  AKILI_HC(kb2_matmul_softmax, kb2_matmul_softmax_arg_t, job_kb2_matmul_softmax)
  AKILI_HC(kb2_matmul_scale_residadd_clamp, kb2_matmul_scale_residadd_clamp_arg_t, job_kb2_clamp)
  AKILI_HC(kb2_matmul_sum_max_avgpool, kb2_matmul_sum_max_avgpool_arg_t, job_kb2_sum_max_avgpool)
  AKILI_HC(kb2_gemm_rmsnorm_swiglu, kb2_gemm_rmsnorm_swiglu_arg_t, job_kb2_rmsnorm_swiglu)
  AKILI_HC(kb2_gemm_silu_mul, kb2_gemm_silu_mul_arg_t, job_kb2_silu_mul)
#undef AKILI_HC
  return AKILI_E_UNSUPPORTED;
}

int akili_device_status(uint32_t* status, int clear) {
  if (!status) return AKILI_E_NULL_ARG;
  DevInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();
    return AKILI_E_LAUNCH;
  }
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_status, sizeof(v)) != cudaSuccess) return AKILI_E_LAUNCH;
  *status = v;
  if (clear) {
    unsigned int z = 0;
    if (cudaMemcpyToSymbol(g_status, &z, sizeof(z)) != cudaSuccess) return AKILI_E_LAUNCH;
  }
  return v ? AKILI_E_DEVICE_TIMEOUT : AKILI_OK;
}

int akili_selftest_wait_timeout(uint32_t limit_us, akili_stream_t s) {
  if (limit_us == 0 || limit_us > 1000000u) return AKILI_E_SHAPE;
  DevInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  selftest_wait_kernel<<<1, 32, 0, S(s)>>>(uint64_t(limit_us) * 1000ull);
  return launch_status();
}

uint64_t akili_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int akili_sm_clock_read(uint64_t* cycles, uint64_t* ns, int clear) {
  if (!cycles || !ns) return AKILI_E_NULL_ARG;
  DevInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();
    return AKILI_E_LAUNCH;
  }
  unsigned long long v[2] = {0, 0};
  if (cudaMemcpyFromSymbol(v, g_clock_acc, sizeof(v)) != cudaSuccess) return AKILI_E_LAUNCH;
  *cycles = v[0];
  *ns = v[1];
  if (clear) {
    const unsigned long long z[2] = {0, 0};
    if (cudaMemcpyToSymbol(g_clock_acc, z, sizeof(z)) != cudaSuccess) return AKILI_E_LAUNCH;
  }
  return AKILI_OK;
}

uint32_t akili_abi_version(void) { return AKILI_ABI_VERSION; }

}  // extern "C"
