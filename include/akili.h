/*
 * akili.h — C ABI of the B200 (sm_100a) backend for akili-bench's tensor-core
 * fused-op benchmarks (the kbt_* family) and the flash-attention forward.
 *
 * Each benchmark keeps its reference argument block byte for byte: the
 * structs below have the same field order, types, sizes and offsets as the
 * `kernel_arg_t` of benchmarks/<bench>/common.h in akili-bench, so a harness
 * that filled a `kernel_arg_t` for `vx_upload_bytes` can hand the very same
 * bytes to `akili_<bench>()`.  The `*_addr` fields hold device addresses
 * (CUDA device pointers cast to uint64_t) exactly as they held Vortex device
 * addresses from `vx_mem_address`.
 *
 * Entry points replace the Vortex launch pair
 *     vx_upload_bytes(arg) ; vx_start(device, kernel, args) ; vx_ready_wait(...)
 * (e.g. benchmarks/kbt_gemm_add_relu/main.cpp:114-118) by one asynchronous
 * call on a CUDA stream.  `grid_dim`/`block_dim` are Vortex launch hints and
 * are ignored.
 *
 * Two forms per op:
 *   akili_<bench>(arg, stream)          reference semantics: fp32 buffers,
 *                                       operands rounded to fp16 on the
 *                                       device (the kernels' f2h), fp32
 *                                       accumulation, fp32 outputs.
 *   akili_<bench>_ex(arg, ex, stream)   same struct plus an `akili_ex_t`:
 *                                       fp16 inputs/outputs, flash
 *                                       batch/heads/scale, caller workspace.
 *
 * Return value: 0 (AKILI_OK) or a negative AKILI_E_* code.  Nothing here
 * calls exit().  Calls are asynchronous with respect to the host; device-side
 * wait timeouts are reported by akili_device_status().
 *
 * Ownership: the caller owns every buffer and the stream.  Scratch fields of
 * the reference structs (norm_addr, gate_addr, temp_addr) may be written.
 */
#ifndef AKILI_H_
#define AKILI_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t (cuda_runtime_api.h: typedef struct CUstream_st *cudaStream_t). */
struct CUstream_st;
typedef struct CUstream_st* akili_stream_t;

#define AKILI_ABI_VERSION 1u

/* ---- status codes -------------------------------------------------------- */
#define AKILI_OK                  0
#define AKILI_E_NULL_ARG         (-1)  /* arg block or a required buffer address is 0      */
#define AKILI_E_SHAPE            (-2)  /* a size is 0 (other than M) or not a multiple of 8 */
#define AKILI_E_ALIGN            (-3)  /* a buffer address is not 16-byte aligned           */
#define AKILI_E_DTYPE            (-4)  /* unsupported in_dtype / out_dtype                  */
#define AKILI_E_UNSUPPORTED      (-5)  /* e.g. causal=1 on a GEMM op, head_dim > 128        */
#define AKILI_E_NO_DEVICE        (-6)  /* current device is not an sm_100 part              */
#define AKILI_E_ALLOC            (-7)  /* internal scratch pool could not grow              */
#define AKILI_E_LAUNCH           (-8)  /* a CUDA launch or tensor-map encode failed         */
#define AKILI_E_DEVICE_TIMEOUT   (-9)  /* a device-side wait ran out (see device status)    */
#define AKILI_E_ABI             (-10)  /* ex->abi_version != AKILI_ABI_VERSION              */
#define AKILI_E_WORKSPACE       (-11)  /* ex->workspace given but smaller than required     */
#define AKILI_E_SCRATCH_LIMIT   (-12)  /* problem needs more than the fixed no-alloc scratch */

#define AKILI_DTYPE_F32 0u
#define AKILI_DTYPE_F16 1u

/* ---- reference argument blocks (byte-identical to akili-bench) ---------- */

/* benchmarks/kbt_sgemm/common.h:4-13 — C[MxN] = A[MxK] . B[KxN] */
typedef struct {
  uint32_t grid_dim[3];
  uint32_t block_dim[3];
  uint32_t M, N, K;
  uint64_t a_addr, b_addr, c_addr;
} kbt_sgemm_arg_t;

/* benchmarks/kbt_gemm_add_relu/common.h:4-14 — ReLU(x.W + bias) */
typedef struct {
  uint32_t grid_dim[3];
  uint32_t block_dim[3];
  uint32_t M, N, K;
  uint64_t a_addr, w_addr, bias_addr, c_addr;
} kbt_gemm_add_relu_arg_t;

/* benchmarks/kbt_gemm_mul_leakyrelu/common.h:4-16 — LeakyReLU((x.W + b) * multiplier) */
typedef struct {
  uint32_t grid_dim[3];
  uint32_t block_dim[3];
  uint32_t M, N, K;
  float    multiplier;
  float    negative_slope;
  uint64_t a_addr, w_addr, bias_addr, c_addr;
} kbt_gemm_mul_leakyrelu_arg_t;

/* benchmarks/kbt_gemm_div_sum_scale/common.h:4-14 — c[M] = scaling_factor * sum_j (x.W)[i,j] / 2 */
typedef struct {
  uint32_t grid_dim[3];
  uint32_t block_dim[3];
  uint32_t M, N, K;
  float    scaling_factor;
  uint64_t a_addr, w_addr, c_addr;
} kbt_gemm_div_sum_scale_arg_t;

/* benchmarks/kbt_gemm_layernorm/common.h:4-17 — LayerNorm(x.W + bias) * ln_w + ln_b */
typedef struct {
  uint32_t grid_dim[3];
  uint32_t block_dim[3];
  uint32_t M, N, K;
  float    eps;
  uint64_t a_addr, w_addr, bias_addr, ln_w_addr, ln_b_addr, c_addr;
} kbt_gemm_layernorm_arg_t;

/* benchmarks/kbt_attention_score/common.h:4-13 — softmax(Q.K^T / sqrt(D)), Q[MxD], K[NxD] */
typedef struct {
  uint32_t grid_dim[3];
  uint32_t block_dim[3];
  uint32_t M, N, D;
  uint64_t q_addr, k_addr, c_addr;
} kbt_attention_score_arg_t;

/* benchmarks/kbt_matmul_softmax/common.h:4-13 — softmax(A.B) */
typedef struct {
  uint32_t grid_dim[3];
  uint32_t block_dim[3];
  uint32_t M, N, K;
  uint64_t a_addr, b_addr, c_addr;
} kbt_matmul_softmax_arg_t;

/* benchmarks/kbt_matmul_scale_residadd_clamp/common.h:4-17 —
 * t = clamp(2*scale*(A.B)); lse = LSE_j t; c[i] = lse * mish(lse) */
typedef struct {
  uint32_t grid_dim[3];
  uint32_t block_dim[3];
  uint32_t M, N, K;
  float    scale_factor;
  float    clamp_min;
  float    clamp_max;
  uint64_t a_addr, b_addr, c_addr, temp_addr;
} kbt_matmul_scale_residadd_clamp_arg_t;

/* benchmarks/kbt_matmul_sum_max_avgpool/common.h:4-14 — c[i] = sum_j (x.W + bias)[i,j] */
typedef struct {
  uint32_t grid_dim[3];
  uint32_t block_dim[3];
  uint32_t M, N, K;
  uint64_t a_addr, w_addr, bias_addr, c_addr;
} kbt_matmul_sum_max_avgpool_arg_t;

/* benchmarks/kbt_gemm_rmsnorm_swiglu/common.h:4-18 — SiLU(RMSNorm(x).Wg) * (RMSNorm(x).Wu) */
typedef struct {
  uint32_t grid_dim[3];
  uint32_t block_dim[3];
  uint32_t M, N, K;
  float    eps;
  uint64_t x_addr, rms_w_addr, wg_addr, wu_addr, norm_addr, gate_addr, c_addr;
} kbt_gemm_rmsnorm_swiglu_arg_t;

/* benchmarks/kbt_gemm_silu_mul/common.h:4-17 — SiLU(x.Wa + ba) * (x.Wb + bb) */
typedef struct {
  uint32_t grid_dim[3];
  uint32_t block_dim[3];
  uint32_t M, N, K;
  uint64_t a_addr, wa_addr, ba_addr, wb_addr, bb_addr, gate_addr, c_addr;
} kbt_gemm_silu_mul_arg_t;

/* benchmarks/flash/common.h:8-20 — O = softmax(Q.K^T).V, one head, Q/K/V/O [seq_len x head_dim] */
typedef struct {
  uint32_t grid_dim[1];
  uint32_t block_dim[1];
  uint32_t kernel_type;   /* 0: SIMT, 1: tensor core — both run the same sm_100a kernel here */
  uint32_t seq_len;
  uint32_t head_dim;
  uint32_t block_size_r;
  uint32_t block_size_c;
  uint64_t Q_addr, K_addr, V_addr, O_addr;
} flash_arg_t;

/* benchmarks/attention/common.h: the unfused three-kernel attention (fp32,
 * one head); kernel_id selects 0: S = Q.K (K stored d x N), 1: P =
 * softmax(S) by rows, 2: O = P.V. */
typedef struct {
  uint32_t grid_dim[2];
  uint32_t N;
  uint32_t d;
  uint64_t Q_addr, K_addr, S_addr, P_addr, V_addr, O_addr;
  uint32_t kernel_id;
} attention_arg_t;

/* benchmarks/llama2/common.h:3-12 — the llama2 matmul offload:
 * C[M x N] = A[M x K] . B[K x N], fp32, row-major.  The caller
 * (llama2/vxmath.cpp:82-212) passes the weight matrix as A and the
 * activation vector as B with N = 1 (llama2/llama.cpp:225-233). */
typedef struct {
  uint32_t grid_dim[2];
  uint32_t block_dim[2];
  uint64_t A_addr;
  uint64_t B_addr;
  uint64_t C_addr;
  int32_t M;
  int32_t N;
  int32_t K;
} matmul_kernel_args_t;

/* One segment of a batched matrix-vector product: C[rows] = W[rows x K] . x.
 * The batch replaces the reference's concatenate-then-multiply
 * (llama2/vxmath.cpp:148-221) without copying the weights. */
typedef struct {
  uint64_t W_addr;
  uint64_t C_addr;
  int32_t rows;
  int32_t reserved;
} akili_matvec_seg_t;

/* ---- the kb2_* SIMT family: fp32 operands, fp32 arithmetic --------------
 * benchmarks/kb2_<bench>/common.h: the same ops without the Vortex launch
 * fields.  Their plain entries keep fp32 semantics (no fp16 rounding of the
 * operands): the GEMM runs on the tensor cores with each operand split into
 * two fp16 parts, x = hi + lo, and S = A_hi.B_hi + A_hi.B_lo + A_lo.B_hi
 * accumulated in fp32 (relative error about 2^-21 per product; operands
 * must lie within fp16's range, |x| < 65504). */
typedef struct {                 /* kb2_gemm_add_relu/common.h:4-12 */
  uint32_t M, N, K;
  uint64_t a_addr, w_addr, bias_addr, c_addr;
} kb2_gemm_add_relu_arg_t;
typedef struct {                 /* kb2_gemm_mul_leakyrelu/common.h */
  uint32_t M, N, K;
  float multiplier, negative_slope;
  uint64_t a_addr, w_addr, bias_addr, c_addr;
} kb2_gemm_mul_leakyrelu_arg_t;
typedef struct {                 /* kb2_gemm_div_sum_scale/common.h */
  uint32_t M, N, K;
  float scaling_factor;
  uint64_t a_addr, w_addr, c_addr;
} kb2_gemm_div_sum_scale_arg_t;
typedef struct {                 /* kb2_gemm_layernorm/common.h */
  uint32_t M, N, K;
  float eps;
  uint64_t a_addr, w_addr, bias_addr, ln_w_addr, ln_b_addr, c_addr;
} kb2_gemm_layernorm_arg_t;
typedef struct {                 /* kb2_attention_score/common.h */
  uint32_t M, N, D;
  uint64_t q_addr, k_addr, c_addr;
} kb2_attention_score_arg_t;
typedef struct {                 /* kb2_matmul_softmax/common.h */
  uint32_t M, N, K;
  uint64_t a_addr, b_addr, c_addr;
} kb2_matmul_softmax_arg_t;
typedef struct {                 /* kb2_matmul_scale_residadd_clamp/common.h (adds a bias) */
  uint32_t M, N, K;
  float scale_factor, clamp_min, clamp_max;
  uint64_t a_addr, w_addr, bias_addr, c_addr;
} kb2_matmul_scale_residadd_clamp_arg_t;
typedef struct {                 /* kb2_matmul_sum_max_avgpool/common.h */
  uint32_t M, N, K;
  uint64_t a_addr, w_addr, bias_addr, c_addr;
} kb2_matmul_sum_max_avgpool_arg_t;
typedef struct {                 /* kb2_gemm_rmsnorm_swiglu/common.h (no scratch fields) */
  uint32_t M, N, K;
  float eps;
  uint64_t x_addr, rms_w_addr, wg_addr, wu_addr, c_addr;
} kb2_gemm_rmsnorm_swiglu_arg_t;
typedef struct {                 /* kb2_gemm_silu_mul/common.h */
  uint32_t M, N, K;
  uint64_t a_addr, wa_addr, ba_addr, wb_addr, bb_addr, c_addr;
} kb2_gemm_silu_mul_arg_t;

/* ---- extension block for the fp16 / batched forms ------------------------ */
typedef struct {
  uint32_t abi_version;     /* must be AKILI_ABI_VERSION                                  */
  uint32_t in_dtype;        /* AKILI_DTYPE_F32 or AKILI_DTYPE_F16: activations + weights  */
  uint32_t out_dtype;       /* AKILI_DTYPE_F32 or AKILI_DTYPE_F16                          */
  uint32_t batch;           /* flash: batch size (0 means 1)                               */
  uint32_t heads;           /* flash: heads per batch entry (0 means 1)                    */
  float    softmax_scale;   /* flash: scale of Q.K^T, >= 0 (0 means 1: the unscaled reference) */
  uint32_t causal;          /* flash: 1 masks key j > query i; must be 0 for the other ops */
  uint32_t flags;           /* reserved; must be 0                                         */
  uint64_t workspace;       /* optional device scratch; 0 means the internal pool          */
  uint64_t workspace_bytes; /* size of `workspace`                                         */
} akili_ex_t;
/* Vectors (bias, ln_w, ln_b, rms_w, ba, bb) are fp32 in every form.
 * Scratch fields in the fp16 form: norm_addr holds M*K fp16, gate_addr and
 * temp_addr are not written. */

/* ---- entry points ---------------------------------------------------------
 * Each replaces the device launch of benchmarks/<bench>/kernel.cpp, i.e. the
 * vx_upload_bytes + vx_start + vx_ready_wait sequence of
 * benchmarks/<bench>/main.cpp (line ranges per op below).                   */

/* kbt_sgemm/main.cpp:107-111, device kernel_body kbt_sgemm/kernel.cpp:20-84 */
int akili_kbt_sgemm(const kbt_sgemm_arg_t* arg, akili_stream_t stream);
int akili_kbt_sgemm_ex(const kbt_sgemm_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* kbt_gemm_add_relu/main.cpp:114-118, kernel.cpp:23-88 */
int akili_kbt_gemm_add_relu(const kbt_gemm_add_relu_arg_t* arg, akili_stream_t stream);
int akili_kbt_gemm_add_relu_ex(const kbt_gemm_add_relu_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* kbt_gemm_mul_leakyrelu/main.cpp:120-124, kernel.cpp:23-90 */
int akili_kbt_gemm_mul_leakyrelu(const kbt_gemm_mul_leakyrelu_arg_t* arg, akili_stream_t stream);
int akili_kbt_gemm_mul_leakyrelu_ex(const kbt_gemm_mul_leakyrelu_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* kbt_gemm_div_sum_scale/main.cpp:110-114, kernel.cpp:24-95 */
int akili_kbt_gemm_div_sum_scale(const kbt_gemm_div_sum_scale_arg_t* arg, akili_stream_t stream);
int akili_kbt_gemm_div_sum_scale_ex(const kbt_gemm_div_sum_scale_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* kbt_gemm_layernorm/main.cpp:136-140, kernel.cpp:24-113 */
int akili_kbt_gemm_layernorm(const kbt_gemm_layernorm_arg_t* arg, akili_stream_t stream);
int akili_kbt_gemm_layernorm_ex(const kbt_gemm_layernorm_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* No counterpart in the reference: a form of kbt_gemm_layernorm that never
 * allocates device memory, for callers that cannot call cudaMalloc — e.g. a
 * serving process whose allocator has already reserved the GPU's memory, or
 * a plugin host whose execute callback must not allocate because cudaMalloc /
 * cudaFree would synchronise the device in the middle of its stream work.
 * The caller passes inputs and outputs as for akili_kbt_gemm_layernorm_ex;
 * operands must be fp16 (ex->in_dtype = AKILI_DTYPE_F16, output fp16 or
 * fp32) and ex->workspace must be 0.  The only scratch, the per-row LayerNorm
 * partial statistics and (for M > 128) one arrival counter per 128-row
 * block, lives in a fixed device array of AKILI_NOALLOC_SCRATCH_BYTES inside
 * the library (held by every GPU that loads it until exit); a problem needing
 * more, i.e. 16 * M * ceil(N / 256) bytes of statistics plus
 * 8 * ceil(M / 256) bytes of counters (each rounded up to 256 bytes)
 * > AKILI_NOALLOC_SCRATCH_BYTES, returns AKILI_E_SCRATCH_LIMIT (M = 16384 at
 * N = 4096 fits).  Each call zeroes the counters on its stream before its
 * GEMM.  The first call on a device looks up that array's device address
 * (once per device and CUDA context, with the device current; after a device
 * reset the next call looks it up again); make that first call before any
 * stream capture.  All calls share the array: calls that overlap on the
 * GPU (different streams, or different host threads on one device) race on
 * it and must be serialised by the caller. */
#define AKILI_NOALLOC_SCRATCH_BYTES ((4u << 20) + (64u << 10))
int akili_kbt_gemm_layernorm_noalloc(const kbt_gemm_layernorm_arg_t* arg, const akili_ex_t* ex,
                                     akili_stream_t stream);

/* kbt_attention_score/main.cpp:107-111, kernel.cpp:25-113 */
int akili_kbt_attention_score(const kbt_attention_score_arg_t* arg, akili_stream_t stream);
int akili_kbt_attention_score_ex(const kbt_attention_score_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* kbt_matmul_softmax/main.cpp:107-111, kernel.cpp:24-105 */
int akili_kbt_matmul_softmax(const kbt_matmul_softmax_arg_t* arg, akili_stream_t stream);
int akili_kbt_matmul_softmax_ex(const kbt_matmul_softmax_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* kbt_matmul_scale_residadd_clamp/main.cpp:119-123, kernel.cpp:24-117 */
int akili_kbt_matmul_scale_residadd_clamp(const kbt_matmul_scale_residadd_clamp_arg_t* arg, akili_stream_t stream);
int akili_kbt_matmul_scale_residadd_clamp_ex(const kbt_matmul_scale_residadd_clamp_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* kbt_matmul_sum_max_avgpool/main.cpp:114-118, kernel.cpp:25-96 */
int akili_kbt_matmul_sum_max_avgpool(const kbt_matmul_sum_max_avgpool_arg_t* arg, akili_stream_t stream);
int akili_kbt_matmul_sum_max_avgpool_ex(const kbt_matmul_sum_max_avgpool_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* kbt_gemm_rmsnorm_swiglu/main.cpp:137-141, kernel.cpp:70-124 */
int akili_kbt_gemm_rmsnorm_swiglu(const kbt_gemm_rmsnorm_swiglu_arg_t* arg, akili_stream_t stream);
int akili_kbt_gemm_rmsnorm_swiglu_ex(const kbt_gemm_rmsnorm_swiglu_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* kbt_gemm_silu_mul/main.cpp:136-140, kernel.cpp:25-146 */
int akili_kbt_gemm_silu_mul(const kbt_gemm_silu_mul_arg_t* arg, akili_stream_t stream);
int akili_kbt_gemm_silu_mul_ex(const kbt_gemm_silu_mul_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* flash/main.cpp:299-307, device entry flash_kernel_entry flash/kernel.cpp:344-417 */
int akili_flash(const flash_arg_t* arg, akili_stream_t stream);
int akili_flash_ex(const flash_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* Flash forward that also writes each query row's softmax statistics, as
 * the reference's flash kernels keep them in their l and m buffers
 * (benchmarks/cupbop_fmha/fmha_cupbop.cu:42,115-116 and
 * benchmarks/cupbop_dao_flash/dao_flash_cupbop.cu:38,124-125):
 *   m[bh][i] = max_j score_ij,  l[bh][i] = sum_j exp(score_ij - m[bh][i]),
 * score = softmax_scale * Q_i.K_j over the keys the row sees (all, or j <= i
 * with ex->causal = 1).  m_addr and l_addr are device fp32 arrays of
 * batch*heads*seq_len entries, 4-byte aligned; logsumexp = m + log(l). */
int akili_flash_ml_ex(const flash_arg_t* arg, const akili_ex_t* ex, uint64_t m_addr, uint64_t l_addr,
                      akili_stream_t stream);

/* benchmarks/attention/main.cpp:218, :288, :378: each of the
 * three vx_start launches, chosen by arg->kernel_id, on fp32 buffers with
 * fp32 CUDA-core arithmetic (S and O summed in the reference's order). */
int akili_attention(const attention_arg_t* arg, akili_stream_t stream);
/* The same launches for batch * heads heads stored one after another (Q, V,
 * O: [heads][N][d]; K: [heads][d][N]; S, P: [heads][N][N]) with the
 * softmax taken of ex->softmax_scale * S.  fp32 buffers run the exact fp32
 * kernels above head by head; fp16 buffers (ex in_dtype = out_dtype = F16;
 * N and d multiples of 8) run the two products on the tensor cores (fp32
 * accumulation, fp16 S and O) and the softmax as one HBM pass over all rows.
 * ex->causal must be 0. */
int akili_attention_ex(const attention_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* llama2/vxmath.cpp:82-141 (vx_matmul_optimized: one vx_start of
 * llama2/matmul_kernel.cpp:4-24 per call): C = A.B in fp32.  N = 1 runs an
 * HBM-bound matrix-vector kernel; N > 1 with M, N, K multiples of 8 and
 * 16-byte aligned pointers runs the tensor-core GEMM in split precision
 * (fp32-level accuracy); other shapes run a tiled fp32 CUDA-core kernel.
 * Pointers need 4-byte alignment; M, N or K may be 0 (K = 0 writes zeros). */
int akili_llama2_matmul(const matmul_kernel_args_t* arg, akili_stream_t stream);

/* The batched products of llama2/vxmath.cpp:143-221 (QKV, FFN w1/w3) as one
 * launch: for each of the nseg (1..4) segments, C_s = W_s . x, W_s row-major
 * [rows_s x K], x and C_s fp32 device vectors. */
int akili_llama2_matvec_batch(const akili_matvec_seg_t* segs, int nseg, uint64_t x_addr, int32_t K,
                              akili_stream_t stream);

/* kb2_* entries: each replaces the vx_upload_bytes + vx_start +
 * vx_ready_wait sequence of benchmarks/kb2_<bench>/main.cpp.  fp32 buffers,
 * fp32 results (see the kb2 structs above); the `_ex` form takes an
 * akili_ex_t only for its workspace (dtype fields must be F32, causal 0). */
/* benchmarks/kb2_gemm_add_relu/main.cpp:104-108 */
int akili_kb2_gemm_add_relu(const kb2_gemm_add_relu_arg_t* arg, akili_stream_t stream);
int akili_kb2_gemm_add_relu_ex(const kb2_gemm_add_relu_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);
/* benchmarks/kb2_gemm_mul_leakyrelu/main.cpp:110-114 */
int akili_kb2_gemm_mul_leakyrelu(const kb2_gemm_mul_leakyrelu_arg_t* arg, akili_stream_t stream);
int akili_kb2_gemm_mul_leakyrelu_ex(const kb2_gemm_mul_leakyrelu_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);
/* benchmarks/kb2_gemm_div_sum_scale/main.cpp:100-104 */
int akili_kb2_gemm_div_sum_scale(const kb2_gemm_div_sum_scale_arg_t* arg, akili_stream_t stream);
int akili_kb2_gemm_div_sum_scale_ex(const kb2_gemm_div_sum_scale_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);
/* benchmarks/kb2_gemm_layernorm/main.cpp:121-125 */
int akili_kb2_gemm_layernorm(const kb2_gemm_layernorm_arg_t* arg, akili_stream_t stream);
int akili_kb2_gemm_layernorm_ex(const kb2_gemm_layernorm_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);
/* benchmarks/kb2_attention_score/main.cpp:96-100 */
int akili_kb2_attention_score(const kb2_attention_score_arg_t* arg, akili_stream_t stream);
int akili_kb2_attention_score_ex(const kb2_attention_score_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);
/* benchmarks/kb2_matmul_softmax/main.cpp:96-100 */
int akili_kb2_matmul_softmax(const kb2_matmul_softmax_arg_t* arg, akili_stream_t stream);
int akili_kb2_matmul_softmax_ex(const kb2_matmul_softmax_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);
/* benchmarks/kb2_matmul_scale_residadd_clamp/main.cpp:112-116 */
int akili_kb2_matmul_scale_residadd_clamp(const kb2_matmul_scale_residadd_clamp_arg_t* arg, akili_stream_t stream);
int akili_kb2_matmul_scale_residadd_clamp_ex(const kb2_matmul_scale_residadd_clamp_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);
/* benchmarks/kb2_matmul_sum_max_avgpool/main.cpp:104-108 */
int akili_kb2_matmul_sum_max_avgpool(const kb2_matmul_sum_max_avgpool_arg_t* arg, akili_stream_t stream);
int akili_kb2_matmul_sum_max_avgpool_ex(const kb2_matmul_sum_max_avgpool_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);
/* benchmarks/kb2_gemm_rmsnorm_swiglu/main.cpp:115-119 */
int akili_kb2_gemm_rmsnorm_swiglu(const kb2_gemm_rmsnorm_swiglu_arg_t* arg, akili_stream_t stream);
int akili_kb2_gemm_rmsnorm_swiglu_ex(const kb2_gemm_rmsnorm_swiglu_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);
/* benchmarks/kb2_gemm_silu_mul/main.cpp:118-122 */
int akili_kb2_gemm_silu_mul(const kb2_gemm_silu_mul_arg_t* arg, akili_stream_t stream);
int akili_kb2_gemm_silu_mul_ex(const kb2_gemm_silu_mul_arg_t* arg, const akili_ex_t* ex, akili_stream_t stream);

/* ---- runtime helpers (no counterpart in the reference beyond RT_CHECK) --- */

/* Human-readable text for an AKILI_E_* code (static storage). */
const char* akili_strerror(int code);

/* Bytes of scratch an `_ex` call with these arguments uses; `op` is the
 * benchmark name without the akili_ prefix, e.g. "kbt_gemm_layernorm".  The
 * `arg` pointer must point at that op's struct.  Returns AKILI_OK. */
int akili_workspace_bytes(const char* op, const void* arg, const akili_ex_t* ex, uint64_t* bytes);

/* One kbt_* / kb2_* GEMM op, or "flash", on HOST buffers: every *_addr field
 * of `arg` (named by `op`, e.g. "kbt_gemm_add_relu") is a host address.  Replaces the
 * harness's whole device round trip (vx_copy_to_dev of the inputs, vx_start,
 * vx_ready_wait, vx_copy_from_dev of the output; e.g.
 * kbt_gemm_add_relu/main.cpp:110-120).  W and the vectors are copied once;
 * the rows then go through in chunks with the host->device copy, the fused
 * GEMM and the device->host copy of successive chunks overlapped on three
 * streams (compute on `stream`).  Returns when the output is in host memory.
 * Page-locked host buffers (cudaHostAlloc / cudaHostRegister) let the copies
 * overlap; pageable ones work but serialise.  The scratch fields (norm, gate,
 * temp) are not written.  ex as for the op's _ex entry (for the GEMM ops
 * batch, heads and causal must be defaults); NULL = fp32 in and out.  Flash
 * goes through in chunks of heads (flash/main.cpp:279-311 is its round
 * trip).  The device buffers it
 * stages through (W and the vectors, three row-chunk slots) are kept per
 * device, grow-only, for later calls until the process exits; calls on one
 * device are serialised by a lock. */
int akili_host_call(const char* op, const void* arg, const akili_ex_t* ex, akili_stream_t stream);

/* Device status word of the current device: 0 when no kernel has timed out
 * on a device-side wait since the last clear, else the code of the first wait
 * that gave up.  Synchronises the device. `clear` != 0 resets it. */
int akili_device_status(uint32_t* status, int clear);

/* Self-test of device-side failure detection: launches one CTA that waits
 * on an mbarrier nothing arrives at, with a limit of `limit_us` microseconds
 * (1..1000000).  The wait gives up, records AKILI_STATUS_SELFTEST in the
 * status word and the kernel returns; the context stays usable.  Returns
 * AKILI_OK once launched; read the outcome with akili_device_status(). */
#define AKILI_STATUS_SELFTEST 0x100Cu
int akili_selftest_wait_timeout(uint32_t limit_us, akili_stream_t stream);

/* Number of kernel launches this library has issued in this process
 * (all devices).  For launch accounting in benchmarks. */
uint64_t akili_launch_count(void);

/* SM clock of the library's own kernels, for benchmarks (no counterpart in
 * the reference).  CTA 0 of every GEMM, flash, fused-softmax and
 * matrix-vector launch adds the SM cycles and globaltimer nanoseconds from
 * its entry to its exit to two device counters of the current device.
 * Returns them in *cycles / *ns; cycles / ns * 1000 is the SM clock in MHz
 * those launches ran at.  Synchronises the device; `clear` != 0 resets the
 * counters. */
int akili_sm_clock_read(uint64_t* cycles, uint64_t* ns, int clear);

/* ABI version compiled into the library. */
uint32_t akili_abi_version(void);

#ifdef __cplusplus
} /* extern "C" */

/* Layout checks against the reference structs (offsets measured with g++ on
 * x86-64 from benchmarks/<bench>/common.h; the same natural alignment holds
 * on RV64). */
#define AKILI_CHECK_LAYOUT(T, sz) static_assert(sizeof(T) == (sz), #T " size")
AKILI_CHECK_LAYOUT(kbt_sgemm_arg_t, 64);
AKILI_CHECK_LAYOUT(kbt_gemm_add_relu_arg_t, 72);
AKILI_CHECK_LAYOUT(kbt_gemm_mul_leakyrelu_arg_t, 80);
AKILI_CHECK_LAYOUT(kbt_gemm_div_sum_scale_arg_t, 64);
AKILI_CHECK_LAYOUT(kbt_gemm_layernorm_arg_t, 88);
AKILI_CHECK_LAYOUT(kbt_attention_score_arg_t, 64);
AKILI_CHECK_LAYOUT(kbt_matmul_softmax_arg_t, 64);
AKILI_CHECK_LAYOUT(kbt_matmul_scale_residadd_clamp_arg_t, 80);
AKILI_CHECK_LAYOUT(kbt_matmul_sum_max_avgpool_arg_t, 72);
AKILI_CHECK_LAYOUT(kbt_gemm_rmsnorm_swiglu_arg_t, 96);
AKILI_CHECK_LAYOUT(kbt_gemm_silu_mul_arg_t, 96);
AKILI_CHECK_LAYOUT(flash_arg_t, 64);
AKILI_CHECK_LAYOUT(akili_ex_t, 48);
AKILI_CHECK_LAYOUT(attention_arg_t, 72);
static_assert(offsetof(attention_arg_t, N) == 8 && offsetof(attention_arg_t, Q_addr) == 16 &&
              offsetof(attention_arg_t, O_addr) == 56 && offsetof(attention_arg_t, kernel_id) == 64,
              "attention offsets");
AKILI_CHECK_LAYOUT(matmul_kernel_args_t, 56);
static_assert(offsetof(matmul_kernel_args_t, A_addr) == 16 && offsetof(matmul_kernel_args_t, C_addr) == 32 &&
              offsetof(matmul_kernel_args_t, M) == 40 && offsetof(matmul_kernel_args_t, K) == 48,
              "matmul_kernel_args_t offsets");
AKILI_CHECK_LAYOUT(akili_matvec_seg_t, 24);
AKILI_CHECK_LAYOUT(kb2_gemm_add_relu_arg_t, 48);
AKILI_CHECK_LAYOUT(kb2_gemm_mul_leakyrelu_arg_t, 56);
AKILI_CHECK_LAYOUT(kb2_gemm_div_sum_scale_arg_t, 40);
AKILI_CHECK_LAYOUT(kb2_gemm_layernorm_arg_t, 64);
AKILI_CHECK_LAYOUT(kb2_attention_score_arg_t, 40);
AKILI_CHECK_LAYOUT(kb2_matmul_softmax_arg_t, 40);
AKILI_CHECK_LAYOUT(kb2_matmul_scale_residadd_clamp_arg_t, 56);
AKILI_CHECK_LAYOUT(kb2_matmul_sum_max_avgpool_arg_t, 48);
AKILI_CHECK_LAYOUT(kb2_gemm_rmsnorm_swiglu_arg_t, 56);
AKILI_CHECK_LAYOUT(kb2_gemm_silu_mul_arg_t, 64);
static_assert(offsetof(kb2_gemm_add_relu_arg_t, a_addr) == 16 && offsetof(kb2_gemm_add_relu_arg_t, c_addr) == 40,
              "kb2_gemm_add_relu offsets");
static_assert(offsetof(kb2_matmul_scale_residadd_clamp_arg_t, clamp_max) == 20 &&
              offsetof(kb2_matmul_scale_residadd_clamp_arg_t, a_addr) == 24, "kb2 clamp offsets");
static_assert(offsetof(kb2_gemm_layernorm_arg_t, eps) == 12 && offsetof(kb2_gemm_layernorm_arg_t, c_addr) == 56,
              "kb2_gemm_layernorm offsets");
static_assert(offsetof(kbt_sgemm_arg_t, M) == 24 && offsetof(kbt_sgemm_arg_t, a_addr) == 40 &&
              offsetof(kbt_sgemm_arg_t, c_addr) == 56, "kbt_sgemm offsets");
static_assert(offsetof(kbt_gemm_mul_leakyrelu_arg_t, multiplier) == 36 &&
              offsetof(kbt_gemm_mul_leakyrelu_arg_t, a_addr) == 48, "mul_leakyrelu offsets");
static_assert(offsetof(kbt_gemm_layernorm_arg_t, eps) == 36 &&
              offsetof(kbt_gemm_layernorm_arg_t, c_addr) == 80, "layernorm offsets");
static_assert(offsetof(kbt_matmul_scale_residadd_clamp_arg_t, clamp_max) == 44 &&
              offsetof(kbt_matmul_scale_residadd_clamp_arg_t, temp_addr) == 72, "clamp offsets");
static_assert(offsetof(kbt_gemm_rmsnorm_swiglu_arg_t, x_addr) == 40 &&
              offsetof(kbt_gemm_rmsnorm_swiglu_arg_t, c_addr) == 88, "swiglu offsets");
static_assert(offsetof(kbt_gemm_silu_mul_arg_t, bb_addr) == 72 &&
              offsetof(kbt_gemm_silu_mul_arg_t, c_addr) == 88, "silu_mul offsets");
static_assert(offsetof(flash_arg_t, kernel_type) == 8 && offsetof(flash_arg_t, block_size_c) == 24 &&
              offsetof(flash_arg_t, Q_addr) == 32 && offsetof(flash_arg_t, O_addr) == 56, "flash offsets");
#undef AKILI_CHECK_LAYOUT
#endif

#endif /* AKILI_H_ */
