"""torch front end of the C ABI: one function per akili-bench op.

Each function fills the op's reference ``kernel_arg_t`` (abi.OPS) with the
device addresses of CUDA tensors and calls ``akili_<bench>`` (fp32 tensors,
reference semantics) or ``akili_<bench>_ex`` (fp16 inputs and/or fp16
output).  The CUDA path is the only path: a missing library or a non-zero
status raises.  Shapes follow the reference: x/a [M, K], W [K, N] row-major,
per-column vectors fp32 [N]; attention-score K is [N, D]; flash tensors are
[B, H, S, D] (or [S, D] for one head).
"""
from __future__ import annotations

import ctypes as C
import threading

import torch

from . import abi


def _stream(stream) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _addr(t: torch.Tensor | None) -> int:
    if t is None:
        return 0
    assert t.is_cuda and t.is_contiguous(), "akili ops take contiguous CUDA tensors"
    return int(t.data_ptr())


_tls = threading.local()


def _a(t: torch.Tensor | None) -> int:
    """Address of an operand of a kbt_* GEMM op: CUDA tensors for the device
    entry, CPU tensors (page-locked to overlap) for akili_host_call.  The
    places of one call's operands are checked together in _launch."""
    if t is None:
        return 0
    assert t.is_contiguous(), "akili ops take contiguous tensors"
    places = getattr(_tls, "places", None)
    if places is None:
        _tls.places = places = set()
    places.add(bool(t.is_cuda))
    return int(t.data_ptr())


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.float16:
        return abi.DTYPE_F16
    if t.dtype == torch.float32:
        return abi.DTYPE_F32
    raise TypeError(f"unsupported dtype {t.dtype}")


def _launch(op: str, arg, in_t: torch.Tensor, out_t: torch.Tensor, stream=None, ex_extra=None,
            workspace: torch.Tensor | None = None) -> None:
    places = getattr(_tls, "places", None) or set()
    _tls.places = set()
    on_gpu = bool(in_t.is_cuda)
    if places and places != {on_gpu}:
        raise ValueError(f"akili_{op}: all tensors of one call must be CUDA tensors, or all host tensors")
    plain = in_t.dtype == torch.float32 and out_t.dtype == torch.float32 and not ex_extra and workspace is None
    ex = None
    if not plain:
        ex = abi.make_ex(_dt(in_t), _dt(out_t), **(ex_extra or {}))
        if workspace is not None:
            ex.workspace = _addr(workspace)
            ex.workspace_bytes = workspace.numel() * workspace.element_size()
    if on_gpu:
        abi.check(op, arg, ex, _stream(stream))
        return
    # host tensors: the pipelined copy-in / run / copy-out of akili_host_call
    if workspace is not None:
        raise ValueError("a device workspace does not apply to a host call")
    rc = abi.load().akili_host_call(op.encode(), C.byref(arg), C.byref(ex) if ex is not None else None,
                                    C.c_void_p(_stream(stream)))
    if rc != abi.OK:
        raise abi.AkiliError(f"host_call({op})", rc)


def _hdr(st, M, N, K, kname="K"):
    a = st()
    a.grid_dim[0] = (M + 7) // 8
    a.grid_dim[1] = a.grid_dim[2] = 1
    a.block_dim[0] = 8
    a.block_dim[1] = a.block_dim[2] = 1
    a.M, a.N = M, N
    setattr(a, kname, K)
    return a


def _out(x, M, N, out_dtype, out):
    if out is not None:
        return out
    shape = (M, N) if N is not None else (M,)
    return torch.empty(shape, device=x.device, dtype=out_dtype or x.dtype, pin_memory=not x.is_cuda)


def kbt_sgemm(a, b, out=None, out_dtype=None, stream=None):
    M, K = a.shape
    N = b.shape[1]
    c = _out(a, M, N, out_dtype or torch.float32, out)
    arg = _hdr(abi.KbtSgemmArg, M, N, K)
    arg.a_addr, arg.b_addr, arg.c_addr = _a(a), _a(b), _a(c)
    _launch("kbt_sgemm", arg, a, c, stream)
    return c


def kbt_gemm_add_relu(x, w, bias, out=None, out_dtype=None, stream=None, workspace=None):
    M, K = x.shape
    N = w.shape[1]
    c = _out(x, M, N, out_dtype, out)
    arg = _hdr(abi.KbtGemmAddReluArg, M, N, K)
    arg.a_addr, arg.w_addr, arg.bias_addr, arg.c_addr = _a(x), _a(w), _a(bias), _a(c)
    _launch("kbt_gemm_add_relu", arg, x, c, stream, workspace=workspace)
    return c


def kbt_gemm_mul_leakyrelu(x, w, bias, multiplier=1.5, negative_slope=0.01, out=None, out_dtype=None,
                           stream=None):
    M, K = x.shape
    N = w.shape[1]
    c = _out(x, M, N, out_dtype, out)
    arg = _hdr(abi.KbtGemmMulLeakyreluArg, M, N, K)
    arg.multiplier, arg.negative_slope = multiplier, negative_slope
    arg.a_addr, arg.w_addr, arg.bias_addr, arg.c_addr = _a(x), _a(w), _a(bias), _a(c)
    _launch("kbt_gemm_mul_leakyrelu", arg, x, c, stream)
    return c


def kbt_gemm_div_sum_scale(x, w, scaling_factor=2.0, out=None, out_dtype=torch.float32, stream=None):
    M, K = x.shape
    N = w.shape[1]
    c = _out(x, M, None, out_dtype, out)
    arg = _hdr(abi.KbtGemmDivSumScaleArg, M, N, K)
    arg.scaling_factor = scaling_factor
    arg.a_addr, arg.w_addr, arg.c_addr = _a(x), _a(w), _a(c)
    _launch("kbt_gemm_div_sum_scale", arg, x, c, stream)
    return c


def kbt_gemm_layernorm(x, w, bias, ln_w, ln_b, eps=1e-5, out=None, out_dtype=None, stream=None, workspace=None):
    M, K = x.shape
    N = w.shape[1]
    c = _out(x, M, N, out_dtype, out)
    arg = _hdr(abi.KbtGemmLayernormArg, M, N, K)
    arg.eps = eps
    arg.a_addr, arg.w_addr, arg.bias_addr = _a(x), _a(w), _a(bias)
    arg.ln_w_addr, arg.ln_b_addr, arg.c_addr = _a(ln_w), _a(ln_b), _a(c)
    _launch("kbt_gemm_layernorm", arg, x, c, stream, workspace=workspace)
    return c


def kbt_attention_score(q, k, out=None, out_dtype=None, stream=None):
    M, D = q.shape
    N = k.shape[0]
    c = _out(q, M, N, out_dtype, out)
    arg = _hdr(abi.KbtAttentionScoreArg, M, N, D, kname="D")
    arg.q_addr, arg.k_addr, arg.c_addr = _a(q), _a(k), _a(c)
    _launch("kbt_attention_score", arg, q, c, stream)
    return c


def kbt_matmul_softmax(a, b, out=None, out_dtype=None, stream=None):
    M, K = a.shape
    N = b.shape[1]
    c = _out(a, M, N, out_dtype, out)
    arg = _hdr(abi.KbtMatmulSoftmaxArg, M, N, K)
    arg.a_addr, arg.b_addr, arg.c_addr = _a(a), _a(b), _a(c)
    _launch("kbt_matmul_softmax", arg, a, c, stream)
    return c


def kbt_matmul_scale_residadd_clamp(a, b, scale_factor=0.5, clamp_min=-2.0, clamp_max=2.0, temp=None, out=None,
                                    out_dtype=torch.float32, stream=None):
    M, K = a.shape
    N = b.shape[1]
    c = _out(a, M, None, out_dtype, out)
    arg = _hdr(abi.KbtMatmulScaleResidaddClampArg, M, N, K)
    arg.scale_factor, arg.clamp_min, arg.clamp_max = scale_factor, clamp_min, clamp_max
    arg.a_addr, arg.b_addr, arg.c_addr, arg.temp_addr = _a(a), _a(b), _a(c), _a(temp)
    _launch("kbt_matmul_scale_residadd_clamp", arg, a, c, stream)
    return c


def kbt_matmul_sum_max_avgpool(x, w, bias, out=None, out_dtype=torch.float32, stream=None):
    M, K = x.shape
    N = w.shape[1]
    c = _out(x, M, None, out_dtype, out)
    arg = _hdr(abi.KbtMatmulSumMaxAvgpoolArg, M, N, K)
    arg.a_addr, arg.w_addr, arg.bias_addr, arg.c_addr = _a(x), _a(w), _a(bias), _a(c)
    _launch("kbt_matmul_sum_max_avgpool", arg, x, c, stream)
    return c


def kbt_gemm_rmsnorm_swiglu(x, rms_w, wg, wu, eps=1e-5, norm=None, out=None, out_dtype=None, stream=None):
    M, K = x.shape
    N = wg.shape[1]
    c = _out(x, M, N, out_dtype, out)
    arg = _hdr(abi.KbtGemmRmsnormSwigluArg, M, N, K)
    arg.eps = eps
    arg.x_addr, arg.rms_w_addr, arg.wg_addr, arg.wu_addr = _a(x), _a(rms_w), _a(wg), _a(wu)
    arg.norm_addr, arg.gate_addr, arg.c_addr = _a(norm), 0, _a(c)
    _launch("kbt_gemm_rmsnorm_swiglu", arg, x, c, stream)
    return c


def kbt_gemm_silu_mul(x, wa, ba, wb, bb, out=None, out_dtype=None, stream=None):
    M, K = x.shape
    N = wa.shape[1]
    c = _out(x, M, N, out_dtype, out)
    arg = _hdr(abi.KbtGemmSiluMulArg, M, N, K)
    arg.a_addr, arg.wa_addr, arg.ba_addr = _a(x), _a(wa), _a(ba)
    arg.wb_addr, arg.bb_addr, arg.gate_addr, arg.c_addr = _a(wb), _a(bb), 0, _a(c)
    _launch("kbt_gemm_silu_mul", arg, x, c, stream)
    return c


def flash(q, k, v, softmax_scale=None, out=None, out_dtype=None, stream=None, kernel_type=1, causal=False,
          return_stats=False):
    """q/k/v [S, D] (one head, reference layout) or [B, H, S, D].

    kernel_type follows the reference's flash_arg_t: 1 = its fp16 tensor-core
    flash (operands rounded to fp16), 0 = its fp32 SIMT flash (with fp32
    inputs the scores are computed in split precision).  causal=True masks
    keys after each query (cupbop_dao_flash).  return_stats=True also returns
    the per-row softmax statistics (m, l), fp32 shaped like q without its
    last dimension: m = row max of the scaled scores, l = sum exp(score - m)."""
    if q.dim() == 2:
        B, H, (S, D) = 1, 1, q.shape
    else:
        B, H, S, D = q.shape
    o = out if out is not None else torch.empty(q.shape, device=q.device, dtype=out_dtype or q.dtype,
                                                pin_memory=not q.is_cuda)
    arg = abi.FlashArg()
    arg.grid_dim[0] = (S + 7) // 8
    arg.block_dim[0] = 8
    arg.kernel_type = kernel_type
    arg.seq_len, arg.head_dim = S, D
    arg.block_size_r = arg.block_size_c = 8
    if not return_stats:  # CPU tensors: the pipelined host call
        arg.Q_addr, arg.K_addr, arg.V_addr, arg.O_addr = _a(q), _a(k), _a(v), _a(o)
    else:
        arg.Q_addr, arg.K_addr, arg.V_addr, arg.O_addr = _addr(q), _addr(k), _addr(v), _addr(o)
    extra = None
    if B * H != 1 or softmax_scale is not None or causal:
        extra = {"batch": B, "heads": H, "softmax_scale": float(softmax_scale or 0.0), "causal": int(causal)}
    if not return_stats:
        _launch("flash", arg, q, o, stream, ex_extra=extra)
        return o
    m = torch.empty(q.shape[:-1], device=q.device, dtype=torch.float32)
    l = torch.empty(q.shape[:-1], device=q.device, dtype=torch.float32)
    ex = abi.make_ex(_dt(q), _dt(o), **(extra or {}))
    rc = abi.load().akili_flash_ml_ex(C.byref(arg), C.byref(ex), _addr(m), _addr(l), C.c_void_p(_stream(stream)))
    if rc != abi.OK:
        raise abi.AkiliError("flash_ml_ex", rc)
    return o, m, l


def kb2_gemm_add_relu(a, w, bias, out=None, stream=None):
    """The fp32 kb2 form: a [M, K], w [K, N], bias [N], out [M, N], all fp32
    (fp32 accuracy through the split-precision GEMM)."""
    M, K = a.shape
    N = w.shape[1]
    c = out if out is not None else torch.empty((M, N), device=a.device, dtype=torch.float32)
    arg = abi.Kb2GemmAddReluArg(M, N, K, _addr(a), _addr(w), _addr(bias), _addr(c))
    abi.check("kb2_gemm_add_relu", arg, None, _stream(stream))
    return c


def attention_unfused(q, k_t, v, softmax_scale=None, s=None, p=None, out=None, stream=None, stages=(0, 1, 2)):
    """The reference's unfused attention (benchmarks/attention/kernel.cpp:6-68)
    over heads [B, H, N, d] (or one head [N, d]): S = Q.K with K stored
    transposed (k_t [B, H, d, N]), P = softmax(softmax_scale * S) by rows,
    O = P.V, each its own launch with S and P materialised.  fp32 tensors run
    the exact fp32 kernels, fp16 tensors the tensor-core path.  Returns
    (O, S, P)."""
    if q.dim() == 2:
        B, H, (N, d) = 1, 1, q.shape
    else:
        B, H, N, d = q.shape
    lead = q.shape[:-2]
    s = s if s is not None else torch.empty((*lead, N, N), device=q.device, dtype=q.dtype)
    p = p if p is not None else torch.empty((*lead, N, N), device=q.device, dtype=q.dtype)
    o = out if out is not None else torch.empty(q.shape, device=q.device, dtype=q.dtype)
    ex = abi.make_ex(_dt(q), _dt(o), batch=B, heads=H, softmax_scale=float(softmax_scale or 0.0))
    arg = abi.AttentionArg()
    arg.N, arg.d = N, d
    arg.Q_addr, arg.K_addr, arg.S_addr = _addr(q), _addr(k_t), _addr(s)
    arg.P_addr, arg.V_addr, arg.O_addr = _addr(p), _addr(v), _addr(o)
    L = abi.load()
    for kid in stages:
        arg.kernel_id = kid
        rc = L.akili_attention_ex(C.byref(arg), C.byref(ex), C.c_void_p(_stream(stream)))
        if rc != abi.OK:
            raise abi.AkiliError("attention_ex", rc)
    return o, s, p


def llama2_matmul(a, b, out=None, stream=None):
    """The llama2 matmul offload (benchmarks/llama2/matmul_kernel.cpp):
    out[M, N] = a[M, K] . b[K, N], fp32.  b may be a vector [K] (N = 1, the
    matrix-vector product every llama2 call makes); out then is [M]."""
    M, K = a.shape
    vec = b.dim() == 1
    N = 1 if vec else b.shape[1]
    c = out if out is not None else torch.empty((M,) if vec else (M, N), device=a.device, dtype=torch.float32)
    arg = abi.MatmulKernelArgs()
    arg.block_dim[0], arg.block_dim[1] = 4, 1 if N == 1 else 4
    arg.grid_dim[0], arg.grid_dim[1] = (M + 3) // 4, (N + arg.block_dim[1] - 1) // arg.block_dim[1]
    arg.A_addr, arg.B_addr, arg.C_addr = _addr(a), _addr(b), _addr(c)
    arg.M, arg.N, arg.K = M, N, K
    rc = abi.load().akili_llama2_matmul(C.byref(arg), C.c_void_p(_stream(stream)))
    if rc != abi.OK:
        raise abi.AkiliError("llama2_matmul", rc)
    return c


def llama2_matvec_batch(ws, x, outs=None, stream=None):
    """One launch of C_s = W_s . x for up to four weight matrices W_s [rows_s, K]
    (the batched QKV / FFN products of benchmarks/llama2/vxmath.cpp)."""
    K = x.shape[0]
    outs = outs if outs is not None else [torch.empty(w.shape[0], device=x.device, dtype=torch.float32) for w in ws]
    segs = (abi.MatvecSeg * len(ws))()
    for i, (w, o) in enumerate(zip(ws, outs)):
        assert w.shape[1] == K
        segs[i].W_addr, segs[i].C_addr, segs[i].rows = _addr(w), _addr(o), w.shape[0]
    rc = abi.load().akili_llama2_matvec_batch(segs, len(ws), _addr(x), K, C.c_void_p(_stream(stream)))
    if rc != abi.OK:
        raise abi.AkiliError("llama2_matvec_batch", rc)
    return outs


def _haddr(t: torch.Tensor | None) -> int:
    if t is None:
        return 0
    assert not t.is_cuda and t.is_contiguous(), "host calls take contiguous CPU tensors (page-locked to overlap)"
    return int(t.data_ptr())


def host_call(op: str, arg, in_dtype, out_dtype, stream=None) -> None:
    """akili_host_call: `arg` holds HOST addresses; blocks until the output
    is in host memory (copies and the fused GEMM pipelined over row chunks)."""
    ex = None
    if in_dtype != torch.float32 or out_dtype != torch.float32:
        ex = abi.make_ex(abi.DTYPE_F16 if in_dtype == torch.float16 else abi.DTYPE_F32,
                         abi.DTYPE_F16 if out_dtype == torch.float16 else abi.DTYPE_F32)
    rc = abi.load().akili_host_call(op.encode(), C.byref(arg), C.byref(ex) if ex is not None else None,
                                    C.c_void_p(_stream(stream)))
    if rc != abi.OK:
        raise abi.AkiliError(f"host_call({op})", rc)


def kbt_gemm_add_relu_host(x, w, bias, out=None, out_dtype=None, stream=None):
    """kbt_gemm_add_relu on CPU tensors (x [M, K], w [K, N], bias [N] fp32):
    the harness's copy-in / run / copy-out as one pipelined call (every kbt_*
    wrapper above takes this path when its tensors are CPU tensors)."""
    assert not x.is_cuda
    return kbt_gemm_add_relu(x, w, bias, out=out, out_dtype=out_dtype, stream=stream)


def launch_count() -> int:
    return int(abi.load().akili_launch_count())


def selftest_wait_timeout(limit_us: int, stream=None) -> None:
    """Launch a kernel whose one wait can never complete; it gives up after
    limit_us and records STATUS_SELFTEST in the device status word."""
    rc = abi.load().akili_selftest_wait_timeout(int(limit_us), C.c_void_p(_stream(stream)))
    if rc != abi.OK:
        raise abi.AkiliError("selftest_wait_timeout", rc)


STATUS_SELFTEST = 0x100C


def device_status(clear: bool = True) -> int:
    v = C.c_uint32(0)
    abi.load().akili_device_status(C.byref(v), 1 if clear else 0)
    return int(v.value)
