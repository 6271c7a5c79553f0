"""Benchmark of the akili-bench kbt_* / flash hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--op NAME|all]

Default workload (one JSON line, the driver contract): kbt_gemm_add_relu,
ReLU(x.W + b) with x[8192,4096] fp16 ~N(0,1), W[4096,4096] fp16 ~N(0,1/4096),
b[4096] fp32 ~N(0,0.1), fp32 accumulation, fp16 output, per GPU.  Inputs are
seeded synthetic data with the configured shapes and distributions.

* value      whole-job TFLOP/s: 2*M*N*K summed over all ranks, over the
             max-over-ranks device time of the K timed steps (CUDA events on
             the launching stream; L2 flushed before every step, outside the
             events).
* e2e        the same metric through the public C ABI with host buffers:
             pinned host->device copies of x, W, b, the op, and the
             device->host copy of the output, all inside the timed region.
* roofline   the fused GEMM kernel against the measured dense tensor peak.
* cpu_baseline  the oracle (a bit-exact restatement of the reference's CPU
             gold loop) on a bounded row sample, rank 0 at N=1: one thread
             (the reference's serial loop), plus a row-parallel run on all
             host threads as "all_cores".
* --impl reference  times that reference CPU path alone (all host threads).
* clocks     sm_mhz of the timed steps measured on the device: the SM
             cycles over the globaltimer nanoseconds of the steps' own kernels
             (their CTA 0 counts both); throttle reasons from nvidia-smi
             sampled over the soak around them.

Multi-GPU (torchrun, one rank per GPU): by default (--scaling strong) the
configured global problem is split across the ranks -- GEMM rows in
contiguous slices, flash (batch, head) pairs -- with no collective in the
timed loop; a weak-scaling run (every rank the full per-GPU workload)
follows and is reported as the line's "weak" field.  Afterwards sampled
output rows are all-gathered over NCCL and checked on rank 0 against the
oracle.  Each rank binds to its GPU's NUMA node before allocating its
page-locked buffers.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fused fp16 GEMM+epilogue TFLOP/s & % tensor peak, 1/2/4/8 B200"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126 * 1024 * 1024
FLASH_SHAPE = [8, 32, 4096, 128]  # batch, heads, seq, head_dim; --flash-shape overrides

# DRAM bytes (read + write) per launch of the dominant kernel, keyed by
# (workload, rows per GPU), from one ncu capture of that launch
# (dram__bytes_read.sum + dram__bytes_write.sum; the capture runs with ncu's
# cache flush, so every operand is read cold).  Workloads or shapes without
# a capture report null.
NCU_TRAFFIC = {
    # gemm_pair_kernel (row-block-major tiles): 111.52 MB read + 49.44 MB written
    ("kbt_gemm_add_relu", 8192): 160.96e6,
    ("kbt_gemm_mul_leakyrelu", 8192): 164.05e6,  # 114.00 + 50.05
    ("kbt_gemm_div_sum_scale", 8192): 104.84e6,  # 101.00 + 3.84 (row partials only)
    ("kbt_matmul_scale_residadd_clamp", 8192): 106.45e6,  # 101.04 + 5.41
    ("kbt_matmul_sum_max_avgpool", 8192): 104.93e6,  # 101.01 + 3.92
    ("kbt_matmul_softmax", 8192): 158.83e6,  # row-fused: 111.48 + 47.35
    ("kbt_gemm_layernorm", 16384): 302.36e6,  # row-fused: 186.20 + 116.16
    # the dual GEMM (groups of row blocks: its 172 MB of weights exceed L2);
    # the RMSNorm pre-pass before it moves another 167.01 + 88.17 MB
    ("kbt_gemm_rmsnorm_swiglu", 16384): 1592.65e6,  # 1240 + 352.65
    ("kbt_gemm_silu_mul", 16384): 1612.56e6,  # 1260 + 352.56
    ("kb2_gemm_add_relu", 8192): 806.58e6,  # split mode, fp32 in and out: 687.75 + 118.83
    # softmax_rows_kernel: 5.52 MB read + 74.69 MB written (part of the
    # output is still in L2 when the kernel ends)
    ("kbt_attention_score", 16384): 80.21e6,
    ("kbt_sgemm", 128): 0.0876e6,  # gemm_kernel, one tile: 87.55 KB read
    # flash_fwd_kernel at B8 H32 S4096 d128: 805.35 / 805.44 MB read (Q, K, V
    # once) + 247.40 / 251.13 MB written
    ("flash", 0): 1052.75e6,
    ("flash_causal", 0): 1056.57e6,
    # matvec_kernel: the QKV launch moved 207.33 MB for 201.39 MB of
    # algorithmic bytes; scaled by that ratio to one token's 26.43 GB (the
    # whole token's 26 GB of weights is too large for a multi-pass capture)
    ("llama2_7b_decode", 0): 27.21e9,
    # matvec_kernel, the 25 launches of one stories15M token captured with
    # --cache-control none (its 61 MB of weights mostly stay in L2):
    # 23.20 MB read + 4.16 MB written
    ("llama2_stories15m_decode", 0): 27.36e6,
}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ----------------------------------------------------------------- workloads --
class Workload:
    """One op at one shape: device inputs, the call, its algorithmic work."""

    def __init__(self, name, desc, flops, make, call, bound="tensor", io_bytes=None, host=None, cpu=None,
                 kernel="gemm_kernel", metric=None, unit="TFLOP/s", scale=1e12, dtype="f16", graph=False,
                 e2e_host=None, e2e_step=None, cpu_fn=None, host_call=None, scratch=()):
        self.name, self.desc, self.flops, self.make, self.call = name, desc, flops, make, call
        self.bound, self.io_bytes, self.host, self.cpu, self.kernel = bound, io_bytes, host, cpu, kernel
        # `flops` is the work of one step in `unit` * `scale` (FLOPs for TFLOP/s, 1 token for tok/s)
        self.metric, self.unit, self.scale, self.dtype = metric or METRIC, unit, scale, dtype
        # graph: time replays of one step captured as a CUDA graph (launch-bound sequences)
        # e2e_host(d) -> pinned host buffers; e2e_step(d, host, stream) -> (h2d, d2h): one
        # end-to-end step through the public API
        # cpu_fn(d) -> cpu_baseline dict
        self.graph, self.e2e_host, self.e2e_step, self.cpu_fn = graph, e2e_host, e2e_step, cpu_fn
        # host_call: the kbt_* GEMM ops measure e2e through akili_host_call (their
        # ops wrapper on page-locked CPU tensors); scratch: inputs that are not copied
        self.host_call = name.startswith("kbt_") if host_call is None else host_call
        self.scratch = scratch


class Gens:
    """Seeded generators: `w` for weights and per-column vectors (identical on
    every rank: replicated parameters), `x` for activations (per-rank shard)."""

    def __init__(self, torch, rank: int):
        self.w = torch.Generator(device="cuda")
        self.w.manual_seed(1234)
        self.x = torch.Generator(device="cuda")
        self.x.manual_seed(99991 + 7919 * rank)


def _rand(torch, gen, shape, std=1.0, mean=0.0, dtype=None):
    t = torch.randn(shape, generator=gen, device="cuda", dtype=torch.float32) * std + mean
    return t.to(dtype) if dtype is not None else t


class Part:
    """This rank's share of a workload.  "strong": the configured global
    problem is split across the ranks (GEMM rows in multiples of 8, flash
    (batch, head) pairs), as the row / head partition of the multi-GPU layout
    prescribes; "weak": every rank runs the full per-GPU workload.  Workloads
    that do not split (kbt_sgemm's one 128-row tile, llama2 decode) run as
    replicas in both modes."""

    def __init__(self, world: int, rank: int, mode: str):
        self.world, self.rank, self.mode = world, rank, mode

    def rows(self, M: int) -> int:
        if self.mode != "strong":
            return M
        from akili_bench_b200 import shard
        r0, r1 = shard.row_range(M, self.world, self.rank)
        return r1 - r0

    def heads(self, B: int, H: int) -> tuple[int, int]:
        """Local (batch, heads) of a [B, H, S, D] attention workload."""
        if self.mode != "strong":
            return B, H
        from akili_bench_b200 import shard
        u0, u1 = shard.unit_range(B * H, self.world, self.rank)
        n = u1 - u0
        return (n // H, H) if n % H == 0 else (1, n)

    def total(self, local_flops: float, global_flops: float) -> float:
        """Work of one step summed over all ranks."""
        return global_flops if self.mode == "strong" else local_flops * self.world


def workloads(torch, ops, part: "Part | None" = None):
    f16, f32 = torch.float16, torch.float32
    W = {}
    part = part or Part(1, 0, "weak")

    def gemm_inputs(M, N, K, bias_std=0.1, dual=False):
        def make(gen):
            d = {"x": _rand(torch, gen.x, (M, K), dtype=f16), "w": _rand(torch, gen.w, (K, N), K ** -0.5, dtype=f16),
                 "b": _rand(torch, gen.w, (N,), bias_std)}
            if dual:
                d["w2"] = _rand(torch, gen.w, (K, N), K ** -0.5, dtype=f16)
                d["b2"] = _rand(torch, gen.w, (N,), bias_std)
            return d
        return make

    G2, N2, K2 = 8192, 4096, 4096  # the C2 shape; G = global rows, M = this rank's rows
    M2 = part.rows(G2)
    W["kbt_gemm_add_relu"] = Workload(
        "kbt_gemm_add_relu", {"M": M2, "N": N2, "K": K2}, 2.0 * M2 * N2 * K2, gemm_inputs(M2, N2, K2),
        lambda d, out, st: ops.kbt_gemm_add_relu(d["x"], d["w"], d["b"], out=out, stream=st),
        host=("x", "w", "b"), cpu="add_relu")
    W["kbt_gemm_mul_leakyrelu"] = Workload(
        "kbt_gemm_mul_leakyrelu", {"M": M2, "N": N2, "K": K2}, 2.0 * M2 * N2 * K2, gemm_inputs(M2, N2, K2),
        lambda d, out, st: ops.kbt_gemm_mul_leakyrelu(d["x"], d["w"], d["b"], 1.5, 0.01, out=out, stream=st))
    W["kbt_gemm_div_sum_scale"] = Workload(
        "kbt_gemm_div_sum_scale", {"M": M2, "N": N2, "K": K2}, 2.0 * M2 * N2 * K2, gemm_inputs(M2, N2, K2),
        lambda d, out, st: ops.kbt_gemm_div_sum_scale(d["x"], d["w"], 2.0, stream=st))
    W["kbt_matmul_softmax"] = Workload(
        "kbt_matmul_softmax", {"M": M2, "N": N2, "K": K2}, 2.0 * M2 * N2 * K2, gemm_inputs(M2, N2, K2),
        lambda d, out, st: ops.kbt_matmul_softmax(d["x"], d["w"], out=out, stream=st))
    W["kbt_matmul_scale_residadd_clamp"] = Workload(
        "kbt_matmul_scale_residadd_clamp", {"M": M2, "N": N2, "K": K2}, 2.0 * M2 * N2 * K2,
        gemm_inputs(M2, N2, K2),
        lambda d, out, st: ops.kbt_matmul_scale_residadd_clamp(d["x"], d["w"], 0.5, -2.0, 2.0, stream=st))
    W["kbt_matmul_sum_max_avgpool"] = Workload(
        "kbt_matmul_sum_max_avgpool", {"M": M2, "N": N2, "K": K2}, 2.0 * M2 * N2 * K2, gemm_inputs(M2, N2, K2),
        lambda d, out, st: ops.kbt_matmul_sum_max_avgpool(d["x"], d["w"], d["b"], stream=st))

    G3 = 16384
    M3 = part.rows(G3)

    def ln_make(gen):
        d = gemm_inputs(M3, N2, K2, 0.02)(gen)
        d["g"] = _rand(torch, gen.w, (N2,), 0.02, 1.0)
        d["beta"] = _rand(torch, gen.w, (N2,), 0.02)
        return d
    W["kbt_gemm_layernorm"] = Workload(
        "kbt_gemm_layernorm", {"M": M3, "N": N2, "K": K2}, 2.0 * M3 * N2 * K2, ln_make,
        lambda d, out, st: ops.kbt_gemm_layernorm(d["x"], d["w"], d["b"], d["g"], d["beta"], 1e-5, out=out,
                                                  stream=st))

    N4 = 11008

    def sw_make(gen):
        return {"x": _rand(torch, gen.x, (M3, K2), dtype=f16), "rw": _rand(torch, gen.w, (K2,), 0.02, 1.0),
                "wg": _rand(torch, gen.w, (K2, N4), K2 ** -0.5, dtype=f16),
                "wu": _rand(torch, gen.w, (K2, N4), K2 ** -0.5, dtype=f16),
                "norm": torch.empty((M3, K2), device="cuda", dtype=f16)}
    W["kbt_gemm_rmsnorm_swiglu"] = Workload(
        "kbt_gemm_rmsnorm_swiglu", {"M": M3, "N": N4, "K": K2}, 4.0 * M3 * N4 * K2, sw_make,
        lambda d, out, st: ops.kbt_gemm_rmsnorm_swiglu(d["x"], d["rw"], d["wg"], d["wu"], 1e-6, norm=d["norm"],
                                                       out=out, stream=st), scratch=("norm",))
    W["kbt_gemm_silu_mul"] = Workload(
        "kbt_gemm_silu_mul", {"M": M3, "N": N4, "K": K2}, 4.0 * M3 * N4 * K2, gemm_inputs(M3, N4, K2, 0.02, True),
        lambda d, out, st: ops.kbt_gemm_silu_mul(d["x"], d["w"], d["b"], d["w2"], d["b2"], out=out, stream=st))

    # kb2: the fp32 SIMT family's add_relu at the C2 shape, fp32 in and out
    def kb2_make(gen):
        return {"x": _rand(torch, gen.x, (M2, K2)), "w": _rand(torch, gen.w, (K2, N2), K2 ** -0.5),
                "b": _rand(torch, gen.w, (N2,), 0.1)}
    W["kb2_gemm_add_relu"] = Workload(
        "kb2_gemm_add_relu", {"M": M2, "N": N2, "K": K2, "precision": "fp32 (split fp16 hi+lo)"},
        2.0 * M2 * N2 * K2, kb2_make, lambda d, out, st: ops.kb2_gemm_add_relu(d["x"], d["w"], d["b"], out=out,
                                                                               stream=st))

    Ga, Na, Da = 16384, 4096, 128
    Ma = part.rows(Ga)

    def as_make(gen):
        return {"q": _rand(torch, gen.x, (Ma, Da), dtype=f16), "k": _rand(torch, gen.w, (Na, Da), dtype=f16)}
    W["kbt_attention_score"] = Workload(
        "kbt_attention_score", {"M": Ma, "N": Na, "D": Da}, 2.0 * Ma * Na * Da, as_make,
        lambda d, out, st: ops.kbt_attention_score(d["q"], d["k"], out=out, stream=st), bound="hbm",
        io_bytes=2.0 * (Ma * Da + Na * Da) + 2.0 * Ma * Na, kernel="softmax_rows_kernel")

    def sg_make(gen):
        return {"a": (torch.rand((128, 128), generator=gen.x, device="cuda") * 2 - 1).to(f16),
                "bm": (torch.rand((128, 128), generator=gen.w, device="cuda") * 2 - 1).to(f16)}
    W["kbt_sgemm"] = Workload(
        "kbt_sgemm", {"M": 128, "N": 128, "K": 128}, 2.0 * 128 ** 3, sg_make,
        lambda d, out, st: ops.kbt_sgemm(d["a"], d["bm"], out=out, out_dtype=f32, stream=st))

    GB, GH, S, D = FLASH_SHAPE
    B, H = part.heads(GB, GH)

    def fl_make(gen):
        return {k: _rand(torch, gen.x, (B, H, S, D), dtype=f16) for k in ("q", "k", "v")}
    W["flash"] = Workload(
        "flash", {"batch": B, "heads": H, "seq": S, "head_dim": D, "causal": False}, 4.0 * B * H * S * S * D,
        fl_make, lambda d, out, st: ops.flash(d["q"], d["k"], d["v"], softmax_scale=D ** -0.5, out=out, stream=st),
        kernel="flash_fwd_kernel", host_call=True)
    # causal: query i sees keys 0..i, so the useful work is 2*B*H*S*(S+1)*D
    W["flash_causal"] = Workload(
        "flash_causal", {"batch": B, "heads": H, "seq": S, "head_dim": D, "causal": True},
        2.0 * B * H * S * (S + 1) * D, fl_make,
        lambda d, out, st: ops.flash(d["q"], d["k"], d["v"], softmax_scale=D ** -0.5, out=out, stream=st,
                                     causal=True),
        kernel="flash_fwd_kernel", host_call=True)

    # The reference's unfused three-kernel attention (benchmarks/attention) at
    # the flash shape, fp16 on the tensor cores, S and P materialised in HBM:
    # the reference point for what the fused flash kernel saves.
    def au_make(gen):
        return {"q": _rand(torch, gen.x, (B, H, S, D), dtype=f16), "k": _rand(torch, gen.x, (B, H, D, S), dtype=f16),
                "v": _rand(torch, gen.x, (B, H, S, D), dtype=f16),
                "s": torch.empty((B, H, S, S), device="cuda", dtype=f16),
                "p": torch.empty((B, H, S, S), device="cuda", dtype=f16)}
    W["attention_unfused"] = Workload(
        "attention_unfused", {"batch": B, "heads": H, "seq": S, "head_dim": D, "S_P_in_HBM": "fp16"},
        4.0 * B * H * S * S * D, au_make,
        lambda d, out, st: ops.attention_unfused(d["q"], d["k"], d["v"], softmax_scale=D ** -0.5, s=d["s"],
                                                 p=d["p"], out=out, stream=st)[0],
        bound="hbm", io_bytes=2.0 * (4 * B * H * S * D + 4 * B * H * S * S), host=("q", "k", "v"),
        kernel="attention_softmax_f16_kernel", graph=True)

    for key, shape in LLAMA2_SHAPES.items():
        W[key] = llama2_workload(torch, ops, key, *shape)
    # work of one step over all ranks, and the partition each workload uses
    for name, wl in W.items():
        if name.startswith("llama2") or name == "kbt_sgemm":
            wl.split, wl.flops_total = "replicas", wl.flops * part.world
        elif "M" in wl.desc:
            G = {"kbt_gemm_layernorm": G3, "kbt_gemm_rmsnorm_swiglu": G3, "kbt_gemm_silu_mul": G3,
                 "kbt_attention_score": Ga}.get(name, G2)
            wl.split = "rows"
            wl.flops_total = part.total(wl.flops, wl.flops * G / max(1, wl.desc["M"]))
            wl.desc["global_M"] = G if part.mode == "strong" else G * part.world
        else:
            wl.split = "heads"
            wl.flops_total = part.total(wl.flops, wl.flops * (GB * GH) / max(1, B * H))
            wl.desc["global_batch_heads"] = GB * GH if part.mode == "strong" else GB * GH * part.world
    return W


# llama2 decode (benchmarks/llama2/llama.cpp:246-407): per token, per layer the
# batched QKV product, wo, the batched FFN w1/w3 product and w2, then the
# classifier; each a matrix-vector product over fp32 weights resident in HBM.
# (dim, hidden_dim, n_layers, kv_dim, vocab_size)
LLAMA2_SHAPES = {
    "llama2_7b_decode": (4096, 11008, 32, 4096, 32000),
    "llama2_stories15m_decode": (288, 768, 6, 288, 32000),  # the reference's model (llama2/Makefile:9)
}


def llama2_calls(dim, hidden, layers, kv_dim, vocab):
    """The offload calls of one token: (rows of each batched matrix, K)."""
    calls = []
    for _ in range(layers):
        calls += [((dim, kv_dim, kv_dim), dim), ((dim,), dim), ((hidden, hidden), dim), ((dim,), hidden)]
    return calls + [((vocab,), dim)]


def llama2_workload(torch, ops, key, dim, hidden, layers, kv_dim, vocab):
    import ctypes as C

    from akili_bench_b200 import abi
    calls = llama2_calls(dim, hidden, layers, kv_dim, vocab)
    n_w = sum(r * K for rows, K in calls for r in rows)
    n_out = sum(r for rows, _ in calls for r in rows)
    n_in = sum(K for _, K in calls)

    def make(gen):
        d = {"x": {K: _rand(torch, gen.x, (K,)) for K in (dim, hidden)}, "calls": []}
        for rows, K in calls:
            ws = [_rand(torch, gen.w, (r, K), K ** -0.5) for r in rows]
            outs = [torch.empty(r, device="cuda", dtype=torch.float32) for r in rows]
            segs = (abi.MatvecSeg * len(rows))()
            for i, (w, o) in enumerate(zip(ws, outs)):
                segs[i].W_addr, segs[i].C_addr, segs[i].rows = w.data_ptr(), o.data_ptr(), w.shape[0]
            d["calls"].append((segs, len(rows), K, ws, outs))
        return d

    def call(d, out, st):
        L = abi.load()
        s = C.c_void_p(int((st or torch.cuda.current_stream()).cuda_stream))
        for segs, n, K, _, _ in d["calls"]:
            rc = L.akili_llama2_matvec_batch(segs, n, d["x"][K].data_ptr(), K, s)
            if rc != abi.OK:
                raise abi.AkiliError("llama2_matvec_batch", rc)
        return d["calls"][-1][4][0]  # the logits

    def e2e_step(d, host, st):
        """The vxmath API's contract per call (llama2/vxmath.cpp:82-145): the
        activation comes from host memory, the product goes back to host
        memory, and the call returns once it is there."""
        L = abi.load()
        s = C.c_void_p(int(st.cuda_stream))
        h2d = d2h = 0
        for i, (segs, n, K, _, outs) in enumerate(d["calls"]):
            x = d["x"][K]
            x.copy_(host["x"][K], non_blocking=True)
            rc = L.akili_llama2_matvec_batch(segs, n, x.data_ptr(), K, s)
            if rc != abi.OK:
                raise abi.AkiliError("llama2_matvec_batch", rc)
            for o, h in zip(outs, host["y"][i]):
                h.copy_(o, non_blocking=True)
            st.synchronize()
            h2d += 4 * K
            d2h += 4 * sum(o.numel() for o in outs)
        return h2d, d2h

    def e2e_host(d):
        return {"x": {K: v.cpu().pin_memory() for K, v in d["x"].items()},
                "y": [[torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in c[4]] for c in d["calls"]]}

    def cpu_fn(d):
        """The reference's CPU matmul (llama2/llama.cpp:236-243, restated by the
        oracle) on rows of the classifier, scaled to one token."""
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle_py
        threads = host_threads()
        wc = d["calls"][-1][3][0]
        rows = min(wc.shape[0], max(threads * 64, (1 << 22) // dim))
        w = wc[:rows].cpu().numpy()
        x = d["x"][dim].cpu().numpy().reshape(dim, 1)
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0 or reps == 0:
            oracle_py.llama2_matmul(np.ascontiguousarray(w[:rows]), x, rows, 1, dim, threads=threads)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        tok_s = (rows * dim / dt) / n_w
        return {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port",
                "sample": f"{rows} rows x K={dim} of the classifier, {reps} repetitions over {threads} threads, "
                          f"scaled by multiply-adds to one token ({n_w / 1e6:.0f} M); oracle restating "
                          "llama2/llama.cpp:236-243"}

    return Workload(
        key, {"dim": dim, "hidden_dim": hidden, "n_layers": layers, "kv_dim": kv_dim, "vocab": vocab,
              "calls_per_token": len(calls), "weights_GB": round(4 * n_w / 1e9, 3)},
        1.0, make, call, bound="hbm", io_bytes=4.0 * (n_w + n_out + n_in), kernel="matvec_kernel",
        metric="llama2 decode matmul offload tokens/s (fp32 weights resident in HBM)", unit="tok/s", scale=1.0,
        dtype="f32", graph=True, e2e_host=e2e_host, e2e_step=e2e_step, cpu_fn=cpu_fn)


# ------------------------------------------------------------------- clocks --
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during timing."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index  # nvidia-smi --id: a UUID ("GPU-...") or an index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (getattr(self, "out", "") or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm),
                "window": "sampled every 200 ms over the timed steps and the untimed soak around them"}


# --------------------------------------------------------------- CPU leg --
def cpu_sample(name: str, d_host: dict, rows: int, threads: int):
    """Time the oracle (the reference CPU gold restated) on `rows` rows."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_py
    x, w, b = d_host["x"], d_host["w"], d_host["b"]
    M, K = x.shape
    N = w.shape[1]
    t0 = time.perf_counter()
    out = oracle_py.kbt_gemm_add_relu(x[:rows].copy(), w, b, rows, N, K, threads=threads)
    dt = time.perf_counter() - t0
    return out, dt, 2.0 * rows * N * K


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def reference_arm(args):
    """--impl reference: the reference's CPU gold path (oracle port), all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = host_threads()
    rng = np.random.default_rng(42)
    M, N, K = 8192, 4096, 4096
    rows_per_step = min(M, max(8, threads * 4))
    x = rng.standard_normal((rows_per_step, K), dtype=np.float32).astype(np.float16).astype(np.float32)
    w = (rng.standard_normal((K, N), dtype=np.float32) * K ** -0.5).astype(np.float16).astype(np.float32)
    b = (rng.standard_normal(N, dtype=np.float32) * 0.1).astype(np.float32)
    d = {"x": x, "w": w, "b": b}
    for _ in range(args.warmup):
        cpu_sample("kbt_gemm_add_relu", d, min(threads, rows_per_step), threads)
    times, flops = [], 0.0
    for _ in range(args.steps):
        _, dt, fl = cpu_sample("kbt_gemm_add_relu", d, rows_per_step, threads)
        times.append(dt)
        flops = fl
    tot = sum(times)
    value = flops * len(times) / tot / 1e12
    _, dt1, fl1 = cpu_sample("kbt_gemm_add_relu", d, min(rows_per_step, 16), 1)
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * tot / len(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": f"kbt_gemm_add_relu M={M} N={N} K={K} (CPU gold loop, sampled rows)",
                       "rows_per_step": rows_per_step},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                             "sample": f"{rows_per_step} of {M} rows per step, rows split over {threads} threads; "
                                       "oracle/oracle.c restates benchmarks/kbt_gemm_add_relu/main.cpp:124-129 "
                                       "bit-exactly (pinned against the reference harness)",
                             "one_core": {"value": fl1 / dt1 / 1e12, "unit": "TFLOP/s", "cores": 1,
                                          "sample": f"{min(rows_per_step, 16)} rows on one thread ({dt1:.1f} s)"},
                             "nproc": threads},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU leg --
def numa_bind(torch, local: int):
    """Bind this process to the CPUs of its GPU's NUMA node, so the
    page-locked host buffers it allocates afterwards sit on that node.
    Returns the node, or None where the topology cannot be read."""
    try:
        p = torch.cuda.get_device_properties(local)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        node = int(open(f"/sys/bus/pci/devices/{bus}/numa_node").read().strip())
        if node < 0:
            return None
        cpus = set()
        for part in open(f"/sys/devices/system/node/node{node}/cpulist").read().strip().split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return node
    except (OSError, ValueError, AttributeError):
        return None


def link_probe(torch, nbytes: int = 256 << 20, reps: int = 4) -> dict:
    """The host link's ceiling for e2e: plain cudaMemcpyAsync copies between
    page-locked host memory and the device, host->device alone,
    device->host alone, and both at once on two streams (duplex)."""
    hu = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    hd = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    du = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    dd = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    s_up, s_dn = torch.cuda.Stream(), torch.cuda.Stream()
    cur = torch.cuda.current_stream()

    def timed(up: bool, dn: bool) -> float:
        best = float("inf")
        for _ in range(reps):
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(cur)
            for s, on in ((s_up, up), (s_dn, dn)):
                if on:
                    s.wait_event(e0)
            if up:
                with torch.cuda.stream(s_up):
                    du.copy_(hu, non_blocking=True)
            if dn:
                with torch.cuda.stream(s_dn):
                    hd.copy_(dd, non_blocking=True)
            for s, on in ((s_up, up), (s_dn, dn)):
                if on:
                    cur.wait_stream(s)
            e1.record(cur)
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1) * 1e-3)
        return best

    t_up, t_dn, t_both = timed(True, False), timed(False, True), timed(True, True)
    del hu, hd, du, dd
    return {"h2d_gbs": nbytes / t_up / 1e9, "d2h_gbs": nbytes / t_dn / 1e9,
            "duplex_gbs": 2 * nbytes / t_both / 1e9,
            "how": f"{nbytes >> 20} MiB cudaMemcpyAsync page-locked<->device, best of {reps}; duplex = "
                   "both directions at once on two streams"}


def cublas_same_shape(torch, d, args, ours: dict):
    """cuBLAS (torch.matmul, fp16) on the line's own x [M, K] and w [K, N],
    timed as the line is: the 252 MiB flush before every step, the same
    soak and step count, CUDA events around each step, nvidia-smi clocks
    sampled meanwhile.  It computes x.w only, with no bias or activation, so
    it does a little less work than the fused op.  None for workloads without
    such operands."""
    x, w = d.get("x"), d.get("w")
    if (x is None or w is None or x.dim() != 2 or w.dim() != 2 or x.dtype != torch.float16 or
            w.dtype != torch.float16 or x.shape[1] != w.shape[0]):
        return None
    M, K = x.shape
    N = w.shape[1]
    out = torch.empty(M, N, device=x.device, dtype=torch.float16)
    flush = torch.empty(2 * L2_BYTES // 4, device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream()

    def step():
        torch.matmul(x, w, out=out)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    try:
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(torch.cuda.current_device()).uuid)
    except Exception:
        gpu_id = str(torch.cuda.current_device())
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(gpu_id) as clk:
        t_end = time.perf_counter() + args.soak
        while time.perf_counter() < t_end:
            for _ in range(8):
                step()
            torch.cuda.synchronize()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    value = 2.0 * M * N * K / (ms * 1e-3) / 1e12
    c = clk.summary()
    return {"value": value, "unit": "TFLOP/s", "ms_per_step": ms, "sm_mhz_smi": c["sm_mhz"],
            "reasons": c["reasons"], "ours_over_cublas": ours["value"] / value,
            "what": f"torch.matmul fp16 (cuBLAS) on the same x [{M}, {K}] and w [{K}, {N}], no bias or "
                    "activation; same flush, soak and step count as the line"}


def cpu_leg(d, threads: int, rows_per_thread: int) -> dict:
    """The reference CPU gold (oracle) on the kbt_gemm_add_relu workload:
    the single-thread figure (the reference's gold is a single-threaded loop,
    kbt_gemm_add_relu/main.cpp:124-129) and a row-parallel run on all host
    threads, each on a bounded row sample."""
    M = 8192
    rows1 = 48
    all_rows = min(M, max(8, threads * rows_per_thread))
    rows = max(rows1, all_rows)
    dh = {"x": d["x"][:rows].float().cpu().numpy(), "w": d["w"].float().cpu().numpy(),
          "b": d["b"].float().cpu().numpy()}
    _, dt1, fl1 = cpu_sample("kbt_gemm_add_relu", dh, rows1, 1)
    _, dtn, fln = cpu_sample("kbt_gemm_add_relu", dh, all_rows, threads)
    return {"value": fl1 / dt1 / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
            "sample": f"{rows1} of {M} rows ({dt1:.1f} s) on one thread; oracle restating "
                      "kbt_gemm_add_relu/main.cpp:124-129 (bit-exact, pinned against the reference harness)",
            "nproc": threads,
            "all_cores": {"value": fln / dtn / 1e12, "unit": "TFLOP/s", "cores": threads,
                          "sample": f"{all_rows} rows ({dtn:.1f} s), rows split over {threads} threads "
                                    "(a labelled row-parallel run; the reference's loop is serial)"}}


class KernelClock:
    """SM clock the timed steps' own kernels ran at: the library's GEMM,
    flash, fused-softmax and matrix-vector kernels each add, from CTA 0, the
    SM cycles (clock64) and globaltimer nanoseconds of their run to two device
    counters (akili_sm_clock_read); read over the timed steps alone, cycles /
    ns is the clock under that load, with nothing running beside them."""

    def __init__(self):
        from akili_bench_b200 import abi
        self.L = abi.load()

    def _read(self, clear):
        import ctypes as C
        cyc, ns = C.c_uint64(0), C.c_uint64(0)
        rc = self.L.akili_sm_clock_read(C.byref(cyc), C.byref(ns), 1 if clear else 0)
        return (int(cyc.value), int(ns.value)) if rc == 0 else (0, 0)

    def reset(self):
        self._read(True)

    def mhz(self):
        cyc, ns = self._read(False)
        return 1e3 * cyc / ns if ns else None


def measure(torch, dist, ops, W, name, args, rank, world, local, pk, pk_kind, barrier, mode):
    """Time one workload: device value, e2e through the public API, the
    verification gather, roofline and clocks.  Returns (line, inputs)."""
    from akili_bench_b200 import shard
    from akili_bench_b200.parity import parity
    wl = W[name]
    d = wl.make(Gens(torch, rank))
    out = wl.call(d, None, None)  # allocates the output
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    flush = torch.empty(2 * L2_BYTES // 4, device="cuda", dtype=torch.float32)
    graph = None
    if wl.graph or args.graph:
        # The timed steps replay the step's launches, captured once in a CUDA
        # graph: a C-ABI call spends tens of microseconds on the host (argument
        # checks, tensor maps, launch), longer than the L2 flush before it, and
        # eager launches would let that host time show up as device idle time
        # inside the events.  The capture stream runs one call first, so any
        # scratch the library keeps per stream exists before the capture.
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        l0 = ops.launch_count()
        with torch.cuda.stream(cap):
            wl.call(d, out, cap)
        torch.cuda.synchronize()
        launches_per_step = ops.launch_count() - l0
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap):
            wl.call(d, out, cap)
        torch.cuda.synchronize()

    def step():
        if graph is not None:
            graph.replay()
        else:
            wl.call(d, out, stream)

    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kclock = KernelClock()

    def soak(seconds):
        # untimed repetitions so the clock sampler sees the GPU under this load
        t_end = time.perf_counter() + seconds
        while time.perf_counter() < t_end:
            for _ in range(8):
                step()
            torch.cuda.synchronize()

    try:
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        gpu_id = str(local)
    with ClockSampler(gpu_id) as clk:
        soak(args.soak)
        torch.cuda.synchronize()
        barrier()
        kclock.reset()
        l0 = ops.launch_count()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
        mhz = kclock.mhz()
        launches = ops.launch_count() - l0 if graph is None else launches_per_step * args.steps
        barrier()
        soak(args.soak / 2)
    per_step = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    graph_used = graph is not None
    dev_ms = float(sum(per_step))
    t = torch.tensor([dev_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    value = wl.flops_total * args.steps / (max_ms * 1e-3) / wl.scale
    status = ops.device_status()
    del graph

    # --- end to end through the public API with host buffers (pinned) ---
    e_s = torch.cuda.Event(enable_timing=True)
    e_e = torch.cuda.Event(enable_timing=True)
    if wl.e2e_step is not None:
        e2e_path = "per call: vector in from page-locked host memory, product back, synchronise"
        host = wl.e2e_host(d)
        for _ in range(max(1, args.warmup // 2)):
            wl.e2e_step(d, host, stream)
        torch.cuda.synchronize()
        barrier()
        e_s.record(stream)
        for _ in range(args.steps):
            h2d, d2h = wl.e2e_step(d, host, stream)
        e_e.record(stream)
        torch.cuda.synchronize()
        del host
    elif wl.host_call:
        e2e_path = "akili_host_call: copies and kernel pipelined over chunks inside one call per step"
        hd = {k: (v.cpu().pin_memory() if k not in wl.scratch else v.cpu()) for k, v in d.items()}
        hout = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        h2d = sum(v.numel() * v.element_size() for k, v in hd.items() if k not in wl.scratch)
        d2h = hout.numel() * hout.element_size()
        for _ in range(max(1, args.warmup // 2)):
            wl.call(hd, hout, stream)
        torch.cuda.synchronize()
        barrier()
        e_s.record(stream)
        for _ in range(args.steps):
            wl.call(hd, hout, stream)
        e_e.record(stream)
        torch.cuda.synchronize()
        del hd
    else:
        e2e_path = "device call, copies in and out in series on the stream"
        keys = wl.host or tuple(d)
        host = {k: d[k].cpu().pin_memory() for k in keys}
        host_out = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        d2 = dict(d)
        d2.update({k: torch.empty_like(d[k]) for k in keys})
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        d2h = out.numel() * out.element_size()
        for _ in range(max(1, args.warmup // 2)):
            for k in keys:
                d2[k].copy_(host[k], non_blocking=True)
            o2 = wl.call(d2, out, stream)
            host_out.copy_(o2, non_blocking=True)
        torch.cuda.synchronize()
        barrier()
        e_s.record(stream)
        for _ in range(args.steps):
            for k in keys:
                d2[k].copy_(host[k], non_blocking=True)
            o2 = wl.call(d2, out, stream)
            host_out.copy_(o2, non_blocking=True)
        e_e.record(stream)
        torch.cuda.synchronize()
    e2e_ms = e_s.elapsed_time(e_e)
    t = torch.tensor([e2e_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_max_ms = float(t.item())
    e2e_value = wl.flops_total * args.steps / (e2e_max_ms * 1e-3) / wl.scale
    link = link_probe(torch) if args.link_probe else None

    # --- verification: sampled rows all-gathered to rank 0, checked against the oracle ---
    check = None
    if name.startswith("llama2") and rank == 0:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle_py
        _, _, K, ws, outs = d["calls"][-1]
        rows = np.linspace(0, ws[0].shape[0] - 1, 256).astype(np.int64)
        a = ws[0][torch.from_numpy(rows).cuda()].cpu().numpy()
        x = d["x"][K].cpu().numpy().reshape(K, 1)
        ref = oracle_py.llama2_matmul(a, x, len(rows), 1, K)[:, 0]
        got = outs[0][torch.from_numpy(rows).cuda()].cpu().numpy()
        lim = 4e-6 * K ** 0.5 * (np.abs(a) @ np.abs(x))[:, 0]
        err = np.abs(got.astype(np.float64) - ref)
        check = {"rows_checked": len(rows), "ok": bool((err <= lim).all()),
                 "max_err_frac": float(err.max() / np.abs(ref).max()), "gather": "local"}
    if name == "kbt_gemm_add_relu":
        sample = torch.tensor(shard.sample_rows(out.shape[0]), device="cuda")
        outs, ins = shard.gather_rows([out.index_select(0, sample).float(),
                                       d["x"].index_select(0, sample).float()], world)
        if rank == 0:
            sys.path.insert(0, os.path.join(ROOT, "oracle"))
            import oracle_py
            w_h = d["w"].float().cpu().numpy()
            b_h = d["b"].float().cpu().numpy()
            worst = shard.check_gathered(outs, ins, lambda xr: oracle_py.kbt_gemm_add_relu(
                np.ascontiguousarray(xr), w_h, b_h, xr.shape[0], w_h.shape[1], w_h.shape[0], threads=4), parity)
            check = {"rows_checked": len(sample) * world, "ok": worst["ok"], "max_err_frac": worst["err_frac"],
                     "min_row_cos": worst["min_cos"], "gather": "all_gather" if world > 1 else "local"}

    # --- roofline of the dominant kernel ---
    mean_s = float(np.mean(per_step)) * 1e-3
    if wl.bound == "tensor":
        # Timed after a power-capped soak, so the sustained peak is the
        # matching denominator; without a soak the burst figure is.
        key = "bf16_tflops_sustained" if args.soak > 0 else "bf16_tflops"
        peak = pk.get(key, FALLBACK_PEAKS[key])
        ach = wl.flops / mean_s / 1e12
        roof = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                "peak_source": f"{pk_kind} {key}" + (" (kernel timed inside sustained load)" if args.soak > 0
                                                    else " (burst)"),
                "frac_of_burst_peak": ach / pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])}
    else:
        peak = pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
        ach = wl.io_bytes / mean_s / 1e9
        roof = {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                "peak_source": f"{pk_kind} hbm_gbs"}
    roof["traffic"] = NCU_TRAFFIC.get((name, wl.desc.get("M", 0)))
    roof["kernel"] = wl.kernel if wl.kernel != "gemm_kernel" or wl.desc.get("M", 0) <= 128 else "gemm_pair_kernel"

    cl = clk.summary()
    cl["sm_mhz_smi"] = cl["sm_mhz"]
    if mhz:
        cl["sm_mhz"] = round(mhz, 1)
        cl["sm_mhz_source"] = ("device: SM cycles / globaltimer ns of the timed steps' own kernels (CTA 0 of each "
                               "launch, akili_sm_clock_read); sm_mhz_smi = nvidia-smi median over the soak around "
                               "the steps")
        roof["achieved_per_mhz"] = ach / mhz
    e2e = {"value": e2e_value, "unit": wl.unit, "path": e2e_path, "h2d_bytes_per_step": int(h2d),
           "d2h_bytes_per_step": int(d2h)}
    if link:
        moved = (h2d + d2h) * args.steps / (e2e_ms * 1e-3) / 1e9
        e2e["link"] = link
        e2e["host_link_gbs"] = moved
        e2e["frac_of_duplex"] = moved / link["duplex_gbs"]
    if getattr(args, "numa_node", None) is not None:
        e2e["numa_node"] = args.numa_node
    line = {"metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": max_ms / args.steps, "higher_is_better": True,
            "scaling": "weak" if wl.split == "replicas" or mode == "weak" else "strong",
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic",
            "config": {"workload": f"{name} " + " ".join(f"{k}={v}" for k, v in wl.desc.items()) + " per GPU",
                       "parallelism": (f"{world} independent replica(s)" if wl.split == "replicas" else
                                       f"{wl.split} split over {world} GPU(s) ({mode} scaling), "
                                       "no collective in the timed loop"),
                       "l2": "flushed (a 252 MiB write, twice L2) before every timed step, outside the events",
                       "launch": ("each timed step replays the step's launches from a CUDA graph" if graph_used
                                  else "eager launches"),
                       "inputs": "seeded synthetic, distributions of the configured workload"},
            "roofline": roof, "e2e": e2e, "gpu_launches": int(launches), "device_status": status, "clocks": cl}
    if check is not None:
        line["check"] = check
    del flush
    return line, d


def run_ours(args):
    import torch
    import torch.distributed as dist

    from akili_bench_b200 import ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    args.numa_node = numa_bind(torch, local) if world > 1 else None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    pk, pk_kind = peaks()
    names = None
    modes = [args.scaling] + (["weak"] if world > 1 and args.scaling == "strong" and not args.no_weak else [])
    results = {}
    for mode in modes:
        if args.shard_of > 1:
            # one rank's share of an N-way row split, measured alone on this GPU
            W = workloads(torch, ops, Part(args.shard_of, 0, "strong"))
            for wl in W.values():
                wl.flops_total = wl.flops * world
                wl.desc["shard"] = f"rank 0 of {args.shard_of}"
        else:
            W = workloads(torch, ops, Part(world, rank, mode))
        names = list(W) if args.op == "all" else [args.op]
        for name in names:
            if mode == "weak" and W[name].split == "replicas":
                continue
            line, d = measure(torch, dist, ops, W, name, args, rank, world, local, pk, pk_kind, barrier, mode)
            if mode == modes[0]:
                results[name] = (line, d)
            else:
                main_line = results[name][0]
                main_line["weak"] = {k: line[k] for k in ("value", "ms_per_step", "scaling")}
                main_line["weak"]["workload"] = line["config"]["workload"]
                main_line["weak"]["gpu_launches"] = line["gpu_launches"]
                if "check" in line:
                    main_line["weak"]["check"] = line["check"]
                del d

    if rank == 0:
        for name in names:
            line, d = results[name]
            if world == 1 and name == "kbt_gemm_add_relu" and not args.no_cpu:
                line["cpu_baseline"] = cpu_leg(d, host_threads(), args.cpu_rows_per_thread)
            elif world == 1 and not args.no_cpu and W[name].cpu_fn is not None:
                line["cpu_baseline"] = W[name].cpu_fn(d)
            if world == 1 and args.vs_cublas:
                cb = cublas_same_shape(torch, d, args, line)
                if cb is not None:
                    line["cublas_same_shape"] = cb
            print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    # A throughput number over wrong results is not a result: fail loudly.
    bad = [n for n, (line, _) in results.items() if (line.get("check") and not line["check"]["ok"]) or
           (line.get("weak", {}).get("check") and not line["weak"]["check"]["ok"])]
    if bad:
        print(f"verification failed for {bad}", file=sys.stderr)
        return 3
    return 0


def main():
    ap = argparse.ArgumentParser(description="akili-bench kbt_*/flash on B200")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--op", default="kbt_gemm_add_relu")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--vs-cublas", action="store_true",
                    help="(1 GPU) also time cuBLAS's x.w on the line's own operands, same flush and soak")
    ap.add_argument("--cpu-rows-per-thread", type=int, default=48)
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="strong: the configured global problem split across the GPUs (default); weak: every GPU "
                         "runs the full per-GPU workload.  With strong at N>1 a weak run follows as a second field")
    ap.add_argument("--no-weak", action="store_true", help="skip the second (weak) run at N>1")
    ap.add_argument("--shard-of", type=int, default=1, metavar="G",
                    help="measure rank 0's share of a G-way strong split on this GPU alone (profiling the small "
                         "per-GPU problems of the multi-GPU split); value is then this GPU's work")
    ap.add_argument("--eager", dest="graph", action="store_false",
                    help="launch the timed steps eagerly instead of replaying a captured CUDA graph")
    ap.add_argument("--no-link-probe", dest="link_probe", action="store_false",
                    help="skip the host-link copy probe that states e2e against the link's ceiling")
    ap.add_argument("--soak", type=float, default=1.0,
                    help="seconds of untimed load before (and half after) the timed steps, for clock sampling")
    ap.add_argument("--flash-shape", type=int, nargs=4, metavar=("B", "H", "S", "D"), default=None,
                    help="flash workload shape (default: configs[4], 8 32 4096 128); smaller for profiling")
    ap.add_argument("--llama2-layers", type=int, default=None,
                    help="layers of the llama2 decode workloads (default: the model's); fewer for profiling")
    args = ap.parse_args()
    if args.flash_shape:
        FLASH_SHAPE[:] = args.flash_shape
    if args.llama2_layers:
        for k, v in LLAMA2_SHAPES.items():
            LLAMA2_SHAPES[k] = (v[0], v[1], args.llama2_layers, v[3], v[4])
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
