"""Generate the golden vectors under tests/golden/ from akili-bench itself.

Run here, where the reference tree exists:
    python oracle/build_oracle.py        # builds oracle/_ref/pin/<bench>
    python tests/golden/make_golden.py

Each case runs the reference's own, unchanged ``benchmarks/<bench>/main.cpp``
(built into ``oracle/_ref/pin/<bench>``) with

* ``AKILI_HOST_DEVICE=zero`` — the stand-in device leaves every output at 0,
* ``AKILI_CAPTURE_DIR`` — the argument block and every host->device upload
  (the harness's own ``srand``/``rand()`` inputs) are written to files,
* ``AKILI_PROBE=record`` — every ``fabsf``/``std::fabs`` argument of the
  harness's verify loop is recorded.  With the output at 0 the first call per
  element is ``fabsf(0 - expected)`` (flash: ``std::fabs(expected - 0)``),
  so the reference gold values come out exactly, sign included.

The result per case is ``<bench>__<tag>.npz`` holding the inputs (fp32, by
the harness's buffer names), ``arg`` (the raw argument block bytes),
``argv`` and ``expected`` (the reference gold output, fp32).
"""
from __future__ import annotations

import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
PIN = os.path.join(ROOT, "oracle", "_ref", "pin")

# Buffer names in the order each harness uploads them (benchmarks/<bench>/main.cpp).
INPUTS = {
    "kbt_sgemm": ["a", "b"],
    "kbt_gemm_add_relu": ["a", "w", "bias"],
    "kbt_gemm_mul_leakyrelu": ["a", "w", "bias"],
    "kbt_gemm_div_sum_scale": ["a", "w"],
    "kbt_gemm_layernorm": ["a", "w", "bias", "ln_w", "ln_b"],
    "kbt_attention_score": ["q", "k"],
    "kbt_matmul_softmax": ["a", "b"],
    "kbt_matmul_scale_residadd_clamp": ["a", "b"],
    "kbt_matmul_sum_max_avgpool": ["a", "w", "bias"],
    "kbt_gemm_rmsnorm_swiglu": ["x", "rms_w", "wg", "wu"],
    "kbt_gemm_silu_mul": ["a", "wa", "ba", "wb", "bb"],
    "flash": ["Q", "K", "V", "O_init"],
    "kb2_gemm_add_relu": ["a", "w", "bias"],
    "kb2_gemm_mul_leakyrelu": ["a", "w", "bias"],
    "kb2_gemm_div_sum_scale": ["a", "w"],
    "kb2_gemm_layernorm": ["a", "w", "bias", "ln_w", "ln_b"],
    "kb2_attention_score": ["q", "k"],
    "kb2_matmul_softmax": ["a", "b"],
    "kb2_matmul_scale_residadd_clamp": ["a", "w", "bias"],
    "kb2_matmul_sum_max_avgpool": ["a", "w", "bias"],
    "kb2_gemm_rmsnorm_swiglu": ["x", "rms_w", "wg", "wu"],
    "kb2_gemm_silu_mul": ["a", "wa", "ba", "wb", "bb"],
}

# Verify-loop shape: ("rel", thr) = diff, fabsf(expected), and a third call
# when |expected| > thr; "abs" = one call; "flash" = two calls, first is +ref.
PATTERN = {
    "kbt_sgemm": ("rel", np.float32(1e-3)),
    "kbt_gemm_add_relu": ("rel", np.float32(1e-6)),
    "kbt_gemm_mul_leakyrelu": ("rel", np.float32(1e-6)),
    "kbt_gemm_div_sum_scale": ("rel", np.float32(1e-6)),
    "flash": ("flash", None),
    # kb2 relative checks: fabsf(expected) first, then one more call per element
    **{b: ("first", None) for b in ["kb2_gemm_add_relu", "kb2_gemm_mul_leakyrelu", "kb2_gemm_div_sum_scale",
                                    "kb2_gemm_layernorm", "kb2_gemm_rmsnorm_swiglu", "kb2_gemm_silu_mul"]},
    # kb2 ulp checks: std::abs(actual_bits - expected_bits), one int per element
    **{b: ("ulp", None) for b in ["kb2_attention_score", "kb2_matmul_softmax", "kb2_matmul_scale_residadd_clamp",
                                  "kb2_matmul_sum_max_avgpool"]},
}

CASES = {
    "kbt_sgemm": {"default": [], "m24n40p56": ["-m24", "-n40", "-p56"], "m8n136p72": ["-m8", "-n136", "-p72"]},
    "kbt_attention_score": {"default": [], "m24n40d16": ["-m24", "-n40", "-d16"], "m32n64d64": ["-m32", "-n64", "-d64"]},
    "kb2_attention_score": {"default": [], "m24n40d16": ["-m24", "-n40", "-d16"], "m32n64d64": ["-m32", "-n64", "-d64"]},
    "flash": {"n64d8tcu": ["-n", "64", "-d", "8", "-t", "1"], "n128d16simt": ["-n", "128", "-d", "16", "-t", "0"],
              "n16d8tcu": ["-n", "16", "-d", "8", "-t", "1"]},
}
GEMM_DEFAULT_CASES = {"default": [], "m24n40p56": ["-m24", "-n40", "-p56"], "m40n24p72": ["-m40", "-n24", "-p72"]}


def parse_expected(bench: str, rec: np.ndarray) -> np.ndarray:
    kind, thr = PATTERN.get(bench, ("abs", None))
    if kind == "abs":
        return -rec
    if kind == "first":
        return rec[0::2].copy()
    if kind == "ulp":  # recorded int32 x = 0 - expected_bits
        return (-rec.view(np.int32)).astype(np.int32).view(np.float32)
    out = []
    i = 0
    if kind == "flash":
        while i < len(rec):
            out.append(rec[i])
            i += 2
        return np.array(out, dtype=np.float32)
    while i < len(rec):
        e = np.float32(-rec[i])
        out.append(e)
        i += 2
        if abs(e) > thr:
            i += 1
    return np.array(out, dtype=np.float32)


def run_case(bench: str, tag: str, argv: list[str]) -> str:
    exe = os.path.join(PIN, bench)
    with tempfile.TemporaryDirectory() as td:
        env = dict(os.environ, AKILI_HOST_DEVICE="zero", AKILI_CAPTURE_DIR=td,
                   AKILI_PROBE="record", AKILI_PROBE_FILE=os.path.join(td, "probe.bin"))
        r = subprocess.run([exe, *argv], env=env, capture_output=True, text=True, cwd=td)
        # Zero output means the harness reports FAILED (non-zero exit); that is expected here.
        if "start device" not in r.stdout:
            raise RuntimeError(f"{bench} {argv}: harness did not run\n{r.stdout}\n{r.stderr}")
        data = {}
        for idx, name in enumerate(INPUTS[bench]):
            data[name] = np.fromfile(os.path.join(td, f"in_{idx}.bin"), dtype=np.float32)
        data["arg"] = np.fromfile(os.path.join(td, "arg.bin"), dtype=np.uint8)
        rec = np.fromfile(os.path.join(td, "probe.bin"), dtype=np.float32)
        data["expected"] = parse_expected(bench, rec)
        data["argv"] = np.array(argv if argv else ["<default>"])
    out = os.path.join(HERE, f"{bench}__{tag}.npz")
    np.savez_compressed(out, **data)
    return out


def main() -> int:
    only = sys.argv[1:]  # optional: bench names (or prefixes) to (re)generate
    for bench in INPUTS:
        if only and not any(bench.startswith(o) for o in only):
            continue
        cases = CASES.get(bench, GEMM_DEFAULT_CASES)
        for tag, argv in cases.items():
            p = run_case(bench, tag, argv)
            d = np.load(p)
            print(f"{os.path.basename(p)}: expected {d['expected'].shape}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
