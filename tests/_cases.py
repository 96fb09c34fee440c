"""Shared parity cases: the reference's golden vectors and known answers.

* ``golden_cases()`` — tests/parity_test/out/fixtures of the reference
  (copied to tests/golden by make_golden.py) expressed as dispatches of the
  packaged kernels, with the thresholds of
  tests/parity_test/generate_fixtures.py:108-113 /
  tests/parity_test/compare_outputs.py:10-15.
* ``selftest_cases()`` — the 15 known-answer cases of
  source/tflite_loader/src/engine.rs:15-174 (input [0.25 .. 4], rhs 2.0,
  gate ``compare(.., 1e-5)``).
* ``compare`` — source/tflite_loader/src/tensor.rs:35-54.
"""
from __future__ import annotations

import hashlib
import json
import struct
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def read_f32(name: str) -> np.ndarray:
    return np.fromfile(GOLDEN / f"{name}.raw.f32", dtype="<f4")


def manifest() -> dict:
    return json.loads((GOLDEN / "manifest.json").read_text())


def sha256_ok() -> dict[str, bool]:
    m = manifest()
    return {k: hashlib.sha256((GOLDEN / v["path"]).read_bytes()).hexdigest() == v["sha256"]
            for k, v in m["files"].items()}


def ulp_dist(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """compare_outputs.py:25-32: distance in the ordered-int32 view."""
    def ordered(x):
        bits = np.asarray(x, np.float32).view(np.int32).astype(np.int64)
        return np.where(bits < 0, -2147483648 - bits, bits)
    return np.abs(ordered(a) - ordered(b))


def compare(actual, expected, eps: float) -> dict:
    """tensor.rs:35-54: mismatch count at |a-e| > eps, max abs / rel error."""
    a = np.asarray(actual, np.float32).reshape(-1)
    e = np.asarray(expected, np.float32).reshape(-1)
    n = min(a.size, e.size)
    d = np.abs(a[:n].astype(np.float32) - e[:n])
    rel = d / np.maximum(np.abs(e[:n]), 1e-30)
    return {"mismatch_count": int((d > eps).sum()) + abs(a.size - e.size),
            "max_abs_error": float(d.max()) if n else 0.0,
            "max_rel_error": float(rel.max()) if n else 0.0}


def check_threshold(name: str, out: np.ndarray, ref: np.ndarray) -> tuple[bool, dict]:
    """compare_outputs.py:49-62 per-kernel rule."""
    t = manifest()["thresholds"][name]
    u = ulp_dist(out, ref)
    absd = np.abs(out.astype(np.float64) - ref.astype(np.float64))
    rel = absd / np.maximum(np.abs(out.astype(np.float64)), 1e-30)
    if name == "relu":
        bad = u != 0
    elif "max_abs" in t:
        bad = (u > t["max_ulp"]) | (absd > t["max_abs"])
    else:
        bad = (u > t["max_ulp"]) | (rel > t["max_rel"])
    stats = {"max_ulp": int(u.max()), "max_abs": float(absd.max()), "max_rel": float(rel.max()),
             "mismatches": int(bad.sum())}
    return not bad.any(), stats


def golden_cases():
    """Yields (name, runner) where runner(run_kernel) -> output vector.

    ``run_kernel(kernel, in0, in1, nout, push) -> np.ndarray``.
    """
    def relu(rk):
        x = read_f32("relu_input")
        return rk("relu.spv", x, np.zeros(1, np.float32), x.size, [x.size])

    def softmax(rk):
        x = read_f32("softmax_input")
        return rk("softmax1000.spv", x, np.zeros(1, np.float32), x.size, [x.size])

    def batchnorm(rk):
        # generate_fixtures.py:36-39: inv = f32(1/sqrt(f32(var+eps))) is a host
        # scalar; the per-element chain is (x - mean) * inv * gamma + beta.
        x = read_f32("batchnorm_input")
        mean, var, gamma, beta, eps = read_f32("batchnorm_params")
        inv = np.float32(1.0 / np.sqrt(np.float64(np.float32(var + eps))))
        full = lambda v: np.full(x.size, v, np.float32)
        n = [x.size]
        t = rk("sub.spv", x, full(mean), x.size, n)
        t = rk("mul.spv", t, full(inv), x.size, n)
        t = rk("mul.spv", t, full(gamma), x.size, n)
        return rk("add.spv", t, full(beta), x.size, n)

    def conv1d(rk):
        # 16 positions x 64 channels, filter [3][64][32], pad 1: an NHWC/HWIO
        # convolution with H = 1, W = 16, KH = 1, KW = 3 (hlo_conv_nhwc_hwio).
        x, f = read_f32("conv1d_input"), read_f32("conv1d_filter")
        push = [1, 1, 16, 64, 1, 3, 32, 1, 16, 1, 1, 0, 1, 16 * 32]
        return rk("hlo_conv_nhwc_hwio.spv", x, f, 16 * 32, push)

    return [("relu", relu), ("softmax", softmax), ("batchnorm", batchnorm), ("conv1d", conv1d)]


SELFTEST_INPUT = np.array([0.25, 0.5, 0.75, 1.0, 1.25, 2.0, 3.0, 4.0], np.float32)


def selftest_cases():
    """engine.rs:21-174: (kernel, push, input1, expected)."""
    x = SELFTEST_INPUT
    rhs = np.full(x.size, 2.0, np.float32)
    un = np.zeros(x.size, np.float32)
    n = [x.size]
    f = np.float32
    alpha_bits = struct.unpack("<i", struct.pack("<f", 0.1))[0]
    with np.errstate(all="ignore"):
        return [
            ("abs", n, un, np.abs(x)),
            ("exp", n, un, np.exp(x)),
            ("log", n, un, np.log(x)),
            ("neg", n, un, -x),
            ("sqrt", n, un, np.sqrt(x)),
            ("rsqrt", n, un, (f(1.0) / np.sqrt(x)).astype(f)),
            ("sub", n, rhs, x - rhs),
            ("mul", n, rhs, x * rhs),
            ("div", n, rhs, x / rhs),
            ("pow", n, rhs, np.power(x, rhs)),
            ("min", n, rhs, np.minimum(x, rhs)),
            ("max", n, rhs, np.maximum(x, rhs)),
            ("leaky_relu", [x.size, alpha_bits], un, np.maximum(x, f(0.1) * x)),
            ("sigmoid", n, un, (f(1.0) / (f(1.0) + np.exp(-x))).astype(f)),
            ("tanh", n, un, ((np.exp(x) - np.exp(-x)) / (np.exp(x) + np.exp(-x))).astype(f)),
        ]
