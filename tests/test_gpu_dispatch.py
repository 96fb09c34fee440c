"""GPU parity of the drop-in boundary (spx_run_kernel through the C ABI)
against the CPU oracle, the reference golden vectors and the reference's
kernel self-test."""
import struct

import numpy as np
import pytest

from _cases import check_threshold, compare, golden_cases, read_f32, selftest_cases
from _cases import SELFTEST_INPUT
from spirv_inference_b200 import _lib, dispatch

pytestmark = pytest.mark.gpu


def spx_rk(kernel, in0, in1, nout, push):
    run = dispatch.KernelRun("test", kernel, np.asarray(in0, np.float32),
                             np.asarray(in1, np.float32), int(nout), 0, list(push))
    return dispatch.run_kernel(0, run).values


@pytest.mark.parametrize("name,runner", golden_cases(), ids=[c[0] for c in golden_cases()])
def test_golden_vectors(gpu, name, runner):
    out = runner(spx_rk)
    ok, stats = check_threshold(name, out, read_f32(f"{name}_ref"))
    assert ok, stats
    if name == "relu":
        assert np.array_equal(out.view(np.int32), read_f32("relu_ref").view(np.int32))


def test_kernel_self_test(gpu):
    for kernel, push, in1, expected in selftest_cases():
        out = spx_rk(kernel + ".spv", SELFTEST_INPUT, in1, SELFTEST_INPUT.size, push)
        c = compare(out, expected, 1e-5)
        assert c["mismatch_count"] == 0, (kernel, c)


def test_kernel_output_info(gpu):
    r = dispatch.run_kernel("nvidia", dispatch.KernelRun("relu", "relu.spv", np.ones(64),
                                                         np.zeros(1), 64, 1, [64]))
    assert r.vendor_id == 0x10DE and r.device_name
    assert r.elapsed_ms >= 0.0


def test_loaded_code_is_sm100(gpu):
    import ctypes
    from spirv_inference_b200 import _lib
    v = ctypes.c_int(0)
    assert _lib.lib().spx_binary_version(gpu, ctypes.byref(v)) == 0, _lib.lib().spx_last_error()
    assert v.value == 100


RNG = np.random.default_rng(11)


def _r(*shape, scale=1.0):
    return (RNG.uniform(-1, 1, size=shape) * scale).astype(np.float32)


def _cases():
    """(kernel, in0, in1, nout, push, tolerance) — tolerance None = bit-exact."""
    c = []
    for un in ["abs", "neg", "relu", "relu6", "reshape"]:
        x = _r(1000, scale=8)
        c.append((un, x, [], 1000, [1000], None))
    for un in ["exp", "sigmoid", "tanh", "sine", "logistic"]:
        x = _r(777, scale=4)
        c.append((un, x, [], 777, [777], 2e-6))
    xp = np.abs(_r(513, scale=4)) + 0.01
    for un in ["log", "sqrt", "rsqrt"]:
        c.append((un, xp, [], 513, [513], 2e-6))
    c.append(("leaky_relu", _r(300, scale=3), [], 300, [300, struct.unpack("<i", struct.pack("<f", 0.2))[0]], None))
    a, b = _r(1031, scale=3), _r(1031, scale=3)
    for bn in ["add", "sub", "mul", "min", "max"]:
        c.append((bn, a, b, 1031, [1031], None))
    c.append(("div", a, b + 4.0, 1031, [1031], 1e-6))
    c.append(("pow", np.abs(a) + 0.1, b, 1031, [1031], 4e-6))
    c.append(("concat", a[:400], b[:600], 1000, [400, 1000], None))
    y = _r(2, 3, 4, 5)
    c.append(("transpose", y, [], 120, [2, 3, 4, 5, 4, 2, 5, 3, 2, 0, 3, 1, 120], None))
    c.append(("pad", y, [0.5], 3 * 5 * 6 * 8, [3, 5, 6, 8, 2, 3, 4, 5, 1, 1, 1, 2, 720], None))
    # conv2d NCHW: 3x3 s2 SAME-style offsets, 1x1, 5x5 with odd channels
    for (n, ic, ih, iw, oc, k, s, pt, pl) in [(2, 3, 15, 13, 8, 3, 2, 0, 0),
                                               (1, 16, 7, 7, 24, 1, 1, 0, 0),
                                               (2, 5, 9, 11, 7, 5, 1, 2, 2)]:
        oh, ow = (ih + 2 * pt - k) // s + 1, (iw + 2 * pl - k) // s + 1
        tot = n * oc * oh * ow
        c.append(("conv2d", _r(n, ic, ih, iw), _r(oc * ic * k * k + oc), tot,
                  [n, ic, ih, iw, oc, oh, ow, k, k, s, s, 1, pt, pl, tot], 1e-5))
    for (n, ch, ih, iw, k, s, dil) in [(2, 8, 12, 12, 3, 2, 1), (1, 5, 9, 9, 5, 1, 1),
                                       (1, 4, 10, 10, 3, 1, 2)]:
        eff = (k - 1) * dil + 1
        pt = eff // 2
        oh = (ih + 2 * pt - eff) // s + 1
        tot = n * ch * oh * oh
        c.append(("depthwise_conv2d", _r(n, ch, ih, iw), _r(ch * k * k + ch), tot,
                  [n, ch, ih, iw, oh, oh, k, k, s, s, 1, pt, pt, dil, dil, tot], 1e-5))
    c.append(("fully_connected", _r(5, 37), _r(11 * 37 + 11), 55, [5, 37, 11, 55], 1e-5))
    c.append(("fully_connected", _r(64, 1280), _r(1000 * 1280 + 1000), 64000,
              [64, 1280, 1000, 64000], ("norm", 1280)))
    c.append(("hlo_conv_nhwc_hwio", _r(2, 9, 9, 6), _r(3 * 3 * 6 * 10), 2 * 5 * 5 * 10,
              [2, 9, 9, 6, 3, 3, 10, 5, 5, 2, 2, 1, 1, 500], 1e-5))
    c.append(("hlo_conv_nhwc_hwio", _r(1, 14, 14, 64), _r(64 * 96), 14 * 14 * 96,
              [1, 14, 14, 64, 1, 1, 96, 14, 14, 1, 1, 0, 0, 14 * 14 * 96], 1e-5))
    c.append(("hlo_dot_rank2", _r(33, 70), _r(70, 45), 33 * 45, [33, 70, 45, 33 * 45], 1e-5))
    c.append(("hlo_dot_batched", _r(3, 17, 64), _r(3, 64, 19), 3 * 17 * 19,
              [3, 17, 64, 19, 3 * 17 * 19], 1e-5))
    x4 = _r(2, 3, 40, 50)
    c.append(("hlo_reduce_rank4", x4, [], 2 * 3, [4, 2, 3, 40, 50, 2, 3, 1, 1, 0, 0, 1, 1, 0, 6], 1e-4))
    c.append(("hlo_reduce_rank4", x4, [], 2 * 3 * 40, [4, 2, 3, 40, 50, 2, 3, 40, 1, 0, 0, 0, 1, 1, 240], None))
    c.append(("hlo_reduce_rank4", x4, [], 3 * 50, [4, 2, 3, 40, 50, 1, 3, 1, 50, 1, 0, 1, 0, 0, 150], 1e-4))
    xw = _r(2, 11, 11, 8)
    c.append(("hlo_reduce_window_rank4", xw, [], 2 * 6 * 6 * 8,
              [2, 11, 11, 8, 6, 6, 3, 3, 2, 2, 1, 1, 1, 576], None))
    c.append(("hlo_reduce_window_rank4", xw, [], 2 * 6 * 6 * 8,
              [2, 11, 11, 8, 6, 6, 3, 3, 2, 2, 1, 1, 0, 576], 1e-5))
    xm = _r(2, 3, 11, 11)
    c.append(("max_pool2d", xm, [], 2 * 3 * 6 * 6, [2, 3, 11, 11, 6, 6, 3, 3, 2, 2, 1, 1, 1, 216], None))
    c.append(("global_avg_pool_sum", xm, [], 6, [2, 3, 11, 11], 1e-5))
    c.append(("global_avg_pool_finalize", _r(6), [], 6, [2, 3, 11, 11], None))
    c.append(("softmax1000", _r(1001, scale=6), [], 1001, [1001], 1e-6))
    c.append(("softmax10", _r(10, scale=6), [], 10, [], 1e-6))
    c.append(("l2norm", _r(99), [], 99, [99, struct.unpack("<i", struct.pack("<f", 3.5))[0]], 1e-7))
    c.append(("resize_bilinear", _r(1, 2, 5, 4), [], 2 * 7 * 9, [1, 2, 5, 4, 7, 9, 0, 1, 126], 1e-6))
    return c


CASES = _cases()


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-{i}" for i, c in enumerate(CASES)])
def test_kernel_vs_oracle(gpu, oracle_built, case):
    kernel, in0, in1, nout, push, tol = case
    want = oracle_built.run_kernel(kernel, in0, in1, nout, push)
    got = spx_rk(kernel, in0, in1, nout, push)
    if tol is None:
        assert np.array_equal(got.view(np.int32), want.view(np.int32)), kernel
    elif isinstance(tol, tuple):
        # Dense contractions that may run on the tensor cores: the 3xTF32
        # accumulate truncates, so the error grows with the K/8 accumulation
        # steps.  Normwise bound: max|got - want| <= (2.5e-8 K + 1e-6) max|want|.
        K = tol[1]
        err = float(np.abs(got - want).max()) / float(np.abs(want).max())
        assert err <= 2.5e-8 * K + 1e-6, (kernel, err)
    else:
        np.testing.assert_allclose(got, want, rtol=tol, atol=tol)


def test_every_registry_kernel_covered():
    covered = {c[0] for c in CASES} | {"add", "sub", "mul"}
    assert set(dispatch.registry()) <= covered, set(dispatch.registry()) - covered


def test_short_buffers_are_rejected(gpu):
    with pytest.raises(_lib.SpxError) as e:
        spx_rk("conv2d", np.ones(10), np.ones(10), 100,
               [1, 3, 8, 8, 4, 8, 8, 3, 3, 1, 1, 1, 1, 1, 256])
    assert e.value.code == _lib.SPX_ERR_INVALID_ARGUMENT
    with pytest.raises(_lib.SpxError):
        spx_rk("add", np.ones(10), np.ones(5), 10, [10])
    # the library stays usable after rejected calls
    assert np.array_equal(spx_rk("relu", [-1.0, 2.0], [], 2, [2]), [0.0, 2.0])
