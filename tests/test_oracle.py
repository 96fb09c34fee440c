"""Pins the CPU oracle: the reference's golden vectors, its known-answer
self-test, and an independent float64 numpy formulation of every kernel."""
import numpy as np
import pytest

import _np_ref as R
from _cases import check_threshold, compare, golden_cases, read_f32, selftest_cases, sha256_ok
from _cases import SELFTEST_INPUT


def test_golden_fixture_hashes():
    ok = sha256_ok()
    assert ok and all(ok.values()), ok


@pytest.mark.parametrize("name,runner", golden_cases(), ids=[c[0] for c in golden_cases()])
def test_oracle_golden(oracle_built, name, runner):
    out = runner(oracle_built.run_kernel)
    ok, stats = check_threshold(name, out, read_f32(f"{name}_ref"))
    assert ok, stats
    if name == "relu":  # signed zero: -0.0 must come out +0.0 (generate_fixtures.py:21-25)
        assert np.array_equal(out.view(np.int32), read_f32("relu_ref").view(np.int32))


def test_oracle_selftest(oracle_built):
    for kernel, push, in1, expected in selftest_cases():
        out = oracle_built.run_kernel(kernel + ".spv", SELFTEST_INPUT, in1, SELFTEST_INPUT.size,
                                      push)
        c = compare(out, expected, 1e-5)
        assert c["mismatch_count"] == 0, (kernel, c)


def test_oracle_unknown_kernel(oracle_built):
    with pytest.raises(KeyError):
        oracle_built.run_kernel("not_a_kernel", [1.0], [], 1, [1])


RNG = np.random.default_rng(7)


def _r(*shape):
    return RNG.uniform(-1, 1, size=shape).astype(np.float32)


@pytest.mark.parametrize("n,ic,ih,iw,oc,k,s,pt,pl", [
    (1, 3, 9, 9, 4, 3, 2, 0, 0), (2, 5, 7, 6, 3, 3, 1, 1, 1), (1, 4, 5, 5, 6, 1, 1, 0, 0),
    (1, 2, 8, 8, 3, 5, 2, 2, 1)])
def test_oracle_conv2d(oracle_built, n, ic, ih, iw, oc, k, s, pt, pl):
    oh = (ih + 2 * pt - k) // s + 1
    ow = (iw + 2 * pl - k) // s + 1
    x, w, b = _r(n, ic, ih, iw), _r(oc, ic, k, k), _r(oc)
    total = n * oc * oh * ow
    out = oracle_built.run_kernel("conv2d", x, np.concatenate([w.ravel(), b]), total,
                                  [n, ic, ih, iw, oc, oh, ow, k, k, s, s, 1, pt, pl, total])
    ref = R.conv_nchw(x, w, b, (s, s), (pt, pl), (oh, ow))
    np.testing.assert_allclose(out.reshape(ref.shape), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("c,k,s,dil", [(3, 3, 1, 1), (5, 3, 2, 1), (4, 5, 1, 2)])
def test_oracle_depthwise(oracle_built, c, k, s, dil):
    n, ih, iw = 2, 9, 8
    eff = (k - 1) * dil + 1
    pt = pl = eff // 2
    oh, ow = (ih + 2 * pt - eff) // s + 1, (iw + 2 * pl - eff) // s + 1
    x, w, b = _r(n, c, ih, iw), _r(c, k, k), _r(c)
    total = n * c * oh * ow
    out = oracle_built.run_kernel("depthwise_conv2d", x, np.concatenate([w.ravel(), b]), total,
                                  [n, c, ih, iw, oh, ow, k, k, s, s, 1, pt, pl, dil, dil, total])
    ref = R.depthwise_nhwc(x.transpose(0, 2, 3, 1), w.transpose(1, 2, 0), b, (s, s), (pt, pl),
                           (oh, ow), (dil, dil)).transpose(0, 3, 1, 2)
    np.testing.assert_allclose(out.reshape(ref.shape), ref, rtol=1e-5, atol=1e-5)


def test_oracle_fc_and_dots(oracle_built):
    x, w, b = _r(3, 17), _r(5, 17), _r(5)
    out = oracle_built.run_kernel("fully_connected", x, np.concatenate([w.ravel(), b]), 15,
                                  [3, 17, 5, 15])
    np.testing.assert_allclose(out.reshape(3, 5), x.astype(np.float64) @ w.T.astype(np.float64) + b,
                               rtol=1e-5, atol=1e-5)
    a, bb = _r(4, 7), _r(7, 6)
    out = oracle_built.run_kernel("hlo_dot_rank2", a, bb, 24, [4, 7, 6, 24])
    np.testing.assert_allclose(out.reshape(4, 6), a.astype(np.float64) @ bb, rtol=1e-5, atol=1e-5)
    a, bb = _r(3, 4, 7), _r(3, 7, 6)
    out = oracle_built.run_kernel("hlo_dot_batched", a, bb, 72, [3, 4, 7, 6, 72])
    np.testing.assert_allclose(out.reshape(3, 4, 6), a.astype(np.float64) @ bb, rtol=1e-5,
                               atol=1e-5)


def test_oracle_hlo_conv(oracle_built):
    x, w = _r(2, 7, 7, 3), _r(3, 3, 3, 4)
    out = oracle_built.run_kernel("hlo_conv_nhwc_hwio", x, w, 2 * 4 * 4 * 4,
                                  [2, 7, 7, 3, 3, 3, 4, 4, 4, 2, 2, 1, 1, 2 * 4 * 4 * 4])
    ref = R.conv_nhwc(x, w, (2, 2), (1, 1), (4, 4))
    np.testing.assert_allclose(out.reshape(ref.shape), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dims,axes,kind", [((2, 3, 4, 5), (1, 2), 0), ((2, 3, 4, 5), (3,), 1),
                                            ((6, 7), (0,), 0), ((2, 3, 4), (0, 2), 1)])
def test_oracle_reduce(oracle_built, dims, axes, kind):
    x = _r(*dims)
    ref = x.astype(np.float64).max(axis=axes) if kind else x.astype(np.float64).sum(axis=axes)
    d = list(dims) + [1] * (4 - len(dims))
    r = [1 if i in axes else 0 for i in range(4)]
    od = [1] * 4
    oshape = [s for i, s in enumerate(dims) if i not in axes]
    cur = 0
    for i in range(len(dims)):
        if i not in axes:
            od[i] = oshape[cur]
            cur += 1
    total = int(np.prod(oshape)) if oshape else 1
    out = oracle_built.run_kernel("hlo_reduce_rank4", x, [], total,
                                  [len(dims)] + d + od + r + [kind, total])
    np.testing.assert_allclose(out.reshape(ref.shape), ref, rtol=1e-5, atol=1e-5)


def test_oracle_reduce_window_and_pools(oracle_built):
    x = _r(2, 9, 9, 3)
    for kind in (0, 1):
        out = oracle_built.run_kernel("hlo_reduce_window_rank4", x, [], 2 * 5 * 5 * 3,
                                      [2, 9, 9, 3, 5, 5, 3, 3, 2, 2, 1, 1, kind, 150])
        ref = R.pool_nhwc(x, (3, 3), (2, 2), (1, 1), (5, 5), kind)
        np.testing.assert_allclose(out.reshape(ref.shape), ref, rtol=1e-5, atol=1e-5)
    xc = x.transpose(0, 3, 1, 2).copy()
    out = oracle_built.run_kernel("max_pool2d", xc, [], 150,
                                  [2, 3, 9, 9, 5, 5, 3, 3, 2, 2, 1, 1, 1, 150])
    ref = R.pool_nhwc(x, (3, 3), (2, 2), (1, 1), (5, 5), 1).transpose(0, 3, 1, 2)
    np.testing.assert_allclose(out.reshape(ref.shape), ref)
    s = oracle_built.run_kernel("global_avg_pool_sum", xc, [], 6, [2, 3, 9, 9])
    f = oracle_built.run_kernel("global_avg_pool_finalize", s, [], 6, [2, 3, 9, 9])
    np.testing.assert_allclose(f.reshape(2, 3), xc.astype(np.float64).mean(axis=(2, 3)),
                               rtol=1e-5, atol=1e-6)


def test_oracle_softmax_pad_transpose_concat(oracle_built):
    x = _r(1001) * 5
    out = oracle_built.run_kernel("softmax1000", x, [], 1001, [1001])
    np.testing.assert_allclose(out, R.softmax_rows(x), rtol=1e-5, atol=1e-7)
    out = oracle_built.run_kernel("softmax10", x[:10], [], 10, [])
    np.testing.assert_allclose(out, R.softmax_rows(x[:10]), rtol=1e-5, atol=1e-7)
    y = _r(2, 3, 4, 5)
    padded = oracle_built.run_kernel("pad", y, [7.5], 3 * 5 * 6 * 8,
                                     [3, 5, 6, 8, 2, 3, 4, 5, 1, 1, 1, 2, 3 * 5 * 6 * 8])
    ref = np.pad(y, ((1, 0), (1, 1), (1, 1), (2, 1)), constant_values=7.5)
    np.testing.assert_array_equal(padded.reshape(ref.shape), ref)
    t = oracle_built.run_kernel("transpose", y, [], y.size,
                                [2, 3, 4, 5, 4, 2, 5, 3, 2, 0, 3, 1, y.size])
    np.testing.assert_array_equal(t.reshape(4, 2, 5, 3), y.transpose(2, 0, 3, 1))
    c = oracle_built.run_kernel("concat", y[0].ravel(), y[1].ravel(), y.size, [60, 120])
    np.testing.assert_array_equal(c, y.ravel())


def test_oracle_resize_bilinear(oracle_built):
    x = _r(1, 2, 5, 4)
    for ac, hp in ((0, 0), (1, 0), (0, 1)):
        out = oracle_built.run_kernel("resize_bilinear", x, [], 2 * 7 * 9,
                                      [1, 2, 5, 4, 7, 9, ac, hp, 2 * 7 * 9])
        ref = R.resize_bilinear_nchw(x, 7, 9, ac, hp)
        np.testing.assert_allclose(out.reshape(ref.shape), ref, rtol=1e-5, atol=1e-6)
