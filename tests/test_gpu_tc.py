"""GPU tests of the tcgen05 3xTF32 tensor-core GEMM (forced with
gemm_path = 2) against float64 numpy and the exact-fp32 SIMT path."""
import numpy as np
import pytest

import _np_ref as R
from spirv_inference_b200 import _lib
from spirv_inference_b200.graph import Graph

pytestmark = pytest.mark.gpu
RNG = np.random.default_rng(21)


@pytest.fixture
def g(gpu):
    _lib.set_option("gemm_path", 2)
    try:
        with Graph(gpu) as graph:
            yield graph
    finally:
        _lib.set_option("gemm_path", 0)


def _r(*shape, scale=1.0):
    return (RNG.uniform(-1, 1, size=shape) * scale).astype(np.float32)


SHAPES = [  # M, N, K
    (128, 16, 32), (200, 24, 16), (1000, 96, 24), (517, 144, 96), (4096, 240, 960),
    (333, 1001, 1280), (2048, 1280, 320), (64, 1000, 1280), (130, 48, 36), (5, 8, 4),
    # projection layers at batch 256: odd and even stage rings, two converter
    # groups, two epilogue groups (N <= 32), three epilogue warps per quarter
    (50176, 64, 384), (50176, 32, 192), (200704, 24, 144), (802816, 16, 32),
    (200704, 96, 16), (200704, 160, 24),
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_tc_gemm_matches_fp64(g, M, N, K):
    a = _r(M, K)
    w = _r(N, K, scale=1.0 / np.sqrt(K))
    bias = _r(N)
    dc = g.alloc((M, N))
    g.gemm(g.tensor(a), g.tensor(w), dc, m=M, n=N, k=K, a_strides=(0, K, 1), b_strides=(0, 1, K),
           c_strides=(0, N), bias=g.tensor(bias))
    out = dc.download()
    ref = a.astype(np.float64) @ w.T.astype(np.float64) + bias
    # 3xTF32: per-product relative error ~2^-21 -> well inside fp32-level tolerance
    np.testing.assert_allclose(out, ref, rtol=2e-5, atol=2e-6 * np.sqrt(K))


def test_tc_pointwise_conv_epilogue(g):
    n, h, w, ic, oc = 2, 56, 56, 24, 144
    x = _r(n, h, w, ic)
    wt = _r(oc, 1, 1, ic, scale=0.3)
    b = _r(oc)
    res = _r(n, h, w, oc)
    dy = g.alloc((n, h, w, oc))
    g.conv2d_nhwc(g.tensor(x), g.tensor(wt), g.tensor(b), dy, activation=_lib.ACT_RELU6,
                  residual=g.tensor(res))
    ref = np.clip(x.reshape(-1, ic).astype(np.float64) @ wt.reshape(oc, ic).T + b
                  + res.reshape(-1, oc), 0, 6).reshape(n, h, w, oc)
    np.testing.assert_allclose(dy.download(), ref, rtol=2e-5, atol=2e-5)


def test_tc_and_simt_agree(gpu):
    M, N, K = 3000, 96, 144
    a, w = _r(M, K), _r(N, K, scale=0.1)
    outs = []
    for path in (1, 2):
        _lib.set_option("gemm_path", path)
        try:
            with Graph(gpu) as g:
                dc = g.alloc((M, N))
                g.gemm(g.tensor(a), g.tensor(w), dc, m=M, n=N, k=K, a_strides=(0, K, 1),
                       b_strides=(0, 1, K), c_strides=(0, N))
                outs.append(dc.download())
        finally:
            _lib.set_option("gemm_path", 0)
    np.testing.assert_allclose(outs[0], outs[1], rtol=2e-5, atol=2e-5)


def test_tc_ineligible_shape_reports_unsupported(g):
    a, w = _r(10, 6), _r(8, 6)  # K = 6 is not a multiple of 4 (TMA row pitch)
    dc = g.alloc((10, 8))
    with pytest.raises(_lib.SpxError) as e:
        g.gemm(g.tensor(a), g.tensor(w), dc, m=10, n=8, k=6, a_strides=(0, 6, 1),
               b_strides=(0, 1, 6), c_strides=(0, 8))
    assert e.value.code == _lib.SPX_ERR_UNSUPPORTED


@pytest.mark.parametrize("M,N,K", [(1000, 96, 24), (4096, 240, 960), (333, 1001, 1280),
                                   (12544, 160, 960), (256, 1280, 320)])
def test_tc_presplit_weights_match_on_chip_split(g, M, N, K):
    a = _r(M, K)
    w = _r(N, K, scale=1.0 / np.sqrt(K))
    res = _r(M, N)
    da, dw, dr = g.tensor(a), g.tensor(w), g.tensor(res)
    hi, lo = g.weights_split(dw)
    h, l = hi.download(), lo.download()
    assert np.all((h.view(np.uint32) & 0x1FFF) == 0) and np.all((l.view(np.uint32) & 0x1FFF) == 0)
    np.testing.assert_allclose(h.astype(np.float64) + l, w, rtol=2 ** -21, atol=0)
    outs = []
    for split in (None, (hi, lo)):
        dc = g.alloc((M, N))
        g.gemm(da, dw, dc, m=M, n=N, k=K, a_strides=(0, K, 1), b_strides=(0, 1, K),
               c_strides=(0, N), residual=dr, activation=_lib.ACT_RELU, b_split=split)
        outs.append(dc.download())
    # the same tf32 terms enter the same MMAs: identical results
    np.testing.assert_array_equal(outs[0], outs[1])
    ref = np.maximum(a.astype(np.float64) @ w.T.astype(np.float64) + res, 0)
    err = np.abs(outs[1] - ref).max() / np.abs(ref).max()
    assert err <= 2.5e-8 * K + 1e-6, err


@pytest.mark.parametrize("n,ih,ic,oc,k,s,pad", [(2, 56, 64, 64, 3, 1, 1), (2, 56, 64, 128, 3, 2, 1),
                                               (3, 7, 64, 96, 3, 1, 1), (2, 14, 32, 64, 3, 1, 1),
                                               (2, 28, 128, 64, 1, 2, 0), (1, 15, 32, 48, 5, 1, 2),
                                               (5, 7, 128, 32, 3, 2, 1), (2, 9, 32, 40, 3, 1, 0)])
def test_conv_tc_implicit_gemm(g, n, ih, ic, oc, k, s, pad):
    """KxK / strided convs as implicit GEMM on tensor cores (4-D TMA boxes of
    the NHWC input per tap, zero fill as padding) against float64."""
    oh = (ih + 2 * pad - k) // s + 1
    x = _r(n, ih, ih, ic)
    w = _r(oc, k, k, ic, scale=1.0 / np.sqrt(k * k * ic))   # OHWI
    b, res = _r(oc), _r(n, oh, oh, oc)
    dx, dw, db, dr = g.tensor(x), g.tensor(w), g.tensor(b), g.tensor(res)
    ref = R.conv_nhwc(x, np.transpose(w, (1, 2, 3, 0)), (s, s), (pad, pad), (oh, oh)) + b + res
    ref = np.maximum(ref, 0)
    outs = []
    for split in (None, g.weights_split(dw)):
        dy = g.alloc((n, oh, oh, oc))
        _lib.set_option("gemm_path", 2)
        try:
            g.conv2d_nhwc(dx, dw, db, dy, stride=(s, s), pad=(pad, pad), residual=dr,
                          activation=_lib.ACT_RELU, w_split=split)
        finally:
            _lib.set_option("gemm_path", 0)
        outs.append(dy.download())
    np.testing.assert_array_equal(outs[0], outs[1])
    K = k * k * ic
    err = np.abs(outs[0] - ref).max() / np.abs(ref).max()
    assert err <= 2.5e-8 * K + 1e-6, err


@pytest.mark.parametrize("M,N,K", [(802816, 24, 144), (50176, 64, 384), (4096, 768, 768),
                                   (517, 144, 96), (12544, 1280, 320)])
def test_tc_lo_terms_in_tmem_match_shared_memory(g, M, N, K):
    """Option tc_lo_tmem: the activations' lo terms written to tensor memory
    (the lo*hi MMA reads A from TMEM) give bit-identical results to the
    shared-memory lo tiles — the same tf32 terms in the same MMA order."""
    a = _r(M, K)
    w = _r(N, K, scale=1.0 / np.sqrt(K))
    bias = _r(N)
    da, dw, db = g.tensor(a), g.tensor(w), g.tensor(bias)
    split = g.weights_split(dw)
    outs = []
    _lib.set_option("tc_cat", 0)  # the three-product form, the one lo_tmem issues
    try:
        for lo_tmem in (0, 1):
            _lib.set_option("tc_lo_tmem", lo_tmem)
            try:
                dc = g.alloc((M, N))
                g.gemm(da, dw, dc, m=M, n=N, k=K, a_strides=(0, K, 1), b_strides=(0, 1, K),
                       c_strides=(0, N), bias=db, activation=_lib.ACT_RELU6, b_split=split)
                outs.append(dc.download())
            finally:
                _lib.set_option("tc_lo_tmem", 0)
    finally:
        _lib.set_option("tc_cat", 1)
    np.testing.assert_array_equal(outs[0], outs[1])
    ref = np.clip(a[:4096].astype(np.float64) @ w.T.astype(np.float64) + bias, 0, 6)
    err = np.abs(outs[1][:4096] - ref).max() / max(np.abs(ref).max(), 1e-30)
    assert err <= 2.5e-8 * K + 1e-6, err


def test_conv_tc_lo_terms_in_tmem(g):
    n, ih, ic, oc, k, s, pad = 2, 28, 64, 96, 3, 1, 1
    oh = (ih + 2 * pad - k) // s + 1
    x = _r(n, ih, ih, ic)
    w = _r(oc, k, k, ic, scale=1.0 / np.sqrt(k * k * ic))
    b = _r(oc)
    dx, dw, db = g.tensor(x), g.tensor(w), g.tensor(b)
    split = g.weights_split(dw)
    outs = []
    _lib.set_option("tc_cat", 0)  # the three-product form, the one lo_tmem issues
    try:
        for lo_tmem in (0, 1):
            _lib.set_option("tc_lo_tmem", lo_tmem)
            try:
                dy = g.alloc((n, oh, oh, oc))
                g.conv2d_nhwc(dx, dw, db, dy, stride=(s, s), pad=(pad, pad),
                              activation=_lib.ACT_RELU, w_split=split)
                outs.append(dy.download())
            finally:
                _lib.set_option("tc_lo_tmem", 0)
    finally:
        _lib.set_option("tc_cat", 1)
    np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.parametrize("M,N,K,conv", [(802816, 24, 144, 0), (50176, 64, 384, 0), (517, 144, 96, 0),
                                        (4096, 32, 200, 0), (2, 64, 576, 1)])
def test_tc_concatenated_product_matches_three_products(g, M, N, K, conv):
    """Option tc_cat: raw A x [hi; lo] as one product of twice the tile width
    plus lo x hi, against the three separate products and float64 (same
    terms, another summation order: equal within the 3xTF32 bound).  conv = 1
    runs a 3x3 implicit-GEMM convolution (n = M images of 16 x 16 x 64)."""
    outs = []
    if conv:
        x = _r(M, 16, 16, 64)
        w = _r(N, 3, 3, 64, scale=1.0 / np.sqrt(K))
        b = _r(N)
        dx, dw, db = g.tensor(x), g.tensor(w), g.tensor(b)
        split = g.weights_split(dw)
        for cat in (0, 1):
            _lib.set_option("tc_cat", cat)
            try:
                dy = g.alloc((M, 16, 16, N))
                g.conv2d_nhwc(dx, dw, db, dy, pad=(1, 1), w_split=split)
                outs.append(dy.download())
            finally:
                _lib.set_option("tc_cat", 1)
        ref = R.conv_nhwc(x, w.transpose(1, 2, 3, 0), (1, 1), (1, 1), (16, 16)) + b
    else:
        a = _r(M, K)
        w = _r(N, K, scale=1.0 / np.sqrt(K))
        bias = _r(N)
        da, dw, db = g.tensor(a), g.tensor(w), g.tensor(bias)
        split = g.weights_split(dw)
        for cat in (0, 1):
            _lib.set_option("tc_cat", cat)
            try:
                dc = g.alloc((M, N))
                g.gemm(da, dw, dc, m=M, n=N, k=K, a_strides=(0, K, 1), b_strides=(0, 1, K),
                       c_strides=(0, N), bias=db, b_split=split)
                outs.append(dc.download())
            finally:
                _lib.set_option("tc_cat", 1)
        ref = a[:4096].astype(np.float64) @ w.T.astype(np.float64) + bias
        outs = [o[:4096] for o in outs]
    scale = np.abs(ref).max()
    for o in outs:
        assert np.abs(o - ref).max() / scale <= 2.5e-8 * K + 1e-6
    assert np.abs(outs[0] - outs[1]).max() / scale <= 2 * (2.5e-8 * K + 1e-6)


@pytest.mark.parametrize("M,N,K", [(3211264, 96, 16), (802816, 144, 24), (50000, 160, 8),
                                   (300001, 128, 20), (200704, 64, 24)])
def test_tc_more_accumulators_give_identical_results(g, M, N, K):
    """Option tc_acc4: one-k-block tiles on three or four accumulators issue
    the three separate products, so they must give the bits of the
    three-product form on two accumulators (tc_cat = 0, tc_acc4 = 0), and
    stay within the 3xTF32 bound of float64."""
    a = _r(M, K)
    w = _r(N, K, scale=1.0 / np.sqrt(K))
    bias = _r(N)
    da, dw, db = g.tensor(a), g.tensor(w), g.tensor(bias)
    split = g.weights_split(dw)
    outs = []
    try:
        for cat, acc4 in ((0, 0), (1, 1)):
            _lib.set_option("tc_cat", cat)
            _lib.set_option("tc_acc4", acc4)
            assert _lib.gemm_tc_plan(M, N, K)["nacc"] == (2 if not acc4 else
                                                          (4 if N <= 128 else 3))
            dc = g.alloc((M, N))
            g.gemm(da, dw, dc, m=M, n=N, k=K, a_strides=(0, K, 1), b_strides=(0, 1, K),
                   c_strides=(0, N), bias=db, b_split=split)
            outs.append(dc.download())
    finally:
        _lib.set_option("tc_cat", 1)
        _lib.set_option("tc_acc4", 1)
    np.testing.assert_array_equal(outs[0], outs[1])
    ref = a[:4096].astype(np.float64) @ w.T.astype(np.float64) + bias
    assert np.abs(outs[1][:4096] - ref).max() / np.abs(ref).max() <= 2.5e-8 * K + 1e-6
