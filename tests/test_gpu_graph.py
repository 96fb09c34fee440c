"""GPU tests of the device-resident graph API (NHWC ops with fused
epilogues) against float64 numpy formulations and the oracle."""
import numpy as np
import pytest

import _np_ref as R
from spirv_inference_b200 import _lib
from spirv_inference_b200.graph import Graph

pytestmark = pytest.mark.gpu
RNG = np.random.default_rng(5)


def _r(*shape, scale=1.0):
    return (RNG.uniform(-1, 1, size=shape) * scale).astype(np.float32)


def _act(y, act):
    if act == _lib.ACT_RELU:
        return np.maximum(y, 0)
    if act == _lib.ACT_RELU6:
        return np.clip(y, 0, 6)
    return y


@pytest.fixture
def g(gpu):
    with Graph(gpu) as graph:
        yield graph


CONV_CASES = [
    # n, ih, iw, ic, oc, k, s, pad, dil, act, residual, layout
    (2, 16, 16, 32, 64, 1, 1, 0, 1, _lib.ACT_RELU6, False, _lib.WEIGHT_OHWI),
    (2, 16, 16, 96, 24, 1, 1, 0, 1, _lib.ACT_NONE, True, _lib.WEIGHT_OHWI),
    (3, 15, 17, 3, 32, 3, 2, 0, 1, _lib.ACT_RELU6, False, _lib.WEIGHT_OHWI),
    (1, 9, 9, 5, 7, 5, 1, 2, 1, _lib.ACT_RELU, False, _lib.WEIGHT_HWIO),
    (1, 12, 12, 8, 16, 3, 1, 2, 2, _lib.ACT_NONE, False, _lib.WEIGHT_HWIO),
    (2, 7, 7, 320, 1280, 1, 1, 0, 1, _lib.ACT_RELU6, False, _lib.WEIGHT_OHWI),
    (4, 1, 1, 1280, 1001, 1, 1, 0, 1, _lib.ACT_NONE, False, _lib.WEIGHT_OHWI),
    (1, 30, 30, 64, 16, 3, 2, 1, 1, _lib.ACT_RELU, True, _lib.WEIGHT_HWIO),
    (2, 10, 11, 4, 16, 3, 1, 1, 1, _lib.ACT_RELU, True, _lib.WEIGHT_HWIO),   # direct small-K
    (1, 13, 13, 3, 64, 3, 2, 1, 1, _lib.ACT_RELU6, False, _lib.WEIGHT_OHWI),  # direct small-K
    (2, 112, 112, 3, 32, 3, 2, 1, 1, _lib.ACT_RELU6, True, _lib.WEIGHT_HWIO),  # 3x3x3 stem
    (1, 33, 31, 3, 32, 3, 1, 1, 1, _lib.ACT_NONE, False, _lib.WEIGHT_OHWI),   # stem, ragged
]


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv2d_nhwc(g, case):
    n, ih, iw, ic, oc, k, s, pad, dil, act, use_res, layout = case
    eff = (k - 1) * dil + 1
    oh, ow = (ih + 2 * pad - eff) // s + 1, (iw + 2 * pad - eff) // s + 1
    x = _r(n, ih, iw, ic)
    w_hwio = _r(k, k, ic, oc, scale=1.0 / np.sqrt(k * k * ic))
    b = _r(oc)
    res = _r(n, oh, ow, oc) if use_res else None
    w_dev = w_hwio if layout == _lib.WEIGHT_HWIO else np.ascontiguousarray(w_hwio.transpose(3, 0, 1, 2))
    dx, dw, db = g.tensor(x), g.tensor(w_dev), g.tensor(b)
    dr = g.tensor(res) if use_res else None
    dy = g.alloc((n, oh, ow, oc))
    g.conv2d_nhwc(dx, dw, db, dy, stride=(s, s), pad=(pad, pad), dilation=(dil, dil),
                  weight_layout=layout, activation=act, residual=dr)
    ref = R.conv_nhwc(x, w_hwio, (s, s), (pad, pad), (oh, ow), (dil, dil)) + b
    if use_res:
        ref = ref + res
    ref = _act(ref, act)
    np.testing.assert_allclose(dy.download(), ref, rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("n,ih,c,k,s,dil,act", [(2, 14, 32, 3, 1, 1, _lib.ACT_RELU6),
                                               (1, 56, 144, 3, 1, 1, _lib.ACT_RELU6),
                                               (2, 28, 192, 3, 1, 1, _lib.ACT_NONE),
                                               (1, 15, 96, 3, 2, 1, _lib.ACT_RELU6),
                                               (2, 9, 5, 5, 1, 1, _lib.ACT_NONE),
                                               (1, 12, 8, 3, 1, 2, _lib.ACT_RELU),
                                               (2, 15, 40, 5, 2, 1, _lib.ACT_RELU6),
                                               (1, 14, 112, 5, 1, 1, _lib.ACT_RELU6),
                                               (3, 7, 160, 3, 1, 1, _lib.ACT_NONE),
                                               (1, 13, 24, 3, 2, 1, _lib.ACT_RELU6),
                                               (2, 15, 144, 3, 2, 1, _lib.ACT_RELU6),
                                               (1, 20, 64, 5, 2, 1, _lib.ACT_RELU6),
                                               (2, 9, 32, 5, 1, 1, _lib.ACT_NONE),
                                               (3, 17, 48, 3, 1, 1, _lib.ACT_RELU),
                                               (1, 56, 144, 3, 1, 1, _lib.ACT_RELU6)])
def test_depthwise_nhwc(g, n, ih, c, k, s, dil, act):
    eff = (k - 1) * dil + 1
    # TFLite SAME: floor(total/2) on top/left
    oh = -(-ih // s)
    tot = max((oh - 1) * s + eff - ih, 0)
    pt = tot // 2
    x, w, b = _r(n, ih, ih, c), _r(k, k, c), _r(c)
    dy = g.alloc((n, oh, oh, c))
    g.depthwise_nhwc(g.tensor(x), g.tensor(w), g.tensor(b), dy, stride=(s, s), pad=(pt, pt),
                     dilation=(dil, dil), activation=act)
    ref = _act(R.depthwise_nhwc(x, w, b, (s, s), (pt, pt), (oh, oh), (dil, dil)), act)
    np.testing.assert_allclose(dy.download(), ref, rtol=1e-5, atol=1e-5)


def test_gemm_strided_batched(g):
    # C[b] = A[b] @ B[b]^T with A k-contiguous and B stored [n][k]
    B, M, N, K = 3, 37, 29, 70
    a, bt = _r(B, M, K), _r(B, N, K)
    dc = g.alloc((B, M, N))
    g.gemm(g.tensor(a), g.tensor(bt), dc, m=M, n=N, k=K, batch=B, a_strides=(M * K, K, 1),
           b_strides=(N * K, 1, K), c_strides=(M * N, N), alpha=0.5)
    ref = 0.5 * np.einsum("bmk,bnk->bmn", a.astype(np.float64), bt.astype(np.float64))
    np.testing.assert_allclose(dc.download(), ref, rtol=1e-5, atol=1e-5)
    # m-contiguous A (A stored [k][m]) with bias + relu
    at = _r(K, M)
    b2 = _r(K, N)
    bias = _r(N)
    dc2 = g.alloc((M, N))
    g.gemm(g.tensor(at), g.tensor(b2), dc2, m=M, n=N, k=K, a_strides=(0, 1, M),
           b_strides=(0, N, 1), c_strides=(0, N), bias=g.tensor(bias), activation=_lib.ACT_RELU)
    ref2 = np.maximum(at.T.astype(np.float64) @ b2 + bias, 0)
    np.testing.assert_allclose(dc2.download(), ref2, rtol=1e-5, atol=1e-5)


def test_gemm_grouped_heads(g):
    # attention-style: 2 outer batches x 8 query heads, K/V heads shared by 4
    Bo, H, Hkv, S, D = 2, 8, 2, 9, 16
    q = _r(Bo, S, H, D)
    k = _r(Bo, S, Hkv, D)
    dq, dk = g.tensor(q), g.tensor(k)
    dsc = g.alloc((Bo, H, S, S))
    g.gemm(dq, dk, dsc, m=S, n=S, k=D, batch=Bo, batch_inner=H, b_inner_div=H // Hkv,
           a_strides=(S * H * D, H * D, 1), b_strides=(S * Hkv * D, 1, Hkv * D),
           c_strides=(H * S * S, S), inner_strides=(D, D, S * S))
    kk = np.repeat(k, H // Hkv, axis=2)
    ref = np.einsum("bqhd,bkhd->bhqk", q.astype(np.float64), kk.astype(np.float64))
    np.testing.assert_allclose(dsc.download(), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("kind", [_lib.POOL_MAX, _lib.POOL_SUM, _lib.POOL_AVG])
@pytest.mark.parametrize("c", [64, 3])
def test_pool_nhwc(g, kind, c):
    x = _r(2, 17, 17, c)
    dy = g.alloc((2, 9, 9, c))
    g.pool2d_nhwc(g.tensor(x), dy, kernel=(3, 3), stride=(2, 2), pad=(1, 1), kind=kind)
    ref = R.pool_nhwc(x, (3, 3), (2, 2), (1, 1), (9, 9), kind)
    np.testing.assert_allclose(dy.download(), ref, rtol=1e-5, atol=1e-5)


def test_gap_softmax_rows(g):
    x = _r(4, 7, 7, 1280)
    dy = g.alloc((4, 1280))
    g.global_avg_pool_nhwc(g.tensor(x), dy)
    np.testing.assert_allclose(dy.download(), x.astype(np.float64).mean(axis=(1, 2)), rtol=1e-5,
                               atol=1e-6)
    z = _r(256, 1001, scale=8)
    ds = g.alloc((256, 1001))
    g.softmax_rows(g.tensor(z), ds, 256, 1001)
    out = ds.download()
    np.testing.assert_allclose(out, R.softmax_rows(z), rtol=1e-5, atol=1e-7)
    assert np.all(np.argmax(out, 1) == np.argmax(z, 1))


def test_attention_softmax_causal(g):
    rows, q_len, cols = 2 * 3 * 5, 5, 9  # q positions 4..8 of a 9-key window
    x = _r(rows, cols, scale=4)
    dy = g.alloc((rows, cols))
    g.attention_softmax(g.tensor(x), dy, rows, cols, scale=0.125, causal=True, q_len=q_len,
                        q_offset=4)
    out = dy.download()
    ref = np.zeros((rows, cols))
    for r in range(rows):
        lim = 4 + r % q_len + 1
        ref[r, :lim] = R.softmax_rows(x[r, :lim] * 0.125)
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-7)


def test_norms_rope_embedding_argmax_swiglu(g):
    rows, cols = 33, 768
    x, res = _r(rows, cols), _r(rows, cols)
    gamma, beta = _r(cols), _r(cols)
    dy, dxo = g.alloc((rows, cols)), g.alloc((rows, cols))
    g.layernorm(g.tensor(x), g.tensor(gamma), g.tensor(beta), dy, rows, cols, 1e-12,
                residual=g.tensor(res), x_out=dxo)
    h = (x + res).astype(np.float64)
    mu, var = h.mean(1, keepdims=True), h.var(1, keepdims=True)
    np.testing.assert_allclose(dy.download(), (h - mu) / np.sqrt(var + 1e-12) * gamma + beta,
                               rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(dxo.download(), x + res, rtol=0, atol=0)
    dr = g.alloc((rows, cols))
    g.rmsnorm(g.tensor(x), g.tensor(gamma), dr, rows, cols, 1e-5)
    xd = x.astype(np.float64)
    np.testing.assert_allclose(dr.download(),
                               gamma * xd / np.sqrt((xd ** 2).mean(1, keepdims=True) + 1e-5),
                               rtol=1e-5, atol=1e-6)
    T, H, D = 3, 4, 64
    q = _r(T, H, D)
    pos = np.array([0, 7, 31], np.int32)
    dq = g.tensor(q)
    g.rope(dq, g.tensor(pos, np.int32), T, H, D, 10000.0)
    inv = 1.0 / (10000.0 ** (np.arange(0, D, 2) / D))
    ang = pos[:, None] * inv[None]
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    x1, x2 = q[..., :D // 2].astype(np.float64), q[..., D // 2:].astype(np.float64)
    ref = np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)
    np.testing.assert_allclose(dq.download(), ref, rtol=1e-5, atol=2e-5)
    table = _r(50, 24)
    ids = np.array([3, 0, 49, 3], np.int32)
    de = g.alloc((4, 24))
    g.embedding(g.tensor(table), g.tensor(ids, np.int32), de, 4, 24)
    np.testing.assert_array_equal(de.download(), table[ids])
    z = _r(5, 32000)
    z[2, 17] = z[2, 900] = 5.0  # tie: first index wins
    di = g.alloc((5,), np.int32)
    g.argmax_rows(g.tensor(z), di, 5, 32000)
    np.testing.assert_array_equal(di.download(), np.argmax(z, 1))
    ga, up = _r(1000), _r(1000)
    dsw = g.alloc((1000,))
    g.swiglu(g.tensor(ga), g.tensor(up), dsw, 1000)
    gd = ga.astype(np.float64)
    np.testing.assert_allclose(dsw.download(), gd / (1 + np.exp(-gd)) * up, rtol=1e-5, atol=1e-6)


def test_binary_broadcast_and_unary(g):
    a = _r(2, 3, 4, 5)
    b = _r(1, 3, 1, 5)
    dy = g.alloc((2, 3, 4, 5))
    g.binary("mul", g.tensor(a), g.tensor(b), dy, (2, 3, 4, 5), (60, 20, 5, 1), (0, 5, 0, 1))
    np.testing.assert_allclose(dy.download(), a * b, rtol=0, atol=0)
    du = g.alloc((2, 3, 4, 5))
    g.unary("gelu_erf", g.tensor(a), du)
    from math import erf
    ref = np.vectorize(lambda v: 0.5 * v * (1 + erf(v / np.sqrt(2))))(a.astype(np.float64))
    np.testing.assert_allclose(du.download(), ref, rtol=1e-5, atol=1e-6)


def test_compare_and_select(g):
    a = _r(2, 3, 4, 5)
    b = _r(1, 3, 1, 5)
    a[0, 0, 0, :2] = b[0, 0, 0, :2]                 # equal entries
    da, db = g.tensor(a), g.tensor(b)
    st_a, st_b = (60, 20, 5, 1), (0, 5, 0, 1)
    bb = np.broadcast_to(b, a.shape)
    for op, f in (("gt", np.greater), ("ge", np.greater_equal), ("lt", np.less),
                  ("le", np.less_equal), ("eq", np.equal), ("ne", np.not_equal)):
        dy = g.alloc(a.shape)
        g.binary(op, da, db, dy, a.shape, st_a, st_b)
        np.testing.assert_array_equal(dy.download(), f(a, bb).astype(np.float32))
    # select never mixes the branches: inf / nan in the branch not taken stay out
    t = a.copy()
    t[0, 1, 2, 3] = np.inf
    e = _r(2, 3, 4, 5)
    e[1, 2, 3, 4] = np.nan
    pred = (a > 0).astype(np.float32)
    dp, dt, de, dy = g.tensor(pred), g.tensor(t), g.tensor(e), g.alloc(a.shape)
    g.select(dp, dt, de, dy, a.shape, st_a, st_a, st_a)
    np.testing.assert_array_equal(dy.download(), np.where(pred != 0, t, e))
    # broadcast predicate and scalar branch
    dz = g.alloc(a.shape)
    g.select(db, dt, g.tensor(np.array([5.0], np.float32)), dz, a.shape, st_b, st_a, (0, 0, 0, 0))
    np.testing.assert_array_equal(dz.download(), np.where(bb != 0, t, np.float32(5.0)))


def test_cuda_graph_capture_and_launch_count(g):
    x = _r(2, 8, 8, 16)
    dx, dy, dz = g.tensor(x), g.alloc((2, 8, 8, 16)), g.alloc((2, 8, 8, 16))
    w = g.tensor(_r(16, 1, 1, 16))
    g.reset_launch_count()
    g.capture_begin()
    g.conv2d_nhwc(dx, w, None, dy, activation=_lib.ACT_RELU)
    g.unary("relu6", dy, dz)
    g.capture_end()
    assert g.launch_count == 0
    for _ in range(3):
        g.replay()
    g.sync()
    assert g.launch_count == 6
    first = dz.download()
    g.upload(dx, x * 2)
    g.replay()
    second = dz.download()
    assert not np.array_equal(first, second)
    ref = np.clip(np.maximum(np.einsum("nhwc,oc->nhwo", (x * 2).astype(np.float64),
                                       w.download()[:, 0, 0, :].astype(np.float64)), 0), 0, 6)
    np.testing.assert_allclose(second, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("n,ih,c,k,s", [(3, 7, 96, 3, 1), (2, 14, 64, 3, 1), (2, 14, 32, 3, 2),
                                        (2, 16, 32, 3, 1), (2, 14, 64, 5, 1), (3, 7, 32, 5, 2),
                                        (1, 15, 32, 3, 2)])
@pytest.mark.parametrize("path", [0, 1])
def test_depthwise_small_maps_all_paths(g, n, ih, c, k, s, path):
    """Maps up to 16 x 16 through the automatic choice (TMA tiles where they
    apply, path 0) and the register sliding window (path 1), against the
    float64 reference."""
    oh = -(-ih // s)
    tot = max((oh - 1) * s + k - ih, 0)
    pt = tot // 2
    x, w, b = _r(n, ih, ih, c), _r(k, k, c), _r(c)
    dy = g.alloc((n, oh, oh, c))
    _lib.set_option("dw_path", path)
    try:
        g.depthwise_nhwc(g.tensor(x), g.tensor(w), g.tensor(b), dy, stride=(s, s), pad=(pt, pt),
                         activation=_lib.ACT_RELU6)
    finally:
        _lib.set_option("dw_path", 0)
    ref = _act(R.depthwise_nhwc(x, w, b, (s, s), (pt, pt), (oh, oh), (1, 1)), _lib.ACT_RELU6)
    np.testing.assert_allclose(dy.download(), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("n,ih,cin,ce,s", [(2, 112, 16, 96, 2), (2, 56, 24, 144, 1),
                                           (2, 56, 24, 144, 2), (3, 28, 32, 192, 1),
                                           (2, 28, 32, 192, 2), (1, 15, 16, 40, 1),
                                           (2, 13, 24, 100, 2)])
def test_expand_dw_fused(g, n, ih, cin, ce, s):
    """1x1 expand + ReLU6 then 3x3 depthwise + ReLU6 in one kernel, against
    the float64 composition of the two ops (SAME padding of the depthwise
    applies to the expanded tensor)."""
    oh = -(-ih // s)
    tot = max((oh - 1) * s + 3 - ih, 0)
    pt = tot // 2
    x = _r(n, ih, ih, cin)
    we, be = _r(ce, 1, 1, cin, scale=0.5), _r(ce)
    wd, bd = _r(3, 3, ce), _r(ce)
    e = np.clip(x.astype(np.float64) @ we.reshape(ce, cin).T.astype(np.float64) + be, 0, 6)
    ref = np.clip(R.depthwise_nhwc(e, wd, bd, (s, s), (pt, pt), (oh, oh), (1, 1)), 0, 6)
    dx, dwe, dbe, dwd, dbd = g.tensor(x), g.tensor(we), g.tensor(be), g.tensor(wd), g.tensor(bd)
    # CUDA-core expand, then the tensor-core expand (pre-split weights)
    for split in (None, g.weights_split(dwe)):
        dy = g.alloc((n, oh, oh, ce))
        g.expand_dw_nhwc(dx, dwe, dbe, dwd, dbd, dy, stride=s, pad=(pt, pt), w_split=split)
        np.testing.assert_allclose(dy.download(), ref, rtol=1e-5, atol=2e-5)
