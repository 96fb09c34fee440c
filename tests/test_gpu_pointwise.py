"""GPU tests of the CUDA-core pointwise (1x1) convolution kernel that takes
the short-reduction expand / project layers: float64 numpy reference, every
chunking mode (K <= 64 with N in chunks; K > 64 in 32-channel reduction
chunks, a partial last one included), ragged pixel tiles, residual and
activations, and agreement with the tensor-core path.  The kernel is
opt-in (option pw_path = 1)."""
import numpy as np
import pytest

from spirv_inference_b200 import _lib
from spirv_inference_b200.graph import Graph

pytestmark = pytest.mark.gpu
RNG = np.random.default_rng(33)


@pytest.fixture
def g(gpu):
    _lib.set_option("pw_path", 1)
    try:
        with Graph(gpu) as graph:
            yield graph
    finally:
        _lib.set_option("pw_path", 0)


def _r(*shape, scale=1.0):
    return (RNG.uniform(-1, 1, size=shape) * scale).astype(np.float32)


def _ref(x, wt, b, res, act):
    n, h, w, ic = x.shape
    oc = wt.shape[0]
    y = x.reshape(-1, ic).astype(np.float64) @ wt.reshape(oc, ic).T.astype(np.float64) + b
    if res is not None:
        y = y + res.reshape(-1, oc)
    if act == _lib.ACT_RELU6:
        y = np.clip(y, 0, 6)
    elif act == _lib.ACT_RELU:
        y = np.maximum(y, 0)
    return y.reshape(n, h, w, oc)


# (n, h, w, ic, oc): MobileNetV2 / EfficientNet-Lite0 shapes plus ragged tiles.
CASES = [
    (2, 112, 112, 32, 16), (2, 112, 112, 16, 96), (3, 56, 56, 96, 24), (2, 56, 56, 24, 144),
    (2, 56, 56, 144, 24), (2, 28, 28, 144, 32), (2, 28, 28, 32, 192), (2, 28, 28, 192, 32),
    (2, 28, 28, 144, 40), (1, 7, 9, 100, 16), (1, 5, 5, 4, 8), (1, 13, 11, 60, 40),
]


@pytest.mark.parametrize("n,h,w,ic,oc", CASES)
@pytest.mark.parametrize("act,with_res", [(_lib.ACT_RELU6, False), (_lib.ACT_NONE, True)])
def test_pointwise_matches_fp64(g, n, h, w, ic, oc, act, with_res):
    x = _r(n, h, w, ic)
    wt = _r(oc, 1, 1, ic, scale=1.0 / np.sqrt(ic))
    b = _r(oc)
    res = _r(n, h, w, oc) if with_res else None
    dy = g.alloc((n, h, w, oc))
    launches = g.launch_count
    g.conv2d_nhwc(g.tensor(x), g.tensor(wt), g.tensor(b), dy, activation=act,
                  residual=g.tensor(res) if res is not None else None)
    out = dy.download()
    assert g.launch_count == launches + 1
    # Exact fp32 products accumulated in channel order: fp32 rounding only.
    np.testing.assert_allclose(out, _ref(x, wt, b, res, act), rtol=1e-5, atol=2e-6 * np.sqrt(ic))


def test_pointwise_agrees_with_tensor_core_path(g):
    n, h, w, ic, oc = 4, 56, 56, 24, 144
    x, wt, b = _r(n, h, w, ic), _r(oc, 1, 1, ic, scale=0.3), _r(oc)
    ys = []
    for path in (1, 0):
        _lib.set_option("pw_path", path)
        dy = g.alloc((n, h, w, oc))
        g.conv2d_nhwc(g.tensor(x), g.tensor(wt), g.tensor(b), dy, activation=_lib.ACT_RELU6)
        ys.append(dy.download())
    np.testing.assert_allclose(ys[0], ys[1], rtol=2e-5, atol=2e-5)


def test_pointwise_option_range():
    with pytest.raises(Exception):
        _lib.set_option("pw_path", 2)
    assert _lib.get_option("pw_path") == 0
    assert _lib.get_option("tc_wide_epilogue") == 1
