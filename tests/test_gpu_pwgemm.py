"""The resident-tile pointwise GEMM (k_pwgemm.cu) behind conv2d_nhwc for 1x1
convolutions with a short reduction and a wide output (the expand convs on
14x14 / 7x7 maps): against float64 (3xTF32 normwise bound) and against the
row-tiled tensor-core GEMM (`pw_gemm` = 0, the default), ragged M and N, K
not a multiple of 32, bias + ReLU6."""
import numpy as np
import pytest

from spirv_inference_b200 import _lib
from spirv_inference_b200.graph import Graph

pytestmark = pytest.mark.gpu
RNG = np.random.default_rng(41)


@pytest.fixture
def g(gpu):
    with Graph(gpu) as graph:
        yield graph


@pytest.mark.parametrize("n,h,cin,cout", [(2, 14, 64, 384), (3, 7, 160, 960), (1, 9, 96, 576),
                                          (2, 5, 20, 132), (4, 3, 128, 1280)])
def test_pwgemm_matches_float64_and_row_tiled(g, n, h, cin, cout):
    x = RNG.uniform(0, 4, (n, h, h, cin)).astype(np.float32)
    w = (RNG.standard_normal((cout, 1, 1, cin)) * np.sqrt(2.0 / cin)).astype(np.float32)
    b = RNG.uniform(-0.1, 0.1, cout).astype(np.float32)
    dx, dw, db = g.tensor(x), g.tensor(w), g.tensor(b)
    split = g.weights_split(dw)
    outs = []
    for pw in (1, 0):
        _lib.set_option("pw_gemm", pw)
        try:
            dy = g.alloc((n, h, h, cout))
            g.conv2d_nhwc(dx, dw, db, dy, activation=_lib.ACT_RELU6, w_split=split)
            outs.append(dy.download())
        finally:
            _lib.set_option("pw_gemm", 0)
    ref = np.clip(x.reshape(-1, cin).astype(np.float64) @ w.reshape(cout, cin).T + b, 0, 6)
    ref = ref.reshape(n, h, h, cout)
    scale = np.abs(ref).max()
    for o in outs:
        assert np.abs(o - ref).max() / scale <= 2.5e-8 * cin + 1e-6
    assert np.abs(outs[0] - outs[1]).max() / scale <= 2 * (2.5e-8 * cin + 1e-6)
