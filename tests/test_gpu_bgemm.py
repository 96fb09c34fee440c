"""Batched attention products on the tensor cores (k_bgemm.cu): Q.K^T with
K-contiguous operands and P.V with an N-contiguous B (transposed on chip),
per (batch, head), grouped-query sharing of B heads, ragged M / N, against
float64.  "gemm_path" = 2 makes the tensor-core path mandatory, so a shape
that silently fell back to the CUDA-core GEMM would fail here.  Tolerance:
the 3xTF32 normwise bound of the other tensor-core tests."""
import numpy as np
import pytest

from spirv_inference_b200 import _lib
from spirv_inference_b200.graph import Graph

pytestmark = pytest.mark.gpu
RNG = np.random.default_rng(31)


@pytest.fixture
def g(gpu):
    with Graph(gpu) as graph:
        _lib.set_option("gemm_path", 2)
        try:
            yield graph
        finally:
            _lib.set_option("gemm_path", 0)


def _bound(k):
    return 2.5e-8 * k + 1e-6


@pytest.mark.parametrize("B,H,S,D", [(2, 12, 128, 64), (1, 3, 77, 32), (3, 2, 200, 16)])
def test_qk_transpose_per_head(g, B, H, S, D):
    hid = H * D
    q = RNG.standard_normal((B, S, hid)).astype(np.float32)
    k = RNG.standard_normal((B, S, hid)).astype(np.float32)
    dq, dk, dc = g.tensor(q), g.tensor(k), g.alloc((B, H, S, S))
    alpha = 1.0 / np.sqrt(D)
    # A = Q[b, :, h, :] (rows stride hid), B = K[b, :, h, :] stored [n][k]
    g.gemm(dq, dk, dc, m=S, n=S, k=D, batch=B, a_strides=(S * hid, hid, 1),
           b_strides=(S * hid, 1, hid), c_strides=(H * S * S, S), alpha=alpha, batch_inner=H,
           inner_strides=(D, D, S * S))
    q4 = q.reshape(B, S, H, D).astype(np.float64)
    k4 = k.reshape(B, S, H, D).astype(np.float64)
    ref = np.einsum("bshd,bthd->bhst", q4, k4) * alpha
    got = dc.download()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= _bound(D)


@pytest.mark.parametrize("B,H,S,D,div", [(2, 12, 128, 64, 1), (1, 8, 96, 64, 4), (2, 4, 52, 32, 2)])
def test_pv_with_n_contiguous_b(g, B, H, S, D, div):
    hid_v = (H // div) * D
    p = RNG.uniform(0, 1, (B, H, S, S)).astype(np.float32)
    v = RNG.standard_normal((B, S, hid_v)).astype(np.float32)
    dp, dv, dc = g.tensor(p), g.tensor(v), g.alloc((B, H, S, D))
    # A = P[b, h] (K = S contiguous); B = V[b, :, h / div, :]: element (k, n) at k*hid_v + n
    g.gemm(dp, dv, dc, m=S, n=D, k=S, batch=B, a_strides=(H * S * S, S, 1),
           b_strides=(S * hid_v, hid_v, 1), c_strides=(H * S * D, D), batch_inner=H,
           b_inner_div=div, inner_strides=(S * S, D, S * D))
    v4 = v.reshape(B, S, H // div, D).astype(np.float64)
    v4 = np.repeat(v4, div, axis=2)
    ref = np.einsum("bhst,bthd->bhsd", p.astype(np.float64), v4)
    got = dc.download()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= _bound(S)


def test_long_reduction_is_not_taken(g):
    """K > 128 is outside the batched kernel: with the tensor-core path
    mandatory the call is refused rather than silently run elsewhere."""
    a = RNG.standard_normal((2, 16, 200)).astype(np.float32)
    b = RNG.standard_normal((2, 8, 200)).astype(np.float32)
    with pytest.raises(_lib.SpxError) as e:
        g.gemm(g.tensor(a), g.tensor(b), g.alloc((2, 16, 8)), m=16, n=8, k=200, batch=2,
               a_strides=(3200, 200, 1), b_strides=(1600, 1, 200), c_strides=(128, 8))
    assert e.value.code == _lib.SPX_ERR_UNSUPPORTED
