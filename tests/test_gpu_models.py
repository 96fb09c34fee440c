"""Model-level parity on the GPU.

The fused NHWC executor and the drop-in per-op lowering through
spx_run_kernel are both compared with the reference scheduler's semantics
executed on the CPU oracle, on the same seeded inputs and weights.  Gate
identical top-1 and max |softmax difference| <= 1e-4.
"""
import numpy as np
import pytest

from spirv_inference_b200 import dispatch, lowering, nets
from spirv_inference_b200.executor import CnnExecutor

pytestmark = pytest.mark.gpu
SOFTMAX_ATOL = 1e-4


def spx_rk(kernel, in0, in1, nout, push):
    return dispatch.run_kernel(0, dispatch.KernelRun("t", kernel, in0, in1, nout, 0, push)).values


@pytest.fixture(scope="module")
def oracle_outputs(oracle_built):
    out = {}
    for name in ("mobilenet_v2", "efficientnet_lite0"):
        m = nets.MODELS[name](seed=0)
        x = nets.make_input(m, 3, seed=99)
        ref, rep = lowering.run_graph(m, x, oracle_built.run_kernel, keep=True)
        out[name] = (m, x, ref, rep)
    return out


@pytest.mark.parametrize("name", ["mobilenet_v2", "efficientnet_lite0"])
def test_fused_executor_matches_oracle(gpu, oracle_outputs, name):
    m, x, ref, rep = oracle_outputs[name]
    ex = CnnExecutor(m, batch=x.shape[0], device=gpu)
    try:
        got = ex.forward(x)
        assert got.shape == ref.shape
        np.testing.assert_array_equal(lowering.top1(got), lowering.top1(ref))
        assert float(np.abs(got - ref).max()) <= SOFTMAX_ATOL
        # an intermediate feature map (an expand conv's output: the depthwise
        # outputs stay on chip in the fused kernel), NHWC on the device vs NCHW
        # in the oracle
        mid = [op.inputs[0] for op in m.ops if op.type == "DEPTHWISE_CONV_2D"][8]
        assert mid not in ex.fused_away
        h, w, c = m.shapes[mid]
        ref_mid = rep["tensors"][mid].reshape(x.shape[0], c, h, w).transpose(0, 2, 3, 1)
        np.testing.assert_allclose(ex.tensor(mid), ref_mid, rtol=1e-3, atol=1e-3)
        # CUDA-graph replay reproduces the eager result bit for bit
        ex.capture()
        ex.g.upload(ex.input, x)
        ex.run()
        again = ex.g.download(ex.output)
        np.testing.assert_array_equal(again, got)
    finally:
        ex.close()


def test_dropin_lowering_matches_oracle(gpu, oracle_built, oracle_outputs):
    m, x, ref, _ = oracle_outputs["mobilenet_v2"]
    got, rep = lowering.run_graph(m, x[:1], spx_rk)
    ref1, _ = lowering.run_graph(m, x[:1], oracle_built.run_kernel)
    np.testing.assert_array_equal(lowering.top1(got), lowering.top1(ref1))
    assert float(np.abs(got - ref1).max()) <= SOFTMAX_ATOL
    assert rep["num_dispatches"] == 102


def test_executor_batch_shards_are_independent(gpu, oracle_outputs):
    """Batch sharding (the multi-GPU plan) is exact: image i's output does not
    depend on which shard or batch size it ran in."""
    m, x, _, _ = oracle_outputs["mobilenet_v2"]
    full = CnnExecutor(m, batch=3, device=gpu)
    one = CnnExecutor(m, batch=1, device=gpu)
    try:
        a = full.forward(x)
        b = one.forward(x[2:3])
        np.testing.assert_allclose(a[2:3], b, rtol=0, atol=1e-6)
    finally:
        full.close()
        one.close()


def test_mnv2_expand_dw_fusion_matches_unfused(gpu):
    """The fused expand -> depthwise path (opt-in) against the default
    executor on the same MobileNetV2 batch."""
    import numpy as np
    from spirv_inference_b200 import nets
    from spirv_inference_b200.executor import CnnExecutor
    m = nets.mobilenet_v2(seed=0)
    x = nets.make_input(m, 4, seed=11)
    outs = []
    for fuse in (False, True):
        ex = CnnExecutor(m, batch=4, device=gpu, fuse_expand_dw=fuse)
        try:
            outs.append(ex.forward(x))
            if fuse:
                assert sum(k == "expand_dw" for k, _ in ex._plan) == 6
        finally:
            ex.close()
    assert np.abs(outs[0] - outs[1]).max() <= 1e-4
    assert np.array_equal(outs[0].argmax(1), outs[1].argmax(1))
