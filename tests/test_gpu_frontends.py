"""The reference's own front-end inputs executed by libspx on the GPU.

* HLO text (source/xla_hlo/src/parser.rs:5-264): the reference's exported
  graphs bert_base.stablehlo.txt (one attention block) and
  resnet50.stablehlo.txt (batch 1, BatchNorm unfused: every add / multiply /
  rsqrt / subtract of the inference-mode BN runs as its own HLO op), parsed
  by hlo_text and committed as tests/golden/*.hlo.json by
  tests/golden/make_hlo_fixtures.py, run through HloExecutor and compared
  with the reference executor semantics (hlo.run_hlo, compiler.rs:267-668)
  on the CPU oracle, same seeded parameters.
* TFLite FlatBuffer (source/tflite_loader/src/model.rs:260-362): the seeded
  CNNs written as .tflite bytes, read back by tflite.read_tflite, run on
  CnnExecutor, compared with the oracle on the original graph.
"""
import numpy as np
import pytest

from spirv_inference_b200 import hlo, lowering, nets, tflite
from spirv_inference_b200.executor import CnnExecutor
from spirv_inference_b200.executor_hlo import HloExecutor
from spirv_inference_b200.hlo import HloGraph

pytestmark = pytest.mark.gpu
from _hlo_fixtures import bind, load_fixture  # noqa: E402


@pytest.mark.parametrize("name", ["bert_base", "resnet50"])
@pytest.mark.parametrize("fuse", [True, False])
def test_reference_hlo_fixture_on_gpu(gpu, oracle_built, name, fuse):
    g, feeds = bind(load_fixture(name), seed=17)
    ref, _ = hlo.run_hlo(g, feeds, oracle_built.run_kernel)
    ex = HloExecutor(g, device=gpu, fuse=fuse)
    try:
        got = ex.forward(feeds)
    finally:
        ex.close()
    assert got.shape == ref.shape
    if name == "resnet50":
        # the graph ends in a softmax: the north-star softmax gate
        assert float(np.abs(got - ref).max()) <= 1e-4
        assert int(np.argmax(got)) == int(np.argmax(ref))
    else:
        err = float(np.abs(got - ref).max() / np.abs(ref).max())
        assert err <= 1e-3, err


@pytest.mark.parametrize("name", ["mobilenet_v2", "efficientnet_lite0"])
def test_tflite_bytes_on_gpu(gpu, oracle_built, name):
    m = nets.MODELS[name](seed=0)
    data = tflite.write_tflite(m)
    assert data[4:8] == b"TFL3"
    r = tflite.read_tflite(data)
    x = nets.make_input(m, 4, seed=21)
    ex = CnnExecutor(r, batch=4, device=gpu)
    try:
        got = ex.forward(x)
    finally:
        ex.close()
    ref, _ = lowering.run_graph(m, x, oracle_built.run_kernel)
    np.testing.assert_array_equal(lowering.top1(got), lowering.top1(ref))
    assert float(np.abs(got - ref).max()) <= 1e-4
