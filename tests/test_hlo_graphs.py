"""CPU tests of the HLO-path graphs and the reference-semantics lowering
(hlo.run_hlo on the oracle) against an independent float64 interpreter."""
import numpy as np
import pytest

import _np_ref as R
from spirv_inference_b200 import hlo, nets_hlo


def test_resnet50_structure():
    g = nets_hlo.resnet50(hw=224)
    h = g.histogram()
    assert h["convolution"] == 53 and h["reduce-window"] == 1 and h["dot"] == 1
    assert g.op(g.output).shape == (1, 1000)
    convs = [o for o in g.ops if o.opcode == "convolution"]
    assert convs[0].shape == (1, 112, 112, 64) and convs[-1].shape == (1, 7, 7, 2048)


def test_bert_structure():
    g = nets_hlo.bert_encoder(seq=128, layers=12)
    assert g.histogram()["dot"] == 12 * 8
    assert g.op(g.output).shape == (1, 128, 768)


@pytest.mark.parametrize("case", ["resnet", "bert", "fixture"])
def test_run_hlo_oracle_matches_float64(oracle_built, case):
    if case == "resnet":
        g = nets_hlo.resnet50(seed=3, hw=48)
        x = nets_hlo.make_image_batch(1, 48, seed=9)
    elif case == "bert":
        g = nets_hlo.bert_encoder(seed=4, seq=8, layers=1)
        x = nets_hlo.bert_embed(4, np.arange(8)[None] * 37)
    else:
        g, x = nets_hlo.bert_block_fixture()
    feeds = {g.inputs[0]: x}
    out, rep = hlo.run_hlo(g, feeds, oracle_built.run_kernel)
    ref = R.eval_hlo_f64(g, feeds)
    assert np.abs(out - ref).max() / np.abs(ref).max() < 1e-5
    # compiler.rs dispatches exactly the device-lowered ops
    devops = sum(v for k, v in g.histogram().items()
                 if k in ("convolution", "reduce-window", "reduce", "dot", "pad") or k in hlo.ELEMENTWISE)
    assert rep["num_dispatches"] == devops


def test_host_broadcast_semantics():
    src = np.arange(3, dtype=np.float32)
    out = hlo.broadcast_host(src, (2, 3), (1,))
    np.testing.assert_array_equal(out, [[0, 1, 2], [0, 1, 2]])
    assert hlo.infer_broadcast_dims((3,), (2, 4, 3)) == [2]
    np.testing.assert_array_equal(hlo.broadcast_host(np.array(5.0, np.float32), (2, 2), ()),
                                  np.full((2, 2), 5.0))
