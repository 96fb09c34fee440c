"""TFLite FlatBuffer front-end: the seeded CNN graphs written as .tflite
files and read back (ops, options, shapes and weights identical), the
reference loader's rejections (model.rs:260-270: too small, missing TFL3
identifier) and an unsupported operator code; the scheduler semantics give identical outputs on
the read-back graph (CPU oracle)."""
import numpy as np
import pytest

from spirv_inference_b200 import lowering, nets, tflite


@pytest.fixture(scope="module", params=["mobilenet_v2", "efficientnet_lite0"])
def roundtrip(request):
    m = nets.MODELS[request.param](seed=0)
    return m, tflite.read_tflite(tflite.write_tflite(m))


def test_roundtrip_graph(roundtrip):
    m, r = roundtrip
    assert (r.input, r.output) == (m.input, m.output)
    assert [o.type for o in r.ops] == [o.type for o in m.ops]
    for a, b in zip(m.ops, r.ops):
        assert (a.inputs, a.output) == (b.inputs, b.output)
        for k, v in a.attrs.items():
            assert b.attrs[k] == v, (a.type, k)
    assert set(r.weights) == set(m.weights)
    for k, v in m.weights.items():
        assert np.array_equal(r.weights[k], v)
    for k, v in m.shapes.items():
        if k not in m.weights:
            assert r.shapes[k] == tuple(v)


def test_rejections():
    with pytest.raises(tflite.TFLiteError, match="too small"):
        tflite.read_tflite(b"1234")
    with pytest.raises(tflite.TFLiteError, match="TFL3"):
        tflite.read_tflite(b"\0" * 16)


def test_unsupported_opcode_is_rejected(monkeypatch):
    m = nets.mobilenet_v2(seed=0)
    monkeypatch.setitem(tflite.CODE, "CONV_2D", 99)
    data = tflite.write_tflite(m)
    monkeypatch.undo()
    with pytest.raises(tflite.TFLiteError, match="unsupported builtin operator code 99"):
        tflite.read_tflite(data)


def test_scheduler_outputs_identical(oracle_built):
    m = nets.mobilenet_v2(seed=0)
    r = tflite.read_tflite(tflite.write_tflite(m))
    x = nets.make_input(m, 1, seed=3)
    a = lowering.run_graph(m, x, oracle_built.run_kernel)[0]
    b = lowering.run_graph(r, x, oracle_built.run_kernel)[0]
    assert np.array_equal(a, b)
