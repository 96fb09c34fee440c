"""The XLA HLO text front-end on the reference's exported graphs.

The committed parses (tests/golden/*.hlo.json, made by
tests/golden/make_hlo_fixtures.py) are checked here: op census, parameter
order and shapes, and evaluation through the reference executor's lowering
with the CPU oracle as the kernel boundary against an independent float64
evaluation.  Where a reference checkout is named by SPX_REFERENCE_ROOT, the
HLO text itself is parsed again (tinyllama included) and compared with the
committed parse; without it those tests are skipped."""
import hashlib
import os
from pathlib import Path

import numpy as np
import pytest

import _np_ref
from _hlo_fixtures import bind, load_fixture
from spirv_inference_b200 import hlo, hlo_text

_ROOT = os.environ.get("SPX_REFERENCE_ROOT")
FIX = Path(_ROOT) / "source" / "xla_hlo" / "fixtures" if _ROOT else None
needs_ref = pytest.mark.skipif(FIX is None or not FIX.exists(),
                               reason="SPX_REFERENCE_ROOT does not name a reference checkout")


def _parse(name):
    return hlo_text.parse((FIX / f"{name}.stablehlo.txt").read_text())


@needs_ref
def test_tinyllama_census():
    g = _parse("tinyllama")
    h = g.histogram()
    assert len(g.inputs) == 4 + 22 * 9 + 2
    assert h["dot"] == 199 and h["rsqrt"] == 45 and h["logistic"] == 22
    assert g.op(g.output).shape == (1, 64, 32000)
    assert g.op(g.inputs[5]).shape == (2048, 2048) and g.op(g.inputs[6]).shape == (2048, 256)
    kinds = {o.attrs["kind"] for o in g.ops if o.opcode == "reduce"}
    assert kinds == {"sum", "max"}


@needs_ref
@pytest.mark.parametrize("name", ["bert_base", "resnet50"])
def test_committed_parse_is_current(name):
    text = (FIX / f"{name}.stablehlo.txt").read_text()
    g, c = hlo_text.parse(text), load_fixture(name)
    import json
    meta = json.loads((Path(__file__).parent / "golden" / f"{name}.hlo.json").read_text())
    assert meta["source_sha256"] == hashlib.sha256(text.encode()).hexdigest()
    assert (g.inputs, g.output) == (c.inputs, c.output)
    assert [(o.name, o.opcode, o.operands, o.shape) for o in g.ops] == \
        [(o.name, o.opcode, o.operands, o.shape) for o in c.ops]
    for a, b in zip(g.ops, c.ops):
        assert set(a.attrs) == set(b.attrs)
        for k in a.attrs:
            assert np.array_equal(np.asarray(a.attrs[k], dtype=object),
                                  np.asarray(b.attrs[k], dtype=object)), (a.name, k)


def test_resnet50_census():
    g = load_fixture("resnet50")
    h = g.histogram()
    assert h["convolution"] == 53 and h["reduce-window"] == 1 and h["dot"] == 1
    assert h["rsqrt"] == 53 and len(g.inputs) == 321
    conv = next(o for o in g.ops if o.opcode == "convolution" and o.shape[1] == 112)
    assert conv.attrs["stride"] == (2, 2)
    rw = next(o for o in g.ops if o.opcode == "reduce-window")
    assert rw.attrs["kind"] == "max" and rw.attrs["size"] == (3, 3) and rw.attrs["stride"] == (2, 2)


def test_bert_block_runs_with_reference_lowering(oracle_built):
    g = load_fixture("bert_base")
    rng = np.random.default_rng(0)
    feeds = {n: (rng.standard_normal(g.op(n).shape) * 0.05).astype(np.float32) for n in g.inputs}
    out, rep = hlo.run_hlo(g, feeds, oracle_built.run_kernel)
    ref = _np_ref.eval_hlo_f64(g, feeds)
    assert rep["num_dispatches"] > 0
    assert np.abs(out - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())


def test_resnet50_fixture_oracle_vs_float64(oracle_built):
    """The bound ResNet-50 fixture (the GPU front-end test's case) through the
    reference lowering on the oracle against float64: a non-degenerate
    softmax, identical argmax."""
    g, feeds = bind(load_fixture("resnet50"), seed=17)
    out, _ = hlo.run_hlo(g, feeds, oracle_built.run_kernel)
    allf = dict(feeds)
    allf.update(g.params)
    ref = _np_ref.eval_hlo_f64(g, allf)
    assert 1e-3 < out.max() < 0.5            # not saturated to one-hot
    assert np.abs(out - ref).max() <= 1e-6
    assert int(np.argmax(out)) == int(np.argmax(ref))
