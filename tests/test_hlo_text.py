"""The XLA HLO text front-end on the reference's exported graphs: op census,
parameter order and shapes, and (for BERT's small block) evaluation through
the reference executor's lowering with the CPU oracle as the kernel
boundary against an independent float64 evaluation.  Skipped where the
reference checkout is not mounted."""
from pathlib import Path

import numpy as np
import pytest

import _np_ref
from spirv_inference_b200 import hlo, hlo_text

FIX = Path("/root/reference/source/xla_hlo/fixtures")
pytestmark = pytest.mark.skipif(not FIX.exists(), reason="reference fixtures not mounted")


def _parse(name):
    return hlo_text.parse((FIX / f"{name}.stablehlo.txt").read_text())


def test_tinyllama_census():
    g = _parse("tinyllama")
    h = g.histogram()
    assert len(g.inputs) == 4 + 22 * 9 + 2
    assert h["dot"] == 199 and h["rsqrt"] == 45 and h["logistic"] == 22
    assert g.op(g.output).shape == (1, 64, 32000)
    assert g.op(g.inputs[5]).shape == (2048, 2048) and g.op(g.inputs[6]).shape == (2048, 256)
    kinds = {o.attrs["kind"] for o in g.ops if o.opcode == "reduce"}
    assert kinds == {"sum", "max"}


def test_resnet50_census():
    g = _parse("resnet50")
    h = g.histogram()
    assert h["convolution"] == 53 and h["reduce-window"] == 1 and h["dot"] == 1
    conv = next(o for o in g.ops if o.opcode == "convolution" and o.shape[1] == 112)
    assert conv.attrs["stride"] == (2, 2)
    rw = next(o for o in g.ops if o.opcode == "reduce-window")
    assert rw.attrs["kind"] == "max" and rw.attrs["size"] == (3, 3) and rw.attrs["stride"] == (2, 2)


def test_bert_block_runs_with_reference_lowering(oracle_built):
    g = _parse("bert_base")
    rng = np.random.default_rng(0)
    feeds = {n: (rng.standard_normal(g.op(n).shape) * 0.05).astype(np.float32) for n in g.inputs}
    out, rep = hlo.run_hlo(g, feeds, oracle_built.run_kernel)
    ref = _np_ref.eval_hlo_f64(g, feeds)
    assert rep["num_dispatches"] > 0
    assert np.abs(out - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())
