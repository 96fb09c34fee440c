"""The reference's exported HLO graphs, as parsed and committed under
tests/golden/*.hlo.json by tests/golden/make_hlo_fixtures.py, with seeded
parameter values bound to them."""
import sys
from pathlib import Path

import numpy as np

from spirv_inference_b200.hlo import HloGraph

GOLDEN = Path(__file__).resolve().parent / "golden"
if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))
import make_hlo_fixtures  # noqa: E402


def load_fixture(name: str) -> HloGraph:
    return make_hlo_fixtures.load(GOLDEN / f"{name}.hlo.json")


def _consumer_chain(g: HloGraph, name: str, depth: int = 3) -> list[str]:
    cons: dict[str, list] = {}
    for o in g.ops:
        for x in o.operands:
            cons.setdefault(x, []).append(o)
    out, cur = [], name
    for _ in range(depth):
        c = cons.get(cur)
        if not c:
            break
        out.append(c[0].opcode)
        cur = c[0].name
    return out


def bind(g: HloGraph, seed: int) -> tuple[HloGraph, dict]:
    """Seeded values for every parameter: parameter 0 is fed per run, the
    others are bound as weights.  Rank-4 HWIO filters He-normal, rank-2
    matrices N(0, 1/in); rank-1 vectors by the role their first consumers
    give them in an inference-mode BatchNorm: the variance (the operand of
    `add` -> `rsqrt`) U[1, 2], the scale (`multiply` -> `reshape`) U[0.5, 1],
    the others N(0, 0.05).  The fed input is N(0, 1)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    params = {}
    for name in g.inputs[1:]:
        shape = g.op(name).shape
        ch = _consumer_chain(g, name)
        if len(shape) == 4:
            fan = shape[0] * shape[1] * shape[2]
            a = rng.standard_normal(shape) * np.sqrt(2.0 / fan)
        elif len(shape) == 2:
            a = rng.standard_normal(shape) / np.sqrt(shape[0])
        elif "rsqrt" in ch:
            a = rng.uniform(1.0, 2.0, shape)
        elif ch[1:3] == ["multiply", "reshape"]:
            a = rng.uniform(0.5, 1.0, shape)
        else:
            a = rng.standard_normal(shape) * 0.05
        params[name] = a.astype(np.float32)
    bound = HloGraph(g.name, g.ops, params, [g.inputs[0]], g.output)
    x = rng.standard_normal(g.op(g.inputs[0]).shape).astype(np.float32)
    return bound, {g.inputs[0]: x}
