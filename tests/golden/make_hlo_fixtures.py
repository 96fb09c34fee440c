"""Generates the parsed-HLO fixtures used by the GPU front-end tests.

The reference exports its StableHLO/XLA graphs as HLO text under
source/xla_hlo/fixtures/ (bert_base.stablehlo.txt: one BERT attention block
with three parameters; resnet50.stablehlo.txt: ResNet-50 at batch 1 with
BatchNorm left unfused, 321 parameters).  This script parses them with
spirv_inference_b200.hlo_text (the front-end under test, parser.rs:5-264
semantics) and writes the parsed graphs as compact JSON next to this file, so
that the tests that run on a GPU machine (where the reference checkout is not
present) execute exactly the graphs the parser produced here.  Each JSON
records the sha256 of the HLO text it came from.

Usage: python tests/golden/make_hlo_fixtures.py <reference checkout root>
       (or set SPX_REFERENCE_ROOT)
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from spirv_inference_b200 import hlo_text  # noqa: E402
from spirv_inference_b200.hlo import HloGraph, HloOp  # noqa: E402

NAMES = ("bert_base", "resnet50")


def _jsonable(v):
    if isinstance(v, (tuple, list)):
        return [_jsonable(x) for x in v]
    if isinstance(v, float) and (v != v or v in (float("inf"), float("-inf"))):
        return {"float": repr(v)}
    return v


def _unjson(v):
    if isinstance(v, list):
        return tuple(_unjson(x) for x in v)
    if isinstance(v, dict) and "float" in v:
        return float(v["float"])
    return v


def dump(g: HloGraph, source_sha256: str) -> dict:
    return {"name": g.name, "source_sha256": source_sha256, "inputs": list(g.inputs),
            "output": g.output,
            "ops": [[o.name, o.opcode, list(o.operands), list(o.shape),
                     {k: _jsonable(v) for k, v in o.attrs.items()}] for o in g.ops]}


def load(path: Path) -> HloGraph:
    """The parsed graph back as an HloGraph (no bound parameters)."""
    d = json.loads(Path(path).read_text())
    ops = [HloOp(n, oc, list(opr), tuple(sh), {k: _unjson(v) for k, v in at.items()})
           for n, oc, opr, sh, at in d["ops"]]
    return HloGraph(d["name"], ops, {}, list(d["inputs"]), d["output"])


def main(ref_root: str) -> None:
    fix = Path(ref_root) / "source" / "xla_hlo" / "fixtures"
    for name in NAMES:
        text = (fix / f"{name}.stablehlo.txt").read_text()
        g = hlo_text.parse(text)
        sha = hashlib.sha256(text.encode()).hexdigest()
        out = HERE / f"{name}.hlo.json"
        out.write_text(json.dumps(dump(g, sha), separators=(",", ":")))
        print(f"{out.name}: {len(g.ops)} ops, {len(g.inputs)} parameters")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SPX_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: make_hlo_fixtures.py <reference root> (or SPX_REFERENCE_ROOT)")
    main(root)
