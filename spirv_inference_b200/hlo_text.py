"""XLA HLO text front-end: parses the reference's exported graphs
(source/xla_hlo/fixtures/*.stablehlo.txt, XLA HLO text form) into the
`hlo.HloGraph` IR, so they run through `hlo.run_hlo` (the reference
executor's lowering semantics) or the device executor.

Follows the reference parser (source/xla_hlo/src/parser.rs:5-264): only the
ENTRY computation's instructions become ops; other computations are the
reducers named by `to_apply=`.  A reduce is a max-reduce when its reducer is
named %max... or its init value is -inf, a sum otherwise (the rule of
compiler.rs:1722-1728).  Shapes drop their layout suffix ({2,1,0}); integer
and predicate element types are carried as float32, as the reference
executor does.  Ops are kept in dependency order (the textual order of an
XLA dump, re-sorted stably if an operand would otherwise come later).
"""
from __future__ import annotations

import re

import numpy as np

from .hlo import HloGraph, HloOp

_SHAPE = re.compile(r"^\(?\s*([a-z0-9]+)\[([0-9,]*)\]")
_INSTR = re.compile(r"^(ROOT\s+)?%([\w.\-]+)\s*=\s*(.+?)\s+([a-z][a-z0-9\-]*)\((.*)$")


def _shape(text: str) -> tuple[int, ...]:
    m = _SHAPE.match(text.strip())
    if not m:
        return ()
    dims = m.group(2)
    return tuple(int(d) for d in dims.split(",")) if dims else ()


def _split_args(s: str) -> tuple[str, str]:
    """Splits 'a, b), attr=...' at the parenthesis closing the operand list."""
    depth = 1
    for i, ch in enumerate(s):
        if ch in "({[":
            depth += 1
        elif ch in ")}]":
            depth -= 1
            if depth == 0:
                return s[:i], s[i + 1:]
    return s, ""


def _top_split(s: str, sep: str = ",") -> list[str]:
    out, depth, cur = [], 0, []
    for ch in s:
        if ch in "({[":
            depth += 1
        elif ch in ")}]":
            depth -= 1
        if ch == sep and depth == 0:
            out.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
    if "".join(cur).strip():
        out.append("".join(cur))
    return [x.strip() for x in out]


def _ints(s: str) -> tuple[int, ...]:
    s = s.strip().strip("{}")
    return tuple(int(x) for x in s.split(",") if x.strip())


def _attrs(tail: str) -> dict[str, str]:
    out = {}
    for part in _top_split(tail.lstrip(", ")):
        if "=" in part:
            k, v = part.split("=", 1)
            out[k.strip()] = v.strip()
    return out


def _window(spec: str) -> dict:
    """window={size=3x3 stride=2x2 pad=0_1x0_1} -> sizes, strides, pads."""
    spec = spec.strip("{}")
    out = {}
    for item in spec.split():
        k, v = item.split("=", 1)
        if k == "pad":
            out[k] = tuple(tuple(int(x) for x in p.split("_")) for p in v.split("x"))
        else:
            out[k] = tuple(int(x) for x in v.split("x"))
    return out


def _constant(arg: str) -> float:
    a = arg.strip().strip("{}").strip()
    if a in ("-inf", "-Inf"):
        return -np.inf
    if a in ("inf", "Inf"):
        return np.inf
    if a in ("true", "false"):
        return 1.0 if a == "true" else 0.0
    try:
        return float(a)
    except ValueError:
        vals = [float(x) for x in re.split(r"[,\s{}]+", a) if x]
        if len(set(vals)) != 1:
            raise NotImplementedError(f"array constant with distinct values: {arg[:40]}")
        return vals[0]


def parse(text: str, name: str | None = None) -> HloGraph:
    """Parses XLA HLO text into an HloGraph whose inputs are the ENTRY
    parameters in parameter-number order."""
    comps: dict[str, list[str]] = {}
    entry = None
    cur = None
    for line in text.splitlines():
        t = line.strip()
        if not t or t.startswith("HloModule"):
            continue
        head = re.match(r"^(ENTRY\s+)?%([\w.\-]+)\s*\(.*\)\s*->.*\{$", t)
        if head:
            cur = head.group(2)
            comps[cur] = []
            if head.group(1):
                entry = cur
            continue
        if t == "}":
            cur = None
            continue
        if cur is not None:
            comps[cur].append(t)
    if entry is None:
        raise ValueError("no ENTRY computation")

    def reducer_kind(comp: str) -> str | None:
        for ln in comps.get(comp, []):
            m = _INSTR.match(ln)
            if m and m.group(1):
                return m.group(4)
        return None

    ops: list[HloOp] = []
    params: dict[int, str] = {}
    consts: dict[str, float] = {}
    root = None
    for ln in comps[entry]:
        m = _INSTR.match(ln)
        if not m:
            continue
        is_root, res, rtype, opcode, rest = m.groups()
        args_s, tail = _split_args(rest)
        shape = _shape(rtype)
        attrs = _attrs(tail)
        operands = re.findall(r"%([\w.\-]+)", args_s) if opcode not in ("parameter",
                                                                        "constant") else []
        a: dict = {}
        if opcode == "parameter":
            params[int(args_s.strip())] = res
        elif opcode == "constant":
            a["value"] = _constant(args_s)
            consts[res] = a["value"]
        elif opcode in ("broadcast", "transpose", "reduce", "concatenate"):
            a["dimensions"] = _ints(attrs.get("dimensions", "{}"))
        if opcode == "reduce":
            init = consts.get(operands[1], 0.0) if len(operands) > 1 else 0.0
            ap = attrs.get("to_apply", "").lstrip("%")
            a["kind"] = "max" if (ap.startswith("max") or (np.isinf(init) and init < 0)
                                  or reducer_kind(ap) == "maximum") else "sum"
        elif opcode == "dot":
            for k in ("lhs_contracting_dims", "rhs_contracting_dims", "lhs_batch_dims",
                      "rhs_batch_dims"):
                a[k] = _ints(attrs.get(k, "{}"))
        elif opcode == "slice":
            rngs = re.findall(r"\[(-?\d+):(-?\d+)(?::(-?\d+))?\]", attrs.get("slice", ""))
            a["slice"] = tuple((int(s), int(e), int(st) if st else 1) for s, e, st in rngs)
        elif opcode == "get-tuple-element":
            a["index"] = int(attrs.get("index", "0"))
        elif opcode == "compare":
            a["direction"] = attrs.get("direction", "GT")
        elif opcode == "pad":
            a["padding"] = tuple(tuple(int(x) for x in p.split("_")[:2])
                                 for p in attrs.get("padding", "").split("x"))
        elif opcode == "convolution":
            w = _window(attrs.get("window", "{}"))
            a["stride"] = w.get("stride", (1, 1))
            a["pad"] = w.get("pad", ((0, 0), (0, 0)))
            a["dim_labels"] = attrs.get("dim_labels", "b01f_01io->b01f")
        elif opcode == "reduce-window":
            w = _window(attrs.get("window", "{}"))
            # NHWC windows: the spatial entries of a rank-4 window spec.
            size, st = w.get("size", (1, 1, 1, 1)), w.get("stride", (1, 1, 1, 1))
            pd = w.get("pad", ((0, 0),) * len(size))
            a["size"], a["stride"], a["pad"] = size[1:3], st[1:3], pd[1:3]
            init = consts.get(operands[1], 0.0) if len(operands) > 1 else 0.0
            ap = attrs.get("to_apply", "").lstrip("%")
            a["kind"] = "max" if (ap.startswith("max") or (np.isinf(init) and init < 0)
                                  or reducer_kind(ap) == "maximum") else "sum"
        ops.append(HloOp(res, opcode, operands, shape, a))
        if is_root:
            root = res
    # Dependency order (stable): an op after all of its operands.
    by_name = {o.name: o for o in ops}
    placed: set[str] = set()
    ordered: list[HloOp] = []

    def place(o: HloOp, depth=0):
        if o.name in placed:
            return
        for d in o.operands:
            if d in by_name and d not in placed:
                place(by_name[d], depth + 1)
        placed.add(o.name)
        ordered.append(o)

    import sys
    limit = sys.getrecursionlimit()
    sys.setrecursionlimit(max(limit, 4 * len(ops) + 100))
    try:
        for o in ops:
            place(o)
    finally:
        sys.setrecursionlimit(limit)
    inputs = [params[i] for i in sorted(params)]
    return HloGraph(name or entry, ordered, {}, inputs, root or ordered[-1].name)
