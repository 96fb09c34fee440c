"""HLO-style graphs and their per-op lowering with the reference executor's
semantics (source/xla_hlo/src/compiler.rs:267-668).

A graph is a list of `HloOp`s in program order (the reference walks the op
list in textual order, compiler.rs:284, no topological sort).  Shapes are
row-major; activations NHWC, convolution weights HWIO
(`dim_labels=b01f_01io->b01f`, compiler.rs:785-790).

`run_hlo(graph, feeds, rk)` executes it the way compiler.rs does:
convolution, reduce-window, reduce (rank <= 4), dot / dot_general, pad and
the elementwise ops are dispatched through `rk` (the drop-in boundary, same
kernel names and push constants as compiler.rs:694-1135); broadcast,
transpose, compare, select, slice and concatenate run on the host, and an
elementwise operand whose size differs from the output is broadcast on the
host first (compiler.rs:705-729).  Dot operands are transposed on the host to
[batch, M, K] and [batch, K, N] (transpose_flat, compiler.rs:1043-1058).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable

import numpy as np

RunKernel = Callable[[str, np.ndarray, np.ndarray, int, list], np.ndarray]

# compiler.rs:1155-1228 kernel_mapping: opcode -> (kernel, arity)
ELEMENTWISE = {
    "add": ("add", 2), "subtract": ("sub", 2), "multiply": ("mul", 2), "divide": ("div", 2),
    "maximum": ("max", 2), "minimum": ("min", 2), "power": ("pow", 2), "abs": ("abs", 1),
    "exponential": ("exp", 1), "log": ("log", 1), "sqrt": ("sqrt", 1), "rsqrt": ("rsqrt", 1),
    "negate": ("neg", 1), "tanh": ("tanh", 1), "logistic": ("sigmoid", 1), "sine": ("sine", 1),
    "convert": ("reshape", 1),
}


@dataclass
class HloOp:
    name: str
    opcode: str
    operands: list[str]
    shape: tuple[int, ...]
    attrs: dict = field(default_factory=dict)


@dataclass
class HloGraph:
    name: str
    ops: list[HloOp]
    params: dict[str, np.ndarray]      # weights / constants bound to parameter ops
    inputs: list[str]                  # parameter names fed per run
    output: str

    def op(self, name: str) -> HloOp:
        for o in self.ops:
            if o.name == name:
                return o
        raise KeyError(name)

    def histogram(self) -> dict[str, int]:
        h: dict[str, int] = {}
        for o in self.ops:
            h[o.opcode] = h.get(o.opcode, 0) + 1
        return h


class Builder:
    """Helper that appends ops and tracks shapes."""

    def __init__(self, name: str):
        self.name = name
        self.ops: list[HloOp] = []
        self.params: dict[str, np.ndarray] = {}
        self.inputs: list[str] = []
        self.shapes: dict[str, tuple[int, ...]] = {}
        self.n = 0

    def _new(self, opcode, operands, shape, **attrs) -> str:
        self.n += 1
        name = f"{opcode.replace('-', '_')}.{self.n}"
        self.ops.append(HloOp(name, opcode, list(operands), tuple(int(s) for s in shape), attrs))
        self.shapes[name] = tuple(int(s) for s in shape)
        return name

    def input(self, shape) -> str:
        name = self._new("parameter", [], shape, index=len(self.inputs))
        self.inputs.append(name)
        return name

    def weight(self, value: np.ndarray) -> str:
        name = self._new("parameter", [], value.shape, index=-1)
        self.params[name] = np.ascontiguousarray(value, dtype=np.float32)
        return name

    def constant(self, v: float) -> str:
        return self._new("constant", [], (), value=float(v))

    def broadcast(self, x: str, shape, dims) -> str:
        return self._new("broadcast", [x], shape, dimensions=tuple(dims))

    def binary(self, opcode: str, a: str, b: str) -> str:
        return self._new(opcode, [a, b], self.shapes[a])

    def unary(self, opcode: str, a: str) -> str:
        return self._new(opcode, [a], self.shapes[a])

    def reshape(self, x: str, shape) -> str:
        return self._new("reshape", [x], shape)

    def transpose(self, x: str, perm) -> str:
        s = self.shapes[x]
        return self._new("transpose", [x], tuple(s[p] for p in perm), dimensions=tuple(perm))

    def pad(self, x: str, low, high, value: float = 0.0) -> str:
        s = self.shapes[x]
        out = tuple(d + lo + hi for d, lo, hi in zip(s, low, high))
        c = self.constant(value)
        return self._new("pad", [x, c], out, padding=tuple(zip(low, high)))

    def conv(self, x: str, w: str, stride=(1, 1), pad=((0, 0), (0, 0))) -> str:
        n, ih, iw, _ = self.shapes[x]
        kh, kw, _, oc = self.shapes[w]
        oh = (ih + pad[0][0] + pad[0][1] - kh) // stride[0] + 1
        ow = (iw + pad[1][0] + pad[1][1] - kw) // stride[1] + 1
        return self._new("convolution", [x, w], (n, oh, ow, oc), stride=tuple(stride),
                         pad=tuple(tuple(p) for p in pad), dim_labels="b01f_01io->b01f")

    def reduce_window(self, x: str, size, stride, pad, kind: str) -> str:
        n, ih, iw, c = self.shapes[x]
        oh = (ih + pad[0][0] + pad[0][1] - size[0]) // stride[0] + 1
        ow = (iw + pad[1][0] + pad[1][1] - size[1]) // stride[1] + 1
        init = self.constant(-np.inf if kind == "max" else 0.0)
        return self._new("reduce-window", [x, init], (n, oh, ow, c), size=tuple(size),
                         stride=tuple(stride), pad=tuple(tuple(p) for p in pad), kind=kind)

    def reduce(self, x: str, dims, kind: str) -> str:
        s = self.shapes[x]
        out = tuple(d for i, d in enumerate(s) if i not in dims)
        init = self.constant(-np.inf if kind == "max" else 0.0)
        return self._new("reduce", [x, init], out, dimensions=tuple(dims), kind=kind)

    def dot(self, a: str, b: str, lhs_contract, rhs_contract, lhs_batch=(), rhs_batch=()) -> str:
        sa, sb = self.shapes[a], self.shapes[b]
        batch = [sa[d] for d in lhs_batch]
        lf = [sa[d] for d in range(len(sa)) if d not in lhs_batch and d not in lhs_contract]
        rf = [sb[d] for d in range(len(sb)) if d not in rhs_batch and d not in rhs_contract]
        return self._new("dot", [a, b], tuple(batch + lf + rf), lhs_contracting_dims=tuple(lhs_contract),
                         rhs_contracting_dims=tuple(rhs_contract), lhs_batch_dims=tuple(lhs_batch),
                         rhs_batch_dims=tuple(rhs_batch))

    def graph(self, out: str) -> HloGraph:
        return HloGraph(self.name, self.ops, self.params, self.inputs, out)


# ---- host-side helpers with compiler.rs semantics ---------------------------
def broadcast_host(src: np.ndarray, out_shape, dims) -> np.ndarray:
    """compiler.rs:1361-1393: output coordinate -> source coordinate through
    `dims`; size-1 source axes broadcast."""
    out_shape = tuple(out_shape)
    if src.size == int(np.prod(out_shape)) and src.shape == out_shape:
        return src.copy()
    if src.size == 1:
        return np.full(out_shape, src.reshape(-1)[0], np.float32)
    view_shape = [1] * len(out_shape)
    for sa, oa in enumerate(dims):
        view_shape[oa] = src.shape[sa]
    return np.ascontiguousarray(np.broadcast_to(src.reshape(view_shape), out_shape), np.float32)


def infer_broadcast_dims(src_shape, out_shape):
    """compiler.rs:1566-1572: trailing alignment."""
    off = len(out_shape) - len(src_shape)
    return [a + off for a in range(len(src_shape))]


def run_hlo(g: HloGraph, feeds: dict[str, np.ndarray], rk: RunKernel,
            keep: bool = False) -> tuple[np.ndarray, dict]:
    vals: dict[str, np.ndarray] = {}
    log: list[str] = []
    unused = np.zeros(1, np.float32)
    for op in g.ops:
        oc = op.opcode
        ins = [vals[o] for o in op.operands]
        if oc == "parameter":
            v = feeds[op.name] if op.name in feeds else g.params[op.name]
            vals[op.name] = np.asarray(v, np.float32).reshape(op.shape)
            continue
        if oc == "constant":
            vals[op.name] = np.array(op.attrs["value"], np.float32)
            continue
        if oc == "broadcast":
            vals[op.name] = broadcast_host(ins[0], op.shape, op.attrs["dimensions"])
        elif oc == "reshape":
            vals[op.name] = ins[0].reshape(op.shape)
        elif oc == "transpose":
            vals[op.name] = np.ascontiguousarray(np.transpose(ins[0], op.attrs["dimensions"]))
        elif oc == "pad":
            # compiler.rs:1086-1135: rank <= 4, dims right-aligned into 4 slots
            x = ins[0]
            r = x.ndim
            od, idd, pl = [1] * 4, [1] * 4, [0] * 4
            for i in range(r):
                idd[4 - r + i] = x.shape[i]
                od[4 - r + i] = op.shape[i]
                pl[4 - r + i] = op.attrs["padding"][i][0]
            total = int(np.prod(op.shape))
            out = rk("pad.spv", x, np.array([float(ins[1])], np.float32), total,
                     od + idd + pl + [total])
            vals[op.name] = out.reshape(op.shape)
            log.append("pad.spv")
        elif oc == "convolution":
            x, w = ins
            n, ih, iw, ic = x.shape
            kh, kw, _, ocn = w.shape
            _, oh, ow, _ = op.shape
            st, pd = op.attrs["stride"], op.attrs["pad"]
            total = int(np.prod(op.shape))
            out = rk("hlo_conv_nhwc_hwio.spv", x, w, total,
                     [n, ih, iw, ic, kh, kw, ocn, oh, ow, st[0], st[1], pd[0][0], pd[1][0], total])
            vals[op.name] = out.reshape(op.shape)
            log.append("hlo_conv_nhwc_hwio.spv")
        elif oc == "reduce-window":
            x = ins[0]
            n, ih, iw, c = x.shape
            _, oh, ow, _ = op.shape
            sz, st, pd = op.attrs["size"], op.attrs["stride"], op.attrs["pad"]
            total = int(np.prod(op.shape))
            kind = 1 if op.attrs["kind"] == "max" else 0
            out = rk("hlo_reduce_window_rank4.spv", x, unused, total,
                     [n, ih, iw, c, oh, ow, sz[0], sz[1], st[0], st[1], pd[0][0], pd[1][0], kind,
                      total])
            vals[op.name] = out.reshape(op.shape)
            log.append("hlo_reduce_window_rank4.spv")
        elif oc == "reduce":
            x = ins[0]
            dims = op.attrs["dimensions"]
            d = list(x.shape) + [1] * (4 - x.ndim)
            flags = [1 if i in dims else 0 for i in range(4)]
            od = [1] * 4
            cur = 0
            for a in range(x.ndim):
                if not flags[a]:
                    od[a] = op.shape[cur]
                    cur += 1
            total = max(int(np.prod(op.shape)), 1)
            kind = 1 if op.attrs["kind"] == "max" else 0
            out = rk("hlo_reduce_rank4.spv", x, unused, total,
                     [x.ndim] + d + od + flags + [kind, total])
            vals[op.name] = out.reshape(op.shape)
            log.append("hlo_reduce_rank4.spv")
        elif oc == "dot":
            a, b = ins
            lc, rc = list(op.attrs["lhs_contracting_dims"]), list(op.attrs["rhs_contracting_dims"])
            lb, rb = list(op.attrs["lhs_batch_dims"]), list(op.attrs["rhs_batch_dims"])
            lf = [d for d in range(a.ndim) if d not in lb and d not in lc]
            rf = [d for d in range(b.ndim) if d not in rb and d not in rc]
            B = int(np.prod([a.shape[d] for d in lb])) if lb else 1
            M = int(np.prod([a.shape[d] for d in lf])) if lf else 1
            K = a.shape[lc[0]]
            N = int(np.prod([b.shape[d] for d in rf])) if rf else 1
            at = np.ascontiguousarray(np.transpose(a, lb + lf + lc))   # transpose_flat
            bt = np.ascontiguousarray(np.transpose(b, rb + rc + rf))
            total = B * M * N
            out = rk("hlo_dot_batched.spv", at, bt, total, [B, M, K, N, total])
            vals[op.name] = out.reshape(op.shape)
            log.append("hlo_dot_batched.spv")
        elif oc == "slice":
            # host side, as compiler.rs does for slice / concatenate
            sl = tuple(slice(a, b, st) for a, b, st in op.attrs["slice"])
            vals[op.name] = np.ascontiguousarray(ins[0][sl])
        elif oc == "concatenate":
            vals[op.name] = np.concatenate(ins, axis=op.attrs["dimensions"][0])
        elif oc in ("tuple", "get-tuple-element"):
            # single-element tuples (the exported graphs' return wrappers)
            vals[op.name] = ins[op.attrs.get("index", 0)] if oc == "get-tuple-element" else ins[0]
        elif oc == "compare":
            a, b = ins
            b = broadcast_host(b, op.shape, infer_broadcast_dims(b.shape, op.shape))
            fn = {"LT": np.less, "LE": np.less_equal, "EQ": np.equal, "NE": np.not_equal,
                  "GE": np.greater_equal}.get(op.attrs.get("direction"), np.greater)
            vals[op.name] = fn(a, b).astype(np.float32)
        elif oc == "select":
            p, t, f = (broadcast_host(v, op.shape, infer_broadcast_dims(v.shape, op.shape))
                       for v in ins)
            vals[op.name] = np.where(p != 0, t, f).astype(np.float32)
        elif oc in ELEMENTWISE:
            kname, arity = ELEMENTWISE[oc]
            total = int(np.prod(op.shape))
            xs = []
            for v in ins[:arity]:
                if v.size != total:
                    v = broadcast_host(v, op.shape, infer_broadcast_dims(v.shape, op.shape))
                xs.append(np.ascontiguousarray(v, np.float32))
            rhs = xs[1] if arity == 2 else unused
            out = rk(kname + ".spv", xs[0], rhs, total, [total])
            vals[op.name] = out.reshape(op.shape)
            log.append(kname + ".spv")
        else:
            raise NotImplementedError(f"no lowering for HLO op {oc}")
    report = {"dispatches": log, "num_dispatches": len(log)}
    if keep:
        report["tensors"] = vals
    return vals[g.output], report
