"""Device executor for HLO-style graphs (the xla_hlo path), B200-resident.

The reference executor (source/xla_hlo/src/compiler.rs:267-668) runs
broadcast, transpose and the pre-dispatch operand broadcasts on the host and
round-trips every op through host memory.  Here every op stays on the GPU:

* broadcast / reshape / transpose become *views* (shape + element strides over
  an existing buffer) and are folded into the strided operands of the
  consuming kernel (binary ops take rank-4 strides, dots take batch / row / k
  strides); a view is only materialised (device transpose kernel) when a
  consumer needs a contiguous input;
* common producer -> consumer chains are fused into single kernels:
  `convolution -> add(bias) [-> add(residual)] [-> maximum(0)]`,
  `dot -> add(bias) [-> tanh-GELU chain] [-> add(residual)]`,
  `[multiply(scale) ->] reduce-max -> subtract -> exp -> reduce-sum -> divide`
  (softmax), the reduce-mean / rsqrt LayerNorm chain, and
  `reduce-sum(1,2) -> divide` (global average pool);
* 1x1 stride-1 convolutions and linear layers run on the tcgen05 tensor-core
  GEMM with weights pre-split once at load (OHWI copies of HWIO weights are
  made on the host at load, not per call as the reference repacks).

Fusions change only rounding (fp32 throughout), never the math.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _lib
from .graph import DeviceTensor, Graph
from .hlo import HloGraph, HloOp


@dataclass
class View:
    """A (possibly broadcast / transposed) view of a device buffer, or a scalar."""
    shape: tuple
    strides: tuple | None = None      # element strides; None for scalars
    t: DeviceTensor | None = None
    scalar: float | None = None

    @property
    def contiguous(self) -> bool:
        if self.t is None:
            return False
        exp, acc = [], 1
        for d in reversed(self.shape):
            exp.append(acc)
            acc *= d
        exp = tuple(reversed(exp))
        return all(s == e or d == 1 for s, e, d in zip(self.strides, exp, self.shape))


def _row_major(shape):
    st, acc = [], 1
    for d in reversed(shape):
        st.append(acc)
        acc *= d
    return tuple(reversed(st))


class HloExecutor:
    def __init__(self, g: HloGraph, device: int = 0, graph: Graph | None = None,
                 fuse: bool = True, presplit: bool = True):
        self.hg = g
        self.g = graph or Graph(device)
        self.fuse = fuse
        self.presplit = presplit
        self.v: dict[str, View] = {}
        self.plan: list = []
        self.scalars: dict[float, DeviceTensor] = {}
        self.uses: dict[str, int] = {}
        self.consumers: dict[str, list[HloOp]] = {}
        for op in g.ops:
            for o in op.operands:
                self.uses[o] = self.uses.get(o, 0) + 1
            for o in dict.fromkeys(op.operands):  # each consuming op once
                self.consumers.setdefault(o, []).append(op)
        self.byname = {op.name: op for op in g.ops}
        self.done: set[str] = set()
        self.folded_pad: dict[str, tuple] = {}  # pad op -> (source, top, left) folded into consumers
        self.nonneg: set[str] = set()            # tensors known to be >= 0 (ReLU outputs)
        self.deferred_scale: dict[str, float] = {}
        self.weights_np = g.params
        self._build()

    # -- helpers ----------------------------------------------------------------
    def _scalar_buf(self, value: float) -> DeviceTensor:
        if value not in self.scalars:
            self.scalars[value] = self.g.tensor(np.array([value], np.float32))
        return self.scalars[value]

    def _new(self, shape) -> View:
        t = self.g.alloc(shape)
        return View(tuple(shape), _row_major(shape), t)

    def _contig(self, v: View) -> View:
        """Materialises a view into a contiguous buffer (device transpose)."""
        if v.t is not None and v.contiguous:
            return v
        out = self._new(v.shape)
        if v.t is None:  # broadcast scalar
            self._binary("add", View(v.shape, None, None, v.scalar),
                         View(v.shape, None, None, 0.0), out)
            return out
        self._copy_strided(v, out)
        return out

    def _pad4(self, shape, *stride_lists):
        r = len(shape)
        if r > 4:
            raise NotImplementedError("rank > 4")
        d = [1] * (4 - r) + list(shape)
        sts = [[0] * (4 - r) + list(s) for s in stride_lists]
        return d, sts

    def _copy_strided(self, v: View, out: View):
        zero = self._scalar_buf(0.0)
        d, (sa,) = self._pad4(v.shape, v.strides)
        self.plan.append(("binary", "add", v.t, zero, out.t, d, sa, [0, 0, 0, 0]))

    def _operand(self, v: View):
        """(buffer, strides padded to the output rank) for a binary operand."""
        if v.t is None:
            return self._scalar_buf(v.scalar), None
        return v.t, v.strides

    def _binary(self, opn: str, a: View, b: View, out: View):
        ta, sa = self._operand(a)
        tb, sb = self._operand(b)
        r = len(out.shape)
        sa = [0] * r if sa is None else list(sa)
        sb = [0] * r if sb is None else list(sb)
        d, (sa4, sb4) = self._pad4(out.shape, sa, sb)
        self.plan.append(("binary", opn, ta, tb, out.t, d, sa4, sb4))

    def _is_const_bcast(self, name: str, value: float | None = None) -> bool:
        op = self.byname.get(name)
        if op is None or op.opcode != "broadcast":
            return False
        src = self.byname.get(op.operands[0])
        return src is not None and src.opcode == "constant" and (
            value is None or abs(src.attrs["value"] - value) < 1e-12)

    def _const_of(self, name: str) -> float:
        return self.byname[self.byname[name].operands[0]].attrs["value"]

    def _bias_param(self, name: str):
        """broadcast(parameter weight of rank 1 onto the last axis) -> weight name."""
        op = self.byname.get(name)
        if op is None or op.opcode != "broadcast":
            return None
        src = self.byname.get(op.operands[0])
        if src is None or src.opcode != "parameter" or src.name not in self.weights_np:
            return None
        if len(src.shape) != 1 or tuple(op.attrs["dimensions"]) != (len(op.shape) - 1,):
            return None
        return src.name

    def _single_consumer(self, name: str, opcode: str | None = None):
        cs = self.consumers.get(name, [])
        if len(cs) != 1 or self.uses.get(name, 0) != 1 or name == self.hg.output:
            return None
        if opcode and cs[0].opcode != opcode:
            return None
        return cs[0]

    def _other(self, op: HloOp, name: str) -> str:
        return op.operands[1] if op.operands[0] == name else op.operands[0]

    def _weight_buf(self, name: str, arr: np.ndarray | None = None, tag: str = "") -> DeviceTensor:
        """Device copy of a weight; `arr` + `tag` name a repacked variant."""
        key = (name, tag if arr is not None else "")
        if key not in self._wcache:
            self._wcache[key] = self.g.tensor(self.weights_np[name] if arr is None else arr)
        return self._wcache[key]

    # -- fusion matchers ----------------------------------------------------------
    def _match_bias_chain(self, root: str):
        """root -> add(bias) [-> add(residual)] [-> maximum(0)]: returns
        (last_name, bias_param, residual_name, relu, consumed)."""
        consumed = []
        c = self._single_consumer(root, "add")
        if c is None:
            return None
        bias = self._bias_param(self._other(c, root))
        if bias is None:
            return None
        consumed.append(c.name)
        last, res, relu = c.name, None, False
        c2 = self._single_consumer(last, "add")
        if c2 is not None and not self._is_const_bcast(self._other(c2, last)):
            other = self._other(c2, last)
            # only a residual that is already computed (program order) fuses
            if self.byname[other].shape == c2.shape and other in self.v:
                res = other
                consumed.append(c2.name)
                last = c2.name
        c3 = self._single_consumer(last, "maximum")
        if c3 is not None and self._is_const_bcast(self._other(c3, last), 0.0):
            relu = True
            consumed.append(c3.name)
            last = c3.name
        return last, bias, res, relu, consumed

    def _match_gelu(self, x: str):
        """tanh-GELU chain built by nets_hlo._gelu_tanh, rooted at x."""
        cs = [c for c in self.consumers.get(x, [])]
        # x feeds: mul(x,x), mul(.,x) [x3], add(x, ...) [inner], mul(x, add(t,1))
        if len(cs) != 4:
            return None
        try:
            m1 = next(c for c in cs if c.opcode == "multiply" and c.operands == [x, x])
            m2 = self._single_consumer(m1.name, "multiply")
            m3 = self._single_consumer(m2.name, "multiply")          # x3 * 0.044715
            inner = self._single_consumer(m3.name, "add")            # x + ...
            m4 = self._single_consumer(inner.name, "multiply")       # * c
            th = self._single_consumer(m4.name, "tanh")
            a1 = self._single_consumer(th.name, "add")               # t + 1
            m5 = self._single_consumer(a1.name, "multiply")          # x * (t + 1)
            m6 = self._single_consumer(m5.name, "multiply")          # * 0.5
        except (StopIteration, AttributeError):
            return None
        if None in (m2, m3, inner, m4, th, a1, m5, m6):
            return None
        if not (self._is_const_bcast(self._other(m3, m2.name), 0.044715)
                and self._is_const_bcast(self._other(a1, th.name), 1.0)
                and self._is_const_bcast(self._other(m6, m5.name), 0.5)
                and abs(self._const_of(self._other(m4, inner.name)) - 0.7978845608028654) < 1e-9):
            return None
        return m6.name, [m1.name, m2.name, m3.name, inner.name, m4.name, th.name, a1.name,
                         m5.name, m6.name]

    def _match_softmax(self, rmax: HloOp):
        """[x] reduce-max(last) -> subtract -> exp -> reduce-sum -> divide."""
        x = rmax.operands[0]
        last_axis = len(self.byname[x].shape) - 1
        if rmax.attrs.get("kind") != "max" or tuple(rmax.attrs["dimensions"]) != (last_axis,):
            return None
        bm = self._single_consumer(rmax.name, "broadcast")
        sub = bm and self._single_consumer(bm.name, "subtract")
        ex = sub and self._single_consumer(sub.name, "exponential")
        if not ex or sub.operands[0] != x:
            return None
        cs = self.consumers.get(ex.name, [])
        if len(cs) != 2:
            return None
        rs = next((c for c in cs if c.opcode == "reduce"), None)
        dv = next((c for c in cs if c.opcode == "divide"), None)
        if rs is None or dv is None or dv.operands[0] != ex.name:
            return None
        bs = self._single_consumer(rs.name, "broadcast")
        if bs is None or dv.operands[1] != bs.name:
            return None
        return dv.name, [rmax.name, bm.name, sub.name, ex.name, rs.name, bs.name, dv.name]

    def _match_layernorm(self, rsum: HloOp):
        x = rsum.operands[0]
        xs = self.byname[x].shape
        if rsum.attrs.get("kind") != "sum" or tuple(rsum.attrs["dimensions"]) != (len(xs) - 1,):
            return None
        try:
            dv = self._single_consumer(rsum.name, "divide")
            bmean = self._single_consumer(dv.name, "broadcast")
            xc = self._single_consumer(bmean.name, "subtract")
            xcs = [c for c in self.consumers[xc.name]]
            sq = next(c for c in xcs if c.opcode == "multiply" and c.operands == [xc.name, xc.name])
            norm = next(c for c in xcs if c.opcode == "multiply" and c is not sq)
            r2 = self._single_consumer(sq.name, "reduce")
            dv2 = self._single_consumer(r2.name, "divide")
            ad = self._single_consumer(dv2.name, "add")
            rs = self._single_consumer(ad.name, "rsqrt")
            br = self._single_consumer(rs.name, "broadcast")
            mg = self._single_consumer(norm.name, "multiply")
            ab = self._single_consumer(mg.name, "add")
        except (StopIteration, AttributeError, KeyError):
            return None
        if None in (dv, bmean, xc, r2, dv2, ad, rs, br, mg, ab) or len(xcs) != 2:
            return None
        if norm.operands != [xc.name, br.name]:
            return None
        gamma = self._bias_param(self._other(mg, norm.name))
        beta = self._bias_param(self._other(ab, mg.name))
        if gamma is None or beta is None or not self._is_const_bcast(self._other(ad, dv2.name)):
            return None
        eps = self._const_of(self._other(ad, dv2.name))
        names = [rsum.name, dv.name, bmean.name, xc.name, sq.name, norm.name, r2.name, dv2.name,
                 ad.name, rs.name, br.name, mg.name, ab.name]
        return ab.name, gamma, beta, eps, names

    # -- build --------------------------------------------------------------------
    def _build(self):
        self._wcache = {}
        self.inputs: dict[str, View] = {}
        for op in self.hg.ops:
            if op.name in self.done:
                continue
            fn = getattr(self, "_op_" + op.opcode.replace("-", "_"), None)
            if fn is None:
                raise NotImplementedError(f"HLO op {op.opcode} has no device lowering")
            fn(op)
        self.output_view = self._contig(self.v[self.hg.output])
        self.output = self.output_view.t

    def _set(self, name: str, view: View):
        self.v[name] = view

    def _op_parameter(self, op):
        if op.name in self.hg.params:
            t = self._weight_buf(op.name)
            self._set(op.name, View(op.shape, _row_major(op.shape), t))
        else:
            v = self._new(op.shape)
            self.inputs[op.name] = v
            self._set(op.name, v)

    def _op_constant(self, op):
        self._set(op.name, View((), None, None, float(op.attrs["value"])))

    def _op_broadcast(self, op):
        src = self.v[op.operands[0]]
        if src.t is None:
            self._set(op.name, View(op.shape, None, None, src.scalar))
            return
        st = [0] * len(op.shape)
        for sa, oa in enumerate(op.attrs["dimensions"]):
            st[oa] = 0 if src.shape[sa] == 1 else src.strides[sa]
        self._set(op.name, View(op.shape, tuple(st), src.t))

    def _op_reshape(self, op):
        src = self._contig(self.v[op.operands[0]])
        self._set(op.name, View(op.shape, _row_major(op.shape), src.t))

    _op_convert = _op_reshape

    def _op_transpose(self, op):
        src = self.v[op.operands[0]]
        perm = op.attrs["dimensions"]
        if src.t is None:
            self._set(op.name, src)
            return
        self._set(op.name, View(op.shape, tuple(src.strides[p] for p in perm), src.t))

    def _foldable_pad(self, op) -> bool:
        """A spatial pad of an NHWC tensor whose every consumer can take it as
        its own low-side padding: a convolution (zero pad), or a max
        reduce-window whose padded taps cannot win (pad value -inf, or 0 over
        a tensor known to be >= 0, e.g. a fused conv + ReLU output)."""
        if not self.fuse or len(op.shape) != 4:
            return False
        padding = op.attrs["padding"]
        if padding[0] != (0, 0) or padding[3] != (0, 0) or any(lo < 0 or hi < 0
                                                               for lo, hi in padding):
            return False
        pv = self.v[op.operands[1]].scalar
        cs = self.consumers.get(op.name, [])
        if not cs:
            return False
        for c in cs:
            if c.operands[0] != op.name:
                return False
            if c.opcode == "convolution" and pv == 0.0:
                continue
            if (c.opcode == "reduce-window" and c.attrs["kind"] == "max"
                    and (pv == -np.inf or (pv == 0.0 and op.operands[0] in self.nonneg))):
                continue
            return False
        return True

    def _op_pad(self, op):
        if self._foldable_pad(op):
            # No kernel: the consumer reads the unpadded tensor with its low-side
            # padding grown by this pad (out-of-map taps are zero / ignored).
            self.folded_pad[op.name] = (op.operands[0], op.attrs["padding"][1][0],
                                        op.attrs["padding"][2][0])
            return
        src = self._contig(self.v[op.operands[0]])
        pv = self.v[op.operands[1]].scalar
        r = len(op.shape)
        od = [1] * (4 - r) + list(op.shape)
        idd = [1] * (4 - r) + list(src.shape)
        pl = [0] * (4 - r) + [p[0] for p in op.attrs["padding"]]
        out = self._new(op.shape)
        total = int(np.prod(op.shape))
        self.plan.append(("pad4", src.t, out.t, float(pv), od + idd + pl + [total]))
        self._set(op.name, out)

    def _unfold(self, name: str):
        """(source view, extra top pad, extra left pad) of an operand."""
        if name in self.folded_pad:
            src, pt, pl = self.folded_pad[name]
            return self._contig(self.v[src]), pt, pl
        return self._contig(self.v[name]), 0, 0

    def _op_convolution(self, op):
        x, ept, epl = self._unfold(op.operands[0])
        wname = op.operands[1]
        w = self.weights_np[wname]
        kh, kw, ic, oc = w.shape
        st, pd = op.attrs["stride"], op.attrs["pad"]
        pd = ((pd[0][0] + ept, pd[0][1]), (pd[1][0] + epl, pd[1][1]))
        fused = self._match_bias_chain(op.name) if self.fuse else None
        bias = res = None
        relu = False
        last = op.name
        if fused:
            last, bname, rname, relu, consumed = fused
            bias = self._weight_buf(bname)
            res = self._contig(self.v[rname]).t if rname else None
            self.done.update(consumed)
        out = self._new(op.shape)
        pointwise = kh == 1 and kw == 1 and tuple(st) == (1, 1)
        # A 3x3 / 7x7 stride-2 stem over 3 channels (ResNet-50's first conv):
        # the tensor-core stem, im2col on chip, weights padded and split once.
        if (self.presplit and ic == 3 and kh == kw and kh in (3, 7) and tuple(st) == (2, 2)
                and res is None and pd[0][0] < kh and pd[1][0] < kw
                and self.g.stem_supported(x.t, out.t, pad=(pd[0][0], pd[1][0]), kernel=kh)):
            wt = self._weight_buf(wname)
            split = self.g.stem_weights(np.ascontiguousarray(w.transpose(3, 0, 1, 2)))
            self.plan.append(("conv", dict(x=x.t, w=wt, bias=bias, y=out.t, stride=tuple(st),
                                           pad=(pd[0][0], pd[1][0]), weight_layout=_lib.WEIGHT_HWIO,
                                           activation=_lib.ACT_RELU if relu else _lib.ACT_NONE,
                                           residual=None, w_split=split, stem=kh)))
            self._set(last, out)
            if relu:
                self.nonneg.add(last)
            if last != op.name:
                self._set(op.name, out)
            return
        # Tensor-core convs (pointwise GEMM, or the implicit GEMM of KxK /
        # strided convs over 32-channel blocks) take an OHWI copy, pre-split once.
        if pointwise or w.shape[2] % 32 == 0:
            wt = self._weight_buf(wname, np.ascontiguousarray(w.transpose(3, 0, 1, 2)), "ohwi")
            split = self.g.weights_split(wt) if self.presplit else None
            layout = _lib.WEIGHT_OHWI
        else:
            wt, split, layout = self._weight_buf(wname), None, _lib.WEIGHT_HWIO
        self.plan.append(("conv", dict(x=x.t, w=wt, bias=bias, y=out.t, stride=tuple(st),
                                       pad=(pd[0][0], pd[1][0]), weight_layout=layout,
                                       activation=_lib.ACT_RELU if relu else _lib.ACT_NONE,
                                       residual=res, w_split=split)))
        self._set(last, out)
        if relu:
            self.nonneg.add(last)
        if last != op.name:
            self._set(op.name, out)

    def _op_reduce_window(self, op):
        x, ept, epl = self._unfold(op.operands[0])
        sz, st, pd = op.attrs["size"], op.attrs["stride"], op.attrs["pad"]
        pd = ((pd[0][0] + ept, pd[0][1]), (pd[1][0] + epl, pd[1][1]))
        out = self._new(op.shape)
        kind = _lib.POOL_MAX if op.attrs["kind"] == "max" else _lib.POOL_SUM
        self.plan.append(("pool", x.t, out.t, tuple(sz), tuple(st), (pd[0][0], pd[1][0]), kind))
        self._set(op.name, out)

    def _op_reduce(self, op):
        x = self.v[op.operands[0]]
        dims = tuple(op.attrs["dimensions"])
        if self.fuse and op.attrs["kind"] == "max":
            m = self._match_softmax(op)
            if m is not None:
                last, names = m
                scale = self.deferred_scale.pop(op.operands[0], 1.0)
                xc = self._contig(x)
                cols = xc.shape[-1]
                rows = int(np.prod(xc.shape)) // cols
                out = self._new(self.byname[last].shape)
                self.plan.append(("softmax", xc.t, out.t, rows, cols, scale))
                self.done.update(names)
                self._set(last, out)
                return
        if self.fuse and op.attrs["kind"] == "sum":
            ln = self._match_layernorm(op)
            if ln is not None:
                last, gamma, beta, eps, names = ln
                res = None  # a residual add before LayerNorm is fused into the producing GEMM
                xc = self._contig(x)
                cols = xc.shape[-1]
                rows = int(np.prod(xc.shape)) // cols
                out = self._new(self.byname[last].shape)
                self.plan.append(("layernorm", xc.t, res, self._weight_buf(gamma),
                                  self._weight_buf(beta), out.t, rows, cols, float(eps)))
                self.done.update(names)
                self._set(last, out)
                return
            # global average pool: reduce-sum over H, W of NHWC -> divide by H*W
            xs = self.byname[op.operands[0]].shape
            dv = self._single_consumer(op.name, "divide")
            if (self.fuse and len(xs) == 4 and dims == (1, 2) and dv is not None
                    and self._is_const_bcast(dv.operands[1], float(xs[1] * xs[2]))):
                xc = self._contig(x)
                out = self._new(dv.shape)
                self.plan.append(("gap", xc.t, out.t))
                self.done.add(dv.name)
                self._set(dv.name, out)
                return
        xc = self._contig(x)
        s = xc.shape
        if len(s) > 4:
            raise NotImplementedError("reduce of rank > 4")
        d = list(s) + [1] * (4 - len(s))
        flags = [1 if i in dims else 0 for i in range(4)]
        od = [1] * 4
        cur = 0
        for a in range(len(s)):
            if not flags[a]:
                od[a] = op.shape[cur]
                cur += 1
        total = max(int(np.prod(op.shape)), 1)
        out = self._new(op.shape)
        self.plan.append(("reduce", xc.t, out.t,
                          [len(s)] + d + od + flags + [1 if op.attrs["kind"] == "max" else 0, total]))
        self._set(op.name, out)

    def _op_dot(self, op):
        a, b = self.v[op.operands[0]], self.v[op.operands[1]]
        lc, rc = list(op.attrs["lhs_contracting_dims"]), list(op.attrs["rhs_contracting_dims"])
        lb, rb = list(op.attrs["lhs_batch_dims"]), list(op.attrs["rhs_batch_dims"])
        lf = [d for d in range(len(a.shape)) if d not in lb + lc]
        rf = [d for d in range(len(b.shape)) if d not in rb + rc]
        if len(lc) != 1 or len(lb) > 2 or len(rf) != 1:
            raise NotImplementedError("dot form")

        def collapse(view, dims):
            """Strides of `dims` collapsed into one row index, or None."""
            if not dims:
                return 1, 0
            size, st = view.shape[dims[-1]], view.strides[dims[-1]]
            for d in reversed(dims[:-1]):
                if view.strides[d] != st * size:
                    return None
                size *= view.shape[d]
            return size, st

        if a.t is None or b.t is None:
            a, b = self._contig(a), self._contig(b)
        ca = collapse(a, lf)
        if ca is None:
            a = self._contig(a)
            ca = collapse(a, lf)
        M, a_ms = ca
        K = a.shape[lc[0]]
        a_ks = a.strides[lc[0]]
        N = b.shape[rf[0]]
        b_ns, b_ks = b.strides[rf[0]], b.strides[rc[0]]
        batch, inner = 1, 1
        a_bs = b_bs = c_bs = a_bis = b_bis = c_bis = 0
        if len(lb) >= 1:
            batch = a.shape[lb[0]]
            a_bs, b_bs = a.strides[lb[0]], b.strides[rb[0]]
        if len(lb) == 2:
            inner = a.shape[lb[1]]
            a_bis, b_bis = a.strides[lb[1]], b.strides[rb[1]]
        c_ms = N
        c_bis = M * N
        c_bs = inner * M * N
        out = self._new(op.shape)
        # Fused linear epilogue: add(bias) [-> GELU] [-> add(residual)].
        bias = res = None
        act = _lib.ACT_NONE
        last = op.name
        is_linear = not lb and self.fuse and b.t is not None and op.operands[1] in self.hg.params
        if is_linear:
            c = self._single_consumer(op.name, "add")
            bname = c and self._bias_param(self._other(c, op.name))
            if bname:
                bias = self._weight_buf(bname)
                self.done.add(c.name)
                last = c.name
                gl = self._match_gelu(last)
                if gl is not None:
                    last, names = gl
                    self.done.update(names)
                    act = _lib.ACT_GELU_TANH
                c2 = self._single_consumer(last, "add")
                if c2 is not None and act == _lib.ACT_NONE:
                    other = self._other(c2, last)
                    if self.byname[other].shape == c2.shape and other in self.v:
                        res = self._contig(self.v[other]).t
                        self.done.add(c2.name)
                        last = c2.name
        split = None
        if is_linear and b_ks == 1 and self.presplit:
            split = self.g.weights_split(b.t)
        elif is_linear and b_ns == 1 and b_ks == N:
            # [K][N] weights: a transposed [N][K] copy makes the B operand
            # K-contiguous, the tensor-core GEMM's layout.
            wt = self._weight_buf(op.operands[1], np.ascontiguousarray(self.weights_np[op.operands[1]].T),
                                   "nk")
            b = View((N, K), (K, 1), wt)
            b_ns, b_ks = K, 1
            split = self.g.weights_split(wt) if self.presplit else None
        self.plan.append(("gemm", dict(a=a.t, b=b.t, c=out.t, m=M, n=N, k=K, batch=batch,
                                       a_strides=(a_bs, a_ms, a_ks), b_strides=(b_bs, b_ks, b_ns),
                                       c_strides=(c_bs, c_ms), bias=bias, residual=res,
                                       activation=act, batch_inner=inner,
                                       inner_strides=(a_bis, b_bis, c_bis), b_split=split)))
        self._set(last, out)
        if last != op.name:
            self._set(op.name, out)

    def _elementwise(self, op, opn: str):
        a = self.v[op.operands[0]]
        b = self.v[op.operands[1]]
        out = self._new(op.shape)
        self._binary(opn, a, b, out)
        self._set(op.name, out)

    def _op_add(self, op): self._elementwise(op, "add")
    def _op_subtract(self, op): self._elementwise(op, "sub")
    def _op_multiply(self, op):
        # multiply(scores, constant) feeding only a softmax: the scale moves
        # into the fused softmax kernel instead of a separate pass.
        if self.fuse and self._is_const_bcast(op.operands[1]):
            cs = self.consumers.get(op.name, [])
            rmax = next((c for c in cs if c.opcode == "reduce" and c.attrs.get("kind") == "max"), None)
            if rmax is not None and len(cs) == 2 and self._match_softmax(rmax) is not None:
                self.deferred_scale[op.name] = self._const_of(op.operands[1])
                self._set(op.name, self.v[op.operands[0]])
                return
        self._elementwise(op, "mul")
    def _op_divide(self, op): self._elementwise(op, "div")

    _CMP = {"GT": "gt", "GE": "ge", "LT": "lt", "LE": "le", "EQ": "eq", "NE": "ne"}

    def _op_compare(self, op):
        # a 0 / 1 float mask; the reference evaluates compare on the host
        self._elementwise(op, self._CMP[op.attrs.get("direction", "GT")])

    def _op_select(self, op):
        views = [self.v[o] for o in op.operands]
        out = self._new(op.shape)
        r = len(op.shape)
        ops_ = []
        for v in views:
            t, st = self._operand(v)
            ops_.append((t, [0] * r if st is None else list(st)))
        d, strides = self._pad4(op.shape, *(st for _, st in ops_))
        self.plan.append(("select", ops_[0][0], ops_[1][0], ops_[2][0], out.t, d, *strides))
        self._set(op.name, out)

    def _op_tuple(self, op):
        self._set(op.name, self.v[op.operands[0]])

    def _op_get_tuple_element(self, op):
        if op.attrs.get("index", 0) != 0:
            raise NotImplementedError("get-tuple-element of a tuple element other than 0")
        self._set(op.name, self.v[op.operands[0]])
    def _op_maximum(self, op): self._elementwise(op, "max")
    def _op_minimum(self, op): self._elementwise(op, "min")
    def _op_power(self, op): self._elementwise(op, "pow")

    def _unary(self, op, name: str):
        x = self._contig(self.v[op.operands[0]])
        out = self._new(op.shape)
        self.plan.append(("unary", name, x.t, out.t))
        self._set(op.name, out)

    def _op_exponential(self, op): self._unary(op, "exp")
    def _op_log(self, op): self._unary(op, "log")
    def _op_sqrt(self, op): self._unary(op, "sqrt")
    def _op_rsqrt(self, op): self._unary(op, "rsqrt")
    def _op_negate(self, op): self._unary(op, "neg")
    def _op_abs(self, op): self._unary(op, "abs")
    def _op_tanh(self, op): self._unary(op, "tanh")
    def _op_logistic(self, op): self._unary(op, "sigmoid")

    # -- run ------------------------------------------------------------------------
    def record(self):
        g = self.g
        for step in self.plan:
            k = step[0]
            if k == "binary":
                _, opn, ta, tb, ty, d, sa, sb = step
                g.binary(opn, ta, tb, ty, d, sa, sb)
            elif k == "unary":
                g.unary(step[1], step[2], step[3])
            elif k == "select":
                _, tp, ta, tb, ty, d, sp, sa, sb = step
                g.select(tp, ta, tb, ty, d, sp, sa, sb)
            elif k == "conv" and step[1].get("stem"):
                p = step[1]
                g.stem_conv_nhwc(p["x"], p["w_split"], p["bias"], p["y"], stride=p["stride"],
                                 pad=p["pad"], activation=p["activation"], kernel=p["stem"])
            elif k == "conv":
                p = step[1]
                g.conv2d_nhwc(p["x"], p["w"], p["bias"], p["y"], stride=p["stride"], pad=p["pad"],
                              weight_layout=p["weight_layout"], activation=p["activation"],
                              residual=p["residual"], w_split=p["w_split"])
            elif k == "gemm":
                p = dict(step[1])
                a, b, c = p.pop("a"), p.pop("b"), p.pop("c")
                g.gemm(a, b, c, **p)
            elif k == "pool":
                _, x, y, sz, st, pd, kind = step
                g.pool2d_nhwc(x, y, kernel=sz, stride=st, pad=pd, kind=kind)
            elif k == "gap":
                g.global_avg_pool_nhwc(step[1], step[2])
            elif k == "softmax":
                _, x, y, rows, cols, scale = step
                g.attention_softmax(x, y, rows, cols, scale)
            elif k == "layernorm":
                _, x, res, gm, bt, y, rows, cols, eps = step
                g.layernorm(x, gm, bt, y, rows, cols, eps, residual=res)
            elif k == "reduce":
                g.reduce_rank4(step[1], step[2], step[3])
            elif k == "pad4":
                g.pad4(step[1], step[2], step[3], step[4])
            else:
                raise AssertionError(k)

    @property
    def kernels_per_run(self) -> int:
        return len(self.plan)

    def op_costs(self) -> list[dict]:
        """Algorithmic flops / HBM bytes per planned kernel (fp32; inputs,
        weights, bias, residual read once, output written once)."""
        out = []
        for st in self.plan:
            k = st[0]
            if k == "conv":
                p = st[1]
                x, w, y = p["x"], p["w"], p["y"]
                kk = int(np.prod(w.shape)) // y.shape[-1]
                f = 2 * y.size * kk
                b = x.size + w.size + y.size + (y.size if p["residual"] is not None else 0)
                label = f"conv{'1x1' if kk == x.shape[-1] else 'kxk'}"
            elif k == "gemm":
                p = st[1]
                bt = p["batch"] * p["batch_inner"]
                f = 2 * bt * p["m"] * p["n"] * p["k"]
                b = bt * (p["m"] * p["k"] + p["m"] * p["n"]) + p["b"].size + \
                    (p["c"].size if p["residual"] is not None else 0)
                label = "gemm" if p["bias"] is not None else "attn_gemm"
            elif k in ("softmax", "layernorm"):
                n = st[1].size
                f, b, label = 5 * n, 2 * n, k
            elif k == "binary":
                n = st[4].size
                f, b, label = n, 3 * n, "elementwise"
            elif k in ("pool", "gap", "reduce", "pad4", "unary"):
                src = st[1] if k != "unary" else st[2]
                dst = st[2] if k != "unary" else st[3]
                f, b, label = src.size, src.size + dst.size, k
            else:
                f, b, label = 0, 0, k
            out.append({"kind": k, "label": label, "flops": int(f), "bytes": int(4 * b)})
        return out

    def record_op(self, i: int) -> None:
        plan, self.plan = self.plan, [self.plan[i]]
        try:
            self.record()
        finally:
            self.plan = plan

    @property
    def input(self):
        return next(iter(self.inputs.values())).t

    def capture(self):
        self.g.sync()
        self.g.capture_begin()
        self.record()
        self.g.capture_end()
        self._captured = True

    def run(self):
        if getattr(self, "_captured", False):
            self.g.replay()
        else:
            self.record()

    def forward(self, feeds: dict[str, np.ndarray]) -> np.ndarray:
        for name, v in self.inputs.items():
            self.g.upload(v.t, np.asarray(feeds[name], np.float32).reshape(v.shape))
        self.run()
        return self.g.download(self.output).reshape(self.hg.op(self.hg.output).shape)

    def close(self):
        self.g.close()
