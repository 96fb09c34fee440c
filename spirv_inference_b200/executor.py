"""Device-resident executor for TFLite-style CNN graphs (NHWC, fused).

Where the reference scheduler round-trips every op through the host and
issues activations and residual adds as extra dispatches
(source/tflite_loader/src/scheduler.rs:75-1039, 1146-1197), this executor:

* uploads weights once in their native TFLite layouts (Conv2D OHWI is the
  implicit-GEMM B operand as is; depthwise [1,kh,kw,c] is read as
  [kh][kw][c]; FullyConnected [out][in] is read transposed by strides),
* keeps every activation in HBM in NHWC,
* fuses bias + activation into every conv / depthwise / FC epilogue and the
  residual ADD of an inverted-residual block into the projecting 1x1 conv,
* by default (fuse_dw_project) runs a block's 3x3 depthwise conv, the 1x1
  projection after it and the residual add as one kernel
  (spx_op_dw_project_nhwc), the depthwise output staying on chip,
* optionally (fuse_expand_dw) runs a block's 1x1 expand conv and the 3x3
  depthwise after it as one kernel, the expanded tensor staying on chip;
  off by default: its CUDA-core expand (exact fp32, ~14 TFLOP/s) is slower
  than the tensor-core expand plus TMA depthwise it replaces on every
  MobileNetV2 block but one,
* treats RESHAPE as an alias, and
* records the whole graph on one stream, optionally captured once into a
  CUDA graph and replayed.
"""
from __future__ import annotations

import numpy as np

from . import _lib
from .graph import DeviceTensor, Graph
from .lowering import same_padding_offsets
from .nets import Model, Op


class _Shape:
    """Shape-only stand-in for a DeviceTensor (eligibility checks at planning)."""

    def __init__(self, shape):
        self.shape = tuple(shape)


class CnnExecutor:
    def __init__(self, model: Model, batch: int, device: int = 0, graph: Graph | None = None,
                 fuse_residual: bool = True, presplit: bool = True,
                 fuse_expand_dw: bool = False, fuse_dw_project: bool = True,
                 tc_stem: bool = True):
        self.model = model
        self.batch = batch
        self.g = graph or Graph(device)
        self.fuse_residual = fuse_residual
        self.fuse_expand_dw = fuse_expand_dw
        self.fuse_dw_project = fuse_dw_project and presplit
        self.tc_stem = tc_stem and presplit
        self.fused_away: set[str] = set()   # tensors that never reach HBM
        self.presplit = presplit
        self._splits: dict = {}
        self.w: dict[str, DeviceTensor] = {}
        for name, arr in model.weights.items():
            self.w[name] = self.g.tensor(arr)
        self.t: dict[str, DeviceTensor] = {}
        self._plan = []
        self._build()
        self._captured = False

    # -- planning ------------------------------------------------------------
    def _split(self, wname: str):
        """Tensor-core (3xTF32) hi / lo terms of a weight, made once at load."""
        if not self.presplit:
            return None
        if wname not in self._splits:
            self._splits[wname] = self.g.weights_split(self.w[wname])
        return self._splits[wname]

    def _buf(self, name: str) -> DeviceTensor:
        if name not in self.t:
            self.t[name] = self.g.alloc((self.batch,) + tuple(self.model.shapes[name]))
        return self.t[name]

    def _build(self) -> None:
        m = self.model
        uses: dict[str, int] = {}
        for op in m.ops:
            for i in op.inputs:
                uses[i] = uses.get(i, 0) + 1
        # Residual fusion: ADD(conv_out, skip) where conv_out feeds only the ADD
        # and the conv has no activation -> conv epilogue adds `skip`.
        fused_into: dict[str, tuple[str, str]] = {}  # conv output -> (add output, skip)
        if self.fuse_residual:
            producers = {op.output: op for op in m.ops}
            for op in m.ops:
                if op.type != "ADD" or op.attrs.get("activation", 0):
                    continue
                for ci, si in ((0, 1), (1, 0)):
                    p = producers.get(op.inputs[ci])
                    if (p is not None and p.type == "CONV_2D" and uses[p.output] == 1
                            and p.attrs.get("activation", 0) == 0):
                        fused_into[p.output] = (op.output, op.inputs[si])
                        break
        skip_adds = {v[0] for v in fused_into.values()}
        # Expand -> depthwise fusion: a 1x1 stride-1 conv with 16 / 24 / 32
        # input channels whose only consumer is a 3x3 depthwise (SAME, no
        # dilation, depth multiplier 1) with 4-aligned channels.
        expand_of: dict[str, Op] = {}  # depthwise output -> expand op
        expanded: set[str] = set()     # expand outputs that never materialise
        if self.fuse_expand_dw:
            producers = {op.output: op for op in m.ops}
            for op in m.ops:
                if op.type != "DEPTHWISE_CONV_2D":
                    continue
                a = op.attrs
                p = producers.get(op.inputs[0])
                wd = m.weights[op.inputs[1]]
                if (p is None or p.type != "CONV_2D" or uses[p.output] != 1
                        or p.output in fused_into):
                    continue
                we = m.weights[p.inputs[1]]
                if (we.shape[1:3] != (1, 1) or tuple(p.attrs["stride"]) != (1, 1)
                        or we.shape[3] not in (16, 24, 32) or wd.shape[1:3] != (3, 3)
                        or tuple(a.get("dilation", (1, 1))) != (1, 1)
                        or a.get("depth_multiplier", 1) != 1 or a.get("padding") != "SAME"
                        or a["stride"][0] != a["stride"][1] or a["stride"][0] not in (1, 2)
                        or wd.shape[3] % 4):
                    continue
                expand_of[op.output] = p
                expanded.add(p.output)
        # Depthwise -> projection fusion: a 3x3 depthwise (SAME, no dilation,
        # depth multiplier 1, equal strides 1 / 2) whose only consumer is a
        # 1x1 stride-1 conv; the conv's residual ADD (if fused) comes along.
        proj_of: dict[str, Op] = {}   # depthwise output -> projecting conv
        if self.fuse_dw_project:
            consumers: dict[str, list] = {}
            for op in m.ops:
                for i in op.inputs:
                    consumers.setdefault(i, []).append(op)
            for op in m.ops:
                if op.type != "DEPTHWISE_CONV_2D" or op.output in expand_of:
                    continue
                a = op.attrs
                wd = m.weights[op.inputs[1]]
                cs = consumers.get(op.output, [])
                if len(cs) != 1 or cs[0].type != "CONV_2D":
                    continue
                pc = cs[0]
                wp = m.weights[pc.inputs[1]]
                if (wp.shape[1:3] != (1, 1) or tuple(pc.attrs["stride"]) != (1, 1)
                        or pc.inputs[0] != op.output or wd.shape[1:3] != (3, 3)
                        or tuple(a.get("dilation", (1, 1))) != (1, 1)
                        or a.get("depth_multiplier", 1) != 1
                        or a["stride"][0] != a["stride"][1]):
                    continue
                h, w_, c = m.shapes[op.inputs[0]]
                oh, ow, cout = m.shapes[pc.output]
                pt, pl = same_padding_offsets(a["padding"], h, w_, oh, ow, 3, 3, *a["stride"])
                if not self.g.dw_project_supported(
                        _Shape((self.batch, h, w_, c)), _Shape((self.batch, oh, ow, cout)),
                        stride=a["stride"][0], pad=(pt, pl), act_dw=a.get("activation", 0),
                        act_proj=pc.attrs.get("activation", 0)):
                    continue
                proj_of[op.output] = pc
        proj_convs = {pc.output: d for d, pc in proj_of.items()}
        self._buf(m.input)
        for op in m.ops:
            a = op.attrs
            if op.type == "DEPTHWISE_CONV_2D" and op.output in proj_of:
                self.fused_away.add(op.output)
                continue  # runs inside the projection that consumes it
            if op.type == "CONV_2D" and op.output in proj_convs:
                dname = proj_convs[op.output]
                dop = next(o for o in m.ops if o.output == dname)
                da = dop.attrs
                x = self._buf(dop.inputs[0])
                res = None
                out_name = op.output
                if op.output in fused_into:
                    out_name, skip = fused_into[op.output]
                    res = self._buf(skip)
                y = self._buf(out_name)
                self.t[op.output] = y
                pt, pl = same_padding_offsets(da["padding"], x.shape[1], x.shape[2], y.shape[1],
                                              y.shape[2], 3, 3, *da["stride"])
                wd = self.w[dop.inputs[1]]
                self._plan.append(("dwproj", dict(
                    x=x, wd=wd.view((3, 3, wd.shape[3])), bd=self.w[dop.inputs[2]],
                    w=self.w[op.inputs[1]], w_split=self._split(op.inputs[1]),
                    bp=self.w[op.inputs[2]], y=y, residual=res, stride=da["stride"][0],
                    pad=(pt, pl), act_dw=da.get("activation", 0),
                    act_proj=a.get("activation", 0))))
                continue
            if op.type == "CONV_2D" and op.output in expanded:
                continue  # runs inside the depthwise that consumes it
            if op.type == "DEPTHWISE_CONV_2D" and op.output in expand_of:
                p = expand_of[op.output]
                x, y = self._buf(p.inputs[0]), self._buf(op.output)
                wd = self.w[op.inputs[1]]
                ce = wd.shape[3]
                s_ = a["stride"][0]
                ih = x.shape[1]
                pt, pl = same_padding_offsets("SAME", ih, x.shape[2], y.shape[1], y.shape[2],
                                              3, 3, s_, s_)
                self._plan.append(("expand_dw", dict(
                    x=x, we=self.w[p.inputs[1]], we_split=self._split(p.inputs[1]),
                    be=self.w[p.inputs[2]],
                    wd=wd.view((3, 3, ce)), bd=self.w[op.inputs[2]], y=y, stride=s_,
                    pad=(pt, pl), act_e=p.attrs.get("activation", 0),
                    act_d=a.get("activation", 0))))
                continue
            if op.type == "CONV_2D":
                x = self._buf(op.inputs[0])
                res = None
                out_name = op.output
                if op.output in fused_into:
                    out_name, skip = fused_into[op.output]
                    res = self._buf(skip)
                y = self._buf(out_name)
                self.t[op.output] = y
                w = self.w[op.inputs[1]]
                kh, kw = w.shape[1], w.shape[2]
                ih, iw = x.shape[1], x.shape[2]
                oh, ow = y.shape[1], y.shape[2]
                pt, pl = same_padding_offsets(a["padding"], ih, iw, oh, ow, kh, kw, *a["stride"])
                pointwise = (kh, kw) == (1, 1) and tuple(a["stride"]) == (1, 1)
                split = self._split(op.inputs[1]) if pointwise else None
                if (self.tc_stem and res is None and (kh, kw) == (3, 3) and x.shape[3] == 3
                        and self.g.stem_supported(x, y, stride=tuple(a["stride"]), pad=(pt, pl),
                                                  activation=a.get("activation", 0))):
                    self._plan.append(("stem", dict(
                        x=x, w=w, w_split=self.g.stem_weights(m.weights[op.inputs[1]]),
                        bias=self.w[op.inputs[2]], y=y, stride=tuple(a["stride"]), pad=(pt, pl),
                        activation=a.get("activation", 0))))
                    continue
                self._plan.append(("conv", dict(x=x, w=w, bias=self.w[op.inputs[2]], y=y,
                                                stride=a["stride"], pad=(pt, pl),
                                                activation=a.get("activation", 0),
                                                residual=res, w_split=split)))
            elif op.type == "DEPTHWISE_CONV_2D":
                x, y = self._buf(op.inputs[0]), self._buf(op.output)
                w = self.w[op.inputs[1]]
                kh, kw = w.shape[1], w.shape[2]
                dil = a.get("dilation", (1, 1))
                pt, pl = same_padding_offsets(a["padding"], x.shape[1], x.shape[2], y.shape[1],
                                              y.shape[2], (kh - 1) * dil[0] + 1,
                                              (kw - 1) * dil[1] + 1, *a["stride"])
                self._plan.append(("dw", dict(x=x, w=w.view((kh, kw, w.shape[3])),
                                              bias=self.w[op.inputs[2]], y=y, stride=a["stride"],
                                              pad=(pt, pl), dilation=dil,
                                              activation=a.get("activation", 0))))
            elif op.type == "ADD":
                if op.output in skip_adds:
                    continue
                a_, b_ = self._buf(op.inputs[0]), self._buf(op.inputs[1])
                self._plan.append(("add", dict(a=a_, b=b_, y=self._buf(op.output))))
            elif op.type == "AVERAGE_POOL_2D":
                x, y = self._buf(op.inputs[0]), self._buf(op.output)
                self._plan.append(("gap", dict(x=x, y=y)))
            elif op.type == "RESHAPE":
                x = self._buf(op.inputs[0])
                self.t[op.output] = x.view((self.batch,) + tuple(m.shapes[op.output]))
            elif op.type == "FULLY_CONNECTED":
                x, y = self._buf(op.inputs[0]), self._buf(op.output)
                w = self.w[op.inputs[1]]
                out, inp = w.shape
                self._plan.append(("fc", dict(x=x, w=w, bias=self.w[op.inputs[2]], y=y, m=self.batch,
                                              n=out, k=inp, activation=a.get("activation", 0),
                                              w_split=self._split(op.inputs[1]))))
            elif op.type == "SOFTMAX":
                x, y = self._buf(op.inputs[0]), self._buf(op.output)
                self._plan.append(("softmax", dict(x=x, y=y, rows=self.batch,
                                                   cols=x.size // self.batch)))
            else:
                raise NotImplementedError(f"op {op.type}")
        self.input = self.t[m.input]
        self.output = self.t[m.output]

    # -- execution -------------------------------------------------------------
    def record(self) -> None:
        """Records the whole graph onto the graph's stream (asynchronous)."""
        g = self.g
        for kind, p in self._plan:
            if kind == "conv":
                g.conv2d_nhwc(p["x"], p["w"], p["bias"], p["y"], stride=p["stride"], pad=p["pad"],
                              activation=p["activation"], residual=p["residual"],
                              w_split=p["w_split"])
            elif kind == "expand_dw":
                g.expand_dw_nhwc(p["x"], p["we"], p["be"], p["wd"], p["bd"], p["y"],
                                 stride=p["stride"], pad=p["pad"], act_expand=p["act_e"],
                                 act_dw=p["act_d"], w_split=p["we_split"])
            elif kind == "stem":
                g.stem_conv_nhwc(p["x"], p["w_split"], p["bias"], p["y"], stride=p["stride"],
                                 pad=p["pad"], activation=p["activation"])
            elif kind == "dwproj":
                g.dw_project_nhwc(p["x"], p["wd"], p["bd"], p["w_split"], p["bp"], p["y"],
                                  stride=p["stride"], pad=p["pad"], act_dw=p["act_dw"],
                                  act_proj=p["act_proj"], residual=p["residual"])
            elif kind == "dw":
                g.depthwise_nhwc(p["x"], p["w"], p["bias"], p["y"], stride=p["stride"],
                                 pad=p["pad"], dilation=p["dilation"], activation=p["activation"])
            elif kind == "add":
                g.add(p["a"], p["b"], p["y"])
            elif kind == "gap":
                g.global_avg_pool_nhwc(p["x"], p["y"])
            elif kind == "fc":
                g.gemm(p["x"], p["w"], p["y"], m=p["m"], n=p["n"], k=p["k"],
                       a_strides=(0, p["k"], 1), b_strides=(0, 1, p["k"]), c_strides=(0, p["n"]),
                       bias=p["bias"], activation=p["activation"], b_split=p["w_split"])
            elif kind == "softmax":
                g.softmax_rows(p["x"], p["y"], p["rows"], p["cols"])

    @property
    def kernels_per_run(self) -> int:
        return len(self._plan)

    def op_costs(self) -> list[dict]:
        """Algorithmic cost of each recorded kernel: flops (2 x MACs) and HBM
        bytes (every input / weight / bias / residual read once, the output
        written once, fp32)."""
        out = []
        for kind, p in self._plan:
            if kind in ("conv", "stem"):
                x, w, y = p["x"], p["w"], p["y"]
                k = w.shape[1] * w.shape[2] * w.shape[3]
                f = 2 * y.size * k
                b = (x.size + w.size + y.shape[-1] + y.size
                     + (y.size if p.get("residual") is not None else 0))
                label = f"conv{w.shape[1]}x{w.shape[2]}"
            elif kind == "expand_dw":
                x, y, we = p["x"], p["y"], p["we"]
                ce, cin = we.shape[0], we.shape[3]
                e_px = x.size // cin                       # expanded pixels (input resolution)
                f = 2 * e_px * ce * cin + 2 * y.size * 9
                b = x.size + we.size + ce + p["wd"].size + ce + y.size
                label = "expand_dw"
            elif kind == "dwproj":
                x, wd, w, y = p["x"], p["wd"], p["w"], p["y"]
                c, cout = x.shape[-1], y.shape[-1]
                px = y.size // cout
                f = 2 * px * c * 9 + 2 * px * c * cout
                b = (x.size + wd.size + c + w.size + cout + y.size
                     + (y.size if p["residual"] is not None else 0))
                label = "dw_project"
            elif kind == "dw":
                x, w, y = p["x"], p["w"], p["y"]
                f = 2 * y.size * w.shape[0] * w.shape[1]
                b = x.size + w.size + y.shape[-1] + y.size
                label = f"dw{w.shape[0]}x{w.shape[1]}"
            elif kind == "add":
                f, b, label = p["y"].size, 3 * p["y"].size, "add"
            elif kind == "gap":
                f, b, label = p["x"].size, p["x"].size + p["y"].size, "gap"
            elif kind == "fc":
                f = 2 * p["m"] * p["n"] * p["k"]
                b = p["m"] * p["k"] + p["n"] * p["k"] + p["n"] + p["m"] * p["n"]
                label = "fc"
            else:
                f, b, label = 3 * p["x"].size, 2 * p["x"].size, "softmax"
            out.append({"kind": kind, "label": label, "flops": int(f), "bytes": int(4 * b)})
        return out

    def record_op(self, i: int) -> None:
        """Records only plan entry i (for per-kernel timing)."""
        plan, self._plan = self._plan, [self._plan[i]]
        try:
            self.record()
        finally:
            self._plan = plan

    def capture(self) -> None:
        """Captures one recording into a CUDA graph for replay()."""
        self.g.sync()
        self.g.capture_begin()
        self.record()
        self.g.capture_end()
        self._captured = True

    def run(self) -> None:
        if self._captured:
            self.g.replay()
        else:
            self.record()

    def forward(self, x_nhwc: np.ndarray) -> np.ndarray:
        """Host in, host out: upload, run, download (synchronous)."""
        self.g.upload(self.input, x_nhwc)
        self.run()
        return self.g.download(self.output)

    def tensor(self, name: str) -> np.ndarray:
        if name in self.fused_away:
            raise KeyError(f"{name} stays on chip inside a fused kernel (fuse_dw_project=False "
                           "keeps it)")
        return self.g.download(self.t[name])

    def close(self) -> None:
        self.g.close()
