"""Per-op lowering of a TFLite-style graph onto the dispatch boundary, with
the reference scheduler's semantics (source/tflite_loader/src/scheduler.rs).

This is the drop-in caller of the hot path: every op becomes one or two
``run_kernel`` dispatches exactly as ``scheduler::run_graph`` issues them —
same kernel names, push-constant layouts, NCHW activation layout, host-side
weight packing and a separate activation dispatch after each fused-activation
op.  ``run_kernel`` is injected, so the same lowering drives the sm_100a
library (``dispatch.run_kernel``) or any other implementation of the
boundary with the same signature.

One deliberate generalisation: the reference softmax shaders handle a single
row (softmax1000.comp:10-22 reads row 0 only); for batch > 1 the lowering
issues the same kernel once per row.
"""
from __future__ import annotations

from typing import Callable

import numpy as np

from .nets import Model

RunKernel = Callable[[str, np.ndarray, np.ndarray, int, list], np.ndarray]


def pack_conv_weight(w_ohwi: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """scheduler.rs:1327-1362: OHWI -> OIHW, then the oc biases appended."""
    oc = w_ohwi.shape[0]
    return np.concatenate([np.transpose(w_ohwi, (0, 3, 1, 2)).reshape(-1),
                           bias.reshape(oc)]).astype(np.float32)


def pack_depthwise_weight(w_1hwc: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """scheduler.rs:1364-1400: [1,kh,kw,c] -> [c][kh][kw], then c biases."""
    return np.concatenate([np.transpose(w_1hwc[0], (2, 0, 1)).reshape(-1),
                           bias.reshape(-1)]).astype(np.float32)


def pack_fully_connected_weight(w: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """scheduler.rs:1402-1436: [out][in] followed by out biases."""
    return np.concatenate([w.reshape(-1), bias.reshape(-1)]).astype(np.float32)


def same_padding_offsets(padding: str, ih, iw, oh, ow, kh, kw, sh, sw) -> tuple[int, int]:
    """scheduler.rs:1597-1614: SAME pads floor(total/2) on top/left."""
    if padding != "SAME":
        return 0, 0
    th = max((oh - 1) * sh + kh - ih, 0)
    tw = max((ow - 1) * sw + kw - iw, 0)
    return th // 2, tw // 2


def _activation(rk: RunKernel, act: int, values: np.ndarray, log: list) -> np.ndarray:
    """scheduler.rs:1146-1197: a separate relu / relu6 dispatch."""
    if act == 0:
        return values
    name = {1: "relu.spv", 3: "relu6.spv"}.get(act)
    if name is None:
        raise NotImplementedError(f"fused activation {act} has no scheduler post-op lowering")
    log.append(name)
    return rk(name, values, np.zeros(1, np.float32), values.size, [values.size])


def run_graph(model: Model, x_nhwc: np.ndarray, rk: RunKernel,
              keep: bool = False) -> tuple[np.ndarray, dict]:
    """Runs ``model`` on a batch.  Returns (output values, report).

    The input batch is given NHWC and handed to the first op in NCHW order,
    which is what the reference's 4-D input labelling requires
    (scheduler.rs:58-62 labels a 4-D input NCHW without transposing).
    """
    batch = x_nhwc.shape[0]
    unused = np.zeros(1, np.float32)
    vals: dict[str, np.ndarray] = {model.input: np.ascontiguousarray(
        np.transpose(x_nhwc, (0, 3, 1, 2))).reshape(-1)}
    log: list[str] = []

    def nchw(name):  # per-image NHWC shape -> batch NCHW dims
        s = model.shapes[name]
        return (batch, s[2], s[0], s[1]) if len(s) == 3 else None

    for op in model.ops:
        a = op.attrs
        if op.type in ("CONV_2D", "DEPTHWISE_CONV_2D"):
            x = vals[op.inputs[0]]
            w = model.weights[op.inputs[1]]
            bias = model.weights[op.inputs[2]]
            n, ic, ih, iw = nchw(op.inputs[0])
            _, oc, oh, ow = nchw(op.output)
            dil = a.get("dilation", (1, 1))
            kh, kw = w.shape[1], w.shape[2]
            pt, pl = same_padding_offsets(a["padding"], ih, iw, oh, ow, (kh - 1) * dil[0] + 1,
                                          (kw - 1) * dil[1] + 1, a["stride"][0], a["stride"][1])
            total = n * oc * oh * ow
            same = 1 if a["padding"] == "SAME" else 0
            if op.type == "CONV_2D":
                if dil != (1, 1):
                    raise NotImplementedError("Conv2D dilation is unsupported (scheduler.rs:341)")
                push = [n, ic, ih, iw, oc, oh, ow, kh, kw, a["stride"][0], a["stride"][1], same,
                        pt, pl, total]
                out = rk("conv2d.spv", x, pack_conv_weight(w, bias), total, push)
                log.append("conv2d.spv")
            else:
                if a.get("depth_multiplier", 1) != 1:
                    raise NotImplementedError("depth_multiplier must be 1 (scheduler.rs:457)")
                push = [n, ic, ih, iw, oh, ow, kh, kw, a["stride"][0], a["stride"][1], same, pt,
                        pl, dil[0], dil[1], total]
                out = rk("depthwise_conv2d.spv", x, pack_depthwise_weight(w, bias), total, push)
                log.append("depthwise_conv2d.spv")
            vals[op.output] = _activation(rk, a.get("activation", 0), out, log)
        elif op.type in ("ADD", "SUB", "MUL", "DIV"):
            if a.get("activation", 0):
                raise NotImplementedError("fused activation on binary op (scheduler.rs:151)")
            xa, xb = vals[op.inputs[0]], vals[op.inputs[1]]
            if xa.size != xb.size:
                raise ValueError("binary op requires equal-sized tensors (scheduler.rs:172-180)")
            name = {"ADD": "add", "SUB": "sub", "MUL": "mul", "DIV": "div"}[op.type] + ".spv"
            vals[op.output] = rk(name, xa, xb, xa.size, [xa.size])
            log.append(name)
        elif op.type == "AVERAGE_POOL_2D":
            x = vals[op.inputs[0]]
            n, c, h, w = nchw(op.inputs[0])
            if model.shapes[op.output][:2] != (1, 1):
                raise NotImplementedError("only global average pool (scheduler.rs:563-568)")
            push = [n, c, h, w]
            s = rk("global_avg_pool_sum.spv", x, unused, n * c, push)
            vals[op.output] = rk("global_avg_pool_finalize.spv", s, unused, n * c, push)
            log += ["global_avg_pool_sum.spv", "global_avg_pool_finalize.spv"]
        elif op.type == "RESHAPE":
            x = vals[op.inputs[0]]
            vals[op.output] = rk("reshape.spv", x, unused, x.size, [x.size])
            log.append("reshape.spv")
        elif op.type == "FULLY_CONNECTED":
            x = vals[op.inputs[0]]
            w, bias = model.weights[op.inputs[1]], model.weights[op.inputs[2]]
            out_size, in_size = w.shape
            total = batch * out_size
            out = rk("fully_connected.spv", x, pack_fully_connected_weight(w, bias), total,
                     [batch, in_size, out_size, total])
            log.append("fully_connected.spv")
            vals[op.output] = _activation(rk, a.get("activation", 0), out, log)
        elif op.type == "SOFTMAX":
            x = vals[op.inputs[0]]
            classes = x.size // batch
            rows = []
            for r in range(batch):
                row = x[r * classes:(r + 1) * classes]
                if classes == 10:
                    rows.append(rk("softmax10.spv", row, unused, 10, []))
                    log.append("softmax10.spv")
                else:
                    rows.append(rk("softmax1000.spv", row, unused, classes, [classes]))
                    log.append("softmax1000.spv")
            vals[op.output] = np.concatenate(rows)
        else:
            raise NotImplementedError(f"op {op.type} has no lowering")
    out = vals[model.output].reshape((batch,) + model.shapes[model.output])
    report = {"dispatches": log, "num_dispatches": len(log)}
    if keep:
        report["tensors"] = vals
    return out, report


def top1(probs: np.ndarray) -> np.ndarray:
    """scheduler.rs:1637-1652: index of the largest value per row."""
    return np.argmax(probs.reshape(probs.shape[0], -1), axis=1)
