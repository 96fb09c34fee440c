"""TFLite-style graph descriptions of the CNN configs, with seeded weights.

No ``.tflite`` files are vendored with the reference (its model evidence is
excluded from the package), so the graphs the reference's TFLite scheduler
would load are constructed here directly in TFLite's own terms: NHWC tensor
shapes, Conv2D weights OHWI ``[oc, kh, kw, ic]``, DepthwiseConv2D weights
``[1, kh, kw, c]``, FullyConnected weights ``[out, in]``, separate bias
tensors, SAME/VALID padding and a fused activation per op (the option set
decoded by source/tflite_loader/src/op_decoder.rs:124-211).

Weights are He-normal ``N(0, sqrt(2 / fan_in))`` with BatchNorm folded into
a bias drawn from ``N(0, 0.01)``; the input is ``U[-1, 1]``.  All draws come
from ``numpy.random.Generator(PCG64(seed))`` in a fixed order.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

ACT_NONE, ACT_RELU, ACT_RELU6 = 0, 1, 3


@dataclass
class Op:
    type: str                    # TFLite builtin name, e.g. "CONV_2D"
    inputs: list[str]
    output: str
    attrs: dict = field(default_factory=dict)


@dataclass
class Model:
    name: str
    input: str
    output: str
    shapes: dict[str, tuple[int, ...]]   # per-image shapes (batch dim excluded)
    ops: list[Op]
    weights: dict[str, np.ndarray]

    def op_counts(self) -> dict[str, int]:
        out: dict[str, int] = {}
        for op in self.ops:
            out[op.type] = out.get(op.type, 0) + 1
        return out

    def flops_per_image(self) -> int:
        """2 x MACs of the conv / depthwise / FC ops (algorithmic count)."""
        f = 0
        for op in self.ops:
            if op.type == "CONV_2D":
                oh, ow, oc = self.shapes[op.output]
                w = self.weights[op.inputs[1]]
                f += 2 * oh * ow * oc * w.shape[1] * w.shape[2] * w.shape[3]
            elif op.type == "DEPTHWISE_CONV_2D":
                oh, ow, c = self.shapes[op.output]
                w = self.weights[op.inputs[1]]
                f += 2 * oh * ow * c * w.shape[1] * w.shape[2]
            elif op.type == "FULLY_CONNECTED":
                w = self.weights[op.inputs[1]]
                f += 2 * w.shape[0] * w.shape[1]
        return f


def same_out(size: int, stride: int) -> int:
    return -(-size // stride)


class _Builder:
    def __init__(self, name: str, seed: int, input_hw=(224, 224), in_ch=3):
        self.rng = np.random.Generator(np.random.PCG64(seed))
        self.name = name
        self.ops: list[Op] = []
        self.weights: dict[str, np.ndarray] = {}
        self.shapes: dict[str, tuple[int, ...]] = {"input": (input_hw[0], input_hw[1], in_ch)}
        self.n = 0

    def _t(self, prefix: str) -> str:
        self.n += 1
        return f"{prefix}_{self.n}"

    def _he(self, shape, fan_in):
        return (self.rng.standard_normal(shape, dtype=np.float64) * np.sqrt(2.0 / fan_in)).astype(np.float32)

    def _bias(self, n):
        return (self.rng.standard_normal(n, dtype=np.float64) * 0.01).astype(np.float32)

    def conv(self, x: str, oc: int, k: int, stride: int, act: int) -> str:
        h, w, ic = self.shapes[x]
        wn, bn, y = self._t("conv_w"), self._t("conv_b"), self._t("conv")
        self.weights[wn] = self._he((oc, k, k, ic), k * k * ic)
        self.weights[bn] = self._bias(oc)
        self.shapes[y] = (same_out(h, stride), same_out(w, stride), oc)
        self.ops.append(Op("CONV_2D", [x, wn, bn], y,
                           dict(stride=(stride, stride), padding="SAME", activation=act,
                                dilation=(1, 1))))
        return y

    def dw(self, x: str, k: int, stride: int, act: int) -> str:
        h, w, c = self.shapes[x]
        wn, bn, y = self._t("dw_w"), self._t("dw_b"), self._t("dw")
        self.weights[wn] = self._he((1, k, k, c), k * k)
        self.weights[bn] = self._bias(c)
        self.shapes[y] = (same_out(h, stride), same_out(w, stride), c)
        self.ops.append(Op("DEPTHWISE_CONV_2D", [x, wn, bn], y,
                           dict(stride=(stride, stride), padding="SAME", activation=act,
                                dilation=(1, 1), depth_multiplier=1)))
        return y

    def add(self, a: str, b: str) -> str:
        y = self._t("add")
        self.shapes[y] = self.shapes[a]
        self.ops.append(Op("ADD", [a, b], y, dict(activation=ACT_NONE)))
        return y

    def global_avg_pool(self, x: str) -> str:
        h, w, c = self.shapes[x]
        y = self._t("avgpool")
        self.shapes[y] = (1, 1, c)
        self.ops.append(Op("AVERAGE_POOL_2D", [x], y,
                           dict(filter=(h, w), stride=(1, 1), padding="VALID",
                                activation=ACT_NONE)))
        return y

    def reshape(self, x: str, shape) -> str:
        y = self._t("reshape")
        self.shapes[y] = tuple(shape)
        self.ops.append(Op("RESHAPE", [x], y, {}))
        return y

    def fc(self, x: str, out: int, act: int = ACT_NONE) -> str:
        (inp,) = self.shapes[x]
        wn, bn, y = self._t("fc_w"), self._t("fc_b"), self._t("fc")
        self.weights[wn] = self._he((out, inp), inp)
        self.weights[bn] = self._bias(out)
        self.shapes[y] = (out,)
        self.ops.append(Op("FULLY_CONNECTED", [x, wn, bn], y, dict(activation=act)))
        return y

    def softmax(self, x: str) -> str:
        y = self._t("softmax")
        self.shapes[y] = self.shapes[x]
        self.ops.append(Op("SOFTMAX", [x], y, dict(beta=1.0)))
        return y

    def inverted_residual(self, x: str, out_ch: int, stride: int, expand: int, k: int) -> str:
        ic = self.shapes[x][2]
        h = x
        if expand != 1:
            h = self.conv(h, ic * expand, 1, 1, ACT_RELU6)
        h = self.dw(h, k, stride, ACT_RELU6)
        h = self.conv(h, out_ch, 1, 1, ACT_NONE)
        if stride == 1 and ic == out_ch:
            h = self.add(h, x)
        return h

    def model(self, out: str) -> Model:
        return Model(self.name, "input", out, self.shapes, self.ops, self.weights)


def mobilenet_v2(seed: int = 0, num_classes: int = 1001) -> Model:
    """MobileNetV2 1.0/224 as TFLite lays it out (66 ops: 36 Conv2D,
    17 DepthwiseConv2D, 10 Add, 1 AveragePool2D, 1 Reshape, 1 Softmax — the
    histogram of source/tflite_loader/TFLITE_REPORT.md:16)."""
    b = _Builder("mobilenet_v2", seed)
    x = b.conv("input", 32, 3, 2, ACT_RELU6)
    # (expansion, out channels, repeats, first stride)
    for t, c, n, s in [(1, 16, 1, 1), (6, 24, 2, 2), (6, 32, 3, 2), (6, 64, 4, 2),
                       (6, 96, 3, 1), (6, 160, 3, 2), (6, 320, 1, 1)]:
        for i in range(n):
            x = b.inverted_residual(x, c, s if i == 0 else 1, t, 3)
    x = b.conv(x, 1280, 1, 1, ACT_RELU6)
    x = b.global_avg_pool(x)
    x = b.conv(x, num_classes, 1, 1, ACT_NONE)   # classifier as a 1x1 conv
    x = b.reshape(x, (num_classes,))
    x = b.softmax(x)
    return b.model(x)


def efficientnet_lite0(seed: int = 0, num_classes: int = 1000) -> Model:
    """EfficientNet-Lite0: stem 3x3 s2 -> 32, 16 MBConv blocks without
    squeeze-excite (kernel, expansion, out channels, repeats, stride per stage
    below), ReLU6, 1x1 conv to 1280, global average pool, FC, softmax."""
    b = _Builder("efficientnet_lite0", seed)
    x = b.conv("input", 32, 3, 2, ACT_RELU6)
    for k, t, c, n, s in [(3, 1, 16, 1, 1), (3, 6, 24, 2, 2), (5, 6, 40, 2, 2), (3, 6, 80, 3, 2),
                          (5, 6, 112, 3, 1), (5, 6, 192, 4, 2), (3, 6, 320, 1, 1)]:
        for i in range(n):
            x = b.inverted_residual(x, c, s if i == 0 else 1, t, k)
    x = b.conv(x, 1280, 1, 1, ACT_RELU6)
    x = b.global_avg_pool(x)
    x = b.reshape(x, (1280,))
    x = b.fc(x, num_classes)
    x = b.softmax(x)
    return b.model(x)


def make_input(model: Model, batch: int, seed: int = 1234) -> np.ndarray:
    """Seeded U[-1, 1] input batch, NHWC."""
    rng = np.random.Generator(np.random.PCG64(seed))
    shape = (batch,) + model.shapes[model.input]
    return rng.uniform(-1.0, 1.0, size=shape).astype(np.float32)


MODELS = {"mobilenet_v2": mobilenet_v2, "efficientnet_lite0": efficientnet_lite0}
