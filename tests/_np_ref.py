"""Independent float64 numpy formulations of the kernel math.

Used to cross-check the C++ oracle (a second, structurally different
implementation: vectorised tensor algebra instead of per-output loops) and
the graph-API ops whose layout has no reference kernel (NHWC depthwise etc.).
"""
from __future__ import annotations

import numpy as np


def conv_nhwc(x, w_hwio, stride, pad_tl, out_hw, dilation=(1, 1)):
    """x [n,ih,iw,ic], w [kh,kw,ic,oc]; low-side pad pad_tl, out size out_hw."""
    x = x.astype(np.float64)
    w = w_hwio.astype(np.float64)
    n, ih, iw, ic = x.shape
    kh, kw, _, oc = w.shape
    oh, ow = out_hw
    y = np.zeros((n, oh, ow, oc))
    for ky in range(kh):
        for kx in range(kw):
            iy = np.arange(oh) * stride[0] + ky * dilation[0] - pad_tl[0]
            ix = np.arange(ow) * stride[1] + kx * dilation[1] - pad_tl[1]
            vy = (iy >= 0) & (iy < ih)
            vx = (ix >= 0) & (ix < iw)
            patch = np.zeros((n, oh, ow, ic))
            sub = x[:, np.clip(iy, 0, ih - 1)][:, :, np.clip(ix, 0, iw - 1)]
            mask = (vy[:, None] & vx[None, :])[None, :, :, None]
            patch = np.where(mask, sub, 0.0)
            y += patch @ w[ky, kx]
    return y


def conv_nchw(x, w_oihw, bias, stride, pad_tl, out_hw):
    y = conv_nhwc(np.transpose(x, (0, 2, 3, 1)), np.transpose(w_oihw, (2, 3, 1, 0)), stride,
                  pad_tl, out_hw)
    return np.transpose(y + bias.astype(np.float64), (0, 3, 1, 2))


def depthwise_nhwc(x, w_hwc, bias, stride, pad_tl, out_hw, dilation=(1, 1)):
    x = x.astype(np.float64)
    n, ih, iw, c = x.shape
    kh, kw, _ = w_hwc.shape
    oh, ow = out_hw
    y = np.zeros((n, oh, ow, c)) + (bias.astype(np.float64) if bias is not None else 0.0)
    for ky in range(kh):
        for kx in range(kw):
            iy = np.arange(oh) * stride[0] + ky * dilation[0] - pad_tl[0]
            ix = np.arange(ow) * stride[1] + kx * dilation[1] - pad_tl[1]
            vy = (iy >= 0) & (iy < ih)
            vx = (ix >= 0) & (ix < iw)
            sub = x[:, np.clip(iy, 0, ih - 1)][:, :, np.clip(ix, 0, iw - 1)]
            mask = (vy[:, None] & vx[None, :])[None, :, :, None]
            y += np.where(mask, sub, 0.0) * w_hwc[ky, kx].astype(np.float64)
    return y


def pool_nhwc(x, k, stride, pad_tl, out_hw, kind):
    """kind 1 max, 0 sum, 2 average over in-range taps."""
    x = x.astype(np.float64)
    n, ih, iw, c = x.shape
    oh, ow = out_hw
    acc = np.full((n, oh, ow, c), -3.4028234663852886e38 if kind == 1 else 0.0)
    cnt = np.zeros((1, oh, ow, 1))
    for ky in range(k[0]):
        for kx in range(k[1]):
            iy = np.arange(oh) * stride[0] + ky - pad_tl[0]
            ix = np.arange(ow) * stride[1] + kx - pad_tl[1]
            vy = (iy >= 0) & (iy < ih)
            vx = (ix >= 0) & (ix < iw)
            mask = (vy[:, None] & vx[None, :])[None, :, :, None]
            sub = x[:, np.clip(iy, 0, ih - 1)][:, :, np.clip(ix, 0, iw - 1)]
            cnt += mask
            if kind == 1:
                acc = np.where(mask, np.maximum(acc, sub), acc)
            else:
                acc = acc + np.where(mask, sub, 0.0)
    if kind == 2:
        acc = acc / np.maximum(cnt, 1)
    return acc


def softmax_rows(x):
    x = x.astype(np.float64)
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


def resize_bilinear_nchw(x, oh, ow, align_corners, half_pixel):
    n, c, ih, iw = x.shape

    def coords(o, i_size, o_size):
        o = np.arange(o_size, dtype=np.float64)
        if align_corners and o_size > 1:
            s = o * (i_size - 1) / (o_size - 1)
        elif half_pixel:
            s = (o + 0.5) * i_size / o_size - 0.5
        else:
            s = o * i_size / o_size
        return np.clip(s, 0, i_size - 1)

    ys, xs = coords(None, ih, oh), coords(None, iw, ow)
    y0 = np.floor(ys).astype(int)
    x0 = np.floor(xs).astype(int)
    y1 = np.minimum(y0 + 1, ih - 1)
    x1 = np.minimum(x0 + 1, iw - 1)
    yl = (ys - y0)[:, None]
    xl = (xs - x0)[None, :]
    xd = x.astype(np.float64)
    top = xd[:, :, y0][:, :, :, x0] * (1 - xl) + xd[:, :, y0][:, :, :, x1] * xl
    bot = xd[:, :, y1][:, :, :, x0] * (1 - xl) + xd[:, :, y1][:, :, :, x1] * xl
    return top * (1 - yl) + bot * yl


def eval_hlo_f64(g, feeds):
    """Independent float64 evaluation of an spirv_inference_b200.hlo graph."""
    vals = {}
    for op in g.ops:
        oc, a = op.opcode, op.attrs
        ins = [vals[o] for o in op.operands]
        if oc == "parameter":
            vals[op.name] = np.asarray(feeds.get(op.name, g.params.get(op.name)), np.float64).reshape(op.shape)
            continue
        if oc == "constant":
            vals[op.name] = np.array(a["value"], np.float64)
            continue
        if oc == "broadcast":
            view = [1] * len(op.shape)
            for sa, oa in enumerate(a["dimensions"]):
                view[oa] = ins[0].shape[sa]
            r = np.broadcast_to(ins[0].reshape(view), op.shape)
        elif oc == "reshape":
            r = ins[0].reshape(op.shape)
        elif oc == "transpose":
            r = np.transpose(ins[0], a["dimensions"])
        elif oc == "pad":
            r = np.pad(ins[0], a["padding"], constant_values=float(ins[1]))
        elif oc == "convolution":
            r = conv_nhwc(ins[0], ins[1], a["stride"], (a["pad"][0][0], a["pad"][1][0]), op.shape[1:3])
        elif oc == "reduce-window":
            r = pool_nhwc(ins[0], a["size"], a["stride"], (a["pad"][0][0], a["pad"][1][0]), op.shape[1:3],
                          1 if a["kind"] == "max" else 0)
        elif oc == "reduce":
            f = np.max if a["kind"] == "max" else np.sum
            r = f(ins[0], axis=tuple(a["dimensions"]))
        elif oc == "dot":
            x, y = ins
            lb, rb = list(a["lhs_batch_dims"]), list(a["rhs_batch_dims"])
            lc, rc = list(a["lhs_contracting_dims"]), list(a["rhs_contracting_dims"])
            lf = [d for d in range(x.ndim) if d not in lb + lc]
            rf = [d for d in range(y.ndim) if d not in rb + rc]
            xt = np.transpose(x, lb + lf + lc)
            yt = np.transpose(y, rb + rc + rf)
            Bs = [x.shape[d] for d in lb]
            M, K, N = int(np.prod([x.shape[d] for d in lf])), x.shape[lc[0]], int(np.prod([y.shape[d] for d in rf]))
            r = (xt.reshape(-1, M, K) @ yt.reshape(-1, K, N)).reshape(op.shape)
        elif oc == "slice":
            r = ins[0][tuple(slice(s0, e0, st) for s0, e0, st in a["slice"])]
        elif oc == "concatenate":
            r = np.concatenate(ins, axis=a["dimensions"][0])
        elif oc in ("tuple", "convert"):
            r = ins[0]
        elif oc == "get-tuple-element":
            r = ins[0]
        elif oc == "compare":
            fn = {"LT": np.less, "LE": np.less_equal, "EQ": np.equal, "NE": np.not_equal,
                  "GE": np.greater_equal}.get(a.get("direction"), np.greater)
            r = fn(ins[0], ins[1]).astype(np.float64)
        elif oc == "select":
            r = np.where(ins[0] != 0, ins[1], ins[2])
        else:
            fns = {"add": np.add, "subtract": np.subtract, "multiply": np.multiply, "divide": np.divide,
                   "maximum": np.maximum, "minimum": np.minimum, "power": np.power}
            una = {"exponential": np.exp, "log": np.log, "sqrt": np.sqrt, "rsqrt": lambda v: 1 / np.sqrt(v),
                   "negate": np.negative, "abs": np.abs, "tanh": np.tanh,
                   "logistic": lambda v: 1 / (1 + np.exp(-v))}
            if oc in fns:
                r = fns[oc](ins[0], ins[1])
            else:
                r = una[oc](ins[0])
        vals[op.name] = np.asarray(r, np.float64).reshape(op.shape)
    return vals[g.output]
