"""HLO-style graphs of the HLO-path configs, built with the op set the
reference executor lowers (source/xla_hlo/src/compiler.rs:284-625).

* ResNet-50 v1.5 (Keras layout): pad 3 + 7x7/2 conv, pad 1 + 3x3/2 max
  reduce-window, bottleneck stages [3, 4, 6, 3] (widths 64..512, 4x
  expansion, stride in the 3x3 conv, projection shortcuts), global average
  pool as reduce-sum / divide, FC 1000.  BatchNorm is folded: every conv is
  `convolution -> add(broadcast bias) [-> add(shortcut)] -> maximum(0)`.
* BERT-base encoder layers on embedded input [B, S, 768]: Q/K/V/O and FFN as
  `dot` + bias, attention as batched `dot`s around a reduce-max / exp /
  reduce-sum / divide softmax, LayerNorm as reduce-mean / rsqrt chains, GELU
  in its tanh form (the erf form has no kernel in the reference set).
* `bert_block_fixture`: the single attention block of
  source/xla_hlo/tools/run_tf_reference.py:86-107 (x = linspace(-0.1, 0.1),
  one 0.001-filled matrix used for q = k = v and one for the output), with
  its final GELU in tanh form.

Weights: He-normal for convs / FC (ResNet), N(0, 0.02) for BERT, seeded
PCG64; ResNet inputs N(0, 1).
"""
from __future__ import annotations

import numpy as np

from .hlo import Builder, HloGraph


def _rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def _bias_relu(b: Builder, x: str, bias: np.ndarray, relu: bool, residual: str | None = None):
    s = b.shapes[x]
    y = b.binary("add", x, b.broadcast(b.weight(bias), s, (len(s) - 1,)))
    if residual is not None:
        y = b.binary("add", y, residual)
    if relu:
        y = b.binary("maximum", y, b.broadcast(b.constant(0.0), s, ()))
    return y


def resnet50(seed: int = 0, batch: int = 1, hw: int = 224, stages=(3, 4, 6, 3),
             num_classes: int = 1000) -> HloGraph:
    rng = _rng(seed)
    b = Builder("resnet50")

    def conv(x, oc, k, stride, pad, relu=True, residual=None):
        ic = b.shapes[x][3]
        w = (rng.standard_normal((k, k, ic, oc)) * np.sqrt(2.0 / (k * k * ic))).astype(np.float32)
        bias = (rng.standard_normal(oc) * 0.01).astype(np.float32)
        y = b.conv(x, b.weight(w), (stride, stride), ((pad, pad), (pad, pad)))
        return _bias_relu(b, y, bias, relu, residual)

    x = b.input((batch, hw, hw, 3))
    h = b.pad(x, (0, 3, 3, 0), (0, 3, 3, 0))
    h = conv(h, 64, 7, 2, 0)
    h = b.pad(h, (0, 1, 1, 0), (0, 1, 1, 0))
    h = b.reduce_window(h, (3, 3), (2, 2), ((0, 0), (0, 0)), "max")
    width = 64
    for si, n_blocks in enumerate(stages):
        for bi in range(n_blocks):
            stride = 2 if (bi == 0 and si > 0) else 1
            inp = h
            out_c = width * 4
            t = conv(inp, width, 1, 1, 0)
            t = conv(t, width, 3, stride, 1)
            if bi == 0:
                sc = conv(inp, out_c, 1, stride, 0, relu=False)
            else:
                sc = inp
            h = conv(t, out_c, 1, 1, 0, relu=True, residual=sc)
        width *= 2
    n, hh, ww, c = b.shapes[h]
    s = b.reduce(h, (1, 2), "sum")
    s = b.binary("divide", s, b.broadcast(b.constant(float(hh * ww)), (n, c), ()))
    wfc = (rng.standard_normal((c, num_classes)) * np.sqrt(2.0 / c)).astype(np.float32)
    bfc = (rng.standard_normal(num_classes) * 0.01).astype(np.float32)
    logits = b.dot(s, b.weight(wfc), (1,), (0,))
    logits = b.binary("add", logits, b.broadcast(b.weight(bfc), (n, num_classes), (1,)))
    return b.graph(logits)


def _layernorm(b: Builder, x: str, gamma, beta, eps: float) -> str:
    s = b.shapes[x]
    H = s[-1]
    red = tuple(s[:-1])
    mean = b.binary("divide", b.reduce(x, (len(s) - 1,), "sum"), b.broadcast(b.constant(H), red, ()))
    xc = b.binary("subtract", x, b.broadcast(mean, s, tuple(range(len(s) - 1))))
    var = b.binary("divide", b.reduce(b.binary("multiply", xc, xc), (len(s) - 1,), "sum"),
                   b.broadcast(b.constant(H), red, ()))
    r = b.unary("rsqrt", b.binary("add", var, b.broadcast(b.constant(eps), red, ())))
    y = b.binary("multiply", xc, b.broadcast(r, s, tuple(range(len(s) - 1))))
    y = b.binary("multiply", y, b.broadcast(b.weight(gamma), s, (len(s) - 1,)))
    return b.binary("add", y, b.broadcast(b.weight(beta), s, (len(s) - 1,)))


def _gelu_tanh(b: Builder, x: str) -> str:
    s = b.shapes[x]
    c = lambda v: b.broadcast(b.constant(v), s, ())
    x3 = b.binary("multiply", b.binary("multiply", x, x), x)
    inner = b.binary("add", x, b.binary("multiply", x3, c(0.044715)))
    t = b.unary("tanh", b.binary("multiply", inner, c(0.7978845608028654)))
    return b.binary("multiply", b.binary("multiply", x, b.binary("add", t, c(1.0))), c(0.5))


def _linear(b: Builder, x: str, w: np.ndarray, bias: np.ndarray | None) -> str:
    s = b.shapes[x]
    y = b.dot(x, b.weight(w), (len(s) - 1,), (0,))
    if bias is not None:
        ys = b.shapes[y]
        y = b.binary("add", y, b.broadcast(b.weight(bias), ys, (len(ys) - 1,)))
    return y


def _softmax_last(b: Builder, x: str) -> str:
    s = b.shapes[x]
    keep = tuple(range(len(s) - 1))
    m = b.reduce(x, (len(s) - 1,), "max")
    e = b.unary("exponential", b.binary("subtract", x, b.broadcast(m, s, keep)))
    d = b.reduce(e, (len(s) - 1,), "sum")
    return b.binary("divide", e, b.broadcast(d, s, keep))


def _attention(b: Builder, q: str, k: str, v: str, heads: int, scale: float) -> str:
    B, S, H = b.shapes[q]
    D = H // heads
    qh = b.transpose(b.reshape(q, (B, S, heads, D)), (0, 2, 1, 3))
    kh = b.transpose(b.reshape(k, (B, S, heads, D)), (0, 2, 1, 3))
    vh = b.transpose(b.reshape(v, (B, S, heads, D)), (0, 2, 1, 3))
    sc = b.dot(qh, kh, (3,), (3,), (0, 1), (0, 1))                        # [B, h, S, S]
    sc = b.binary("multiply", sc, b.broadcast(b.constant(scale), b.shapes[sc], ()))
    p = _softmax_last(b, sc)
    ctx = b.dot(p, vh, (3,), (2,), (0, 1), (0, 1))                         # [B, h, S, D]
    ctx = b.transpose(ctx, (0, 2, 1, 3))
    return b.reshape(ctx, (B, S, H))


def bert_encoder(seed: int = 0, batch: int = 1, seq: int = 128, layers: int = 12,
                 hidden: int = 768, heads: int = 12, ffn: int = 3072,
                 eps: float = 1e-12) -> HloGraph:
    rng = _rng(seed)
    nrm = lambda *shape: (rng.standard_normal(shape) * 0.02).astype(np.float32)
    b = Builder("bert_encoder")
    x = b.input((batch, seq, hidden))
    h = _layernorm(b, x, np.ones(hidden, np.float32), np.zeros(hidden, np.float32), eps)
    for _ in range(layers):
        q = _linear(b, h, nrm(hidden, hidden), nrm(hidden))
        k = _linear(b, h, nrm(hidden, hidden), nrm(hidden))
        v = _linear(b, h, nrm(hidden, hidden), nrm(hidden))
        ctx = _attention(b, q, k, v, heads, 1.0 / np.sqrt(hidden // heads))
        o = _linear(b, ctx, nrm(hidden, hidden), nrm(hidden))
        h = _layernorm(b, b.binary("add", o, h), 1 + nrm(hidden), nrm(hidden), eps)
        f = _gelu_tanh(b, _linear(b, h, nrm(hidden, ffn), nrm(ffn)))
        f = _linear(b, f, nrm(ffn, hidden), nrm(hidden))
        h = _layernorm(b, b.binary("add", f, h), 1 + nrm(hidden), nrm(hidden), eps)
    return b.graph(h)


def bert_embed(seed: int, ids: np.ndarray, hidden: int = 768, vocab: int = 30522,
               max_pos: int = 512) -> np.ndarray:
    """Host-side word + position embedding (the reference drivers gather
    embeddings in numpy before the HLO graph runs)."""
    rng = _rng(seed + 7)
    word = (rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float32)
    pos = (rng.standard_normal((max_pos, hidden)) * 0.02).astype(np.float32)
    B, S = ids.shape
    return (word[ids] + pos[None, :S]).astype(np.float32)


def bert_block_fixture(seq: int = 16, hidden: int = 768, heads: int = 12) -> tuple[HloGraph, np.ndarray]:
    """run_tf_reference.py:86-107 with a tanh-form GELU; returns (graph, x)."""
    b = Builder("bert_block_fixture")
    x = b.input((1, seq, hidden))
    wq = np.full((hidden, hidden), 0.001, np.float32)
    wo = np.full((hidden, hidden), 0.001, np.float32)
    q = _linear(b, x, wq, None)
    ctx = _attention(b, q, q, q, heads, 0.125)
    y = _linear(b, ctx, wo, None)
    out = _gelu_tanh(b, b.binary("add", y, x))
    xv = np.linspace(-0.1, 0.1, num=seq * hidden, dtype=np.float32).reshape(1, seq, hidden)
    return b.graph(out), xv


def make_image_batch(batch: int, hw: int = 224, seed: int = 1234) -> np.ndarray:
    return _rng(seed).standard_normal((batch, hw, hw, 3)).astype(np.float32)
