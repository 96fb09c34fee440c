"""Device-resident graph API (``spx_graph_*`` / ``spx_buf_*`` / ``spx_op_*``).

Generalises runtime/chained_graph_runtime/src/main.rs:298-547 — pipelines and
buffers created once, dispatches recorded back to back on one queue — to a
per-graph CUDA stream with device buffers that live for the graph's
lifetime, optional CUDA-graph capture and replay, and NHWC activations.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import check


@dataclass
class DeviceTensor:
    """A device buffer owned by a Graph: pointer, shape, float32/int32."""
    ptr: int
    shape: tuple[int, ...]
    dtype: np.dtype
    graph: "Graph"

    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    @property
    def nbytes(self) -> int:
        return self.size * np.dtype(self.dtype).itemsize

    def upload(self, host: np.ndarray) -> "DeviceTensor":
        self.graph.upload(self, host)
        return self

    def download(self) -> np.ndarray:
        return self.graph.download(self)

    def view(self, shape, offset_elems: int = 0) -> "DeviceTensor":
        """A reshaped (and optionally offset) alias of this buffer."""
        return DeviceTensor(self.ptr + offset_elems * np.dtype(self.dtype).itemsize,
                            tuple(shape), self.dtype, self.graph)


class Graph:
    """One device, one stream, owned device buffers, recorded ops."""

    def __init__(self, device: int = 0, stream: int | None = None):
        self._l = _lib.lib()
        h = ctypes.c_void_p()
        if stream:
            check(self._l.spx_graph_create_on_stream(device, ctypes.c_void_p(stream),
                                                     ctypes.byref(h)))
        else:
            check(self._l.spx_graph_create(device, ctypes.byref(h)))
        self.h = h
        self.device = device

    # -- lifetime ----------------------------------------------------------
    def close(self) -> None:
        if self.h:
            self._l.spx_graph_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return int(self._l.spx_graph_stream(self.h) or 0)

    def sync(self) -> None:
        check(self._l.spx_graph_sync(self.h))

    @property
    def launch_count(self) -> int:
        return int(self._l.spx_graph_launch_count(self.h))

    def reset_launch_count(self) -> None:
        self._l.spx_graph_reset_launch_count(self.h)

    def capture_begin(self) -> None:
        check(self._l.spx_graph_capture_begin(self.h))

    def capture_end(self) -> None:
        check(self._l.spx_graph_capture_end(self.h))

    def replay(self) -> None:
        check(self._l.spx_graph_replay(self.h))

    # -- buffers -----------------------------------------------------------
    def alloc(self, shape, dtype=np.float32) -> DeviceTensor:
        shape = tuple(int(s) for s in shape)
        nbytes = int(np.prod(shape)) * np.dtype(dtype).itemsize if shape else 4
        p = ctypes.c_void_p()
        check(self._l.spx_buf_alloc(self.h, max(nbytes, 16), ctypes.byref(p)))
        return DeviceTensor(int(p.value), shape, np.dtype(dtype), self)

    def tensor(self, host: np.ndarray, dtype=np.float32) -> DeviceTensor:
        host = np.ascontiguousarray(host, dtype=dtype)
        t = self.alloc(host.shape, dtype)
        self.upload(t, host)
        return t

    def upload(self, t: DeviceTensor, host: np.ndarray) -> None:
        host = np.ascontiguousarray(host, dtype=t.dtype)
        assert host.size == t.size, (host.shape, t.shape)
        check(self._l.spx_buf_upload(self.h, ctypes.c_void_p(t.ptr),
                                     host.ctypes.data_as(ctypes.c_void_p), host.nbytes))
        self.sync()  # pageable source: keep the host array alive until copied

    def upload_async(self, t: DeviceTensor, host_ptr: int, nbytes: int) -> None:
        check(self._l.spx_buf_upload(self.h, ctypes.c_void_p(t.ptr), ctypes.c_void_p(host_ptr),
                                     nbytes))

    def download(self, t: DeviceTensor) -> np.ndarray:
        out = np.empty(t.shape, t.dtype)
        check(self._l.spx_buf_download(self.h, out.ctypes.data_as(ctypes.c_void_p),
                                       ctypes.c_void_p(t.ptr), out.nbytes))
        self.sync()
        return out

    def download_async(self, host_ptr: int, t: DeviceTensor, nbytes: int) -> None:
        check(self._l.spx_buf_download(self.h, ctypes.c_void_p(host_ptr), ctypes.c_void_p(t.ptr),
                                       nbytes))

    def copy_d2d(self, dst: DeviceTensor, src_ptr: int, nbytes: int) -> None:
        check(self._l.spx_buf_copy(self.h, ctypes.c_void_p(dst.ptr), ctypes.c_void_p(src_ptr),
                                   nbytes))

    def zero(self, t: DeviceTensor) -> None:
        check(self._l.spx_buf_zero(self.h, ctypes.c_void_p(t.ptr), t.nbytes))

    # -- ops ---------------------------------------------------------------
    @staticmethod
    def _p(t):
        return ctypes.c_void_p(t.ptr) if t is not None else None

    def weights_split(self, w) -> tuple:
        """Pre-splits weights for the tensor-core path: returns (hi, lo)."""
        hi, lo = self.alloc(w.shape), self.alloc(w.shape)
        check(self._l.spx_weights_split(self.h, self._p(w), self._p(hi), self._p(lo), w.size))
        return hi, lo

    def conv2d_nhwc(self, x, w, bias, y, *, stride=(1, 1), pad=(0, 0), dilation=(1, 1),
                    weight_layout=_lib.WEIGHT_OHWI, activation=_lib.ACT_NONE, residual=None,
                    w_split=None):
        n, ih, iw, ic = x.shape
        _, oh, ow, oc = y.shape
        if weight_layout == _lib.WEIGHT_OHWI:
            kh, kw = w.shape[1], w.shape[2]
        else:
            kh, kw = w.shape[0], w.shape[1]
        p = _lib.ConvParams(n, ih, iw, ic, oc, oh, ow, kh, kw, stride[0], stride[1], pad[0],
                            pad[1], dilation[0], dilation[1], weight_layout, activation)
        if w_split is not None:
            check(self._l.spx_op_conv2d_nhwc_split(
                self.h, self._p(x), self._p(w), self._p(w_split[0]), self._p(w_split[1]),
                self._p(bias), self._p(residual), self._p(y), ctypes.byref(p)))
        else:
            check(self._l.spx_op_conv2d_nhwc(self.h, self._p(x), self._p(w), self._p(bias),
                                             self._p(residual), self._p(y), ctypes.byref(p)))

    def depthwise_nhwc(self, x, w, bias, y, *, stride=(1, 1), pad=(0, 0), dilation=(1, 1),
                       activation=_lib.ACT_NONE):
        n, ih, iw, c = x.shape
        _, oh, ow, _ = y.shape
        kh, kw = w.shape[0], w.shape[1]
        p = _lib.DwParams(n, ih, iw, c, oh, ow, kh, kw, stride[0], stride[1], pad[0], pad[1],
                          dilation[0], dilation[1], activation)
        check(self._l.spx_op_depthwise_conv2d_nhwc(self.h, self._p(x), self._p(w), self._p(bias),
                                                   self._p(y), ctypes.byref(p)))

    def gemm(self, a, b, c, *, m, n, k, batch=1, a_strides, b_strides, c_strides, bias=None,
             residual=None, alpha=1.0, activation=_lib.ACT_NONE, batch_inner=1, b_inner_div=1,
             inner_strides=(0, 0, 0), b_split=None):
        """C[b][m][n] = act(alpha * A.B + bias + R).  *_strides = (batch, row/k, k/col)."""
        p = _lib.GemmParams(batch, m, n, k, batch_inner, b_inner_div, a_strides[0], a_strides[1],
                            a_strides[2], b_strides[0], b_strides[1], b_strides[2], c_strides[0],
                            c_strides[1], inner_strides[0], inner_strides[1], inner_strides[2],
                            alpha, activation)
        if b_split is not None:
            check(self._l.spx_op_gemm_split(self.h, self._p(a), self._p(b), self._p(b_split[0]),
                                            self._p(b_split[1]), self._p(bias),
                                            self._p(residual), self._p(c), ctypes.byref(p)))
        else:
            check(self._l.spx_op_gemm(self.h, self._p(a), self._p(b), self._p(bias),
                                      self._p(residual), self._p(c), ctypes.byref(p)))

    def linear(self, x, w_t, y, bias=None, activation=_lib.ACT_NONE, residual=None):
        """y[m][n] = x[m][k] @ w_t[k][n] (+bias, +residual), row-major 2-D views."""
        m, k = x.shape[0], x.shape[-1]
        n = w_t.shape[-1]
        self.gemm(x, w_t, y, m=m, n=n, k=k, a_strides=(0, k, 1), b_strides=(0, n, 1),
                  c_strides=(0, n), bias=bias, residual=residual, activation=activation)

    def pool2d_nhwc(self, x, y, *, kernel, stride, pad=(0, 0), kind=_lib.POOL_MAX):
        n, ih, iw, c = x.shape
        _, oh, ow, _ = y.shape
        p = _lib.PoolParams(n, ih, iw, c, oh, ow, kernel[0], kernel[1], stride[0], stride[1],
                            pad[0], pad[1], kind)
        check(self._l.spx_op_pool2d_nhwc(self.h, self._p(x), self._p(y), ctypes.byref(p)))

    def global_avg_pool_nhwc(self, x, y):
        n, h, w, c = x.shape
        check(self._l.spx_op_global_avg_pool_nhwc(self.h, self._p(x), self._p(y), n, h * w, c))

    def softmax_rows(self, x, y, rows, cols):
        check(self._l.spx_op_softmax_rows(self.h, self._p(x), self._p(y), rows, cols))

    def attention_softmax(self, x, y, rows, cols, scale, causal=False, q_len=0, q_offset=0):
        check(self._l.spx_op_attention_softmax(self.h, self._p(x), self._p(y), rows, cols,
                                               scale, int(causal), q_len, q_offset))

    def unary(self, op: str, x, y, n=None, alpha=0.0):
        n = x.size if n is None else n
        check(self._l.spx_op_unary(self.h, _lib.UNARY[op], self._p(x), self._p(y), n, alpha))

    def binary(self, op: str, a, b, y, dims, a_strides, b_strides):
        p = _lib.BcastParams((ctypes.c_int32 * 4)(*dims), (ctypes.c_int64 * 4)(*a_strides),
                             (ctypes.c_int64 * 4)(*b_strides))
        check(self._l.spx_op_binary(self.h, _lib.BINARY[op], self._p(a), self._p(b), self._p(y),
                                    ctypes.byref(p)))

    def select(self, pred, a, b, y, dims, p_strides, a_strides, b_strides):
        p = _lib.SelectParams((ctypes.c_int32 * 4)(*dims), (ctypes.c_int64 * 4)(*p_strides),
                              (ctypes.c_int64 * 4)(*a_strides), (ctypes.c_int64 * 4)(*b_strides))
        check(self._l.spx_op_select(self.h, self._p(pred), self._p(a), self._p(b), self._p(y),
                                    ctypes.byref(p)))

    def add(self, a, b, y):
        n = y.size
        self.binary("add", a, b, y, (1, 1, 1, n), (0, 0, 0, 1), (0, 0, 0, 1))

    def reduce_rank4(self, x, y, push):
        q = (ctypes.c_int32 * 15)(*push)
        check(self._l.spx_op_reduce_rank4(self.h, self._p(x), self._p(y), q))

    def layernorm(self, x, gamma, beta, y, rows, cols, eps, residual=None, x_out=None):
        check(self._l.spx_op_layernorm(self.h, self._p(x), self._p(residual), self._p(x_out),
                                       self._p(gamma), self._p(beta), self._p(y), rows, cols,
                                       eps))

    def rmsnorm(self, x, gamma, y, rows, cols, eps):
        check(self._l.spx_op_rmsnorm(self.h, self._p(x), self._p(gamma), self._p(y), rows, cols,
                                     eps))

    def rope(self, x, positions, tokens, heads, head_dim, theta):
        check(self._l.spx_op_rope(self.h, self._p(x), self._p(positions), tokens, heads,
                                  head_dim, theta))

    def embedding(self, table, ids, y, tokens, dim):
        check(self._l.spx_op_embedding(self.h, self._p(table), self._p(ids), self._p(y), tokens,
                                       dim))

    def argmax_rows(self, x, idx, rows, cols, val=None):
        check(self._l.spx_op_argmax_rows(self.h, self._p(x), self._p(idx), self._p(val), rows,
                                         cols))

    def swiglu(self, gate, up, y, n):
        check(self._l.spx_op_swiglu(self.h, self._p(gate), self._p(up), self._p(y), n))

    def expand_dw_nhwc(self, x, w_expand, b_expand, w_dw, b_dw, y, *, stride, pad,
                       act_expand=_lib.ACT_RELU6, act_dw=_lib.ACT_RELU6, w_split=None):
        """Fused 1x1 expand conv + 3x3 depthwise (x NHWC [n][ih][iw][cin],
        w_expand OHWI [ce][1][1][cin], w_dw [3][3][ce] (or [1][3][3][ce]))."""
        n, ih, iw, cin = x.shape
        _, oh, ow, ce = y.shape
        p = _lib.ExpandDwParams(n, ih, iw, cin, ce, oh, ow, stride, pad[0], pad[1], act_expand,
                                act_dw)
        if w_split is not None:
            check(self._l.spx_op_expand_dw_nhwc_split(
                self.h, self._p(x), self._p(w_expand), self._p(w_split[0]), self._p(w_split[1]),
                self._p(b_expand), self._p(w_dw), self._p(b_dw), self._p(y), ctypes.byref(p)))
            return
        check(self._l.spx_op_expand_dw_nhwc(self.h, self._p(x), self._p(w_expand),
                                            self._p(b_expand), self._p(w_dw), self._p(b_dw),
                                            self._p(y), ctypes.byref(p)))

    @staticmethod
    def _stem_params(x, y, stride, pad, activation, kernel=3):
        n, ih, iw, ic = x.shape
        _, oh, ow, oc = y.shape
        return _lib.ConvParams(n, ih, iw, ic, oc, oh, ow, kernel, kernel, stride[0], stride[1],
                               pad[0], pad[1], 1, 1, _lib.WEIGHT_OHWI, activation)

    def stem_supported(self, x, y, *, stride=(2, 2), pad=(0, 0),
                       activation=_lib.ACT_NONE, kernel=3) -> bool:
        p = self._stem_params(x, y, stride, pad, activation, kernel)
        return bool(self._l.spx_stem_conv_supported(ctypes.byref(p)))

    def stem_weights(self, w_ohwi: np.ndarray) -> tuple:
        """[oc][k][k][3] OHWI weights (k = 3 or 7) -> tensor-core (hi, lo) of
        the [oc][kpad] copy (k*k*3 taps, zero-padded to a multiple of 32) for
        stem_conv_nhwc."""
        w = np.asarray(w_ohwi, np.float32)
        oc, taps = w.shape[0], int(np.prod(w.shape[1:]))
        pad = np.zeros((oc, -(-taps // 32) * 32), np.float32)
        pad[:, :taps] = w.reshape(oc, taps)
        return self.weights_split(self.tensor(pad))

    def stem_conv_nhwc(self, x, w_split, bias, y, *, stride=(2, 2), pad=(0, 0),
                       activation=_lib.ACT_NONE, kernel=3):
        p = self._stem_params(x, y, stride, pad, activation, kernel)
        check(self._l.spx_op_stem_conv_nhwc(self.h, self._p(x), self._p(w_split[0]),
                                            self._p(w_split[1]), self._p(bias), self._p(y),
                                            ctypes.byref(p)))

    @staticmethod
    def _dwproj_params(x, y, *, stride, pad, act_dw, act_proj, kernel=3):
        n, ih, iw, c = x.shape
        _, oh, ow, cout = y.shape
        return _lib.DwProjParams(n, ih, iw, c, oh, ow, kernel, stride, pad[0], pad[1], act_dw,
                                 cout, act_proj)

    def dw_project_supported(self, x, y, *, stride, pad, act_dw=_lib.ACT_RELU6,
                             act_proj=_lib.ACT_NONE, kernel=3) -> bool:
        p = self._dwproj_params(x, y, stride=stride, pad=pad, act_dw=act_dw, act_proj=act_proj,
                                kernel=kernel)
        return bool(self._l.spx_dw_project_supported(ctypes.byref(p)))

    def dw_project_nhwc(self, x, w_dw, b_dw, w_split, b_proj, y, *, stride, pad,
                        act_dw=_lib.ACT_RELU6, act_proj=_lib.ACT_NONE, residual=None):
        """Fused 3x3 depthwise + 1x1 projection (+ residual): x NHWC
        [n][ih][iw][c], w_dw [3][3][c], w_split = pre-split projection weights
        (hi, lo) [cout][c], y NHWC [n][oh][ow][cout]."""
        p = self._dwproj_params(x, y, stride=stride, pad=pad, act_dw=act_dw, act_proj=act_proj)
        check(self._l.spx_op_dw_project_nhwc(
            self.h, self._p(x), self._p(w_dw), self._p(b_dw), self._p(w_split[0]),
            self._p(w_split[1]), self._p(b_proj), self._p(residual), self._p(y), ctypes.byref(p)))

    # -- decode path -------------------------------------------------------
    def rope_kv_append(self, qkv, ld_qkv, cos_t, sin_t, state, q_out, k_cache, v_cache, *,
                       batch, q_len, q_heads, kv_heads, head_dim, max_seq):
        p = _lib.KvParams(batch, q_len, q_heads, kv_heads, head_dim, max_seq)
        check(self._l.spx_op_rope_kv_append(self.h, self._p(qkv), ld_qkv, self._p(cos_t),
                                            self._p(sin_t), self._p(state), self._p(q_out),
                                            self._p(k_cache), self._p(v_cache), ctypes.byref(p)))

    def attention_kv(self, q, k_cache, v_cache, out, state, *, batch, q_len, q_heads, kv_heads,
                     head_dim, max_seq, scale):
        p = _lib.KvParams(batch, q_len, q_heads, kv_heads, head_dim, max_seq)
        check(self._l.spx_op_attention_kv(self.h, self._p(q), self._p(k_cache), self._p(v_cache),
                                          self._p(out), self._p(state), ctypes.byref(p), scale))

    def swiglu_linear(self, a, lda, w, ldw, m, f, k, c, ldc, rms_eps=-1.0):
        check(self._l.spx_op_swiglu_linear(self.h, self._p(a), lda, self._p(w), ldw, m, f, k,
                                           rms_eps, self._p(c), ldc))

    def rms_linear(self, x, ldx, w, ldw, m, n, k, c, ldc, *, rms_eps=-1.0, residual=None,
                   argmax_keys=None):
        check(self._l.spx_op_rms_linear(self.h, self._p(x), ldx, self._p(w), ldw, m, n, k,
                                        rms_eps, self._p(residual), self._p(c), ldc,
                                        self._p(argmax_keys)))

    def swiglu_rows(self, gu, ld, y, ldy, rows, f):
        check(self._l.spx_op_swiglu_rows(self.h, self._p(gu), ld, self._p(y), ldy, rows, f))

    def token_commit(self, ids, hist, state, batch, advance, hist_cap, argmax_keys=None):
        check(self._l.spx_op_token_commit(self.h, self._p(ids), self._p(hist), self._p(state),
                                          batch, advance, hist_cap, self._p(argmax_keys)))

    def argmax_partial(self, x, ldx, rows, cols, col_offset, packed):
        check(self._l.spx_op_argmax_partial(self.h, self._p(x), ldx, rows, cols, col_offset,
                                            self._p(packed)))

    def argmax_merge(self, packed, parts, rows, ids):
        check(self._l.spx_op_argmax_merge(self.h, self._p(packed), parts, rows, self._p(ids)))

    def pad4(self, x, y, pad_value, push):
        q = (ctypes.c_int32 * 13)(*push)
        check(self._l.spx_op_pad4(self.h, self._p(x), self._p(y), pad_value, q))

    def transpose4(self, x, y, push):
        q = (ctypes.c_int32 * 13)(*push)
        check(self._l.spx_op_transpose4(self.h, self._p(x), self._p(y), q))


def device_count() -> int:
    return int(_lib.lib().spx_device_count())
