"""GPU test of spx_conv2d_nchw_noalloc, the conv2d entry point that allocates
nothing (for callers whose memory policy forbids a library from calling
cudaMalloc).  Its output must match the regular "conv2d" dispatch and the
CPU oracle's restatement of conv2d.comp on two calls in a row; the second
call uses different data, so stale staging from the first call would show.
A call after the first leaves the device's free memory unchanged.
Collected last on purpose."""
import ctypes

import numpy as np
import pytest

from spirv_inference_b200 import _lib, dispatch
from spirv_inference_b200.graph import Graph

pytestmark = pytest.mark.gpu


def _noalloc(g, x, w, push, nout):
    dx, dw, dy = g.tensor(x), g.tensor(w), g.alloc((nout,))
    q = np.asarray(push, np.int32)
    rc = _lib.lib().spx_conv2d_nchw_noalloc(
        ctypes.c_void_p(dx.ptr), ctypes.c_void_p(dw.ptr), ctypes.c_void_p(dy.ptr),
        q.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), q.size, ctypes.c_void_p(g.stream))
    _lib.check(rc)
    return dy.download()  # downloads on the same stream, after a sync


@pytest.mark.parametrize("n,ic,ih,iw,oc,k,s,pt,pl", [(2, 3, 15, 13, 8, 3, 2, 0, 0),
                                                   (1, 16, 14, 14, 24, 1, 1, 0, 0),
                                                   (2, 5, 9, 11, 7, 5, 1, 2, 2)])
def test_noalloc_matches_regular_dispatch_twice(gpu, oracle_built, n, ic, ih, iw, oc, k, s, pt,
                                                pl):
    oh, ow = (ih + 2 * pt - k) // s + 1, (iw + 2 * pl - k) // s + 1
    total = n * oc * oh * ow
    push = [n, ic, ih, iw, oc, oh, ow, k, k, s, s, 1, pt, pl, total]
    rng = np.random.default_rng(k + ic)
    with Graph(gpu) as g:
        for _ in range(2):
            x = rng.uniform(-1, 1, n * ic * ih * iw).astype(np.float32)
            w = rng.uniform(-1, 1, oc * ic * k * k + oc).astype(np.float32)
            want = dispatch.run_kernel(gpu, dispatch.KernelRun("conv2d", "conv2d.spv", x, w,
                                                               total, 0, push)).values
            got = _noalloc(g, x, w, push, total)
            np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
            ref = oracle_built.run_kernel("conv2d", x, w, total, push)
            np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)
        assert _lib.lib().spx_device_status() == 0


def test_noalloc_call_allocates_nothing(gpu):
    import torch
    n, ic, ih, iw, oc, k = 2, 16, 28, 28, 32, 3
    push = [n, ic, ih, iw, oc, ih, iw, k, k, 1, 1, 1, 1, 1, n * oc * ih * iw]
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, n * ic * ih * iw).astype(np.float32)
    w = rng.uniform(-1, 1, oc * ic * k * k + oc).astype(np.float32)
    with Graph(gpu) as g:
        first = _noalloc(g, x, w, push, push[-1])      # allocates the test's own buffers
        dx, dw, dy = g.tensor(x), g.tensor(w), g.alloc((push[-1],))
        q = np.asarray(push, np.int32)
        g.sync()
        free0 = torch.cuda.mem_get_info(gpu)[0]
        for _ in range(3):
            _lib.check(_lib.lib().spx_conv2d_nchw_noalloc(
                ctypes.c_void_p(dx.ptr), ctypes.c_void_p(dw.ptr), ctypes.c_void_p(dy.ptr),
                q.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), q.size,
                ctypes.c_void_p(g.stream)))
        g.sync()
        assert torch.cuda.mem_get_info(gpu)[0] == free0
        np.testing.assert_array_equal(dy.download(), first)


def test_noalloc_rejects_bad_pads(gpu):
    push = [1, 3, 8, 8, 4, 8, 8, 3, 3, 1, 1, 1, 3, 1, 256]   # pad_top 3 >= kernel 3
    q = np.asarray(push, np.int32)
    with Graph(gpu) as g:
        dummy = g.alloc((16,))
        rc = _lib.lib().spx_conv2d_nchw_noalloc(
            ctypes.c_void_p(dummy.ptr), ctypes.c_void_p(dummy.ptr), ctypes.c_void_p(dummy.ptr),
            q.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), q.size, ctypes.c_void_p(g.stream))
    assert rc == _lib.SPX_ERR_INVALID_ARGUMENT
    assert "pad_top" in _lib.last_error()


def test_noalloc_rejects_oversized(gpu):
    n, ic, ih, iw, oc = 8, 64, 64, 64, 64  # 2 Mi input + 2 Mi output floats > 4 Mi limit
    total = n * oc * ih * iw
    push = [n, ic, ih, iw, oc, ih, iw, 1, 1, 1, 1, 1, 0, 0, total]
    need = 2 * n * ic * ih * iw + oc * ic + oc
    assert need > 4 << 20  # rejected before anything is launched on the dummy buffers
    q = np.asarray(push, np.int32)
    with Graph(gpu) as g:
        dummy = g.alloc((16,))
        rc = _lib.lib().spx_conv2d_nchw_noalloc(
            ctypes.c_void_p(dummy.ptr), ctypes.c_void_p(dummy.ptr), ctypes.c_void_p(dummy.ptr),
            q.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), q.size, ctypes.c_void_p(g.stream))
    assert rc == _lib.SPX_ERR_INVALID_ARGUMENT
    assert "fixed scratch" in _lib.last_error()
