"""ctypes binding of libspx.so (declared in include/spx.h).

Loading fails loudly when the library has not been built: there is no
pure-Python or CPU fallback for any operator.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, c_char, c_char_p, c_double, c_float, c_int, c_int32
from ctypes import c_int64, c_size_t, c_uint32, c_void_p
from pathlib import Path

LIB_PATH = Path(os.environ.get("SPX_LIBRARY") or Path(__file__).resolve().parent / "libspx.so")

SPX_OK = 0
SPX_ERR_INVALID_ARGUMENT = 1
SPX_ERR_UNSUPPORTED = 2
SPX_ERR_CUDA = 3
SPX_ERR_OUT_OF_MEMORY = 4
SPX_ERR_NO_DEVICE = 5

ACT_NONE, ACT_RELU, ACT_RELU_N1_TO_1, ACT_RELU6, ACT_TANH = 0, 1, 2, 3, 4
ACT_GELU_ERF, ACT_GELU_TANH, ACT_SILU = 16, 17, 18
WEIGHT_OHWI, WEIGHT_HWIO = 0, 1
POOL_SUM, POOL_MAX, POOL_AVG = 0, 1, 2
UNARY = {"abs": 0, "exp": 1, "log": 2, "neg": 3, "sqrt": 4, "rsqrt": 5, "sigmoid": 6,
         "tanh": 7, "relu": 8, "relu6": 9, "leaky_relu": 10, "sin": 11, "copy": 12,
         "gelu_erf": 13, "silu": 14}
BINARY = {"add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4, "min": 5, "max": 6,
          "gt": 7, "ge": 8, "lt": 9, "le": 10, "eq": 11, "ne": 12}


class SpxError(RuntimeError):
    """A libspx call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"spx error {code}: {message}")
        self.code = code


class KernelOutputInfo(Structure):
    _fields_ = [("elapsed_ms", c_double), ("device_name", c_char * 256),
                ("vendor_id", c_uint32), ("device_id", c_uint32)]


class ConvParams(Structure):
    _fields_ = [(n, c_int32) for n in (
        "n", "ih", "iw", "ic", "oc", "oh", "ow", "kh", "kw", "stride_h", "stride_w",
        "pad_top", "pad_left", "dilation_h", "dilation_w", "weight_layout", "activation")]


class DwParams(Structure):
    _fields_ = [(n, c_int32) for n in (
        "n", "ih", "iw", "c", "oh", "ow", "kh", "kw", "stride_h", "stride_w", "pad_top",
        "pad_left", "dilation_h", "dilation_w", "activation")]


class GemmParams(Structure):
    _fields_ = ([(n, c_int32) for n in ("batch", "m", "n", "k", "batch_inner", "b_inner_div")]
                + [(n, c_int64) for n in ("a_bs", "a_ms", "a_ks", "b_bs", "b_ks", "b_ns",
                                          "c_bs", "c_ms", "a_bis", "b_bis", "c_bis")]
                + [("alpha", c_float), ("activation", c_int32)])


class ExpandDwParams(Structure):
    _fields_ = [(n, c_int32) for n in ("n", "ih", "iw", "cin", "ce", "oh", "ow", "stride",
                                       "pad_top", "pad_left", "act_expand", "act_dw")]


class DwProjParams(Structure):
    _fields_ = [(n, c_int32) for n in ("n", "ih", "iw", "c", "oh", "ow", "kernel", "stride",
                                       "pad_top", "pad_left", "act_dw", "cout", "act_proj")]


class KvParams(Structure):
    _fields_ = [(n, c_int32) for n in ("batch", "q_len", "q_heads", "kv_heads", "head_dim",
                                       "max_seq")]


class PoolParams(Structure):
    _fields_ = [(n, c_int32) for n in (
        "n", "ih", "iw", "c", "oh", "ow", "kh", "kw", "stride_h", "stride_w", "pad_top",
        "pad_left", "kind")]


class BcastParams(Structure):
    _fields_ = [("d", c_int32 * 4), ("a_stride", c_int64 * 4), ("b_stride", c_int64 * 4)]


class SelectParams(Structure):
    _fields_ = [("d", c_int32 * 4), ("p_stride", c_int64 * 4), ("a_stride", c_int64 * 4),
                ("b_stride", c_int64 * 4)]


_FP = POINTER(c_float)
_IP = POINTER(c_int32)
_lib = None

_SIGS = {
    "spx_last_error": ([], c_char_p),
    "spx_version": ([], c_char_p),
    "spx_device_count": ([], c_int),
    "spx_select_device": ([c_char_p, POINTER(c_int)], c_int),
    "spx_binary_version": ([c_int, POINTER(c_int)], c_int),
    "spx_device_status": ([], c_int),
    "spx_set_option": ([c_char_p, c_int64], c_int),
    "spx_get_option": ([c_char_p], c_int64),
    "spx_gemm_tc_plan": ([c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p,
                          c_int32], c_int),
    "spx_kernel_count": ([], c_int),
    "spx_kernel_name": ([c_int], c_char_p),
    "spx_kernel_push_count": ([c_char_p], c_int),
    "spx_kernel_local_size": ([c_char_p], c_int),
    "spx_run_kernel": ([c_char_p, _FP, c_size_t, _FP, c_size_t, _FP, c_size_t, _IP, c_size_t,
                        c_int, POINTER(KernelOutputInfo)], c_int),
    "spx_conv2d_nchw_noalloc": ([c_void_p, c_void_p, c_void_p, _IP, c_size_t, c_void_p], c_int),
    "spx_graph_create": ([c_int, POINTER(c_void_p)], c_int),
    "spx_graph_create_on_stream": ([c_int, c_void_p, POINTER(c_void_p)], c_int),
    "spx_graph_destroy": ([c_void_p], c_int),
    "spx_graph_stream": ([c_void_p], c_void_p),
    "spx_graph_device": ([c_void_p], c_int),
    "spx_graph_sync": ([c_void_p], c_int),
    "spx_graph_launch_count": ([c_void_p], c_int64),
    "spx_graph_reset_launch_count": ([c_void_p], None),
    "spx_graph_capture_begin": ([c_void_p], c_int),
    "spx_graph_capture_end": ([c_void_p], c_int),
    "spx_graph_replay": ([c_void_p], c_int),
    "spx_buf_alloc": ([c_void_p, c_size_t, POINTER(c_void_p)], c_int),
    "spx_buf_free": ([c_void_p, c_void_p], c_int),
    "spx_buf_upload": ([c_void_p, c_void_p, c_void_p, c_size_t], c_int),
    "spx_buf_download": ([c_void_p, c_void_p, c_void_p, c_size_t], c_int),
    "spx_buf_zero": ([c_void_p, c_void_p, c_size_t], c_int),
    "spx_buf_copy": ([c_void_p, c_void_p, c_void_p, c_size_t], c_int),
    "spx_host_alloc_pinned": ([c_size_t, POINTER(c_void_p)], c_int),
    "spx_host_free_pinned": ([c_void_p], c_int),
    "spx_op_conv2d_nhwc": ([c_void_p] + [c_void_p] * 5 + [POINTER(ConvParams)], c_int),
    "spx_weights_split": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int64], c_int),
    "spx_op_conv2d_nhwc_split": ([c_void_p] + [c_void_p] * 7 + [POINTER(ConvParams)], c_int),
    "spx_op_gemm_split": ([c_void_p] + [c_void_p] * 7 + [POINTER(GemmParams)], c_int),
    "spx_op_depthwise_conv2d_nhwc": ([c_void_p] + [c_void_p] * 4 + [POINTER(DwParams)], c_int),
    "spx_op_gemm": ([c_void_p] + [c_void_p] * 5 + [POINTER(GemmParams)], c_int),
    "spx_op_pool2d_nhwc": ([c_void_p, c_void_p, c_void_p, POINTER(PoolParams)], c_int),
    "spx_op_global_avg_pool_nhwc": ([c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32],
                                    c_int),
    "spx_op_softmax_rows": ([c_void_p, c_void_p, c_void_p, c_int32, c_int32], c_int),
    "spx_op_attention_softmax": ([c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float,
                                  c_int32, c_int32, c_int32], c_int),
    "spx_op_unary": ([c_void_p, c_int32, c_void_p, c_void_p, c_int64, c_float], c_int),
    "spx_op_binary": ([c_void_p, c_int32, c_void_p, c_void_p, c_void_p, POINTER(BcastParams)],
                      c_int),
    "spx_op_select": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, POINTER(SelectParams)],
                      c_int),
    "spx_op_reduce_rank4": ([c_void_p, c_void_p, c_void_p, _IP], c_int),
    "spx_op_layernorm": ([c_void_p] + [c_void_p] * 6 + [c_int32, c_int32, c_float], c_int),
    "spx_op_rmsnorm": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float],
                       c_int),
    "spx_op_rope": ([c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_float], c_int),
    "spx_op_embedding": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32], c_int),
    "spx_op_argmax_rows": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32], c_int),
    "spx_op_swiglu": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int64], c_int),
    "spx_op_rope_kv_append": ([c_void_p, c_void_p, c_int64] + [c_void_p] * 6
                              + [POINTER(KvParams)], c_int),
    "spx_op_attention_kv": ([c_void_p] + [c_void_p] * 5 + [POINTER(KvParams), c_float], c_int),
    "spx_op_swiglu_linear": ([c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32,
                              c_int32, c_float, c_void_p, c_int64], c_int),
    "spx_op_rms_linear": ([c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32,
                           c_int32, c_float, c_void_p, c_void_p, c_int64, c_void_p], c_int),
    "spx_op_swiglu_rows": ([c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32],
                           c_int),
    "spx_op_token_commit": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                             c_void_p], c_int),
    "spx_op_argmax_partial": ([c_void_p, c_void_p, c_int64, c_int32, c_int32, c_int32,
                               c_void_p], c_int),
    "spx_op_argmax_merge": ([c_void_p, c_void_p, c_int32, c_int32, c_void_p], c_int),
    "spx_ar_create": ([c_int32, c_int32, c_int32, ctypes.c_size_t, POINTER(c_void_p)], c_int),
    "spx_ar_handle_size": ([], ctypes.c_size_t),
    "spx_ar_handle": ([c_void_p, c_void_p, ctypes.c_size_t], c_int),
    "spx_ar_open": ([c_void_p, c_void_p], c_int),
    "spx_ar_slot": ([c_void_p, c_int32], c_void_p),
    "spx_op_allreduce": ([c_void_p, c_void_p, c_int32, c_void_p, c_int64], c_int),
    "spx_ar_reset": ([c_void_p], c_int),
    "spx_ar_destroy": ([c_void_p], c_int),
    "spx_op_dw_project_nhwc": ([c_void_p] + [c_void_p] * 8 + [POINTER(DwProjParams)], c_int),
    "spx_dw_project_supported": ([POINTER(DwProjParams)], c_int),
    "spx_op_stem_conv_nhwc": ([c_void_p] * 6 + [POINTER(ConvParams)], c_int),
    "spx_stem_conv_supported": ([POINTER(ConvParams)], c_int),
    "spx_op_expand_dw_nhwc": ([c_void_p] + [c_void_p] * 6 + [POINTER(ExpandDwParams)], c_int),
    "spx_op_expand_dw_nhwc_split": ([c_void_p] + [c_void_p] * 8 + [POINTER(ExpandDwParams)],
                                    c_int),
    "spx_op_pad4": ([c_void_p, c_void_p, c_void_p, c_float, _IP], c_int),
    "spx_op_transpose4": ([c_void_p, c_void_p, c_void_p, _IP], c_int),
}


def lib():
    """Loads libspx.so once; raises if it was never built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m spirv_inference_b200.build` "
                "(there is no CPU fallback)")
        l = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in _SIGS.items():
            fn = getattr(l, name)
            fn.argtypes = args
            fn.restype = res
        _lib = l
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def set_option(name: str, value: int) -> None:
    check(lib().spx_set_option(name.encode(), int(value)))


def get_option(name: str) -> int:
    return int(lib().spx_get_option(name.encode()))


def last_error() -> str:
    return (lib().spx_last_error() or b"").decode(errors="replace")


def check(rc: int) -> None:
    if rc != SPX_OK:
        raise SpxError(rc, last_error())


_PLAN_KEYS = ("BN", "n_tiles", "k_blocks", "last_ksteps", "stages", "stage_bytes", "epi_warps",
              "conv_groups", "groups", "nacc", "tmem_cols", "b_resident", "smem_bytes",
              "m_tiles", "conv_threads", "grid", "lo_tmem")


def gemm_tc_plan(m: int, n: int, k: int, presplit: bool = True, conv: bool = False,
                 vec4: bool = True) -> dict:
    """The tensor-core GEMM's launch plan for an m x n x k product (host only)."""
    out = (c_int32 * 17)()
    check(lib().spx_gemm_tc_plan(m, n, k, int(presplit), int(conv), int(vec4), out, 17))
    return dict(zip(_PLAN_KEYS, list(out)))
