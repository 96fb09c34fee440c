"""Drop-in dispatch boundary: the Python face of ``spx_run_kernel``.

Mirrors the reference's op interface so callers written against it port
line for line:

* ``KernelSpec`` / ``TFLITE_KERNELS`` / ``registry()`` follow
  source/tflite_loader/src/kernels.rs:4-242 (names, binding count, push
  constant names), extended with the HLO kernels that
  source/xla_hlo/src/compiler.rs:768-1135 dispatches.
* ``KernelRun`` / ``KernelOutput`` / ``groups`` / ``run_kernel`` follow
  source/tflite_loader/src/vulkan.rs:18-44.  ``KernelRun.spv`` names the
  kernel (registry name or ``.spv`` file name) instead of carrying SPIR-V
  bytes; the library holds the sm_100a kernel for every name.

Errors raise ``SpxError``: unknown kernels carry ``SPX_ERR_UNSUPPORTED``, the
case the reference reports as ``blocked_unsupported_feature``
(source/tflite_loader/src/main.rs:66-76).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import _lib


@dataclass(frozen=True)
class KernelSpec:
    name: str
    spv: str
    bindings: int
    push_constants: tuple[str, ...]


def _k(name, spv, *push):
    return KernelSpec(name, spv, 3, tuple(push))


_CONV_PUSH = ("n", "ic", "ih", "iw", "oc", "oh", "ow", "kh", "kw", "stride_h", "stride_w",
              "same", "pad_top", "pad_left", "total")
_DW_PUSH = ("n", "c", "ih", "iw", "oh", "ow", "kh", "kw", "stride_h", "stride_w", "same",
            "pad_top", "pad_left", "dilation_h", "dilation_w", "total")
_POOL_PUSH = ("n", "c", "ih", "iw", "oh", "ow", "kh", "kw", "stride_h", "stride_w", "same",
              "pad_top", "pad_left", "total")

# kernels.rs:12-238, in the same order.  ``transpose`` carries the 13 push
# constants its shader declares (kernels/transpose/glsl/transpose.comp); the
# reference registry lists 5 names for it that no call site uses.
TFLITE_KERNELS: tuple[KernelSpec, ...] = (
    _k("add", "add.spv", "total"), _k("sub", "sub.spv", "total"),
    _k("mul", "mul.spv", "total"), _k("div", "div.spv", "total"),
    _k("pow", "pow.spv", "total"), _k("min", "min.spv", "total"),
    _k("max", "max.spv", "total"), _k("exp", "exp.spv", "total"),
    _k("neg", "neg.spv", "total"), _k("abs", "abs.spv", "total"),
    _k("sqrt", "sqrt.spv", "total"), _k("rsqrt", "rsqrt.spv", "total"),
    _k("log", "log.spv", "total"), _k("leaky_relu", "leaky_relu.spv", "total", "alpha_bits"),
    _k("logistic", "sigmoid.spv", "total"), _k("sigmoid", "sigmoid.spv", "total"),
    _k("tanh", "tanh.spv", "total"), _k("relu6", "relu6.spv", "total"),
    _k("relu", "relu.spv", "total"), _k("reshape", "reshape.spv", "total"),
    _k("concat", "concat.spv", "a_total", "total"),
    _k("transpose", "transpose.spv", "in0", "in1", "in2", "in3", "out0", "out1", "out2", "out3",
       "p0", "p1", "p2", "p3", "total"),
    _k("conv2d", "conv2d.spv", *_CONV_PUSH),
    _k("depthwise_conv2d", "depthwise_conv2d.spv", *_DW_PUSH),
    _k("global_avg_pool_sum", "global_avg_pool_sum.spv", "n", "c", "h", "w"),
    _k("max_pool2d", "max_pool2d.spv", *_POOL_PUSH),
    _k("l2norm", "l2norm.spv", "total", "norm_bits"),
    _k("resize_bilinear", "resize_bilinear.spv", "n", "c", "ih", "iw", "oh", "ow",
       "align_corners", "half_pixel_centers", "total"),
    _k("global_avg_pool_finalize", "global_avg_pool_finalize.spv", "n", "c", "h", "w"),
    _k("fully_connected", "fully_connected.spv", "batches", "input_size", "output_size", "total"),
    _k("softmax10", "softmax10.spv"),
    _k("softmax1000", "softmax1000.spv", "classes"),
)

# HLO kernels (compiler.rs:768-1135 push layouts; kernel_mapping 1155-1228
# adds "sine" to the elementwise set).
HLO_KERNELS: tuple[KernelSpec, ...] = (
    _k("sine", "sine.spv", "total"),
    _k("hlo_conv_nhwc_hwio", "hlo_conv_nhwc_hwio.spv", "n", "ih", "iw", "ic", "kh", "kw", "oc",
       "oh", "ow", "stride_h", "stride_w", "pad_top", "pad_left", "total"),
    _k("hlo_dot_rank2", "hlo_dot_rank2.spv", "m", "k", "n", "total"),
    _k("hlo_dot_batched", "hlo_dot_batched.spv", "batch", "m", "k", "n", "total"),
    _k("hlo_reduce_rank4", "hlo_reduce_rank4.spv", "rank", "d0", "d1", "d2", "d3", "od0", "od1",
       "od2", "od3", "r0", "r1", "r2", "r3", "kind", "total"),
    _k("hlo_reduce_window_rank4", "hlo_reduce_window_rank4.spv", "n", "ih", "iw", "c", "oh",
       "ow", "wh", "ww", "stride_h", "stride_w", "pad_top", "pad_left", "kind", "total"),
    _k("pad", "pad.spv", "od0", "od1", "od2", "od3", "id0", "id1", "id2", "id3", "pl0", "pl1",
       "pl2", "pl3", "total"),
)


def registry() -> dict[str, KernelSpec]:
    """kernels.rs:240-242: name -> spec (TFLite set plus the HLO kernels)."""
    return {k.name: k for k in TFLITE_KERNELS + HLO_KERNELS}


def groups(elements: int, local_size: int) -> int:
    """vulkan.rs:38-40: ceil(elements / local_size)."""
    return -(-int(elements) // int(local_size))


@dataclass
class KernelRun:
    """vulkan.rs:27-36.  ``spv`` is the kernel name or its .spv file name."""
    label: str
    spv: str
    input0: np.ndarray
    input1: np.ndarray
    output_elements: int
    dispatch_x: int = 0
    push: list[int] = field(default_factory=list)


@dataclass
class KernelOutput:
    """vulkan.rs:18-25."""
    values: np.ndarray
    device_name: str
    vendor_id: int
    device_id: int
    elapsed_ms: float


def select_device(selector: str | int = "any") -> int:
    """vulkan.rs:204-231 selector ("any" | "nvidia" | "intel") or ordinal."""
    out = ctypes.c_int(-1)
    _lib.check(_lib.lib().spx_select_device(str(selector).encode(), ctypes.byref(out)))
    return out.value


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32).reshape(-1))


def run_kernel(device_selector: str | int, spec: KernelRun) -> KernelOutput:
    """vulkan.rs:42-44: one synchronous dispatch with host buffers."""
    # Integer ordinals go straight to the library, which validates the kernel
    # name and push constants before it looks for the device.
    dev = device_selector if isinstance(device_selector, int) else select_device(device_selector)
    a, b = _f32(spec.input0), _f32(spec.input1)
    out = np.empty(int(spec.output_elements), np.float32)
    q = np.ascontiguousarray(np.asarray(spec.push, dtype=np.int64).astype(np.int32))
    info = _lib.KernelOutputInfo()
    fp = ctypes.POINTER(ctypes.c_float)
    ptr = lambda x: x.ctypes.data_as(fp) if x.size else None
    rc = _lib.lib().spx_run_kernel(
        spec.spv.encode(), ptr(a), a.size, ptr(b), b.size, ptr(out), out.size,
        q.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)) if q.size else None, q.size, dev,
        ctypes.byref(info))
    _lib.check(rc)
    return KernelOutput(out, info.device_name.decode(errors="replace"), int(info.vendor_id),
                        int(info.device_id), float(info.elapsed_ms))


def f32_bits(x: float) -> int:
    """Float -> i32 bit pattern for push constants (kernels.rs:92-97 alpha_bits)."""
    return int(np.array([x], np.float32).view(np.int32)[0])
