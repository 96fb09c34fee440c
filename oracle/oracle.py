"""ctypes binding of liboracle.so — TEST INFRASTRUCTURE ONLY (the checker).

``run_kernel`` mirrors the reference dispatch boundary
(source/tflite_loader/src/vulkan.rs:27-44, ``KernelRun``): a kernel name, two
f32 inputs, an output length and i32 push constants.  The kernels are plain
C++ restatements of kernels/<name>/glsl/<name>.comp (see spx_oracle.cpp).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
_lib = None


def build() -> Path:
    """Compiles liboracle.so with the committed Makefile (g++ -fopenmp)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        l = ctypes.CDLL(str(LIB_PATH))
        fp = ctypes.POINTER(ctypes.c_float)
        l.oracle_run_kernel.argtypes = [ctypes.c_char_p, fp, ctypes.c_size_t, fp, ctypes.c_size_t,
                                        fp, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int32),
                                        ctypes.c_size_t]
        l.oracle_run_kernel.restype = ctypes.c_int
        l.oracle_num_threads.restype = ctypes.c_int
        l.oracle_set_threads.argtypes = [ctypes.c_int]
        l.oracle_set_threads.restype = None
        _lib = l
    return _lib


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def run_kernel(kernel: str, input0, input1, output_elements: int, push) -> np.ndarray:
    """Runs one reference kernel on the CPU and returns the output values."""
    a = np.ascontiguousarray(np.asarray(input0, dtype=np.float32).reshape(-1))
    b = np.ascontiguousarray(np.asarray(input1, dtype=np.float32).reshape(-1))
    if b.size == 0:
        b = np.zeros(1, np.float32)
    out = np.zeros(int(output_elements), np.float32)
    q = np.ascontiguousarray(np.asarray(push, dtype=np.int32).reshape(-1))
    qp = q.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)) if q.size else None
    rc = lib().oracle_run_kernel(kernel.encode(), _fptr(a), a.size, _fptr(b), b.size,
                                 _fptr(out) if out.size else None, out.size, qp, q.size)
    if rc == 2:
        raise KeyError(f"oracle has no kernel {kernel!r}")
    if rc != 0:
        raise ValueError(f"oracle rejected {kernel!r} push={list(q)}")
    return out


def use_all_host_cores() -> int:
    """Sets the OpenMP team to every core this process may run on (launchers
    such as torchrun export OMP_NUM_THREADS=1) and returns the count."""
    import os
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    lib().oracle_set_threads(int(n or 1))
    return num_threads()


def num_threads() -> int:
    return int(lib().oracle_num_threads())
