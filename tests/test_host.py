"""CPU tests of the host side: the C-ABI library loads and exports every
declared symbol, the registry mirrors the reference's, argument errors are
reported without touching a device, and the TFLite-style graphs have the
reference's structure."""
import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from spirv_inference_b200 import _lib, dispatch, lowering, nets

ROOT = Path(__file__).resolve().parent.parent


def _declared_functions() -> list[str]:
    text = (ROOT / "include" / "spx.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(spx_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(spx_built):
    out = subprocess.run(["nm", "-D", "--defined-only", str(spx_built)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (spx_\w+)", out))
    declared = _declared_functions()
    assert declared, "no declarations parsed"
    missing = [d for d in declared if d not in exported]
    assert not missing, missing
    l = _lib.lib()
    for d in declared:
        assert hasattr(l, d)
    assert set(_lib.exported_symbols()) <= set(declared)


def test_build_targets_sm100a_only():
    """Every object is compiled with exactly one -gencode, for sm_100a (the
    loaded code's binary version is checked on the GPU)."""
    from spirv_inference_b200 import build
    gencodes = [build.CFLAGS[i + 1] for i, f in enumerate(build.CFLAGS) if f == "-gencode"]
    assert gencodes == ["arch=compute_100a,code=sm_100a"]
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_registry_matches_library(spx_built):
    l = _lib.lib()
    names = [l.spx_kernel_name(i).decode() for i in range(l.spx_kernel_count())]
    reg = dispatch.registry()
    assert sorted(names) == sorted(reg)
    for name, spec in reg.items():
        assert l.spx_kernel_push_count(name.encode()) == len(spec.push_constants), name
        assert l.spx_kernel_push_count(spec.spv.encode()) == len(spec.push_constants), name
    assert l.spx_kernel_push_count(b"nope") == -1
    # kernels.rs:12-238 order and push names for the TFLite set
    assert [k.name for k in dispatch.TFLITE_KERNELS][:5] == ["add", "sub", "mul", "div", "pow"]
    conv = reg["conv2d"]
    assert conv.push_constants[-1] == "total" and conv.push_constants[11] == "same"


def test_groups():
    assert dispatch.groups(65, 64) == 2 and dispatch.groups(64, 64) == 1


def test_unknown_kernel_is_unsupported(spx_built):
    with pytest.raises(_lib.SpxError) as e:
        dispatch.run_kernel(0, dispatch.KernelRun("x", "warp_drive.spv", np.ones(1), np.ones(1), 1,
                                                  1, [1]))
    assert e.value.code == _lib.SPX_ERR_UNSUPPORTED
    assert "warp_drive" in str(e.value)


def test_bad_push_count_is_invalid(spx_built):
    with pytest.raises(_lib.SpxError) as e:
        dispatch.run_kernel(0, dispatch.KernelRun("x", "conv2d.spv", np.ones(1), np.ones(1), 1, 1,
                                                  [1, 2, 3]))
    assert e.value.code == _lib.SPX_ERR_INVALID_ARGUMENT


def test_no_device_behaviour(spx_built):
    l = _lib.lib()
    if l.spx_device_count() > 0:
        pytest.skip("a CUDA device is present")
    with pytest.raises(_lib.SpxError) as e:
        dispatch.run_kernel("any", dispatch.KernelRun("x", "relu", np.ones(4), np.ones(1), 4, 1, [4]))
    assert e.value.code == _lib.SPX_ERR_NO_DEVICE
    h = ctypes.c_void_p()
    assert l.spx_graph_create(0, ctypes.byref(h)) == _lib.SPX_ERR_NO_DEVICE
    assert l.spx_op_unary(None, 0, None, None, 0, 0.0) == _lib.SPX_ERR_INVALID_ARGUMENT
    o = ctypes.c_int()
    assert l.spx_select_device(b"intel", ctypes.byref(o)) == _lib.SPX_ERR_NO_DEVICE


def test_models_structure():
    m = nets.mobilenet_v2(seed=0)
    # source/tflite_loader/TFLITE_REPORT.md:16 histogram
    assert m.op_counts() == {"CONV_2D": 36, "DEPTHWISE_CONV_2D": 17, "ADD": 10,
                             "AVERAGE_POOL_2D": 1, "RESHAPE": 1, "SOFTMAX": 1}
    assert abs(m.flops_per_image() / 1e9 - 0.6015) < 1e-3
    assert m.shapes[m.output] == (1001,)
    e = nets.efficientnet_lite0(seed=0)
    assert e.op_counts()["DEPTHWISE_CONV_2D"] == 16
    assert e.shapes[e.output] == (1000,)
    # seeded: identical weights on rebuild
    m2 = nets.mobilenet_v2(seed=0)
    for k in m.weights:
        assert np.array_equal(m.weights[k], m2.weights[k])


def test_packing_and_padding():
    w = np.arange(2 * 3 * 3 * 4, dtype=np.float32).reshape(2, 3, 3, 4)
    b = np.array([100, 200], np.float32)
    p = lowering.pack_conv_weight(w, b)
    assert p.size == w.size + 2 and p[-1] == 200
    oihw = p[:-2].reshape(2, 4, 3, 3)
    assert oihw[1, 2, 0, 1] == w[1, 0, 1, 2]
    d = lowering.pack_depthwise_weight(np.arange(9 * 5, dtype=np.float32).reshape(1, 3, 3, 5),
                                       np.zeros(5, np.float32))
    assert d[:-5].reshape(5, 3, 3)[4, 1, 2] == (1 * 3 + 2) * 5 + 4
    # SAME with stride 2 on an even size pads 0 on top, 1 on the bottom
    assert lowering.same_padding_offsets("SAME", 224, 224, 112, 112, 3, 3, 2, 2) == (0, 0)
    assert lowering.same_padding_offsets("SAME", 7, 7, 7, 7, 5, 5, 1, 1) == (2, 2)
    assert lowering.same_padding_offsets("VALID", 7, 7, 5, 5, 3, 3, 1, 1) == (0, 0)


def test_lowering_dispatch_sequence_with_oracle(oracle_built):
    m = nets.mobilenet_v2(seed=3)
    x = nets.make_input(m, 1)
    out, rep = lowering.run_graph(m, x, oracle_built.run_kernel)
    c = {}
    for d in rep["dispatches"]:
        c[d] = c.get(d, 0) + 1
    # 36 conv (+ 35 relu6 post-ops: all but the 17 linear projections and the
    # classifier), 17 depthwise (+17 relu6), 10 adds, 2 pool passes, reshape, softmax
    assert c["conv2d.spv"] == 36 and c["depthwise_conv2d.spv"] == 17
    assert c["relu6.spv"] == 36 - 17 - 1 + 17
    assert c["add.spv"] == 10 and c["softmax1000.spv"] == 1
    assert out.shape == (1, 1001) and abs(float(out.sum()) - 1.0) < 1e-5


def test_process_options(spx_built):
    """Path options are host-side state: defaults, round trip, range errors."""
    defaults = {"gemm_path": 0, "dw_path": 0, "pw_path": 0, "tc_wide_epilogue": 1,
                "tc_conv_groups": 2, "tc_lo_tmem": 0, "pw_gemm": 0, "dwp_groups": 47, "dwp_stages": 4, "dwp_accs": 4, "dwp_epi1": 62, "tc_cat": 1, "tc_acc4": 1, "pdl": 1}
    for name, v in defaults.items():
        assert _lib.get_option(name) == v, name
    assert _lib.get_option("no_such_option") == -1
    for name, v, bad in (("pw_path", 1, 2), ("tc_wide_epilogue", 0, 2), ("tc_conv_groups", 1, 3),
                         ("tc_lo_tmem", 1, 2), ("pw_gemm", 1, 2), ("dwp_groups", 2, 64), ("dwp_stages", 2, 5), ("dwp_accs", 2, 3), ("dwp_epi1", 0, 64), ("tc_cat", 0, 2), ("tc_acc4", 0, 2), ("pdl", 0, 2),
                         ("dw_path", 1, 2), ("gemm_path", 2, 3)):
        try:
            _lib.set_option(name, v)
            assert _lib.get_option(name) == v
            with pytest.raises(_lib.SpxError) as e:
                _lib.set_option(name, bad)
            assert e.value.code == _lib.SPX_ERR_INVALID_ARGUMENT
            assert _lib.get_option(name) == v
        finally:
            _lib.set_option(name, defaults[name])
    with pytest.raises(_lib.SpxError):
        _lib.set_option("no_such_option", 0)


def test_plain_c_host_against_header_and_library(spx_built, tmp_path):
    """include/spx.h compiles as C99 and a C program linked against libspx.so
    (the view of a cgo / FFI binding) passes its host-side checks."""
    here = Path(__file__).resolve().parent
    lib = Path(spx_built)
    exe = tmp_path / "host_check"
    cc = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(here.parent / "include"),
                         str(here / "c_host" / "host_check.c"), "-L", str(lib.parent), "-lspx",
                         f"-Wl,-rpath,{lib.parent}", "-o", str(exe)],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr


def test_ctypes_signatures_match_header():
    """Every ctypes binding declares as many arguments as include/spx.h."""
    text = (ROOT / "include" / "spx.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = dict(re.findall(r"\b(spx_[a-z0-9_]+)\s*\(([^()]*)\)\s*;", text))
    assert decls
    for name, (args, _) in _lib._SIGS.items():
        assert name in decls, name
        params = decls[name].strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert n == len(args), (name, n, len(args))


def test_dw_project_eligibility_on_host(spx_built):
    """Shape eligibility of the fused depthwise -> projection kernel is decided
    on the host (no device needed)."""
    l = _lib.lib()
    ok = _lib.DwProjParams(2, 56, 56, 144, 56, 56, 3, 1, 1, 1, 3, 24, 0)
    assert l.spx_dw_project_supported(ctypes.byref(ok)) == 1
    for field, bad in (("kernel", 5), ("c", 30), ("cout", 600), ("stride", 3)):
        q = _lib.DwProjParams(2, 56, 56, 144, 56, 56, 3, 1, 1, 1, 3, 24, 0)
        setattr(q, field, bad)
        assert l.spx_dw_project_supported(ctypes.byref(q)) == 0, field
    assert l.spx_op_dw_project_nhwc(None, *([None] * 8), ctypes.byref(ok)) == \
        _lib.SPX_ERR_INVALID_ARGUMENT


# (map, channels, stride, outputs) of every fused block of MobileNetV2 and the
# 3x3 ones of EfficientNet-Lite0
_DWP_LAYERS = [(112, 32, 1, 16), (112, 96, 2, 24), (56, 144, 1, 24), (56, 144, 2, 32),
               (28, 192, 1, 32), (28, 192, 2, 64), (14, 384, 1, 64), (14, 384, 1, 96),
               (14, 576, 1, 96), (14, 576, 2, 160), (7, 960, 1, 160), (7, 960, 1, 320),
               (28, 240, 2, 80), (14, 480, 1, 80)]


def test_dw_project_shared_memory_fits_every_option(spx_built):
    """Every tile class fits shared memory (at least two A/B stages and two
    halo slots) for every value of the kernel's options, so no option setting
    turns a supported layer into an unsupported one."""
    l = _lib.lib()
    names = ("dwp_groups", "dwp_stages", "dwp_accs", "dwp_epi1")
    defaults = [_lib.get_option(k) for k in names]
    try:
        for setting in [(g, st, a, e) for g in (0, 63) for st in (2, 3, 4) for a in (2, 4)
                        for e in (0, 63)]:
            for k, v in zip(names, setting):
                _lib.set_option(k, v)
            for h, c, s, cout in _DWP_LAYERS:
                oh = -(-h // s)
                pt = max((oh - 1) * s + 3 - h, 0) // 2
                q = _lib.DwProjParams(256, h, h, c, oh, oh, 3, s, pt, pt, 3, cout, 0)
                assert l.spx_dw_project_supported(ctypes.byref(q)) == 1, (setting, h, c, s, cout)
    finally:
        for k, v in zip(names, defaults):
            _lib.set_option(k, v)
