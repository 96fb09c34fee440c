"""GPU tests of the fused depthwise 3x3 -> 1x1 projection (+ residual)
kernel, spx_op_dw_project_nhwc: against a float64 formulation of the two
reference shaders (depthwise_conv2d.comp then conv2d.comp, plus add.comp),
over every tile configuration (stride 1 / 2, maps wider and narrower than
8 columns), projection widths from 16 to 320 (two n tiles), ragged map
edges, channel counts that are not multiples of 32, and with and without
the residual.  Tolerance: the 3xTF32 bound the tensor-core GEMM tests use,
normwise (2.5e-8 K + 1e-6) relative to the output scale."""
import numpy as np
import pytest

import _np_ref as R
from spirv_inference_b200 import _lib, lowering, nets
from spirv_inference_b200.executor import CnnExecutor
from spirv_inference_b200.graph import Graph

pytestmark = pytest.mark.gpu
RNG = np.random.default_rng(23)


def _r(*shape, scale=1.0):
    return (RNG.uniform(-1, 1, size=shape) * scale).astype(np.float32)


@pytest.fixture
def g(gpu):
    with Graph(gpu) as graph:
        yield graph


CASES = [
    # n, ih, c, s, cout, residual
    (2, 16, 32, 1, 16, False),
    (2, 19, 96, 2, 24, False),     # ragged 10x10 output, s2 (16-channel halo sub-blocks)
    (1, 56, 144, 1, 24, True),     # MobileNetV2 block 3 shape, K = 144 (4.5 K blocks)
    (1, 56, 144, 2, 32, False),
    (2, 28, 192, 1, 32, True),
    (2, 14, 384, 1, 64, True),
    (2, 14, 384, 1, 96, False),    # np = 96: second accumulator at TMEM column 96
    (3, 14, 576, 1, 96, True),
    (3, 112, 32, 1, 16, False),    # MobileNetV2's first block at full map size
    (3, 112, 96, 2, 24, False),    # even map, stride 2: no top / left padding
    (2, 14, 576, 2, 160, False),   # 7x7 output: the narrow-map tile
    (3, 7, 960, 1, 160, True),
    (2, 7, 960, 1, 320, False),    # two n tiles of 160
    (1, 7, 64, 1, 32, True),       # a two-image 7x7 tile with its second image absent
    (5, 6, 48, 1, 40, True),       # 6x6 maps, odd image count
    (1, 9, 40, 1, 52, False),      # c and cout not multiples of 32
    (2, 28, 192, 2, 64, False),    # stride 2, c > 160: 32-channel halo blocks, 64-pixel tiles
    (1, 30, 200, 2, 40, True),     # the same class, ragged: c = 200, 15x15 output
]


@pytest.mark.parametrize("n,ih,c,s,cout,residual", CASES)
def test_dw_project_matches_float64(g, n, ih, c, s, cout, residual):
    oh = -(-ih // s)
    tot = max((oh - 1) * s + 3 - ih, 0)
    pt = tot // 2
    x = _r(n, ih, ih, c, scale=2.0)
    wd, bd = _r(3, 3, c), _r(c, scale=0.1)
    wp = _r(cout, c, scale=np.sqrt(3.0 / c))
    bp = _r(cout, scale=0.1)
    res = _r(n, oh, oh, cout) if residual else None
    dwp = g.tensor(wp)
    split = g.weights_split(dwp)
    dy = g.alloc((n, oh, oh, cout))
    dx = g.tensor(x)
    assert g.dw_project_supported(dx, dy, stride=s, pad=(pt, pt))
    g.dw_project_nhwc(dx, g.tensor(wd), g.tensor(bd), split, g.tensor(bp), dy, stride=s,
                      pad=(pt, pt), act_dw=_lib.ACT_RELU6,
                      residual=g.tensor(res) if residual else None)
    d = np.clip(R.depthwise_nhwc(x, wd, bd, (s, s), (pt, pt), (oh, oh)), 0, 6)
    ref = d @ wp.T.astype(np.float64) + bp
    if residual:
        ref = ref + res
    got = dy.download()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err <= 2.5e-8 * c + 1e-6, err
    # and the unfused depthwise + tensor-core conv of the library agree
    dd = g.alloc((n, oh, oh, c))
    g.depthwise_nhwc(dx, g.tensor(wd), g.tensor(bd), dd, stride=(s, s), pad=(pt, pt),
                     activation=_lib.ACT_RELU6)
    dz = g.alloc((n, oh, oh, cout))
    g.conv2d_nhwc(dd, dwp.view((cout, 1, 1, c)), g.tensor(bp), dz,
                  residual=g.tensor(res) if residual else None, w_split=split)
    assert np.abs(got - dz.download()).max() / np.abs(ref).max() <= 2 * (2.5e-8 * c + 1e-6)


@pytest.mark.parametrize("n,ih,c,s,cout,residual", [CASES[1], CASES[3], CASES[8], CASES[10],
                                                   CASES[11], CASES[13]])
def test_builder_groups_and_stages_give_identical_results(g, n, ih, c, s, cout, residual):
    """One builder group per K block or two taking alternate K blocks, two to
    four A/B stages, two or four TMEM accumulators, one or two epilogue
    groups: every depthwise value is accumulated by one
    thread in the same order and every GEMM in the same k order either way,
    so the outputs are bit-identical."""
    oh = -(-ih // s)
    pt = max((oh - 1) * s + 3 - ih, 0) // 2
    x = g.tensor(_r(n, ih, ih, c, scale=2.0))
    wd, bd = g.tensor(_r(3, 3, c)), g.tensor(_r(c, scale=0.1))
    split = g.weights_split(g.tensor(_r(cout, c, scale=np.sqrt(3.0 / c))))
    bp = g.tensor(_r(cout, scale=0.1))
    res = g.tensor(_r(n, oh, oh, cout)) if residual else None
    outs = []
    names = ("dwp_groups", "dwp_stages", "dwp_accs", "dwp_epi1")
    defaults = [_lib.get_option(k) for k in names]
    try:
        for setting in ((0, 2, 2, 0), (63, 2, 4, 63), (0, 4, 2, 63), (63, 4, 4, 0), (63, 3, 4, 47),
                        (47, 4, 2, 0)):
            for k, v in zip(names, setting):
                _lib.set_option(k, v)
            dy = g.alloc((n, oh, oh, cout))
            g.dw_project_nhwc(x, wd, bd, split, bp, dy, stride=s, pad=(pt, pt),
                              act_dw=_lib.ACT_RELU6, residual=res)
            outs.append(dy.download())
    finally:
        for k, v in zip(names, defaults):
            _lib.set_option(k, v)
    for o in outs[1:]:
        np.testing.assert_array_equal(o, outs[0])


@pytest.mark.parametrize("act_dw,act_proj", [(_lib.ACT_NONE, _lib.ACT_RELU), (_lib.ACT_RELU6, _lib.ACT_TANH),
                                             (_lib.ACT_SILU, _lib.ACT_NONE)])
def test_dw_project_other_activations(g, act_dw, act_proj):
    """Activations outside ReLU6 / none on either side (the kernel's second
    activation-group instantiation) against float64."""
    n, ih, c, s, cout = 2, 14, 96, 1, 40
    x = _r(n, ih, ih, c, scale=2.0)
    wd, bd = _r(3, 3, c), _r(c, scale=0.1)
    wp = _r(cout, c, scale=np.sqrt(3.0 / c))
    bp = _r(cout, scale=0.1)
    dy = g.alloc((n, ih, ih, cout))
    g.dw_project_nhwc(g.tensor(x), g.tensor(wd), g.tensor(bd), g.weights_split(g.tensor(wp)),
                      g.tensor(bp), dy, stride=s, pad=(1, 1), act_dw=act_dw, act_proj=act_proj)
    acts = {_lib.ACT_NONE: lambda v: v, _lib.ACT_RELU: lambda v: np.maximum(v, 0),
            _lib.ACT_RELU6: lambda v: np.clip(v, 0, 6), _lib.ACT_TANH: np.tanh,
            _lib.ACT_SILU: lambda v: v / (1 + np.exp(-v))}
    d = acts[act_dw](R.depthwise_nhwc(x, wd, bd, (s, s), (1, 1), (ih, ih)))
    ref = acts[act_proj](d @ wp.T.astype(np.float64) + bp)
    got = dy.download()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= 2.5e-8 * c + 2e-6


def test_dw_project_rejects_unsupported(g):
    x, y = g.alloc((1, 8, 8, 30)), g.alloc((1, 8, 8, 16))
    assert not g.dw_project_supported(x, y, stride=1, pad=(1, 1))     # c % 4
    x2, y2 = g.alloc((1, 8, 8, 32)), g.alloc((1, 8, 8, 600))
    assert not g.dw_project_supported(x2, y2, stride=1, pad=(1, 1))   # cout > 512
    with pytest.raises(_lib.SpxError):
        g.dw_project_nhwc(x, g.alloc((3, 3, 30)), None, (g.alloc((16, 30)), g.alloc((16, 30))),
                          None, y, stride=1, pad=(1, 1))


def test_mobilenet_v2_fusion_plan_and_parity(gpu, oracle_built):
    m = nets.mobilenet_v2(seed=0)
    x = nets.make_input(m, 3, seed=5)
    outs = []
    for fuse in (True, False):
        ex = CnnExecutor(m, batch=3, device=gpu, fuse_dw_project=fuse)
        try:
            if fuse:
                assert sum(k == "dwproj" for k, _ in ex._plan) == 17
                assert not any(k == "dw" for k, _ in ex._plan)
            outs.append(ex.forward(x))
        finally:
            ex.close()
    ref, _ = lowering.run_graph(m, x, oracle_built.run_kernel)
    # the fused kernel and the unfused depthwise + tensor-core GEMM pipeline
    # (same split, products summed in a different order) agree closely
    assert np.abs(outs[0] - outs[1]).max() <= 2e-5
    for o in outs:
        np.testing.assert_array_equal(lowering.top1(o), lowering.top1(ref))
        assert np.abs(o - ref).max() <= 1e-4


def test_fused_forward_is_deterministic(gpu):
    """Repeated runs of the fused MobileNetV2 step give bit-identical outputs
    (a halo slot refilled while a slow builder still read it, or an A tile
    rewritten under the MMA, would show up as run-to-run differences)."""
    m = nets.mobilenet_v2(seed=0)
    x = nets.make_input(m, 16, seed=5)
    ex = CnnExecutor(m, batch=16, device=gpu)
    try:
        first = ex.forward(x)
        for _ in range(12):
            np.testing.assert_array_equal(ex.forward(x), first)
    finally:
        ex.close()


@pytest.mark.parametrize("n,ih,iw,oc,pad", [(2, 224, 224, 32, (0, 0)), (3, 16, 16, 32, (1, 1)),
                                             (1, 37, 20, 16, (1, 0))])
def test_stem_conv_matches_float64(g, n, ih, iw, oc, pad):
    """The tensor-core stem (3x3 stride 2 over 3 channels, im2col on chip,
    3xTF32) against float64, with ReLU6; pads 0 / 1 exercise the 16-byte
    rounding of the row box start."""
    oh, ow = -(-ih // 2), -(-iw // 2)
    x = _r(n, ih, iw, 3, scale=2.0)
    w = _r(oc, 3, 3, 3, scale=0.5)
    b = _r(oc, scale=0.1)
    dx, dy = g.tensor(x), g.alloc((n, oh, ow, oc))
    assert g.stem_supported(dx, dy, pad=pad, activation=_lib.ACT_RELU6)
    g.stem_conv_nhwc(dx, g.stem_weights(w), g.tensor(b), dy, pad=pad,
                     activation=_lib.ACT_RELU6)
    ref = np.clip(R.conv_nhwc(x, w.transpose(1, 2, 3, 0), (2, 2), pad, (oh, ow)) + b, 0, 6)
    got = dy.download()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= 2.5e-8 * 27 + 1e-6


@pytest.mark.parametrize("n,ih,iw,oc,pad", [(2, 224, 224, 64, (3, 3)), (3, 20, 24, 32, (2, 2)),
                                         (1, 17, 16, 12, (3, 1))])
def test_stem_7x7_matches_float64(g, n, ih, iw, oc, pad):
    """The 7x7 stride-2 tensor-core stem (ResNet-50's first conv: 147 taps in
    five 32-wide K blocks) against float64, with ReLU; pad 3 exercises row box
    starts that round down below the map and past its left edge."""
    oh = (ih + 2 * pad[0] - 7) // 2 + 1
    ow = (iw + 2 * pad[1] - 7) // 2 + 1
    x = _r(n, ih, iw, 3, scale=2.0)
    w = _r(oc, 7, 7, 3, scale=0.2)
    b = _r(oc, scale=0.1)
    dx, dy = g.tensor(x), g.alloc((n, oh, ow, oc))
    assert g.stem_supported(dx, dy, pad=pad, activation=_lib.ACT_RELU, kernel=7)
    g.stem_conv_nhwc(dx, g.stem_weights(w), g.tensor(b), dy, pad=pad,
                     activation=_lib.ACT_RELU, kernel=7)
    ref = np.maximum(R.conv_nhwc(x, w.transpose(1, 2, 3, 0), (2, 2), pad, (oh, ow)) + b, 0)
    got = dy.download()
    assert np.abs(got - ref).max() / np.abs(ref).max() <= 2.5e-8 * 147 + 1e-6


def test_stem_accumulator_count_gives_identical_results(g):
    """Two or four TMEM accumulators in the stem change only which tensor
    memory columns a tile uses, not the arithmetic: identical bits."""
    x = g.tensor(_r(2, 64, 64, 3, scale=2.0))
    w = g.stem_weights(_r(32, 3, 3, 3, scale=0.5))
    b = g.tensor(_r(32, scale=0.1))
    outs = []
    try:
        for accs in (2, 4):
            _lib.set_option("dwp_accs", accs)
            dy = g.alloc((2, 32, 32, 32))
            g.stem_conv_nhwc(x, w, b, dy, pad=(0, 0), activation=_lib.ACT_RELU6)
            outs.append(dy.download())
    finally:
        _lib.set_option("dwp_accs", 4)
    np.testing.assert_array_equal(outs[1], outs[0])


def test_stem_rejects_other_shapes(g):
    x, y = g.alloc((1, 16, 18, 3)), g.alloc((1, 8, 9, 32))
    assert not g.stem_supported(x, y)                     # iw % 4
    x2, y2 = g.alloc((1, 16, 16, 4)), g.alloc((1, 8, 8, 32))
    assert not g.stem_supported(x2, y2)                   # 4 input channels


def test_programmatic_launch_gives_identical_outputs(gpu):
    """Option pdl: the fused and GEMM kernels launched with programmatic
    stream serialisation (set-up overlapping the previous kernel's tail)
    give the same bits as plain launches, in eager runs and graph replays."""
    m = nets.mobilenet_v2(seed=0)
    x = nets.make_input(m, 16, seed=5)
    outs = []
    try:
        for pdl in (0, 1):
            _lib.set_option("pdl", pdl)
            ex = CnnExecutor(m, batch=16, device=gpu)
            try:
                outs += [ex.forward(x), ex.forward(x)]
            finally:
                ex.close()
    finally:
        _lib.set_option("pdl", 1)
    for o in outs[1:]:
        np.testing.assert_array_equal(o, outs[0])
