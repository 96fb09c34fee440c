"""CPU tests of the tensor-core GEMM's per-shape launch plan (host code only,
no device): for every pointwise-conv / linear shape of the configs, the plan
fits shared memory and TMEM, its warp roles add up, and the ring invariants
the kernel's mbarrier parities rely on hold (two converter groups only on an
even stage ring; two epilogue groups only with one chunk per lane quarter)."""
import pytest

from spirv_inference_b200 import _lib, nets

SMEM_LIMIT = 227 * 1024


def _pointwise_shapes(model_name, batches):
    m = nets.MODELS[model_name](seed=0)
    out = set()
    for op in m.ops:
        if op.type != "CONV_2D":
            continue
        w = m.weights[op.inputs[1]]
        if w.shape[1:3] != (1, 1):
            continue
        oh, ow, oc = m.shapes[op.output]
        for b in batches:
            out.add((b * oh * ow, oc, w.shape[3]))
    return sorted(out)


SHAPES = sorted(set(
    _pointwise_shapes("mobilenet_v2", (1, 8, 64, 256))
    + _pointwise_shapes("efficientnet_lite0", (1, 64, 256))
    + [  # ResNet-50 b256 1x1 convs and FC, BERT-base b32 s128 linears, TinyLlama prefill
        (802816, 64, 64), (802816, 256, 64), (200704, 512, 256), (50176, 1024, 512),
        (12544, 2048, 1024), (256, 1000, 2048), (4096, 768, 768), (4096, 2304, 768),
        (4096, 3072, 768), (4096, 768, 3072), (2048, 2560, 2048), (2048, 11264, 2048),
        (333, 1001, 1280), (5, 8, 4), (130, 48, 36),
    ]))


def _check(plan, m, n, k):
    bn = plan["BN"]
    assert bn % 32 == 0 and 32 <= bn <= 256
    assert plan["n_tiles"] == -(-n // bn)
    assert plan["k_blocks"] == -(-k // 32)
    assert 1 <= plan["last_ksteps"] <= 4
    assert (plan["k_blocks"] - 1) * 32 + plan["last_ksteps"] * 8 >= k
    assert 2 <= plan["stages"] <= 8
    assert plan["smem_bytes"] <= SMEM_LIMIT
    assert plan["epi_warps"] in (4, 8, 12)
    # converters are warps max(8, epilogue) .. 15
    assert plan["conv_threads"] == (16 - max(8, plan["epi_warps"])) * 32
    if plan["conv_groups"] == 2:
        assert plan["stages"] % 2 == 0 and plan["k_blocks"] > 1
        assert plan["conv_threads"] % 64 == 0
    if plan["groups"] == 2:
        assert bn == 32 and plan["epi_warps"] == 8
    # two accumulators per epilogue group, or three / four for one-k-block tiles
    assert plan["nacc"] == 2 * plan["groups"] or (
        plan["nacc"] in (3, 4) and plan["groups"] == 1 and plan["k_blocks"] == 1)
    cols = plan["tmem_cols"]
    lo_cols = 64 if plan["lo_tmem"] else 0
    assert cols & (cols - 1) == 0 and 32 <= cols <= 512
    assert cols >= plan["nacc"] * bn + lo_cols
    if plan["lo_tmem"]:  # two 32-column lo slots after the accumulators
        assert plan["k_blocks"] >= 2 and plan["epi_warps"] <= 8
        assert plan["stage_bytes"] == 16384 + 2 * bn * 128
    if plan["b_resident"]:
        assert plan["k_blocks"] == 1 and plan["n_tiles"] == 1
    # every 32-column chunk of a tile has an epilogue warp per lane quarter
    per_quarter = plan["epi_warps"] // plan["groups"] // 4
    assert per_quarter >= 1
    assert plan["grid"] == min(plan["m_tiles"] * plan["n_tiles"], 148)


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_plan_invariants(spx_built, m, n, k):
    for presplit in (True, False):
        for vec4 in (True, False):
            plan = _lib.gemm_tc_plan(m, n, k, presplit=presplit, vec4=vec4)
            _check(plan, m, n, k)
            if not presplit:
                assert plan["b_resident"] == 0 and plan["lo_tmem"] == 0
            if not vec4:  # no TMA stores: one epilogue group
                assert plan["groups"] == 1


def test_plan_options_restore_plain_layout(spx_built):
    try:
        _lib.set_option("tc_wide_epilogue", 0)
        _lib.set_option("tc_conv_groups", 1)
        _lib.set_option("tc_lo_tmem", 0)
        for m, n, k in SHAPES:
            p = _lib.gemm_tc_plan(m, n, k)
            assert p["epi_warps"] in (4, 8) and p["groups"] == 1 and p["conv_groups"] == 1
            assert p["b_resident"] == 0 and p["lo_tmem"] == 0
    finally:
        _lib.set_option("tc_wide_epilogue", 1)
        _lib.set_option("tc_conv_groups", 2)
        _lib.set_option("tc_lo_tmem", 0)


def test_plan_known_configurations(spx_built):
    # expand 16 -> 96 at 112x112, batch 256: 12 epilogue warps, weights resident
    p = _lib.gemm_tc_plan(3211264, 96, 16)
    assert (p["BN"], p["epi_warps"], p["b_resident"], p["last_ksteps"]) == (96, 12, 1, 2)
    # project 32 -> 16: two epilogue groups on four accumulators
    p = _lib.gemm_tc_plan(3211264, 16, 32)
    assert (p["BN"], p["groups"], p["nacc"]) == (32, 2, 4)
    # project 144 -> 24: five k-blocks, two converter groups on an even ring
    p = _lib.gemm_tc_plan(802816, 24, 144)
    assert p["k_blocks"] == 5 and p["lo_tmem"] == 0
    assert p["conv_groups"] == 2 and p["stages"] % 2 == 0
    # with the lo terms in TMEM the stages shrink to raw A + B and the ring deepens
    _lib.set_option("tc_lo_tmem", 1)
    try:
        q = _lib.gemm_tc_plan(802816, 24, 144)
    finally:
        _lib.set_option("tc_lo_tmem", 0)
    assert q["lo_tmem"] == 1 and q["stages"] > p["stages"] and q["stages"] % 2 == 0
    assert q["tmem_cols"] >= q["nacc"] * q["BN"] + 64


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_plan_invariants_lo_in_tmem(spx_built, m, n, k):
    _lib.set_option("tc_lo_tmem", 1)
    try:
        for presplit in (True, False):
            _check(_lib.gemm_tc_plan(m, n, k, presplit=presplit), m, n, k)
    finally:
        _lib.set_option("tc_lo_tmem", 0)


def test_plan_rejects_bad_arguments(spx_built):
    with pytest.raises(_lib.SpxError):
        _lib.gemm_tc_plan(0, 8, 8)
