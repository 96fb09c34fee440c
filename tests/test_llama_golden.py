"""TinyLlama parity pinned to the reference's own exported graph.

tests/golden/tinyllama_step_golden.npz holds the float64 evaluation of the
reference's `llama_step` HLO (source/xla_hlo/fixtures/tinyllama.stablehlo.txt,
made by tests/golden/make_llama_golden.py) on seeded inputs.  The CPU oracle
(oracle/llama_ref.llama_step) must reproduce its next-token logits and the
argmax of every prompt position; the GPU decoder's prefill must too (logits
within 1e-3 relative, the north-star gate)."""
from pathlib import Path

import numpy as np
import pytest

from oracle import llama_ref as R
from spirv_inference_b200 import llama

GOLDEN = Path(__file__).resolve().parent / "golden" / "tinyllama_step_golden.npz"
P, S = 32, 64


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="module")
def weights():
    return llama.make_weights(llama.TINYLLAMA, 0, generator="torch")


def test_prompt_is_the_seeded_one(golden):
    assert np.array_equal(golden["prompt"], llama.make_prompt(llama.TINYLLAMA, 1, P, 4321)[0])


def test_oracle_matches_reference_graph(golden, weights):
    cfg = llama.TINYLLAMA
    prompt = golden["prompt"]
    toks = [int(t) for t in prompt] + [0] * (S - P)
    cos, sin = llama.rope_tables(cfg, S)
    logits = R.llama_step(cfg, weights, weights["embed"][toks], cos, sin, R.causal_mask(S, P))
    ref = golden["last_logits"].astype(np.float64)
    assert np.abs(logits[P - 1] - ref).max() / np.abs(ref).max() <= 1e-4
    assert np.array_equal(logits[:P].argmax(axis=1), golden["argmax"])


@pytest.mark.gpu
def test_decoder_prefill_matches_reference_graph(gpu, golden, weights):
    dec = llama.LlamaDecoder(llama.TINYLLAMA, weights, 1, P, 1, device=gpu)
    try:
        toks = dec.generate(golden["prompt"][None])
        logits = dec.last_logits()[0]
    finally:
        dec.close()
    ref = golden["last_logits"].astype(np.float64)
    assert np.abs(logits - ref).max() / np.abs(ref).max() <= 1e-3
    assert int(toks[0, 0]) == int(golden["argmax"][P - 1])
