"""Parity at the benchmark configurations themselves.

Every configuration the benchmark names runs on the GPU at its full size
(MobileNetV2 b256, EfficientNet-Lite0 b64, ResNet-50 224x224 b256, BERT-base
12 layers s128 b32, TinyLlama 22 layers b1 / b64), with the per-shape kernel
plans those sizes select.  Sampled rows of each batch are compared with the
reference semantics on the CPU oracle run on the same rows (batch rows are
independent in every one of these graphs, which the shard tests check
exactly):

* CNNs (source/tflite_loader/src/scheduler.rs:29-1082 on the oracle):
  identical top-1, max |softmax difference| <= 1e-4.
* HLO graphs (source/xla_hlo/src/compiler.rs:267-668 on the oracle): logits /
  hidden states within 1e-3 relative to the output's max magnitude, identical
  top-1 for ResNet-50.
* TinyLlama (the reference decode loop, run_llama_spirv.py:190-260, restated
  in oracle/llama_ref.generate_full): all 20 greedy tokens identical at b1;
  the b64 run's sampled rows identical as well, with each step's logits
  within 1e-3 relative (teacher-forced KV-cache oracle).
"""
import numpy as np
import pytest

from spirv_inference_b200 import hlo, lowering, nets, nets_hlo
from spirv_inference_b200.executor import CnnExecutor
from spirv_inference_b200.executor_hlo import HloExecutor

pytestmark = pytest.mark.gpu
SOFTMAX_ATOL = 1e-4
LOGIT_RTOL = 1e-3


def _sample_rows(batch: int, n_extra: int, seed: int) -> list[int]:
    rng = np.random.Generator(np.random.PCG64(seed))
    mid = rng.choice(np.arange(1, batch - 1), size=min(n_extra, batch - 2), replace=False)
    return sorted({0, batch - 1, *map(int, mid)})


def _normerr(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


@pytest.mark.parametrize("name,batch", [("mobilenet_v2", 256), ("efficientnet_lite0", 64)])
def test_cnn_config_batch_matches_oracle(gpu, oracle_built, name, batch):
    m = nets.MODELS[name](seed=0)
    x = nets.make_input(m, batch, seed=1234)       # the bench's input
    ex = CnnExecutor(m, batch=batch, device=gpu)
    try:
        ex.capture()                                # the bench's CUDA-graph replay
        ex.g.upload(ex.input, x)
        ex.run()
        got = ex.g.download(ex.output)
    finally:
        ex.close()
    rows = _sample_rows(batch, 6, seed=batch)
    ref, _ = lowering.run_graph(m, x[rows], oracle_built.run_kernel)
    np.testing.assert_array_equal(lowering.top1(got[rows]), lowering.top1(ref))
    err = float(np.abs(got[rows] - ref).max())
    assert err <= SOFTMAX_ATOL, err
    assert np.all(np.isfinite(got))
    # every row is a distribution
    np.testing.assert_allclose(got.sum(axis=1), 1.0, atol=1e-4)


@pytest.fixture(scope="module")
def resnet_ref(oracle_built):
    g2 = nets_hlo.resnet50(seed=0, batch=2, hw=224)
    x = nets_hlo.make_image_batch(256, 224, seed=5)
    ref, _ = hlo.run_hlo(g2, {g2.inputs[0]: x[[0, 255]]}, oracle_built.run_kernel)
    return x, ref


def test_resnet50_224_b2_matches_oracle(gpu, resnet_ref):
    x, ref = resnet_ref
    g = nets_hlo.resnet50(seed=0, batch=2, hw=224)
    ex = HloExecutor(g, device=gpu)
    try:
        got = ex.forward({g.inputs[0]: x[[0, 255]]})
    finally:
        ex.close()
    assert _normerr(got, ref) <= LOGIT_RTOL, _normerr(got, ref)
    np.testing.assert_array_equal(np.argmax(got, 1), np.argmax(ref, 1))


def test_resnet50_224_b256_sampled_rows_match_oracle(gpu, resnet_ref):
    x, ref = resnet_ref
    g = nets_hlo.resnet50(seed=0, batch=256, hw=224)
    ex = HloExecutor(g, device=gpu)
    try:
        got = ex.forward({g.inputs[0]: x})
    finally:
        ex.close()
    assert got.shape == (256, 1000)
    sel = got[[0, 255]]
    assert _normerr(sel, ref) <= LOGIT_RTOL, _normerr(sel, ref)
    np.testing.assert_array_equal(np.argmax(sel, 1), np.argmax(ref, 1))
    assert np.all(np.isfinite(got))


def test_bert_base_12_layers_s128_matches_oracle(gpu, oracle_built):
    batch, seq = 32, 128
    rng = np.random.Generator(np.random.PCG64(2024))
    ids = rng.integers(0, 30522, (batch, seq))
    x = nets_hlo.bert_embed(0, ids)
    g = nets_hlo.bert_encoder(seed=0, batch=batch, seq=seq, layers=12)
    ex = HloExecutor(g, device=gpu)
    try:
        got = ex.forward({g.inputs[0]: x})
    finally:
        ex.close()
    assert got.shape == (batch, seq, 768)
    g2 = nets_hlo.bert_encoder(seed=0, batch=2, seq=seq, layers=12)
    rows = [0, batch - 1]
    ref, _ = hlo.run_hlo(g2, {g2.inputs[0]: x[rows]}, oracle_built.run_kernel)
    assert _normerr(got[rows], ref) <= LOGIT_RTOL, _normerr(got[rows], ref)
    assert np.all(np.isfinite(got))


@pytest.fixture(scope="module")
def tinyllama():
    from spirv_inference_b200 import llama
    cfg = llama.TINYLLAMA
    return cfg, llama.make_weights(cfg, seed=0, generator="torch")


def test_tinyllama_22_layers_b1_tokens_identical(gpu, tinyllama):
    from oracle import llama_ref as R
    from spirv_inference_b200 import llama
    cfg, W = tinyllama
    prompt = llama.make_prompt(cfg, 1, 32)
    dec = llama.LlamaDecoder(cfg, W, 1, 32, 20, device=gpu)
    try:
        toks = dec.generate(prompt)
        last = dec.last_logits()
    finally:
        dec.close()
    rope = llama.rope_tables(cfg, cfg.max_seq)
    full, full_last = R.generate_full(cfg, W, prompt[0], 20, rope, return_logits=True)
    np.testing.assert_array_equal(toks[0], full)
    assert _normerr(last[0], full_last) <= LOGIT_RTOL


def test_tinyllama_22_layers_b64_sampled_rows(gpu, tinyllama):
    from oracle import llama_ref as R
    from spirv_inference_b200 import llama
    cfg, W = tinyllama
    batch = 64
    prompt = llama.make_prompt(cfg, batch, 32, seed=11)
    dec = llama.LlamaDecoder(cfg, W, batch, 32, 20, device=gpu)
    try:
        toks = dec.generate(prompt)
        last = dec.last_logits()
    finally:
        dec.close()
    rope = llama.rope_tables(cfg, cfg.max_seq)
    for b in (0, 37, batch - 1):
        want, logits = R.generate_cached(cfg, W, prompt[b], 20, rope, forced=toks[b])
        # teacher-forced on the device's tokens: equal argmax at every step
        # means the device's greedy sequence is the oracle's
        np.testing.assert_array_equal(toks[b], want)
        assert _normerr(last[b], logits[-1]) <= LOGIT_RTOL
