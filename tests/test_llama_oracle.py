"""CPU tests of the TinyLlama decode oracle and the tensor-parallel packing.

* the KV-cache restatement gives the same greedy tokens as the reference's
  full re-computation loop (run_llama_spirv.py:190-260) on seeded weights;
* tensor-parallel packing at 2 / 4 / 8 ranks (kv heads replicated at 8)
  reproduces the unsharded tokens, simulated in one process and as two gloo
  ranks with a real all-reduce / argmax exchange."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import _llama_np
from oracle import llama_ref as R
from spirv_inference_b200 import llama

CFG = llama.TINY_TEST


@pytest.fixture(scope="module")
def weights():
    return llama.make_weights(CFG, 0)


def test_rope_tables_match_reference_formula():
    cos, sin = llama.rope_tables(llama.TINYLLAMA, 64)
    assert cos.shape == (64, 64) and cos.dtype == np.float32
    inv = 1.0 / (10000.0 ** (np.arange(0, 64, 2, dtype=np.float32) / 64))
    ang = 5.0 * inv
    assert np.allclose(cos[5, :32], np.cos(ang), atol=1e-6)
    assert np.allclose(sin[5, 32:], np.sin(ang), atol=1e-6)
    assert np.all(cos[0] == 1) and np.all(sin[0] == 0)


def test_causal_mask_matches_reference_rule():
    m = R.causal_mask(6, 4)
    for r in range(6):
        for c in range(6):
            assert m[r, c] == (-1e9 if (c > r or c >= 4) else 0.0)


def test_cached_equals_full_recompute(weights):
    rope = llama.rope_tables(CFG, CFG.max_seq)
    prompt = llama.make_prompt(CFG, 2, 32)
    for b in range(2):
        full = R.generate_full(CFG, weights, prompt[b], 20, rope)
        cached = R.generate_cached(CFG, weights, prompt[b], 20, rope)
        assert np.array_equal(full, cached), (full, cached)


def test_forced_logits_consistent(weights):
    rope = llama.rope_tables(CFG, CFG.max_seq)
    prompt = llama.make_prompt(CFG, 1, 8)[0]
    toks = R.generate_cached(CFG, weights, prompt, 5, rope)
    out, logits = R.generate_cached(CFG, weights, prompt, 5, rope, forced=toks)
    assert np.array_equal(out, toks) and logits.shape == (5, CFG.vocab)
    _, last = R.generate_full(CFG, weights, prompt, 5, rope, return_logits=True)
    assert np.max(np.abs(last - logits[-1])) <= 1e-4 * np.max(np.abs(last))


def test_tp_shard_layout():
    full = llama.TINYLLAMA
    s8 = [llama.tp_shard(full, r, 8) for r in range(8)]
    assert [s.kv0 for s in s8] == [0, 0, 1, 1, 2, 2, 3, 3]
    assert all(s.nq == 4 and s.nkv == 1 and s.nf == 704 and s.nv == 4000 for s in s8)
    s2 = [llama.tp_shard(full, r, 2) for r in range(2)]
    assert [(s.q0, s.nq, s.kv0, s.nkv) for s in s2] == [(0, 16, 0, 2), (16, 16, 2, 2)]
    with pytest.raises(ValueError):
        llama.tp_shard(full, 0, 3)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_simulated_matches_unsharded(weights, world):
    rope = llama.rope_tables(CFG, CFG.max_seq)
    prompt = llama.make_prompt(CFG, 1, 32)[0]
    ref = R.generate_cached(CFG, weights, prompt, 8, rope)
    if CFG.heads % world or CFG.ffn % world or CFG.vocab % world:
        pytest.skip("degree does not divide the test config")
    got = _llama_np.tp_generate(CFG, weights, prompt, 8, world)
    assert np.array_equal(ref, got), (ref, got)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _GlooReduce:
    def __init__(self, rank, world):
        self.rank, self.world = rank, world

    def __call__(self, part):
        import torch
        import torch.distributed as dist
        t = torch.from_numpy(np.ascontiguousarray(part))
        dist.all_reduce(t)
        return t.numpy()

    def argmax(self, cand):
        import torch
        import torch.distributed as dist
        mine = torch.tensor([cand[0], float(cand[1])], dtype=torch.float64)
        out = [torch.zeros(2, dtype=torch.float64) for _ in range(self.world)]
        dist.all_gather(out, mine)
        best = None
        for o in out:
            v, i = float(o[0]), int(o[1])
            if best is None or v > best[0] or (v == best[0] and i < best[1]):
                best = (v, i)
        return best[1]


def _tp_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W = llama.make_weights(CFG, 0)
        prompt = llama.make_prompt(CFG, 1, 32)[0]
        toks = _llama_np.tp_generate(CFG, W, prompt, 6, world, reduce=_GlooReduce(rank, world))
        q.put((rank, toks.tolist()))
    finally:
        dist.destroy_process_group()


def test_tp_two_gloo_ranks(weights):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rope = llama.rope_tables(CFG, CFG.max_seq)
    ref = R.generate_cached(CFG, weights, llama.make_prompt(CFG, 1, 32)[0], 6, rope)
    assert res[0] == res[1] == ref.tolist()
