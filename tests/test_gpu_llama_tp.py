"""Tensor-parallel TinyLlama decode on 2 GPUs (one process per GPU, NCCL
all-reduce after the row-parallel projections, vocab-parallel argmax):
greedy tokens equal the single-GPU decoder's.  Skipped with fewer than two
GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from spirv_inference_b200 import llama

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ar_worker(rank, world, port, q):
    """Peer-memory all-reduce kernel on its own: alternating slots, sizes
    from one float4 to 256 KB, repeated so epochs advance."""
    import torch.distributed as dist
    from spirv_inference_b200.comm import PeerAllReduce
    from spirv_inference_b200.graph import Graph
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        g = Graph(rank)
        ar = PeerAllReduce(rank, rank, world, 1 << 20)
        errs = []
        for it, n in enumerate([4, 1000, 65536, 4, 262144 // 4 * 4]):
            slot = it % 2
            data = [np.random.default_rng(100 * r + it).standard_normal(n).astype(np.float32)
                    for r in range(world)]
            part = ar.slot(slot, (n,), g)
            g.upload(part, data[rank])
            out = g.alloc((n,))
            # every rank's slot is written before anyone reduces
            g.sync()
            dist.barrier()
            ar.allreduce(g, slot, out, n)
            got = out.download()
            ref = data[0].astype(np.float64)
            for r in range(1, world):
                ref = ref + data[r]
            errs.append(float(np.abs(got - ref).max()))
        g.sync()
        ar.close()
        g.close()
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def test_peer_allreduce_two_gpus(gpu):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ar_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert max(res[0] + res[1]) <= 1e-5


def _worker(rank, world, port, batch, q, capture=True, peer=False):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        cfg = llama.TINY_TEST
        W = llama.make_weights(cfg, 0)
        prompt = llama.make_prompt(cfg, batch, 32)
        s = torch.cuda.Stream()
        torch.cuda.set_stream(s)
        dec = llama.LlamaDecoder(cfg, W, batch, 32, 12, device=rank, stream=s.cuda_stream,
                                 rank=rank, world=world, capture=capture,
                                 peer_allreduce=peer)
        toks = dec.generate(prompt)
        toks2 = dec.generate(prompt)          # replay of the captured step
        assert np.array_equal(toks, toks2)
        assert dec._captured == capture, "decode step with collectives was not captured"
        dec.close()
        q.put((rank, toks.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch,peer", [(1, False), (12, False), (1, True), (12, True)])
def test_tp2_matches_single_gpu(gpu, batch, peer):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = llama.TINY_TEST
    W = llama.make_weights(cfg, 0)
    prompt = llama.make_prompt(cfg, batch, 32)
    dec = llama.LlamaDecoder(cfg, W, batch, 32, 12, device=gpu)
    ref = dec.generate(prompt)
    dec.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, q, True, peer))
             for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1]
    np.testing.assert_array_equal(np.array(res[0]), ref)
