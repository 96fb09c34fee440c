"""CPU tests of the multi-GPU host logic: shard ranges, per-rank seeds and the
max-over-ranks timing reduction, the last run as two gloo ranks."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from spirv_inference_b200 import sharding


def test_shard_ranges_cover_batch_exactly():
    for total, world in [(256, 1), (2048, 8), (10, 3), (7, 4), (3, 8)]:
        spans = [sharding.shard_range(total, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == total
        for (a, b), (c, d) in zip(spans, spans[1:]):
            assert b == c
        sizes = [b - a for a, b in spans]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(8, 2, 2)


def test_seeds_and_throughput():
    assert len({sharding.shard_seed(1000, r) for r in range(8)}) == 8
    assert sharding.throughput(256, 4, 10.0) == pytest.approx(4 * 256 / 0.010)
    assert sharding.max_over_ranks(3.5) == 3.5  # no process group


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w, r, lr = sharding.dist_env()
    assert (w, r, lr) == (world, rank, rank)
    m = sharding.max_over_ranks(10.0 + rank)  # rank 1 is the slowest
    dist.barrier()
    out[rank] = m
    dist.destroy_process_group()


def test_max_over_ranks_gloo_two_ranks():
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
        assert dict(out) == {0: 11.0, 1: 11.0}


def test_bench_rank_plumbing_two_gloo_ranks():
    """bench.py under the driver's torchrun launch line, two ranks, --dry-run:
    exactly one JSON line (rank 0), the slowest rank's time, the whole-job
    throughput and the per-GPU batch of the config."""
    import json
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    port = _free_port()
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port",
                        str(port), str(root / "bench.py"), "--gpus", "2", "--dry-run"],
                       capture_output=True, text=True, timeout=300, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["n_gpus"] == 2 and d["dry_run"] is True
    assert d["ms_per_step"] == 2.0                      # max over ranks (1 + rank)
    assert d["value"] == pytest.approx(2 * 256 / 0.002)
    assert d["config"]["batch_per_gpu"] == 256 and d["config"]["global_batch"] == 512
