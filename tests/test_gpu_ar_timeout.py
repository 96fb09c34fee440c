"""The peer all-reduce's bounded wait running out (failure detection).

Rank 1 joins the communicator (its memory is exported and opened by rank 0)
but never launches the all-reduce: rank 0's kernel waits for a flag that
nothing sets.  With "ar_wait_limit_us" at 0.2 s the kernel gives up, leaves
the output untouched and records a status; the next graph sync returns
SPX_ERR_CUDA naming the timeout, the status is cleared, and the library keeps
working.  Only rank 0 ever runs a waiting kernel, so the one-GPU form has no
two kernels waiting on each other.  With two GPUs the ranks then reset their
communicators between host barriers and a normal all-reduce on fresh epochs
gives the right sums.  The ranks are spawned child processes that meet only
through host queues (no collective library involved).
"""
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
N = 4096


def _rank(rank, device, to_parent, from_parent):
    from spirv_inference_b200 import _lib
    from spirv_inference_b200.comm import PeerAllReduce
    from spirv_inference_b200.graph import Graph
    out = {"rank": rank}
    try:
        def exchange(mine):
            to_parent.put(("handle", rank, mine))
            return from_parent.get(timeout=60)

        g = Graph(device)
        ar = PeerAllReduce(device, rank, 2, 1 << 16, exchange=exchange)
        data = np.random.default_rng(rank).standard_normal(N).astype(np.float32)
        res = g.alloc((N,))
        if rank == 0:
            l = _lib.lib()
            assert l.spx_set_option(b"ar_wait_limit_us", 200000) == 0
            g.upload(ar.slot(0, (N,), g), data)
            g.upload(res, np.full(N, 7.0, np.float32))
            t0 = time.perf_counter()
            ar.allreduce(g, 0, res, N)
            try:
                g.sync()
                out["error"] = None
            except _lib.SpxError as e:
                out["error"] = (e.code, str(e))
            out["seconds"] = time.perf_counter() - t0
            out["untouched"] = bool(np.all(res.download() == 7.0))
            g.sync()                                  # status was cleared
            x = np.linspace(-2, 2, 1000, dtype=np.float32)
            d = g.tensor(x)
            y = g.alloc((1000,))
            g.softmax_rows(d, y, 1, 1000)
            e = np.exp(x - x.max())
            out["after_ok"] = bool(np.abs(y.download() - e / e.sum()).max() < 1e-6)
            l.spx_set_option(b"ar_wait_limit_us", 2000000)
        to_parent.put(("phase1", rank, out))
        cmd = from_parent.get(timeout=120)
        if cmd == "second_round":
            ar.reset()
            to_parent.put(("reset", rank, None))
            assert from_parent.get(timeout=60) == "go"
            g.upload(ar.slot(1, (N,), g), data)
            g.sync()
            to_parent.put(("written", rank, None))
            assert from_parent.get(timeout=60) == "go"
            ar.allreduce(g, 1, res, N)
            g.sync()
            ref = sum(np.random.default_rng(r).standard_normal(N).astype(np.float64)
                      for r in range(2))
            to_parent.put(("phase2", rank, float(np.abs(res.download() - ref).max())))
        ar.close()
        g.close()
    except Exception as e:  # reported to the parent, which fails the test
        to_parent.put(("exception", rank, repr(e)))


def _collect(q, kind, n=2, timeout=120):
    got = {}
    while len(got) < n:
        k, r, v = q.get(timeout=timeout)
        if k == "exception":
            raise AssertionError(f"rank {r}: {v}")
        assert k == kind, (k, kind)
        got[r] = v
    return got


def test_allreduce_wait_runs_out_and_library_recovers(gpu):
    from spirv_inference_b200.graph import device_count
    two = device_count() >= 2
    ctx = mp.get_context("spawn")
    to_parent = ctx.Queue()
    to_child = [ctx.Queue(), ctx.Queue()]
    procs = [ctx.Process(target=_rank, args=(r, r if two else 0, to_parent, to_child[r]))
             for r in range(2)]
    for p in procs:
        p.start()
    try:
        hs = _collect(to_parent, "handle")
        every = hs[0] + hs[1]
        for q in to_child:
            q.put(every)
        res = _collect(to_parent, "phase1")[0]
        code, msg = res["error"]
        assert code == 3 and "gave up" in msg and "200000 us" in msg, msg
        assert res["seconds"] < 5.0
        assert res["untouched"] and res["after_ok"]
        if two:
            for q in to_child:
                q.put("second_round")
            _collect(to_parent, "reset")
            for q in to_child:
                q.put("go")
            _collect(to_parent, "written")
            for q in to_child:
                q.put("go")
            errs = _collect(to_parent, "phase2")
            assert max(errs.values()) <= 1e-5, errs
        else:
            for q in to_child:
                q.put("stop")
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
