#!/usr/bin/env python3
"""MobileNetV2 fp32 inference throughput on B200 (images/s), the metric of
the reference's operator-dispatch hot path.

One process per GPU (torchrun for N > 1).  Each rank runs the fused NHWC
executor on its own shard of 256 images per step (weak scaling, batch
sharded, no collective on the data path); ranks only meet at the barriers
around the timed region and in the max-over-ranks reduction of its time.

Reported on one JSON line (rank 0):
  value    images/s over all ranks, inputs resident in HBM, CUDA-graph replay
  e2e      the same through the host API: pinned-host input upload, graph
           replay and the softmax download every step (copies overlapped
           with compute by double buffering), device-timed
  roofline the dominant kernel class vs the measured HBM peak
  cpu_baseline  the reference scheduler semantics on the CPU oracle, bounded
           sample, host cores
  --impl reference times that CPU path alone (the reference arm).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MobileNetV2 fp32 images/sec"
UNIT = "images/s"
# Other configs of the same hot path, --model selects.
METRICS = {
    "mobilenet_v2": ("MobileNetV2 fp32 images/sec", "images/s"),
    "efficientnet_lite0": ("EfficientNet-Lite0 fp32 images/sec", "images/s"),
    "resnet50": ("ResNet-50 fp32 images/sec (HLO path)", "images/s"),
    "bert": ("BERT-base encoder fp32 sequences/sec (HLO path, seq 128)", "sequences/s"),
    "tinyllama": ("TinyLlama-1.1B fp32 greedy tokens/sec (prompt 32, 20 new tokens, KV cache)",
                  "tokens/s"),
}
DEFAULT_BATCH = {"mobilenet_v2": 256, "efficientnet_lite0": 64, "resnet50": 256, "bert": 32,
                 "tinyllama": 1}
LLAMA_PROMPT, LLAMA_NEW = 32, 20


def build_model(name: str, batch: int, graph, seed_rank: int, unfused: bool = False):
    """(executor, host input) for a config; inputs are this rank's shard.
    unfused: the CNN step without the fused depthwise->projection kernel and
    with the CUDA-core stem (the kernels the fused path replaces)."""
    from spirv_inference_b200 import nets, nets_hlo
    from spirv_inference_b200.sharding import shard_seed
    if name in ("mobilenet_v2", "efficientnet_lite0"):
        from spirv_inference_b200.executor import CnnExecutor
        model = nets.MODELS[name](seed=0)
        ex = CnnExecutor(model, batch=batch, graph=graph, fuse_dw_project=not unfused,
                         tc_stem=not unfused)
        return ex, nets.make_input(model, batch, seed=shard_seed(1000, seed_rank))
    from spirv_inference_b200.executor_hlo import HloExecutor
    if name == "resnet50":
        g = nets_hlo.resnet50(seed=0, batch=batch)
        x = nets_hlo.make_image_batch(batch, seed=shard_seed(1000, seed_rank))
    else:
        g = nets_hlo.bert_encoder(seed=0, batch=batch, seq=128)
        rng = np.random.default_rng(shard_seed(1000, seed_rank))
        x = nets_hlo.bert_embed(0, rng.integers(0, 30522, (batch, 128)))
    return HloExecutor(g, graph=graph), x


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.rows: list[list[str]] = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.device),
                                      f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits"],
                                     capture_output=True, text=True, timeout=5).stdout
                for line in out.strip().splitlines():
                    self.rows.append([c.strip() for c in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for i, n in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.rows)}


def reference_pass(name: str, batch: int):
    """One pass of the reference executor semantics on the CPU oracle:
    the TFLite scheduler lowering (lowering.run_graph) or the HLO executor
    lowering (hlo.run_hlo), with the oracle as the kernel boundary."""
    from oracle import oracle
    from spirv_inference_b200 import hlo, lowering, nets, nets_hlo
    if name in ("mobilenet_v2", "efficientnet_lite0"):
        model = nets.MODELS[name](seed=0)
        x = nets.make_input(model, batch, seed=4321)
        return lambda: lowering.run_graph(model, x, oracle.run_kernel)
    if name == "resnet50":
        g = nets_hlo.resnet50(seed=0, batch=batch)
        feeds = {g.inputs[0]: nets_hlo.make_image_batch(batch, seed=4321)}
    else:
        g = nets_hlo.bert_encoder(seed=0, batch=batch, seq=128)
        ids = np.random.default_rng(4321).integers(0, 30522, (batch, 128))
        feeds = {g.inputs[0]: nets_hlo.bert_embed(0, ids)}
    return lambda: hlo.run_hlo(g, feeds, oracle.run_kernel)


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), for the baseline lines."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_baseline(name: str, seconds: float = 10.0, max_images: int = 64) -> dict:
    """The reference semantics on the CPU oracle (OpenMP over all host
    cores), one image / sequence per pass, until `seconds` have elapsed."""
    from oracle import oracle
    oracle.use_all_host_cores()
    step = reference_pass(name, 1)
    step()  # warm
    n, t0 = 0, time.perf_counter()
    while n < max_images and (time.perf_counter() - t0) < seconds:
        step()
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
            "cpu": cpu_model(),
            "sample": f"{n} single-{'sequence' if name == 'bert' else 'image'} {name} passes "
                      f"through the reference executor semantics on the C++ oracle ({dt:.1f} s)"}


def dist_setup():
    from spirv_inference_b200.sharding import dist_env
    return dist_env()


def run_reference(args) -> None:
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    from oracle import oracle
    global METRIC, UNIT
    METRIC, UNIT = METRICS[args.model]
    oracle.use_all_host_cores()
    per_step = args.ref_images
    step = reference_pass(args.model, per_step)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    v = per_step * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded U[-1,1] input, seeded He-normal weights)",
        "config": _ref_config(args, world),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
                         "cpu": cpu_model(),
                         "sample": f"{per_step} image(s) per step through the reference "
                                   "scheduler lowering (scheduler.rs semantics) on the C++ "
                                   "restatement of the reference kernels"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


_WORKLOADS = {
    "mobilenet_v2": "mobilenet_v2 224x224x3 fp32 NHWC inference",
    "efficientnet_lite0": "efficientnet_lite0 224x224x3 fp32 NHWC inference",
    "resnet50": "resnet50 v1.5 224x224x3 fp32 NHWC inference (HLO graph)",
    "bert": "bert-base encoder fp32, seq 128 (HLO graph)",
}


def _config(args, world) -> dict:
    l2 = ("step working set larger than L2 (fp32 weights ~440 MB read every step, plus "
          "activations)" if args.model == "bert" else
          "inputs larger than L2 (each step reads a >126 MB input and writes ~GBs of "
          "activations)")
    return {"workload": f"{_WORKLOADS.get(args.model, args.model)}, batch {args.batch} per GPU",
            "batch_per_gpu": args.batch, "global_batch": args.batch * world,
            "parallelism": f"dp{world} (batch-sharded replicas, no collective)",
            "l2": l2, "cuda_graph": True,
            "kernels": ("unfused (depthwise and projection as separate kernels, CUDA-core stem)"
                        if getattr(args, "unfused", False) else
                        "fused depthwise->projection, tensor-core stem")}


def _ref_config(args, world) -> dict:
    """The reference arm's own configuration: the same model and image size,
    but a reduced batch of --ref-images images per step, reported as a
    per-image rate (batch 256 of the CPU path would take minutes per step)."""
    unit = "sequences" if args.model == "bert" else "images"
    return {"workload": f"{_WORKLOADS.get(args.model, args.model)}, reduced batch: "
                        f"{args.ref_images} {unit} per step (batch {args.batch} impractical "
                        f"on the CPU path), per-{unit[:-1]} rate",
            "batch_per_step": args.ref_images, "global_batch": args.ref_images,
            "parallelism": "host cores of rank 0 (OpenMP over outputs)",
            "cuda_graph": False}


def run_dry(args) -> None:
    """The multi-rank plumbing of run_spx without a GPU (CPU tests): gloo
    process group, barrier, MAX over ranks of a stand-in per-rank step time
    (1 + rank ms), whole-job throughput, one JSON line from rank 0."""
    import torch.distributed as dist
    from spirv_inference_b200.sharding import max_over_ranks, throughput
    world, rank, _ = dist_setup()
    if world > 1:
        dist.init_process_group("gloo")
        dist.barrier()
    ms = max_over_ranks(1.0 + rank)
    if world > 1:
        dist.barrier()
    if rank == 0:
        print(json.dumps({"metric": METRICS[args.model][0], "value": throughput(args.batch, world, ms),
                          "unit": METRICS[args.model][1], "n_gpus": world, "ms_per_step": ms,
                          "config": _config(args, world), "dry_run": True}), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_spx(args) -> None:
    import torch

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from spirv_inference_b200.graph import Graph

    global METRIC, UNIT
    METRIC, UNIT = METRICS[args.model]
    B = args.batch
    stream = torch.cuda.Stream()  # a real stream: the legacy default stream cannot be captured
    torch.cuda.set_stream(stream)
    g = Graph(local, stream=stream.cuda_stream)
    ex, x = build_model(args.model, B, g, rank, unfused=args.unfused)  # this rank's shard
    g.upload(ex.input, x)
    ex.capture()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    from spirv_inference_b200.sharding import max_over_ranks as _mor, shard_seed, throughput

    def max_over_ranks(v: float) -> float:
        return _mor(v, device="cuda")

    # ---- device-resident throughput (value) ----
    for _ in range(max(args.warmup, 3)):
        ex.run()
    barrier()
    g.reset_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            ex.run()
        e1.record(stream)
        torch.cuda.synchronize()
    launches = g.launch_count
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    barrier()
    value = throughput(B, world, ms)

    # ---- per-kernel timing of one eager pass (roofline) ----
    costs = ex.op_costs()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(costs) + 1)]
    reps = 3
    times = np.zeros(len(costs))
    for _ in range(reps):
        evs[0].record(stream)
        for i in range(len(costs)):
            ex.record_op(i)
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
        times += np.array([evs[i].elapsed_time(evs[i + 1]) for i in range(len(costs))])
    times /= reps
    peaks = _peaks()
    classes: dict[str, dict] = {}
    for c, t in zip(costs, times):
        k = c["label"]
        d = classes.setdefault(k, {"ms": 0.0, "bytes": 0, "flops": 0, "launches": 0})
        d["ms"] += t
        d["bytes"] += c["bytes"]
        d["flops"] += c["flops"]
        d["launches"] += 1
    total_ms = float(times.sum())
    # fp32-accurate tensor rate for FLOP ceilings: 3xTF32 issues three tf32
    # MMAs per fp32 product and dense tf32 runs at half the measured bf16 rate.
    fp32_tc = peaks["bf16_tflops"] / 2.0 / 3.0
    per_class = {}
    for k, d in sorted(classes.items(), key=lambda kv: -kv[1]["ms"]):
        t_mem = d["bytes"] / (peaks["hbm_gbs"] * 1e9) * 1e3
        per_class[k] = {"share": round(d["ms"] / total_ms, 4), "ms": round(d["ms"], 4),
                        "launches": d["launches"],
                        "achieved_gbs": round(d["bytes"] / (d["ms"] / 1e3) / 1e9, 1),
                        "achieved_tflops": round(d["flops"] / (d["ms"] / 1e3) / 1e12, 2),
                        "hbm_roof_frac": round(t_mem / d["ms"], 4)}
    if args.per_op:
        # one line per recorded kernel on stderr: label, output shape, us, GB/s
        plan = getattr(ex, "_plan", None) or [(c["kind"], {}) for c in costs]
        for (kind, pl), c, t in zip(plan, costs, times):
            y = pl.get("y")
            shape = tuple(y.shape) if y is not None else ()
            print(f"per_op {c['label']:12s} {str(shape):24s} {t * 1000:9.1f} us "
                  f"{c['bytes'] / (t / 1e3) / 1e9:8.0f} GB/s", file=sys.stderr)
    top = max(classes, key=lambda k: classes[k]["ms"])
    d = classes[top]
    per_launch_bytes = d["bytes"] / d["launches"]
    per_launch_s = d["ms"] / d["launches"] / 1e3
    ach = per_launch_bytes / per_launch_s / 1e9
    # DRAM traffic per launch, from an ncu --set full capture of this kernel
    # (expand 16 -> 96 at batch 64): dram read + write = 301.1 MB
    # against 359.6 MB algorithmic for that launch (ratio 0.837; the balance
    # was still in L2 when the kernel ended).  Scaled to this class's average
    # algorithmic bytes per launch; only meaningful for the GEMM class.
    traffic = round(per_launch_bytes * (301.1 / 359.6)) if top == "conv1x1" else None
    traffic_source = ("ncu capture of one gemm_tc launch (expand 16->96, batch 64), dram bytes / "
                      "algorithmic bytes scaled to the class average")
    if top == "dw_project":
        # dram read + write of the 17 dw_project launches of one MobileNetV2
        # step at batch 64 (one ncu pass, dram__bytes_read/write.sum):
        # 1,066.0 MB against 1,167.7 MB algorithmic.  Reads are 1.0015 of the
        # algorithmic reads (halo overlap served by L2); writes read low
        # because outputs still in L2 when a serialised launch ends are not
        # counted.  Scaled to this class's average algorithmic bytes.
        traffic = round(per_launch_bytes * (1066.0 / 1167.7))
        traffic_source = ("ncu dram__bytes_read/write.sum over the 17 dw_project launches of a "
                          "batch-64 step, ratio to their algorithmic bytes (0.913; reads 1.0015) "
                          "scaled to the class average")
    # The dominant class is tensor-bound when its FLOPs per byte exceed the
    # ridge of the fp32-accurate tensor rate.
    ridge = fp32_tc * 1e12 / (peaks["hbm_gbs"] * 1e9)
    if d["bytes"] and d["flops"] / d["bytes"] > ridge:
        ach_tf = d["flops"] / (d["ms"] / 1e3) / 1e12
        roofline = {"bound": "tensor", "achieved": round(ach_tf, 2), "peak": round(fp32_tc, 1),
                    "unit": "TFLOP/s", "frac": round(ach_tf / fp32_tc, 4), "traffic": None,
                    "kernel": top, "peak_source": peaks["source"] + " (bf16 / 2 / 3: the "
                    "3xTF32 fp32-accurate ceiling)",
                    "note": "achieved = fp32 FLOPs of the class / its CUDA-event time in one "
                            "eager pass"}
    else:
        roofline = {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "frac": round(ach / peaks["hbm_gbs"], 4), "traffic": traffic,
                    "traffic_source": traffic_source,
                    "kernel": top, "peak_source": peaks["source"],
                    "note": "achieved = algorithmic bytes per launch / CUDA-event launch time, "
                            "averaged over the class's launches in one eager pass"}
    sum_roof_ms = sum(max(c["bytes"] / (peaks["hbm_gbs"] * 1e9),
                          c["flops"] / (fp32_tc * 1e12)) * 1e3 for c in costs)

    # ---- end to end through the host API (pinned host in/out, overlapped) ----
    copy = torch.cuda.Stream()
    host_in = [torch.from_numpy(x.copy()).pin_memory() for _ in range(2)]
    staging = [torch.empty(x.shape, dtype=torch.float32, device="cuda") for _ in range(2)]
    out_elems = ex.output.size
    host_out = torch.empty(out_elems, dtype=torch.float32).pin_memory()
    up_done = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    n_in = x.nbytes

    def e2e_steps(k):
        for i in range(k):
            s = i % 2
            with torch.cuda.stream(copy):
                if i >= 2:
                    copy.wait_event(free[s])
                staging[s].copy_(host_in[s], non_blocking=True)
                up_done[s].record(copy)
            stream.wait_event(up_done[s])
            g.copy_d2d(ex.input, staging[s].data_ptr(), n_in)
            free[s].record(stream)
            ex.run()
            g.download_async(host_out.data_ptr(), ex.output, out_elems * 4)

    e2e_steps(max(args.warmup, 3))
    barrier()
    e0.record(stream)
    e2e_steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    barrier()
    e2e_value = throughput(B, world, e2e_ms)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded U[-1,1] input, seeded He-normal weights, BN folded)",
            "config": _config(args, world),
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": int(n_in),
                    "d2h_bytes_per_step": int(out_elems * 4), "ms_per_step": round(e2e_ms, 4)},
            "roofline": roofline,
            "per_kernel_class": per_class,
            "sum_of_op_rooflines_ms": round(sum_roof_ms, 4),
            "eager_pass_ms": round(total_ms, 4),
            "gpu_launches": int(launches),
            "kernels_per_step": ex.kernels_per_run,
            "clocks": clk.summary(),
        }
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    ex.close()
    if rank == 0:
        # Timed after the process group is gone: NCCL's polling threads and
        # the other ranks no longer compete for the host cores.
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.model, seconds=args.cpu_seconds)
        print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# TinyLlama decode: greedy generation of 20 tokens
# after a 32-token prompt, batch 1 or 64, tensor-parallel over the N GPUs.

def _llama_config(args, world) -> dict:
    return {"workload": f"tinyllama 1.1B fp32 greedy decode, batch {args.batch}, prompt "
                        f"{LLAMA_PROMPT}, {LLAMA_NEW} new tokens (1 prefill + "
                        f"{LLAMA_NEW - 1} cached decode steps)",
            "global_batch": args.batch, "seq_len": LLAMA_PROMPT + LLAMA_NEW - 1,
            "parallelism": f"tp{world}" + (" (NCCL all-reduce x2 per layer)" if world > 1 else ""),
            "l2": "weights (4.4 GB / tp degree) larger than L2: every step streams them",
            "cuda_graph": world == 1}


def _llama_weights():
    from spirv_inference_b200 import llama
    return llama.make_weights(llama.TINYLLAMA, seed=0, generator="torch")


def llama_cpu_step(W, batch: int = 1, n_tokens: int = 1):
    """The reference's decode loop on the CPU (oracle/llama_ref.generate_full:
    full 64-position re-computation per token), numpy / BLAS on all host
    cores.  One call generates `n_tokens` tokens for each of `batch` prompts."""
    from oracle import llama_ref
    from spirv_inference_b200 import llama
    cfg = llama.TINYLLAMA
    rope = llama.rope_tables(cfg, cfg.max_seq)
    prompt = llama.make_prompt(cfg, batch, LLAMA_PROMPT, seed=4321)
    return lambda: [llama_ref.generate_full(cfg, W, prompt[b], n_tokens, rope)
                    for b in range(batch)]


def llama_cpu_baseline(W, seconds: float) -> dict:
    step = llama_cpu_step(W, 1, 1)
    n, t0 = 0, time.perf_counter()
    while n < 1 or (time.perf_counter() - t0) < seconds:
        step()
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port", "cpu": cpu_model(),
            "sample": f"{n} greedy token(s) of one sequence through the reference's decode loop "
                      f"(full 64-position llama_step per token, numpy fp32 BLAS; {dt:.1f} s)"}


def run_llama_reference(args) -> None:
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    W = _llama_weights()
    step = llama_cpu_step(W, 1, 1)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    v = args.steps / dt
    UNIT_ = METRICS["tinyllama"][1]
    print(json.dumps({
        "impl": "reference", "metric": METRICS["tinyllama"][0], "value": v, "unit": UNIT_,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * dt / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded uniform prompt ids, seeded N(0,0.02) weights)",
        "config": _llama_config(args, world),
        "cpu_baseline": {"value": v, "unit": UNIT_, "cores": os.cpu_count(), "kind": "port", "cpu": cpu_model(),
                         "sample": "1 greedy token of one sequence per step through the "
                                   "reference's decode loop (full 64-position re-computation, "
                                   "numpy fp32 BLAS)"},
        "e2e": {"value": v, "unit": UNIT_, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_llama_spx(args) -> None:
    import torch

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from spirv_inference_b200 import llama
    from spirv_inference_b200.sharding import max_over_ranks as _mor

    B = args.batch
    METRIC_, UNIT_ = METRICS["tinyllama"]
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    W = _llama_weights()
    dec = llama.LlamaDecoder(llama.TINYLLAMA, W, B, LLAMA_PROMPT, LLAMA_NEW, device=local,
                             stream=stream.cuda_stream, rank=rank, world=world)
    prompt = llama.make_prompt(llama.TINYLLAMA, B, LLAMA_PROMPT, seed=4321)
    dec.upload_prompt(prompt)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    for _ in range(max(args.warmup, 3)):
        dec.run()
    barrier()
    g = dec.g
    g.reset_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            dec.run()
        e1.record(stream)
        torch.cuda.synchronize()
    launches = g.launch_count
    ms = _mor(e0.elapsed_time(e1), device="cuda") / args.steps
    barrier()
    value = B * LLAMA_NEW / (ms / 1e3)
    toks = dec.tokens()

    # Per-op timing of one eager prefill + decode step (events between ops).
    marks = []

    def mark(label, nbytes, flops):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        marks.append((label, nbytes, flops, ev))

    cap = dec.capture
    dec.capture = False
    decode_classes: dict[str, dict] = {}
    prefill_ms = decode_ms = 0.0
    for phase in ("prefill", "decode"):
        marks.clear()
        start = torch.cuda.Event(enable_timing=True)
        if phase == "prefill":
            dec.g.zero(dec.state)
            dec._host_pos = 0
            start.record(stream)
            dec._mark = mark
            dec._forward(dec.prompt_ids, LLAMA_PROMPT)
        else:
            for _ in range(8):          # decode at a mid-sequence position
                dec._forward(dec.ids, 1)
            start.record(stream)
            dec._mark = mark
            dec._forward(dec.ids, 1)
        dec._mark = None
        torch.cuda.synchronize()
        prev = start
        for label, nb, fl, ev in marks:
            t = prev.elapsed_time(ev)
            prev = ev
            if phase == "decode":
                d = decode_classes.setdefault(label, {"ms": 0.0, "bytes": 0.0, "flops": 0.0,
                                                      "launches": 0})
                d["ms"] += t
                d["bytes"] += nb
                d["flops"] += fl
                d["launches"] += 1
        total = start.elapsed_time(marks[-1][3])
        if phase == "prefill":
            prefill_ms = total
        else:
            decode_ms = total
    dec.capture = cap
    peaks = _peaks()
    lin = decode_classes["linear"]
    per_launch_bytes = lin["bytes"] / lin["launches"]
    ach = lin["bytes"] / (lin["ms"] / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(ach / peaks["hbm_gbs"], 4), "traffic": None,
                "kernel": "linear (gemm_rows / swiglu_linear at batch <= 8, tensor-core GEMM "
                          "above) in one eager decode step",
                "bytes_per_launch": round(per_launch_bytes),
                "peak_source": peaks["source"],
                "note": "achieved = algorithmic bytes (weights + activations) per launch / "
                        "CUDA-event time, averaged over the step's projection launches"}
    per_class = {k: {"ms": round(d["ms"], 4), "launches": d["launches"],
                     "share": round(d["ms"] / decode_ms, 4),
                     "achieved_gbs": round(d["bytes"] / (d["ms"] / 1e3) / 1e9, 1)}
                 for k, d in sorted(decode_classes.items(), key=lambda kv: -kv[1]["ms"])}
    step_bytes = sum(d["bytes"] for d in decode_classes.values())

    # End to end through the public API: pinned prompt upload, generation,
    # token download, every step.
    host_prompt = torch.from_numpy(prompt.copy()).pin_memory()
    host_tok = torch.empty((LLAMA_NEW, B), dtype=torch.int32).pin_memory()

    def e2e_step():
        g.upload_async(dec.prompt_ids, host_prompt.data_ptr(), prompt.nbytes)
        dec.run()
        g.download_async(host_tok.data_ptr(), dec.hist, host_tok.numel() * 4)

    for _ in range(3):
        e2e_step()
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = _mor(e0.elapsed_time(e1), device="cuda") / args.steps
    barrier()
    if rank == 0:
        line = {
            "metric": METRIC_, "value": round(value, 2), "unit": UNIT_, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded uniform prompt ids, seeded N(0,0.02) weights)",
            "config": _llama_config(args, world),
            "e2e": {"value": round(B * LLAMA_NEW / (e2e_ms / 1e3), 2), "unit": UNIT_,
                    "h2d_bytes_per_step": int(prompt.nbytes),
                    "d2h_bytes_per_step": int(host_tok.numel() * 4),
                    "ms_per_step": round(e2e_ms, 4)},
            "roofline": roofline,
            "prefill_ms": round(prefill_ms, 4), "decode_step_ms_eager": round(decode_ms, 4),
            "decode_step_bytes": round(step_bytes),
            "decode_step_roofline_ms": round(step_bytes / (peaks["hbm_gbs"] * 1e9) * 1e3, 4),
            "per_kernel_class_decode": per_class,
            "gpu_launches": int(launches),
            "tokens_first_sequence": toks[0].tolist(),
            "clocks": clk.summary(),
        }
    # Free the decoder (and its captured CUDA graph, which holds NCCL work on
    # the communicator) before the process group goes away.
    torch.cuda.synchronize()
    dec.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = llama_cpu_baseline(W, args.cpu_seconds)
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["spx", "reference"], default="spx")
    ap.add_argument("--model", default="mobilenet_v2", choices=list(METRICS))
    ap.add_argument("--batch", type=int, default=None, help="per-GPU batch (config default)")
    ap.add_argument("--ref-images", type=int, default=2, help="images per reference-arm step")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--per-op", action="store_true",
                    help="print each kernel's eager-pass time to stderr")
    ap.add_argument("--unfused", action="store_true",
                    help="CNN step without the fused depthwise->projection and tensor-core stem")
    ap.add_argument("--dry-run", action="store_true",
                    help="exercise the rank plumbing on CPU (tests); no GPU work, no timing")
    args = ap.parse_args()
    if args.batch is None:
        args.batch = DEFAULT_BATCH[args.model]
    if args.dry_run:
        run_dry(args)
    elif args.model == "tinyllama":
        run_llama_reference(args) if args.impl == "reference" else run_llama_spx(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_spx(args)


if __name__ == "__main__":
    main()
