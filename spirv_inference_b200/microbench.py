"""Single-kernel timing for profiling: one library call on seeded operands,
timed with CUDA events on the launching stream (after warm-up).  Used to
produce the ncu captures of individual kernels; the model-level numbers come
from bench.py.

    python -m spirv_inference_b200.microbench gemm M N K [reps]
        y[M][N] = x[M][K] W^T + b with pre-split W (the linear / 1x1 path)
    python -m spirv_inference_b200.microbench conv3x3 n h ic oc [reps]
        3x3 stride-1 pad-1 NHWC convolution (implicit GEMM), pre-split OHWI W
    python -m spirv_inference_b200.microbench dwproj n h c stride cout residual [reps]
        fused 3x3 depthwise (ReLU6) -> 1x1 projection (+ residual)
"""
from __future__ import annotations

import sys

import numpy as np


def _time(run, stream, reps: int) -> float:
    import torch
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def main(argv: list[str]) -> None:
    import torch
    from spirv_inference_b200 import _lib
    from spirv_inference_b200.graph import Graph

    kind, args = argv[0], [int(a) for a in argv[1:]]
    rng = np.random.default_rng(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    with Graph(0, stream=stream.cuda_stream) as g:
        if kind == "gemm":
            M, N, K = args[:3]
            reps = args[3] if len(args) > 3 else 20
            da = g.tensor(rng.standard_normal((M, K)).astype(np.float32))
            dw = g.tensor((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
            db = g.tensor(rng.standard_normal(N).astype(np.float32))
            split = g.weights_split(dw)
            dc = g.alloc((M, N))
            ms = _time(lambda: g.gemm(da, dw, dc, m=M, n=N, k=K, a_strides=(0, K, 1),
                                      b_strides=(0, 1, K), c_strides=(0, N), bias=db,
                                      b_split=split), stream, reps)
            print(f"gemm {M}x{N}x{K}: {ms * 1e3:.1f} us, "
                  f"{2 * M * N * K / ms / 1e9:.1f} fp32 TFLOP/s")
        elif kind == "conv3x3":
            n, h, ic, oc = args[:4]
            reps = args[4] if len(args) > 4 else 20
            dx = g.tensor(rng.standard_normal((n, h, h, ic)).astype(np.float32))
            dw = g.tensor((rng.standard_normal((oc, 3, 3, ic)) / np.sqrt(9 * ic))
                          .astype(np.float32))
            db = g.tensor(rng.standard_normal(oc).astype(np.float32))
            split = g.weights_split(dw)
            dy = g.alloc((n, h, h, oc))
            ms = _time(lambda: g.conv2d_nhwc(dx, dw, db, dy, pad=(1, 1), w_split=split),
                       stream, reps)
            print(f"conv3x3 {n}x{h}x{h}x{ic}->{oc}: {ms * 1e3:.1f} us, "
                  f"{2 * n * h * h * oc * 9 * ic / ms / 1e9:.1f} fp32 TFLOP/s")
        elif kind == "dwproj":
            n, h, c, s, cout, res = args[:6]
            reps = args[6] if len(args) > 6 else 20
            oh = -(-h // s)
            pt = max((oh - 1) * s + 3 - h, 0) // 2
            dx = g.tensor(rng.uniform(0, 6, (n, h, h, c)).astype(np.float32))
            dwd = g.tensor(rng.uniform(-1, 1, (3, 3, c)).astype(np.float32))
            dbd = g.tensor(rng.uniform(-.1, .1, c).astype(np.float32))
            split = g.weights_split(g.tensor(
                (rng.uniform(-1, 1, (cout, c)) * np.sqrt(3 / c)).astype(np.float32)))
            dbp = g.tensor(rng.uniform(-.1, .1, cout).astype(np.float32))
            dy = g.alloc((n, oh, oh, cout))
            dr = g.tensor(rng.uniform(-1, 1, (n, oh, oh, cout)).astype(np.float32)) \
                if res else None
            ms = _time(lambda: g.dw_project_nhwc(dx, dwd, dbd, split, dbp, dy, stride=s,
                                                 pad=(pt, pt), act_dw=_lib.ACT_RELU6,
                                                 residual=dr), stream, reps)
            nbytes = 4 * (dx.size + dy.size * (2 if res else 1))
            print(f"dw_project {n}x{h}x{h}x{c} s{s} -> {cout}: {ms * 1e3:.1f} us, "
                  f"{nbytes / ms / 1e6:.0f} GB/s")
        else:
            raise SystemExit(__doc__)


if __name__ == "__main__":
    main(sys.argv[1:])
