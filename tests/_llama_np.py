"""numpy restatement of the device's tensor-parallel TinyLlama pass, built on
the same per-rank packing (llama.pack_layer / tp_shard): each rank computes
its column-parallel Q/K/V, gate/up and vocab slice and its row-parallel
o_proj / down_proj partial; `reduce` sums the partials over ranks."""
import numpy as np

from oracle import llama_ref as R
from spirv_inference_b200 import llama


def tp_generate(cfg, W, prompt, n_new, world, reduce=None):
    """Greedy tokens for one prompt with `world` simulated ranks (or, with
    `reduce`, as one real rank whose partial sums `reduce` all-reduces)."""
    rope = llama.rope_tables(cfg, cfg.max_seq)
    ranks = range(world) if reduce is None else [reduce.rank]
    sh = {r: llama.tp_shard(cfg, r, world) for r in ranks}
    packed = {r: [llama.pack_layer(cfg, L, sh[r]) for L in W["layers"]] for r in ranks}
    caches = {r: [([], []) for _ in W["layers"]] for r in ranks}
    D = cfg.head_dim
    allreduce = (lambda parts: sum(parts.values())) if reduce is None else \
        (lambda parts: reduce(next(iter(parts.values()))))

    def block(ids, pos0):
        T = len(ids)
        x = W["embed"][ids].astype(np.float32)
        cos, sin = rope[0][pos0:pos0 + T], rope[1][pos0:pos0 + T]
        for li in range(cfg.layers):
            parts = {}
            for r in ranks:
                P, s = packed[r][li], sh[r]
                h = R.rms_norm(x, np.float32(1.0), cfg.eps)    # gain folded into wqkv
                qkv = h @ P["wqkv"].T
                q = qkv[:, :s.nq * D].reshape(T, s.nq, D).transpose(1, 0, 2)
                k = qkv[:, s.nq * D:(s.nq + s.nkv) * D].reshape(T, s.nkv, D).transpose(1, 0, 2)
                v = qkv[:, (s.nq + s.nkv) * D:].reshape(T, s.nkv, D).transpose(1, 0, 2)
                q = q * cos + R.rotate_half(q) * sin
                k = k * cos + R.rotate_half(k) * sin
                kc, vc = caches[r][li]
                kc.append(k)
                vc.append(v)
                K = np.repeat(np.concatenate(kc, 1), s.nq // s.nkv, 0)
                V = np.repeat(np.concatenate(vc, 1), s.nq // s.nkv, 0)
                qpos = pos0 + np.arange(T)[:, None]
                mask = np.where(np.arange(K.shape[1])[None, :] > qpos, np.float32(-1e9),
                                np.float32(0)).astype(np.float32)
                att = R.softmax((q @ K.transpose(0, 2, 1)) * np.float32(0.125) + mask) @ V
                parts[r] = att.transpose(1, 0, 2).reshape(T, s.nq * D) @ P["wo"].T
            x = x + allreduce(parts)
            parts = {}
            for r in ranks:
                P, s = packed[r][li], sh[r]
                h = R.rms_norm(x, np.float32(1.0), cfg.eps)    # gain folded into wgu
                gu = h @ P["wgu"].T
                parts[r] = (R.silu(gu[:, :s.nf]) * gu[:, s.nf:]) @ P["wdown"].T
            x = x + allreduce(parts)
        h = R.rms_norm(x[-1:], np.float32(1.0), cfg.eps)
        best = None
        for r in (range(world) if reduce is None else [reduce.rank]):
            s = llama.tp_shard(cfg, r, world)
            lg = (h @ llama.pack_lm_head(cfg, W, s).T)[0]
            cand = (float(lg.max()), s.v0 + int(np.argmax(lg)))
            if reduce is not None:
                return reduce.argmax(cand)
            if best is None or cand[0] > best[0] or (cand[0] == best[0] and cand[1] < best[1]):
                best = cand
        return best[1]

    out = [block([int(t) for t in prompt], 0)]
    pos = len(prompt)
    for _ in range(n_new - 1):
        out.append(block([out[-1]], pos))
        pos += 1
    return np.array(out, np.int32)
