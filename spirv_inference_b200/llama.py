"""TinyLlama-architecture greedy decode on the device, with a KV cache and
optional tensor parallelism.

The reference runs the `llama_step` graph (source/xla_hlo/tools/
export_llama.py:269-365: 22 x [RMSNorm, Q/K/V/O, RoPE, GQA attention,
RMSNorm, SwiGLU MLP], final RMSNorm, lm_head) once per generated token over
the whole padded 64-token window with a causal mask, and takes the argmax at
the last valid position (run_llama_spirv.py:190-260).  This runner computes
the same function with a KV cache:

* prefill: the P prompt tokens of every sequence go through the layers as
  one [B*P, hidden] block (tensor-core GEMMs); K/V of every position are
  appended to the per-layer cache; the lm_head runs on the last position.
* decode: one token per sequence per step ([B, hidden]): weight-streaming
  GEMMs for B <= 8 rows, the gate/up projection fused with SiLU * up,
  attention of the new token over the cache.  The step reads its token ids
  and position from device memory, so it is captured once as a CUDA graph
  and replayed.

Tensor parallelism (world > 1, one process per GPU, torch.distributed NCCL):
Q/K/V and gate/up are split by output column (heads / FFN columns), o_proj
and down_proj by input row; each row-parallel product is summed with one
all-reduce (2 per layer), rank 0 adding the residual; the lm_head is split
by vocabulary and the greedy token is a (value, index) argmax merged over
ranks.  With more ranks than kv heads, kv heads are replicated (rank r uses
kv head r * kv_heads // world).

Weights (seeded, N(0, 0.02); norm gains 1 + N(0, 0.02)) are generated in the
reference's shapes and argument order (export_llama.py:305-316, 360-361) and
packed at load time: projection matrices transposed to [out][in], Q|K|V and
gate|up concatenated.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from .graph import DeviceTensor, Graph


@dataclass(frozen=True)
class LlamaConfig:
    layers: int = 22
    hidden: int = 2048
    heads: int = 32
    kv_heads: int = 4
    head_dim: int = 64
    ffn: int = 5632
    vocab: int = 32000
    eps: float = 1e-5
    theta: float = 10000.0
    max_seq: int = 64          # the reference's window (export_llama.py: S = 64)


TINYLLAMA = LlamaConfig()
# A scaled-down configuration with the same structure (GQA 4:1, head_dim 64)
# for parity tests whose CPU reference must finish in seconds.
TINY_TEST = LlamaConfig(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=64, ffn=1376,
                        vocab=1000)


def make_weights(cfg: LlamaConfig, seed: int = 0, generator: str = "numpy") -> dict:
    """Seeded weights in the reference's shapes ([in, out] matrices).

    generator "numpy": PCG64 standard normals (parity tests); "torch": the
    multi-threaded torch CPU generator seeded with `seed` (the 1.1B-parameter
    benchmark model, where single-threaded numpy would take most of a
    minute)."""
    H, KV, F = cfg.hidden, cfg.kv_heads * cfg.head_dim, cfg.ffn
    if generator == "torch":
        import torch
        tg = torch.Generator().manual_seed(seed)

        def nrm(*shape):
            a = torch.randn(shape, generator=tg, dtype=torch.float32).numpy()
            a *= np.float32(0.02)
            return a
    else:
        rng = np.random.Generator(np.random.PCG64(seed))

        def nrm(*shape):
            a = rng.standard_normal(shape, dtype=np.float32)
            a *= np.float32(0.02)
            return a

    def gain(n):
        return (np.float32(1.0) + nrm(n)).astype(np.float32)

    embed = nrm(cfg.vocab, H)
    layers = []
    for _ in range(cfg.layers):
        layers.append({
            "ln": gain(H), "q": nrm(H, H), "k": nrm(H, KV), "v": nrm(H, KV), "o": nrm(H, H),
            "post_ln": gain(H), "gate": nrm(H, F), "up": nrm(H, F), "down": nrm(F, H),
        })
    return {"embed": embed, "layers": layers, "final_ln": gain(H), "lm_head": nrm(H, cfg.vocab)}


def make_prompt(cfg: LlamaConfig, batch: int, prompt_len: int = 32, seed: int = 7) -> np.ndarray:
    """Prompt ids uniform over the vocabulary, [batch, prompt_len] int32."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(0, cfg.vocab, size=(batch, prompt_len), dtype=np.int64).astype(np.int32)


def rope_tables(cfg: LlamaConfig, seq: int) -> tuple[np.ndarray, np.ndarray]:
    """cos / sin [seq, head_dim] as run_llama_spirv.py:87-97 computes them."""
    D = cfg.head_dim
    inv_freq = 1.0 / (cfg.theta ** (np.arange(0, D, 2, dtype=np.float32) / D))
    pos = np.arange(seq, dtype=np.float32)
    freqs = np.outer(pos, inv_freq)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


@dataclass(frozen=True)
class TpShard:
    """Which heads / columns rank `rank` of `world` owns."""
    rank: int
    world: int
    q0: int
    nq: int
    kv0: int
    nkv: int
    f0: int
    nf: int
    v0: int
    nv: int


def tp_shard(cfg: LlamaConfig, rank: int, world: int) -> TpShard:
    if cfg.heads % world or cfg.ffn % world or cfg.vocab % world:
        raise ValueError(f"tensor parallel degree {world} does not divide heads / ffn / vocab")
    nq = cfg.heads // world
    if world <= cfg.kv_heads:
        if cfg.kv_heads % world:
            raise ValueError("kv heads not divisible by the tensor parallel degree")
        nkv = cfg.kv_heads // world
        kv0 = rank * nkv
    else:
        if world % cfg.kv_heads:
            raise ValueError("tensor parallel degree not a multiple of the kv heads")
        nkv, kv0 = 1, rank * cfg.kv_heads // world
    nf, nv = cfg.ffn // world, cfg.vocab // world
    return TpShard(rank, world, rank * nq, nq, kv0, nkv, rank * nf, nf, rank * nv, nv)


def pack_layer(cfg: LlamaConfig, lw: dict, sh: TpShard) -> dict:
    """Per-rank device layouts: [out][in] matrices, Q|K|V and gate|up fused.

    The RMSNorm gains are folded into the projections they feed
    (rms_norm(x, g) @ W = (x / rms(x)) @ (g[:, None] * W)), so the device
    normalises without a gain, inside the projection for few rows."""
    D = cfg.head_dim
    qs = slice(sh.q0 * D, (sh.q0 + sh.nq) * D)
    ks = slice(sh.kv0 * D, (sh.kv0 + sh.nkv) * D)
    fs = slice(sh.f0, sh.f0 + sh.nf)
    wqkv = np.concatenate([lw["q"][:, qs].T, lw["k"][:, ks].T, lw["v"][:, ks].T], axis=0)
    wgu = np.concatenate([lw["gate"][:, fs].T, lw["up"][:, fs].T], 0)
    return {
        "wqkv": np.ascontiguousarray(wqkv * lw["ln"][None, :]),      # [(nq + 2 nkv) D][H]
        "wo": np.ascontiguousarray(lw["o"][qs, :].T),                # [H][nq D]
        "wgu": np.ascontiguousarray(wgu * lw["post_ln"][None, :]),   # [2 nf][H]
        "wdown": np.ascontiguousarray(lw["down"][fs, :].T),          # [H][nf]
    }


def pack_lm_head(cfg: LlamaConfig, W: dict, sh: TpShard) -> np.ndarray:
    """This rank's vocabulary rows of the lm_head, [nv][H], final gain folded."""
    return np.ascontiguousarray(W["lm_head"][:, sh.v0:sh.v0 + sh.nv].T * W["final_ln"][None, :])


class _CudaArray:
    """Wraps a device pointer for torch.as_tensor (__cuda_array_interface__)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


class LlamaDecoder:
    """Greedy generation for a fixed batch on one device (or one TP rank).

    generate(prompt [B, P] int32, n_new) -> tokens [B, n_new] int32; the first
    token comes from the prefill, the rest from cached decode steps.
    """

    def __init__(self, cfg: LlamaConfig, weights: dict, batch: int, prompt_len: int,
                 n_new: int, *, device: int = 0, stream: int | None = None,
                 rank: int = 0, world: int = 1, group=None, capture: bool = True,
                 peer_allreduce: bool = False):
        self.cfg, self.B, self.P, self.n_new = cfg, batch, prompt_len, n_new
        if prompt_len + n_new - 1 > cfg.max_seq:
            raise ValueError(f"prompt {prompt_len} + {n_new} new tokens exceed max_seq "
                             f"{cfg.max_seq}")
        self.rank, self.world, self.group = rank, world, group
        self.sh = tp_shard(cfg, rank, world)
        self.g = Graph(device, stream=stream)
        g, sh = self.g, self.sh
        H, D = cfg.hidden, cfg.head_dim
        self.nqkv = (sh.nq + 2 * sh.nkv) * D
        # Weights.
        self.embed = g.tensor(weights["embed"])
        self.lm_head = g.tensor(pack_lm_head(cfg, weights, sh))
        self.layers = []
        for lw in weights["layers"]:
            pk = pack_layer(cfg, lw, sh)
            self.layers.append({k: g.tensor(v) for k, v in pk.items()})
        # Tensor-core copies (hi / lo tf32 parts) of every projection: blocks of
        # more than 8 rows (prefill, batch > 8) stream these instead of
        # splitting the fp32 weights on chip; single rows keep the fp32 copy.
        self._split = {}
        for t in [self.lm_head] + [w for L in self.layers for w in L.values()]:
            self._split[t.ptr] = g.weights_split(t)
        cos, sin = rope_tables(cfg, cfg.max_seq)
        self.cos, self.sin = g.tensor(cos), g.tensor(sin)
        # Activations (sized for the prefill block).
        M = batch * prompt_len
        self.h = g.alloc((M, H))
        self.qkv = g.alloc((M, self.nqkv))
        self.q = g.alloc((M, sh.nq * D))
        self.att = g.alloc((M, sh.nq * D))
        self.gu = g.alloc((M, 2 * sh.nf))
        self.mlp = g.alloc((M, sh.nf))
        self.logits = g.alloc((batch, sh.nv))
        self.kc = [g.alloc((batch, sh.nkv, cfg.max_seq, D)) for _ in range(cfg.layers)]
        self.vc = [g.alloc((batch, sh.nkv, cfg.max_seq, D)) for _ in range(cfg.layers)]
        self.keys = g.alloc((batch,), np.uint64)
        g.zero(self.keys)
        self.prompt_ids = g.alloc((M,), np.int32)
        self.ids = g.alloc((batch,), np.int32)
        self.hist = g.alloc((n_new, batch), np.int32)
        self.state = g.alloc((2,), np.int32)
        self._torch_bufs = []
        if world > 1:
            import torch
            dev = torch.device("cuda", device)
            self.x_a = self._torch_buf(torch.empty((M, H), device=dev))
            self.x_b = self._torch_buf(torch.empty((M, H), device=dev))
            self.packed = self._torch_buf(torch.empty((batch, 2), device=dev))
            self.packed_all = self._torch_buf(torch.empty((world, batch, 2), device=dev))
        else:
            self.x_a, self.x_b = g.alloc((M, H)), g.alloc((M, H))
        # Optionally, small all-reduces (decode steps; prefill when it is small
        # too) go over peer memory: one kernel per all-reduce instead of an
        # NCCL call.  Measured on 2 B200s it matches NCCL inside a captured
        # step (b1 678 vs 708 tok/s, b64 15.6k vs 15.8k), so NCCL stays the
        # default.
        self.peer_ar = None
        self._ar_slot = 0
        if world > 1 and peer_allreduce:
            from .comm import PeerAllReduce
            self.peer_ar = PeerAllReduce(device, rank, world,
                                         min(M, 256) * H * 4, group=group)
        self.capture = capture
        self._captured = False
        self._mark = None      # optional callback(label, bytes, flops) after each op
        self._host_pos = 0

    # -- helpers -----------------------------------------------------------
    def _torch_buf(self, t) -> DeviceTensor:
        self._torch_bufs.append(t)
        return DeviceTensor(t.data_ptr(), tuple(t.shape), np.dtype(np.float32), self.g)

    def _torch_view(self, t: DeviceTensor, rows: int, cols: int):
        import torch
        return torch.as_tensor(_CudaArray(t.ptr, (rows, cols), "<f4"),
                               device=torch.device("cuda", self.g.device))

    def _all_reduce(self, t: DeviceTensor, rows: int) -> None:
        import torch.distributed as dist
        dist.all_reduce(self._torch_view(t, rows, self.cfg.hidden), group=self.group)

    def _note(self, label: str, nbytes: float, flops: float = 0.0) -> None:
        if self._mark is not None:
            self._mark(label, nbytes, flops)

    def _linear(self, a: DeviceTensor, lda: int, w: DeviceTensor, m: int, c: DeviceTensor,
                residual: DeviceTensor | None = None, label: str = "linear"):
        n, k = w.shape
        split = self._split.get(w.ptr) if m > 8 else None
        self.g.gemm(a, w, c, m=m, n=n, k=k, a_strides=(0, lda, 1), b_strides=(0, 1, k),
                    c_strides=(0, n), residual=residual, b_split=split)
        wb = 8.0 if split else 4.0
        self._note(label, wb * n * k + 4.0 * (m * k + m * n * (2 if residual is not None else 1)),
                   2.0 * m * n * k)

    def _row_parallel(self, a: DeviceTensor, lda: int, w: DeviceTensor, M: int,
                      x_in: DeviceTensor, x_out: DeviceTensor) -> None:
        """x_out = x_in + sum over ranks of a @ w^T (rank 0 adds the residual)."""
        lead = self.rank == 0
        H = self.cfg.hidden
        if self.world == 1:
            self._linear(a, lda, w, M, x_out, residual=x_in)
            return
        ar = self.peer_ar
        if ar is not None and M * H * 4 <= ar.max_bytes:
            s = self._ar_slot
            self._ar_slot ^= 1
            part = ar.slot(s, (M, H), self.g)
            self._linear(a, lda, w, M, part, residual=x_in if lead else None)
            ar.allreduce(self.g, s, x_out, M * H)
            self._note("all_reduce", 4.0 * M * H * self.world)
            return
        self._linear(a, lda, w, M, x_out, residual=x_in if lead else None)
        self._all_reduce(x_out, M)
        self._note("all_reduce", 4.0 * M * H)

    # -- one pass over T tokens per sequence -------------------------------
    def _forward(self, ids: DeviceTensor, T: int) -> None:
        cfg, g, sh = self.cfg, self.g, self.sh
        B, H, D = self.B, cfg.hidden, cfg.head_dim
        M = B * T
        kv = dict(batch=B, q_len=T, q_heads=sh.nq, kv_heads=sh.nkv, head_dim=D,
                  max_seq=cfg.max_seq)
        lead = self.rank == 0
        g.embedding(self.embed, ids, self.x_a, M, H)
        self._note("small", 8.0 * M * H)
        # Keys read by attention: positions 0 .. state[0] + T - 1 (state[0] is
        # on the device; the host tracks it only for the cost model).
        n_keys = self._host_pos + T
        few = M <= 8          # weight-streaming projections with the norm folded in
        eps = cfg.eps
        for li, L in enumerate(self.layers):
            if few:
                g.rms_linear(self.x_a, H, L["wqkv"], H, M, self.nqkv, H, self.qkv, self.nqkv,
                             rms_eps=eps)
                self._note("linear", 4.0 * (self.nqkv * H + M * H + M * self.nqkv),
                           2.0 * M * self.nqkv * H)
            else:
                g.rmsnorm(self.x_a, None, self.h, M, H, eps)
                self._note("small", 8.0 * M * H)
                self._linear(self.h, H, L["wqkv"], M, self.qkv)
            g.rope_kv_append(self.qkv, self.nqkv, self.cos, self.sin, self.state, self.q,
                             self.kc[li], self.vc[li], **kv)
            self._note("small", 8.0 * M * self.nqkv)
            g.attention_kv(self.q, self.kc[li], self.vc[li], self.att, self.state,
                           scale=float(1.0 / np.sqrt(np.float32(D))), **kv)
            self._note("attention", 4.0 * (2 * B * sh.nkv * n_keys * D + 2 * M * sh.nq * D),
                       4.0 * B * sh.nq * T * n_keys * D)
            self._row_parallel(self.att, sh.nq * D, L["wo"], M, self.x_a, self.x_b)
            if few:
                g.swiglu_linear(self.x_b, H, L["wgu"], H, M, sh.nf, H, self.mlp, sh.nf,
                                rms_eps=eps)
                self._note("linear", 4.0 * (2 * sh.nf * H + M * H + M * sh.nf),
                           4.0 * M * sh.nf * H)
            else:
                g.rmsnorm(self.x_b, None, self.h, M, H, eps)
                self._note("small", 8.0 * M * H)
                self._linear(self.h, H, L["wgu"], M, self.gu)
                g.swiglu_rows(self.gu, 2 * sh.nf, self.mlp, sh.nf, M, sh.nf)
                self._note("small", 12.0 * M * sh.nf)
            self._row_parallel(self.mlp, sh.nf, L["wdown"], M, self.x_b, self.x_a)
        # Final norm + lm_head on the last position of every sequence.
        keys = None
        last_x = self.x_a.view((B, H), offset_elems=(T - 1) * H)
        if B <= 8:
            keys = self.keys if self.world == 1 else None
            g.rms_linear(last_x, T * H, self.lm_head, H, B, sh.nv, H, self.logits, sh.nv,
                         rms_eps=eps, argmax_keys=keys)
            self._note("linear", 4.0 * (sh.nv * H + B * H + B * sh.nv), 2.0 * B * sh.nv * H)
        else:
            g.rmsnorm(self.x_a, None, self.h, M, H, eps)
            self._note("small", 8.0 * M * H)
            last = self.h.view((B, H), offset_elems=(T - 1) * H)
            self._linear(last, T * H, self.lm_head, B, self.logits)
            if self.world == 1:
                g.argmax_rows(self.logits, self.ids, B, sh.nv)
        if self.world > 1:
            import torch.distributed as dist
            g.argmax_partial(self.logits, sh.nv, B, sh.nv, sh.v0, self.packed)
            dist.all_gather_into_tensor(self._torch_view(self.packed_all, self.world, B * 2),
                                        self._torch_view(self.packed, 1, B * 2),
                                        group=self.group)
            g.argmax_merge(self.packed_all, self.world, B, self.ids)
        g.token_commit(self.ids, self.hist, self.state, B, T, self.n_new, argmax_keys=keys)
        self._note("small", 4.0 * B * sh.nv)
        self._host_pos += T

    # -- public ------------------------------------------------------------
    def upload_prompt(self, prompt: np.ndarray) -> None:
        assert prompt.shape == (self.B, self.P), prompt.shape
        self.g.upload(self.prompt_ids, prompt.astype(np.int32))

    def prefill(self) -> None:
        """Resets the position state and runs the prompt block."""
        self.g.zero(self.state)
        self._host_pos = 0
        self._forward(self.prompt_ids, self.P)

    def decode_step(self) -> None:
        """One cached decode step.  With `capture` the step (kernels and, at
        world > 1, its NCCL collectives) is recorded once as a CUDA graph and
        replayed; if recording fails the step runs eagerly from then on."""
        if self.capture and not self._captured:
            try:
                self.g.capture_begin()
                try:
                    self._forward(self.ids, 1)
                finally:
                    self.g.capture_end()
                self._host_pos -= 1          # recorded, not run
                self._captured = True
            except Exception:
                self.capture = False
        if self._captured:
            self.g.replay()
            self._host_pos += 1
        else:
            self._forward(self.ids, 1)

    def run(self) -> None:
        """Prefill + n_new - 1 decode steps, all enqueued on the stream."""
        self.prefill()
        for _ in range(self.n_new - 1):
            self.decode_step()

    def tokens(self) -> np.ndarray:
        return self.hist.download().T.copy()      # [B, n_new]

    def generate(self, prompt: np.ndarray) -> np.ndarray:
        self.upload_prompt(prompt)
        self.run()
        self.g.sync()
        return self.tokens()

    def last_logits(self) -> np.ndarray:
        """Logits of the last step for this rank's vocabulary slice, [B, nv]."""
        return self.logits.download()

    def close(self) -> None:
        self.g.sync()
        if self.peer_ar is not None:
            self.peer_ar.close()
            self.peer_ar = None
        self.g.close()
