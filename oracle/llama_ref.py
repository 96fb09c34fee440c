"""CPU oracle for the TinyLlama decode path (test infrastructure only: imported
by tests/, the smoke check and bench.py's CPU legs, never by the product).

`llama_step` restates the reference's traced forward pass,
source/xla_hlo/tools/export_llama.py:269-365, in numpy float32 (one sequence,
the batch dimension of 1 dropped):

  per layer: h = rms_norm(x, ln) (x * rsqrt(mean(x^2) + eps) * w, :284-286);
  q/k/v = h @ W; heads split [S, heads, 64] -> [heads, S, 64]; RoPE
  x * cos + rotate_half(x) * sin with rotate_half = [-x2, x1] (:288-296);
  kv heads repeated 8x (:333-345); scores = q k^T * rsqrt(64) + mask;
  softmax; att = p v; merged heads @ o_w; residual; rms_norm; silu(h @ gate)
  * (h @ up) @ down; residual.  Then rms_norm(final) @ lm_head.

`generate_full` restates the decode loop of run_llama_spirv.py:190-260: at
every step the whole window of S = 64 positions is recomputed with the
tokens so far padded by id 0, the causal mask of build_causal_mask
(:100-107, -1e9 where column > row or column >= valid), and the argmax of
the logits at the last valid position is appended.

`generate_cached` computes the same tokens with a KV cache (the algorithm
the device runs) so the two can be checked against each other here.
"""
from __future__ import annotations

import numpy as np


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    var = np.mean(np.square(x), axis=-1, keepdims=True, dtype=np.float32)
    return (x * (np.float32(1.0) / np.sqrt(var + np.float32(eps)))) * w


def rotate_half(x: np.ndarray) -> np.ndarray:
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def silu(x: np.ndarray) -> np.ndarray:
    return x * (np.float32(1.0) / (np.float32(1.0) + np.exp(-x)))


def softmax(x: np.ndarray) -> np.ndarray:
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=-1, keepdims=True, dtype=np.float32)


def causal_mask(S: int, valid: int) -> np.ndarray:
    r = np.arange(S)[:, None]
    c = np.arange(S)[None, :]
    return np.where((c > r) | (c >= valid), np.float32(-1e9), np.float32(0.0)).astype(np.float32)


def _attention_block(cfg, L, x, cos, sin, mask):
    S = x.shape[0]
    D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
    h = rms_norm(x, L["ln"], cfg.eps)
    q = (h @ L["q"]).reshape(S, Hq, D).transpose(1, 0, 2)
    k = (h @ L["k"]).reshape(S, Hkv, D).transpose(1, 0, 2)
    v = (h @ L["v"]).reshape(S, Hkv, D).transpose(1, 0, 2)
    q = q * cos + rotate_half(q) * sin
    k = k * cos + rotate_half(k) * sin
    rep = Hq // Hkv
    k = np.repeat(k, rep, axis=0)
    v = np.repeat(v, rep, axis=0)
    scale = np.float32(1.0) / np.sqrt(np.float32(D))
    scores = (q @ k.transpose(0, 2, 1)) * scale + mask
    att = softmax(scores) @ v
    att = att.transpose(1, 0, 2).reshape(S, Hq * D)
    return x + att @ L["o"]


def _mlp_block(cfg, L, x):
    h = rms_norm(x, L["post_ln"], cfg.eps)
    return x + (silu(h @ L["gate"]) * (h @ L["up"])) @ L["down"]


def llama_step(cfg, W: dict, tok_emb: np.ndarray, cos: np.ndarray, sin: np.ndarray,
               mask: np.ndarray) -> np.ndarray:
    """tokens' embeddings [S, H] -> logits [S, vocab] (export_llama.py:269-365)."""
    x = tok_emb.astype(np.float32)
    for L in W["layers"]:
        x = _attention_block(cfg, L, x, cos, sin, mask)
        x = _mlp_block(cfg, L, x)
    return rms_norm(x, W["final_ln"], cfg.eps) @ W["lm_head"]


def generate_full(cfg, W: dict, prompt: np.ndarray, n_new: int, rope, S: int | None = None,
                  return_logits: bool = False):
    """Greedy tokens [n_new] for one prompt, full re-computation per step.
    `rope` = (cos, sin) tables [>= S, head_dim]."""
    S = S or cfg.max_seq
    cos, sin = rope[0][:S], rope[1][:S]
    tokens = [int(t) for t in prompt]
    out, last_logits = [], None
    for _ in range(n_new):
        padded = (tokens + [0] * (S - len(tokens)))[:S]
        emb = W["embed"][padded]
        logits = llama_step(cfg, W, emb, cos, sin, causal_mask(S, len(tokens)))
        last_logits = logits[len(tokens) - 1]
        nxt = int(np.argmax(last_logits))
        out.append(nxt)
        tokens.append(nxt)
    out = np.array(out, np.int32)
    return (out, last_logits) if return_logits else out


def generate_cached(cfg, W: dict, prompt: np.ndarray, n_new: int, rope,
                    return_logits: bool = False, forced=None):
    """The same greedy tokens with a KV cache (prefill, then one token per step).

    With `forced` (a token sequence [n_new]) the step inputs are those tokens
    instead of the oracle's own argmax (teacher forcing), and the logits of
    every step are returned as [n_new, vocab]."""
    cos_t, sin_t = rope
    D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
    caches = [([], []) for _ in W["layers"]]
    scale = np.float32(1.0) / np.sqrt(np.float32(D))

    def block(ids, pos0):
        T = len(ids)
        x = W["embed"][ids].astype(np.float32)
        cos, sin = cos_t[pos0:pos0 + T], sin_t[pos0:pos0 + T]
        for L, (kc, vc) in zip(W["layers"], caches):
            h = rms_norm(x, L["ln"], cfg.eps)
            q = (h @ L["q"]).reshape(T, Hq, D).transpose(1, 0, 2)
            k = (h @ L["k"]).reshape(T, Hkv, D).transpose(1, 0, 2)
            v = (h @ L["v"]).reshape(T, Hkv, D).transpose(1, 0, 2)
            q = q * cos + rotate_half(q) * sin
            k = k * cos + rotate_half(k) * sin
            kc.append(k)
            vc.append(v)
            K = np.repeat(np.concatenate(kc, axis=1), Hq // Hkv, axis=0)
            V = np.repeat(np.concatenate(vc, axis=1), Hq // Hkv, axis=0)
            n_keys = K.shape[1]
            qpos = pos0 + np.arange(T)[:, None]
            mask = np.where(np.arange(n_keys)[None, :] > qpos, np.float32(-1e9),
                            np.float32(0.0)).astype(np.float32)
            att = softmax((q @ K.transpose(0, 2, 1)) * scale + mask) @ V
            x = x + att.transpose(1, 0, 2).reshape(T, Hq * D) @ L["o"]
            x = _mlp_block(cfg, L, x)
        return rms_norm(x[-1:], W["final_ln"], cfg.eps) @ W["lm_head"]

    logits = block([int(t) for t in prompt], 0)[0]
    all_logits = [logits]
    out = [int(np.argmax(logits))]
    pos = len(prompt)
    for i in range(n_new - 1):
        feed = out[-1] if forced is None else int(forced[i])
        logits = block([feed], pos)[0]
        all_logits.append(logits)
        pos += 1
        out.append(int(np.argmax(logits)))
    out = np.array(out, np.int32)
    if forced is not None:
        return out, np.stack(all_logits)
    return (out, logits) if return_logits else out
