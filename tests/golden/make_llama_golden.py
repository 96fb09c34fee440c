"""Golden next-token logits of the reference's own TinyLlama graph.

Parses the reference's exported `llama_step` graph
(source/xla_hlo/fixtures/tinyllama.stablehlo.txt, 22 layers, S = 64) with
spirv_inference_b200.hlo_text, feeds it the seeded synthetic inputs the
tests use (weights: llama.make_weights(TINYLLAMA, seed=0, generator="torch");
prompt: llama.make_prompt(TINYLLAMA, 1, 32, seed=4321) padded with id 0 to
64; the reference's RoPE tables and causal mask) and evaluates it in float64
numpy (tests/_np_ref.eval_hlo_f64).  Saves the logits of the last prompt
position, the argmax of every prompt position and the fixture's sha256 to
tinyllama_step_golden.npz.

Run from the repository root with the reference mounted (about 3 minutes):
    python tests/golden/make_llama_golden.py /path/to/SPIRV_INFERENCE
"""
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE.parent))

from oracle import llama_ref  # noqa: E402
from spirv_inference_b200 import hlo_text, llama  # noqa: E402
import _np_ref  # noqa: E402

PROMPT_SEED, WEIGHT_SEED, P, S = 4321, 0, 32, 64


def feeds_for(graph, W, prompt):
    cfg = llama.TINYLLAMA
    toks = [int(t) for t in prompt] + [0] * (S - len(prompt))
    cos, sin = llama.rope_tables(cfg, S)
    args = [W["embed"][toks][None], cos[None, None], sin[None, None],
            llama_ref.causal_mask(S, len(prompt))[None, None]]
    for L in W["layers"]:
        args += [L[k] for k in ("ln", "q", "k", "v", "o", "post_ln", "gate", "up", "down")]
    args += [W["final_ln"], W["lm_head"]]
    return dict(zip(graph.inputs, args))


def main(ref_root: str) -> None:
    path = Path(ref_root) / "source" / "xla_hlo" / "fixtures" / "tinyllama.stablehlo.txt"
    text = path.read_bytes()
    g = hlo_text.parse(text.decode())
    W = llama.make_weights(llama.TINYLLAMA, WEIGHT_SEED, generator="torch")
    prompt = llama.make_prompt(llama.TINYLLAMA, 1, P, seed=PROMPT_SEED)[0]
    logits = _np_ref.eval_hlo_f64(g, feeds_for(g, W, prompt))[0]
    np.savez_compressed(HERE / "tinyllama_step_golden.npz",
                        prompt=prompt.astype(np.int32),
                        last_logits=logits[P - 1].astype(np.float32),
                        argmax=logits[:P].argmax(axis=1).astype(np.int32),
                        fixture_sha256=np.array(hashlib.sha256(text).hexdigest()))
    print("argmax at the last prompt position:", int(logits[P - 1].argmax()))


if __name__ == "__main__":
    main(sys.argv[1])
