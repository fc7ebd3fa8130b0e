"""Generates tests/golden/llm_ref_small.npz: the reference's own Qwen2 decoder
path (src/llm_manual.cpp: llm_kv_cache_init, then llm_kv_cache_step per step,
compiled in place into oracle/_ref by oracle/Makefile) on seeded random
weights of the real shapes, 2 layers.  Two cases: a 9-token prompt with 3
steps, and a 1-token prompt with 2 steps.

    make -C oracle REF=<tree> && python tests/golden/make_llm_golden.py

Weights and embeddings are regenerated from seeds (dots.tts.cpp_b200/synth.py),
so the file holds the seeds, shapes and reference outputs only."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "dots.tts.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402
import synth  # noqa: E402

SEED, N_LAYERS = 11, 2
CASES = ((9, 3), (1, 2))   # (prompt tokens, steps)


def weights():
    return synth.llm_weights(SEED, n_layers=N_LAYERS)


def inputs(case):
    n_tok, steps = CASES[case]
    prompt = synth.normal(SEED, f"golden.llm_prompt{case}", (n_tok, 1536), 1.0)
    step = synth.normal(SEED, f"golden.llm_step{case}", (steps, 1536), 1.0)
    return prompt, step


def main():
    ref = O.Reference()
    w = weights()
    out = {"seed": SEED, "n_layers": N_LAYERS}
    for c in range(len(CASES)):
        p, s = inputs(c)
        ph, sh = ref.llm_run(w, N_LAYERS, p, s)
        out[f"prompt_hidden{c}"], out[f"step_hidden{c}"] = ph, sh
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "llm_ref_small.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, {k: getattr(v, "shape", v) for k, v in out.items()})


if __name__ == "__main__":
    main()
