"""Generates tests/golden/voc_ref_small.npz: the reference's own BigVGAN decoder
(src/modules/vocoder/bigvgan_cpp.cpp + lstm.cpp, compiled in place into
oracle/_ref by oracle/Makefile) on seeded random weights of the real shapes,
plus the 12 filter taps the reference hard-codes for its AMP activations
(bigvgan_cpp.cpp:27-31), read from the source text.

    make -C oracle REF=<tree> && python tests/golden/make_voc_golden.py <tree>

Weights and latents are regenerated from seeds (dots.tts.cpp_b200/synth.py),
so the file holds the seeds, shapes and reference outputs only."""
import os
import re
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "dots.tts.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402
import synth  # noqa: E402

SEED, N_FRAMES = 5, 2


def inputs():
    w = synth.voc_weights(SEED, aa_filter=O.aa_filter())
    lat = synth.normal(SEED, "golden.voc_latent", (N_FRAMES, 128), 1.0)
    return w, lat


def reference_filter(tree):
    src = open(os.path.join(tree, "src", "modules", "vocoder", "bigvgan_cpp.cpp")).read()
    body = re.search(r"AA_FILTER\[12\]\s*=\s*\{([^}]*)\}", src).group(1)
    vals = [float(v.strip().rstrip("f")) for v in body.split(",") if v.strip()]
    assert len(vals) == 12
    return np.array(vals, np.float32)


def main():
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DTTS_REFERENCE", "")
    if not tree:
        raise SystemExit("usage: make_voc_golden.py REFERENCE_TREE (or set DTTS_REFERENCE)")
    ref = O.Reference()
    w, lat = inputs()
    audio = ref.voc_decode(w, lat)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "voc_ref_small.npz")
    np.savez_compressed(out, seed=SEED, n_frames=N_FRAMES, audio=audio, aa_filter=reference_filter(tree))
    print("wrote", out, audio.shape, float(np.sqrt(np.mean(audio ** 2))))


if __name__ == "__main__":
    main()
