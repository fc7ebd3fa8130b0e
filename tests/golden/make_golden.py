"""Generates tests/golden/dit_ref_small.npz from the reference's own DiT math
(include/dit_manual.h compiled in place into oracle/_ref by oracle/Makefile).

    make -C oracle REF=<tree> && python tests/golden/make_golden.py

Inputs are regenerated from seeds (dots.tts.cpp_b200/synth.py), so the file
holds the seeds, shapes and the reference outputs only.  Small sizes keep the
file a few hundred KB while covering every branch of the reference's block:
mask + position ids, no mask, qk-norm gains, biases, O(1) adaLN modulation."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "dots.tts.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402
import synth  # noqa: E402

SEED, N_LAYERS, ADA_STD = 11, 2, 0.5
L_ATT, L_BLK = 8, 12


def inputs():
    w = synth.dit_weights(SEED, n_layers=N_LAYERS, ada_bias_std=ADA_STD)
    x_att = synth.normal(SEED, "golden.x_att", (L_ATT, 1024), 1.0)
    x_blk = synth.normal(SEED, "golden.x_blk", (L_BLK, 1024), 1.0)
    cond = synth.normal(SEED, "golden.cond", (1024,), 1.0)
    return w, x_att, x_blk, cond


def fm_tables(orc):
    mask = orc.fm_mask(L_BLK, L_BLK - 4, 4)
    pos = orc.fm_pos(L_BLK, L_BLK - 4, 4)
    return mask, pos


def main():
    ref, orc = O.Reference(), O.Oracle()
    w, x_att, x_blk, cond = inputs()
    p = "velocity_field_predictor.blocks.0."
    W = [w[p + n] for n in ("attn.q_proj.weight", "attn.k_proj.weight", "attn.v_proj.weight", "attn.o_proj.weight",
                            "attn.o_proj.bias", "attn.q_norm.weight", "attn.k_norm.weight")]
    mask, pos = fm_tables(orc)
    out = {
        "seed": np.int64(SEED), "n_layers": np.int64(N_LAYERS), "ada_std": np.float64(ADA_STD),
        "attn_nomask": ref.manual_attention(x_att, *W),
        "attn_mask_pos": ref.manual_attention(x_blk, *W, mask=mask, pos=pos),
        "block_per_token": ref.dit_block(w, 0, x_blk, cond, mask, pos, O.FFN_PER_TOKEN),
        "block_nomask": ref.dit_block(w, 1, x_blk, cond, None, None, O.FFN_PER_TOKEN),
        "block_as_written_row0": ref.dit_block(w, 0, x_blk, cond, mask, pos, O.FFN_AS_WRITTEN)[0],
        "velocity": ref.dit_velocity(w, N_LAYERS, x_blk, cond, mask, pos, O.FFN_PER_TOKEN),
    }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "dit_ref_small.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
