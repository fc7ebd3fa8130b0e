"""Generates tests/golden/pipeline_ref_small.npz: outputs of the reference's own
code around the DiT blocks and of its PatchEncoder, compiled in place into
oracle/_ref by oracle/Makefile (oracle/ref_pipeline.cpp):
  src/e2e_pipeline_v4.cpp   compute_cond, apply_latent/hidden/coord_proj,
                            build_fm_attn_mask, build_fm_pos_ids, the EOS head,
                            one patch of the Euler + CFG decode loop
                            (verbatim pieces, oracle/extract_ref.py)
  src/modules/backbone/patchenc.cpp   causal_conv1d_stride2,
                            per_head_attention_cpu, patchenc_forward as written
                            (ggml operators from oracle/shim/ggml_eager.cpp)
on seeded random weights of the real shapes.

    make -C oracle REF=<tree> && python tests/golden/make_pipeline_golden.py

Weights and inputs are regenerated from seeds (dots.tts.cpp_b200/synth.py), so
the file holds the seeds, shapes and reference outputs only; large outputs are
kept as a few rows."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "dots.tts.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402
import synth  # noqa: E402

SEED, N_LAYERS, ADA_STD = 13, 2, 0.5
TIMES = (0.0, 0.3, 0.9)
SPK_SCALE = 1.5
LAYOUTS = ((12, 8, 1), (64, 60, 1), (256, 252, 1), (64, 8, 1), (256, 60, 2))  # (total, fm_len, hidden_patch)
SOLVE_FM_LEN, SOLVE_NFE, SOLVE_CFG = 8, 10, 2.0
PE_CONV_FRAMES = 500
PE_ATT_T = 250
PE_ATT_ROWS = (0, 1, 2, 124, 249)
PE_SMALL_FRAMES = 12     # 3 patches: the as-written pairing differs from adjacent pairs
PE_FULL_FRAMES = 500     # 125 patches, 250 tokens
PE_FULL_ROWS = (0, 1, 62, 123, 124)


def dit_inputs():
    w = synth.dit_weights(SEED, n_layers=N_LAYERS, ada_bias_std=ADA_STD)
    spk = synth.normal(SEED, "golden.spk", (512,), 1.0 / np.sqrt(512))
    z = synth.normal(SEED, "golden.z", (4, 128), 1.0)
    h = synth.normal(SEED, "golden.h", (3, 1536), 1.0)
    fc, fu = synth.fm_history(SEED, 1, SOLVE_FM_LEN, w)
    return w, spk, z, h, fc[0], fu[0]


def pe_inputs():
    pw = synth.pe_weights(SEED + 1, n_layers=N_LAYERS)
    conv_x = synth.normal(SEED, "golden.pe_conv", (PE_CONV_FRAMES, 128), 1.0)
    q, k, v = (synth.normal(SEED, f"golden.pe_{n}", (PE_ATT_T, 1024), 1.0) for n in "qkv")
    small = synth.normal(SEED, "golden.pe_small", (PE_SMALL_FRAMES, 128), 1.0)
    full = synth.normal(SEED, "golden.pe_full", (PE_FULL_FRAMES, 128), 1.0)
    return pw, conv_x, q, k, v, small, full


def main():
    ref = O.Reference()
    w, spk, z, h, fc, fu = dit_inputs()
    out = {"seed": SEED, "n_layers": N_LAYERS}
    out["cond_nospk"] = np.stack([ref.compute_cond(w, t, None, SPK_SCALE) for t in TIMES])
    out["cond_spk"] = np.stack([ref.compute_cond(w, t, spk, SPK_SCALE) for t in TIMES])
    for i, (total, fl, hp) in enumerate(LAYOUTS):
        out[f"mask{i}"] = np.packbits(ref.fm_mask(total, fl, 4, hp))
        out[f"pos{i}"] = ref.fm_pos(total, fl, 4)
    out["latent_proj"] = ref.latent_proj(w, z)
    out["hidden_proj"] = ref.hidden_proj(w, h[0])
    out["coord_proj"] = ref.coord_proj(w, z[1])
    out["eos_prob"] = ref.eos_prob(w, h)
    out["solve_z"] = ref.solve_patch(w, N_LAYERS, fc, fu, z, SOLVE_NFE, SOLVE_CFG)
    out["solve_z_fast"] = ref.solve_patch(w, N_LAYERS, fc, fu, z, SOLVE_NFE, SOLVE_CFG, fast=True)
    pw, conv_x, q, k, v, small, full = pe_inputs()
    out["pe_conv"] = ref.pe_conv(conv_x, pw["patch_encoder.ds_proj.weight"], pw["patch_encoder.ds_proj.bias"])
    out["pe_attention_rows"] = ref.pe_causal_attention(q, k, v)[list(PE_ATT_ROWS)]
    out["pe_small"] = ref.pe_forward(pw, N_LAYERS, small)
    out["pe_full_rows"] = ref.pe_forward(pw, N_LAYERS, full)[list(PE_FULL_ROWS)]
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "pipeline_ref_small.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
