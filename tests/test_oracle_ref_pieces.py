"""The oracle's restatements around the DiT blocks, and of the PatchEncoder,
pinned against the reference's own code (oracle/ref_pipeline.cpp, built into
oracle/_ref from the reference tree):
  * src/e2e_pipeline_v4.cpp: compute_cond (:57-71), the FM projections
    (:81-113), build_fm_attn_mask / build_fm_pos_ids (:120-155), the EOS head
    (:599-619) and one patch of the Euler + CFG decode loop (:381-400,
    :410-533), taken verbatim by oracle/extract_ref.py;
  * src/modules/backbone/patchenc.cpp compiled whole: causal_conv1d_stride2
    (:19-39), per_head_attention_cpu (:59-101) and patchenc_forward (:146-239)
    as written, over the eager ggml stand-in (oracle/shim/ggml_eager.cpp).
Each check runs against the committed golden vectors
(tests/golden/pipeline_ref_small.npz, tests/golden/make_pipeline_golden.py)
everywhere, and against the live reference build where oracle/_ref exists.
The engine's host-side mask and position tables (dtts_fm_layout) are compared
bit for bit.  Integer work (mask, position ids) and the plain-C pieces the two
sides evaluate in the same order (conv, causal attention) must be identical;
fp32 dot products summed in another order agree to 1e-5."""
import os
import sys

import numpy as np
import pytest

import oracle as O
from helpers import rel

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_pipeline_golden as G  # noqa: E402

F32 = 1e-5


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(HERE, "golden", "pipeline_ref_small.npz"))


@pytest.fixture(scope="module")
def dit_in():
    return G.dit_inputs()


@pytest.fixture(scope="module")
def pe_in():
    return G.pe_inputs()


def test_pieces_come_from_the_cited_lines(ref):
    """The verbatim pieces sit where this repository's citations say."""
    assert ref.gen_ranges() == {
        "HIDDEN_PATCH_SIZE": (39, 39), "LATENT_PATCH_SIZE": (40, 40), "compute_cond": (57, 71),
        "apply_latent_proj": (81, 91), "apply_hidden_proj": (94, 102), "apply_coord_proj": (105, 113),
        "build_fm_attn_mask": (120, 146), "build_fm_pos_ids": (149, 155), "solver_locals": (246, 249),
        "fm_input": (381, 400), "euler_loop": (410, 533), "eos_head": (599, 619),
        "raw_compute_cond": (22, 36)}


def test_fm_mask_and_pos_golden(orc, gold, dtts_mod):
    """Oracle and engine host tables against the reference's mask / position ids, bit for bit."""
    for i, (total, fl, hp) in enumerate(G.LAYOUTS):
        want_m = np.unpackbits(gold[f"mask{i}"])[:total * total].reshape(total, total)
        want_p = gold[f"pos{i}"]
        assert np.array_equal(orc.fm_mask(total, fl, 4, hp), want_m), (total, fl, hp)
        assert np.array_equal(orc.fm_pos(total, fl, 4), want_p)
        m, p = dtts_mod.fm_layout(total, fl, 4, hp)
        assert np.array_equal(m, want_m), (total, fl, hp)
        assert np.array_equal(p, want_p)


@pytest.mark.parametrize("total,fm_len", [(12, 8), (64, 60), (256, 252), (16, 4), (256, 8), (130, 126), (5, 1)])
@pytest.mark.parametrize("hidden_patch", [1, 2])
def test_fm_mask_and_pos_live(orc, ref, dtts_mod, total, fm_len, hidden_patch):
    want_m, want_p = ref.fm_mask(total, fm_len, 4, hidden_patch), ref.fm_pos(total, fm_len, 4)
    m, p = dtts_mod.fm_layout(total, fm_len, 4, hidden_patch)
    assert np.array_equal(m, want_m) and np.array_equal(p, want_p)
    assert np.array_equal(orc.fm_mask(total, fm_len, 4, hidden_patch), want_m)
    assert np.array_equal(orc.fm_pos(total, fm_len, 4), want_p)


def test_compute_cond_golden(orc, gold, dit_in):
    w, spk = dit_in[0], dit_in[1]
    for j, t in enumerate(G.TIMES):
        assert rel(orc.compute_cond(w, t, None, G.SPK_SCALE), gold["cond_nospk"][j]) <= F32
        assert rel(orc.compute_cond(w, t, spk, G.SPK_SCALE), gold["cond_spk"][j]) <= F32


def test_compute_cond_live(orc, ref, dit_in):
    w, spk = dit_in[0], dit_in[1]
    for t in (0.05, 0.5, 0.99):
        for s, sc in ((None, 1.0), (spk, 1.0), (spk, 1.5), (spk * 3.0, 0.25)):
            assert rel(orc.compute_cond(w, t, s, sc), ref.compute_cond(w, t, s, sc)) <= F32


def test_compute_cond_of_the_ggml_path_live(orc, ref, dit_in):
    """dit_forward_raw's own compute_cond (src/modules/backbone/dit_forward.cpp:22-36) is the
    pipeline's with the speaker term unscaled."""
    w, spk = dit_in[0], dit_in[1]
    for t in (0.0, 0.4):
        for s in (None, spk):
            assert rel(orc.compute_cond(w, t, s, 1.0), ref.compute_cond_raw(w, t, s)) <= F32


def test_projections_and_eos_golden(orc, gold, dit_in):
    w, spk, z, h, fc, fu = dit_in
    assert rel(orc.linear_rows(z, w["latent_proj.weight"], w["latent_proj.bias"]), gold["latent_proj"]) <= F32
    assert rel(orc.linear_rows(h[:1], w["hidden_proj.weight"], w["hidden_proj.bias"])[0], gold["hidden_proj"]) <= F32
    assert rel(orc.linear_rows(z[1:2], w["coordinate_proj.weight"], w["coordinate_proj.bias"])[0],
               gold["coord_proj"]) <= F32
    # the EOS head as written computes s * SiLU(s) between the layers
    assert rel(orc.eos_prob(w, h, as_written=True), gold["eos_prob"]) <= F32


def test_projections_and_eos_live(orc, ref, dit_in):
    w, spk, z, h, fc, fu = dit_in
    z2 = z * 2.5 - 0.3
    assert rel(orc.linear_rows(z2, w["latent_proj.weight"], w["latent_proj.bias"]), ref.latent_proj(w, z2)) <= F32
    assert rel(orc.linear_rows(h[2:3], w["hidden_proj.weight"], w["hidden_proj.bias"])[0],
               ref.hidden_proj(w, h[2])) <= F32
    zero = np.zeros(1536, np.float32)   # the CFG rows: hidden_proj of zeros = the bias
    assert np.array_equal(ref.hidden_proj(w, zero), w["hidden_proj.bias"])
    assert rel(orc.eos_prob(w, h * 3.0, as_written=True), ref.eos_prob(w, h * 3.0)) <= F32


def test_euler_patch_golden(orc, gold, dit_in):
    """The oracle's Euler + CFG solve (v4 layout and CFG form, no speaker) against
    the reference's own loop: NFE 10, CFG 2.0, and the --fast path (no CFG row)."""
    w, spk, z, h, fc, fu = dit_in
    got = orc.euler_solve(w, G.N_LAYERS, fc[None], fu[None], z[None], None, 1.5, nfe=G.SOLVE_NFE,
                          cfg_scale=G.SOLVE_CFG)[0]
    assert rel(got - z, gold["solve_z"] - z) <= F32
    fast = orc.euler_solve(w, G.N_LAYERS, fc[None], fu[None], z[None], None, 1.5, nfe=G.SOLVE_NFE, cfg_scale=0.0)[0]
    assert rel(fast - z, gold["solve_z_fast"] - z) <= F32


def test_euler_patch_live(orc, ref, dit_in):
    w, spk, z, h, fc, fu = dit_in
    for nfe, cfg in ((3, 1.0), (10, 3.0)):
        got = orc.euler_solve(w, G.N_LAYERS, fc[None], fu[None], z[None], None, 1.5, nfe=nfe, cfg_scale=cfg)[0]
        want = ref.solve_patch(w, G.N_LAYERS, fc, fu, z, nfe, cfg)
        assert rel(got - z, want - z) <= F32, (nfe, cfg)


def test_pe_conv_and_attention_golden(orc, gold, pe_in):
    """The two plain-C pieces of patchenc.cpp at the benchmark's depth (500 frames,
    250 tokens), identical bit for bit."""
    pw, conv_x, q, k, v, small, full = pe_in
    got = orc.pe_conv(conv_x, pw["patch_encoder.ds_proj.weight"], pw["patch_encoder.ds_proj.bias"])
    assert np.array_equal(got, gold["pe_conv"])
    att = orc.pe_causal_attention(q, k, v)
    assert np.array_equal(att[list(G.PE_ATT_ROWS)], gold["pe_attention_rows"])


@pytest.mark.parametrize("T", [250, 500])
def test_pe_conv_and_attention_live(orc, ref, pe_in, T):
    pw = pe_in[0]
    x = np.concatenate([pe_in[1], pe_in[1][::-1]])[:2 * T]
    wc, bc = pw["patch_encoder.ds_proj.weight"], pw["patch_encoder.ds_proj.bias"]
    assert np.array_equal(orc.pe_conv(x, wc, bc), ref.pe_conv(x, wc, bc))
    assert np.array_equal(orc.pe_conv(x, wc, None), ref.pe_conv(x, wc, None))
    rng = np.random.default_rng(T)
    q, k, v = (rng.standard_normal((T, 1024)).astype(np.float32) for _ in range(3))
    assert np.array_equal(orc.pe_causal_attention(q, k, v), ref.pe_causal_attention(q, k, v))


def test_pe_forward_golden(orc, gold, pe_in):
    """patchenc_forward as written: one call over 3 patches (the as-written pairing)
    and over 125 patches (250 tokens, the benchmark's prefill)."""
    pw, conv_x, q, k, v, small, full = pe_in
    assert rel(orc.pe_forward(pw, G.N_LAYERS, small, O.PAIR_AS_WRITTEN), gold["pe_small"]) <= F32
    got = orc.pe_forward(pw, G.N_LAYERS, full, O.PAIR_AS_WRITTEN)
    assert rel(got[list(G.PE_FULL_ROWS)], gold["pe_full_rows"]) <= F32


def test_pe_forward_live(orc, ref, pe_in):
    pw = pe_in[0]
    fr = pe_in[5]
    for n in (4, 12):
        assert rel(orc.pe_forward(pw, G.N_LAYERS, fr[:n], O.PAIR_AS_WRITTEN), ref.pe_forward(pw, G.N_LAYERS, fr[:n])) <= F32
    # one patch: the as-written pairing is the adjacent one
    assert rel(orc.pe_forward(pw, G.N_LAYERS, fr[:4], O.PAIR_ADJACENT), ref.pe_forward(pw, G.N_LAYERS, fr[:4])) <= F32
