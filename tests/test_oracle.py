"""The CPU oracle is pinned before it is trusted:
  * against the reference's own include/dit_manual.h compiled in oracle/_ref
    (attention, block, velocity), when that build is present;
  * against golden outputs of that build committed in tests/golden/;
  * against the one weight-independent known answer the reference's tests
    hold for this path (sinusoid RMS at t = 0, test/test_time_embed.cpp:70);
  * against hand-derived FM mask / position ids
    (src/e2e_pipeline_v4.cpp:120-155)."""
import os

import numpy as np
import pytest

import oracle as O
import synth
from helpers import rel

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "dit_ref_small.npz")
P0 = "velocity_field_predictor.blocks.0."


def _attn_w(w, i=0):
    p = f"velocity_field_predictor.blocks.{i}."
    return [w[p + n] for n in ("attn.q_proj.weight", "attn.k_proj.weight", "attn.v_proj.weight",
                               "attn.o_proj.weight", "attn.o_proj.bias", "attn.q_norm.weight",
                               "attn.k_norm.weight")]


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


@pytest.fixture(scope="module")
def gold_inputs(gold):
    import make_golden  # noqa
    return make_golden.inputs()


@pytest.fixture(scope="module", autouse=True)
def _golden_path():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))


def test_sinusoid_known_answer(orc):
    # test/test_time_embed.cpp:70 of the reference: RMS 0.7071 at t = 0 (cos(0)=1, sin(0)=0)
    se = orc.sinusoid(0.0)
    assert abs(float(np.sqrt((se.astype(np.float64) ** 2).mean())) - 0.70710678) < 1e-6
    assert np.all(se[:128] == 1.0) and np.all(se[128:] == 0.0)


def test_fm_mask_and_pos_hand_derived(orc):
    # total 8, history 5 (block_start 4), 3 latent queries
    m = orc.fm_mask(8, 5, 3)
    want = np.zeros((8, 8), np.uint8)
    for i in range(4):
        want[i, :i + 1] = 1            # causal history
    want[4, :5] = 1                     # last history block sees all history ...
    want[4, 5:] = 1                     # ... and the latent block
    want[5:, :5] = 1                    # latents see history
    want[5:, 5:] = 1                    # and each other
    assert np.array_equal(m, want)
    np.testing.assert_array_equal(orc.fm_pos(8, 5, 3), [0, 1, 2, 3, 4, 5, 6, 7])
    # padding rows between history and latents only see themselves, pos 0
    m2 = orc.fm_mask(9, 5, 3)
    assert m2[5].sum() == 1 and m2[5, 5] == 1
    np.testing.assert_array_equal(orc.fm_pos(9, 5, 3), [0, 1, 2, 3, 4, 0, 5, 6, 7])


def test_oracle_matches_golden(orc, gold, gold_inputs):
    w, x_att, x_blk, cond = gold_inputs
    W = _attn_w(w)
    mask = orc.fm_mask(12, 8, 4)
    pos = orc.fm_pos(12, 8, 4)
    assert rel(orc.attention(x_att, *W), gold["attn_nomask"]) < 1e-6
    assert rel(orc.attention(x_blk, *W, mask=mask, pos=pos), gold["attn_mask_pos"]) < 1e-6
    assert rel(orc.dit_block(w, 0, x_blk, cond, mask, pos), gold["block_per_token"]) < 2e-6
    assert rel(orc.dit_block(w, 1, x_blk, cond), gold["block_nomask"]) < 2e-6
    assert rel(orc.dit_block(w, 0, x_blk, cond, mask, pos, O.FFN_AS_WRITTEN)[0], gold["block_as_written_row0"]) < 2e-6
    assert rel(orc.dit_velocity(w, 2, x_blk, cond, mask, pos), gold["velocity"]) < 2e-6


def test_oracle_matches_reference_build_config1_shape(orc, ref):
    # config 1: X ~ N(0,1) [L=64, 1024] seed 0, Wq/k/v/o ~ N(0,0.02), zero bias,
    # gains 1 + N(0, 0.02), bidirectional, positions 0..63
    w = synth.dit_weights(0, n_layers=1)
    W = _attn_w(w)
    W[4] = np.zeros(1024, np.float32)
    x = synth.normal(0, "c1.x", (64, 1024), 1.0)
    a = orc.attention(x, *W)
    b = ref.manual_attention(x, *W)
    assert rel(a, b) < 1e-6


def test_oracle_matches_reference_build_block_and_velocity(orc, ref):
    w = synth.dit_weights(5, n_layers=2, ada_bias_std=0.5)
    x = synth.normal(5, "x", (10, 1024), 1.0)
    cond = synth.normal(5, "c", (1024,), 1.0)
    mask, pos = orc.fm_mask(10, 6, 4), orc.fm_pos(10, 6, 4)
    assert rel(orc.dit_block(w, 0, x, cond, mask, pos), ref.dit_block(w, 0, x, cond, mask, pos)) < 2e-6
    assert rel(orc.dit_velocity(w, 2, x, cond), ref.dit_velocity(w, 2, x, cond)) < 2e-6
    v1 = orc.dit_velocity(w, 2, x, cond, mask, pos, n_out=4)
    v2 = ref.dit_velocity(w, 2, x, cond, mask, pos, n_out=4)
    assert rel(v1, v2) < 2e-6


def test_as_written_block_differs_only_by_ffn(orc, ref):
    """The shipped block projects the FFN for token 0 only (include/dit_manual.h:185,194);
    row 0 agrees with the per-token block, later rows lack the FFN branch."""
    w = synth.dit_weights(6, n_layers=1, ada_bias_std=0.5)
    x = synth.normal(6, "x", (6, 1024), 1.0)
    cond = synth.normal(6, "c", (1024,), 1.0)
    per_tok = orc.dit_block(w, 0, x, cond)
    as_wr = orc.dit_block(w, 0, x, cond, ffn_mode=O.FFN_AS_WRITTEN)
    assert rel(as_wr[0], per_tok[0]) < 1e-6
    assert rel(as_wr[0], ref.dit_block(w, 0, x, cond, ffn_mode=O.FFN_AS_WRITTEN)[0]) < 2e-6
    assert np.abs(as_wr[1:] - per_tok[1:]).max() > 1e-2


def test_euler_solve_uses_velocity(orc):
    """One Euler step of the oracle solve equals z0 + dt * CFG(velocities) built
    from the oracle's own velocity (src/e2e_pipeline_v4.cpp:410-526)."""
    w = synth.dit_weights(8, n_layers=1)
    fc, fu = synth.fm_history(8, 1, 6, w)
    z0 = synth.normal(8, "z0", (1, 4, 128), 1.0)
    z1 = orc.euler_solve(w, 1, fc, fu, z0, nfe=1, cfg_scale=2.0)
    L = 10
    mask, pos = orc.fm_mask(L, 6, 4), orc.fm_pos(L, 6, 4)
    coord = orc.linear_rows(z0[0], w["coordinate_proj.weight"], w["coordinate_proj.bias"])
    cond = orc.compute_cond(w, 0.0, None, 1.5)
    xc = np.concatenate([fc[0], coord]).astype(np.float32)
    xu = np.concatenate([fu[0], coord]).astype(np.float32)
    vc = orc.dit_velocity(w, 1, xc, cond, mask, pos, n_out=4)
    vu = orc.dit_velocity(w, 1, xu, cond, mask, pos, n_out=4)
    want = z0[0] + (vc + 2.0 * (vc - vu)) * 1.0
    assert rel(z1[0], want) < 1e-6


def test_eos_head_restatement(orc):
    """The EOS head of the v4 pipeline (src/e2e_pipeline_v4.cpp:598-619) against
    a float64 evaluation: SiLU between the layers, or s * SiLU(s) as the shipped
    code computes (:608-609)."""
    import synth
    w = {k: v for k, v in synth.dit_weights(4, n_layers=1).items() if k.startswith("eos_proj")}
    h = synth.normal(4, "eos.h", (3, 1536), 1.0)
    for as_written in (False, True):
        got = orc.eos_prob(w, h, as_written)
        s = h.astype(np.float64) @ w["eos_proj.0.weight"].T.astype(np.float64) + w["eos_proj.0.bias"]
        a = s / (1 + np.exp(-s))
        if as_written:
            a = s * a
        lg = a @ w["eos_proj.2.weight"].T.astype(np.float64) + w["eos_proj.2.bias"]
        want = np.exp(lg[:, 1] - lg.max(1)) / np.exp(lg - lg.max(1, keepdims=True)).sum(1)
        assert np.abs(got - want).max() < 1e-5
    assert np.abs(orc.eos_prob(w, h, False) - orc.eos_prob(w, h, True)).max() > 1e-3
