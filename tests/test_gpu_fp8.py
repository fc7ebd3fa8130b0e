"""DiT FP8 path (DTTS_DTYPE_FP8: e4m3 x e4m3 tcgen05 GEMMs with per-channel
weight scales and per-row activation scales) on the GPU.  Checked two ways:
against the oracle's restatement of the same FP8 recipe (FP8_ORACLE_* in
helpers.py), and against the fp32 reference arithmetic at the FP8 bar (the
quantisation error itself, FP8_REL / FP8_COS).  The e4m3 GEMM and the e4m3
conversion are pinned exactly on their own."""
import numpy as np
import pytest

import dtts
import oracle as O
import synth
from helpers import (assert_fp8_close, assert_fp8_recipe_close, assert_fp8_solve_close,
                     assert_no_worse_than_recipe, rel)

pytestmark = pytest.mark.gpu


@pytest.fixture
def fp8_oracle(orc):
    orc.set_dit_fp8(1)
    yield orc
    orc.set_dit_fp8(0)


def test_device_e4m3_conversion_matches_oracle(orc):
    c = np.arange(256, dtype=np.uint8)
    d = orc.e4m3_decode(c)
    pos = np.sort(d[np.isfinite(d) & (d >= 0)])
    ties = (pos[:-1] + pos[1:]) / 2
    rng = np.random.default_rng(1)
    x = np.concatenate([d[np.isfinite(d)], ties, -ties, rng.standard_normal(5000) * np.exp(rng.uniform(-14, 7, 5000)),
                        [448.5, 464.0, 479.0, 1e6, -1e6, 1e-7, -1e-7, 2.0 ** -10, 3 * 2.0 ** -10]]).astype(np.float32)
    got = dtts.selftest_e4m3(x)
    want = orc.e4m3_encode(x)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, [(float(x[i]), int(got[i]), int(want[i])) for i in bad[:8]]


@pytest.mark.parametrize("bn", [128, 256])
def test_e4m3_gemm_matches_exact_product(orc, bn):
    """kind::f8f6f4 GEMM on e4m3 bytes with row and column scales: every product
    of two e4m3 values is exact in fp32, so the result equals the float64
    product up to the fp32 accumulation."""
    rng = np.random.default_rng(5)
    M, N, K = 300, 512, 1024
    finite = np.array([c for c in range(256) if c not in (0x7F, 0xFF)], np.uint8)
    A = rng.choice(finite, size=(M, K)).astype(np.uint8)
    B = rng.choice(finite, size=(N, K)).astype(np.uint8)
    sa = rng.uniform(0.5, 2.0, M).astype(np.float32) / 448
    sb = rng.uniform(0.5, 2.0, N).astype(np.float32) / 448
    bias = rng.standard_normal(N).astype(np.float32)
    got = dtts.selftest_gemm_e4m3(A, sa, B, sb, bias, bn=bn)
    lut = orc.e4m3_decode(np.arange(256, dtype=np.uint8)).astype(np.float64)
    lut[~np.isfinite(lut)] = 0
    want = (lut[A] @ lut[B].T) * sa[:, None].astype(np.float64) * sb[None, :].astype(np.float64) + bias
    assert rel(got, want) <= 1e-5, rel(got, want)


def _case(orc, L=64, rows=4, seed=21):
    w = synth.dit_weights(seed, n_layers=2, ada_bias_std=0.5)
    x = synth.normal(seed, "fp8.x", (rows, L, 1024), 1.0)
    cond = synth.normal(seed, "fp8.c", (rows, 1024), 1.0)
    mask, pos = orc.fm_mask(L, L - 4, 4), orc.fm_pos(L, L - 4, 4)
    return w, x, cond, mask, pos


def test_fp8_velocity_two_layers(orc, fp8_oracle):
    w, x, cond, mask, pos = _case(orc)
    eng = dtts.DiT(w, n_layers=2, dtype=dtts.DTYPE_FP8)
    got = eng.velocity(x, cond, mask, pos)
    eng.close()
    want8 = np.stack([fp8_oracle.dit_velocity(w, 2, x[r], cond[r], mask, pos) for r in range(x.shape[0])])
    assert_fp8_recipe_close(got, want8, "FP8 velocity vs FP8 oracle")
    orc.set_dit_fp8(0)
    want32 = np.stack([orc.dit_velocity(w, 2, x[r], cond[r], mask, pos) for r in range(x.shape[0])])
    assert_fp8_close(got, want32, "FP8 velocity vs fp32")
    assert_no_worse_than_recipe(got, want8, want32, "FP8 velocity")


@pytest.mark.parametrize("L", [17, 100, 256])
def test_fp8_blocks_ragged_and_long(orc, fp8_oracle, L):
    """One block at a ragged length (partial tiles) and past the short-attention
    limit (the tiled attention kernel's e4m3 output)."""
    w = synth.dit_weights(22, n_layers=1, ada_bias_std=0.5)
    h = synth.normal(22, "fp8.h", (3, L, 1024), 1.0)
    cond = synth.normal(22, "fp8.c", (3, 1024), 1.0)
    eng = dtts.DiT(w, n_layers=1, dtype=dtts.DTYPE_FP8)
    got = eng.blocks(h, cond)
    eng.close()
    want = np.stack([fp8_oracle.dit_block(w, 0, h[r], cond[r]) for r in range(3)])
    assert_fp8_recipe_close(got - h, want - h, f"FP8 block L={L}")


def test_fp8_solve_18_layers(orc, fp8_oracle):
    w = synth.dit_weights(1, n_layers=18)
    n_utt, fm_len = 2, 60
    fc, fu = synth.fm_history(9, n_utt, fm_len, w)
    z0 = synth.normal(9, "z0", (n_utt, 4, 128), 1.0)
    spk = synth.normal(9, "spk", (n_utt, 512), 1.0 / np.sqrt(512))
    eng = dtts.DiT(w, n_layers=18, dtype=dtts.DTYPE_FP8)
    got = eng.solve(fc, fu, z0, spk, nfe=3, cfg_scale=2.0)
    eng.close()
    want8 = fp8_oracle.euler_solve(w, 18, fc, fu, z0, spk, 1.5, nfe=3, cfg_scale=2.0)
    assert_fp8_solve_close(got - z0, want8 - z0, "FP8 18-layer solve vs FP8 oracle")
    orc.set_dit_fp8(0)
    want32 = orc.euler_solve(w, 18, fc, fu, z0, spk, 1.5, nfe=3, cfg_scale=2.0)
    assert_fp8_solve_close(got - z0, want32 - z0, "FP8 18-layer solve vs fp32")
    assert_no_worse_than_recipe(got - z0, want8 - z0, want32 - z0, "FP8 18-layer solve")


def test_fp8_config3_as_benchmarked(orc, fp8_oracle):
    """The FP8 twin of config 3 as benchmarked (64 utterances, NFE 10, CFG 2.0):
    utterances 0 and 63 against the FP8 recipe oracle and against fp32."""
    w = synth.dit_weights(1, n_layers=18)
    seed = 1000
    fc, fu = synth.fm_history(seed, 64, 60, w)
    z0 = synth.normal(seed, "z0", (64, 4, 128), 1.0)
    spk = synth.normal(seed, "spk", (64, 512), 1.0 / np.sqrt(512.0))
    eng = dtts.DiT(w, n_layers=18, dtype=dtts.DTYPE_FP8)
    got = eng.solve(fc, fu, z0, spk, nfe=10, cfg_scale=2.0)
    eng.close()
    for u in (0, 63):
        sl = slice(u, u + 1)
        fp8_oracle.set_dit_fp8(1)
        want8 = fp8_oracle.euler_solve(w, 18, fc[sl], fu[sl], z0[sl], spk[sl], 1.5, nfe=10, cfg_scale=2.0)[0]
        orc.set_dit_fp8(0)
        want32 = orc.euler_solve(w, 18, fc[sl], fu[sl], z0[sl], spk[sl], 1.5, nfe=10, cfg_scale=2.0)[0]
        d = got[u] - z0[u]
        assert_fp8_solve_close(d, want8 - z0[u], f"FP8 config 3 utterance {u} vs FP8 oracle")
        assert_fp8_solve_close(d, want32 - z0[u], f"FP8 config 3 utterance {u} vs fp32")
        assert_no_worse_than_recipe(d, want8 - z0[u], want32 - z0[u], f"FP8 config 3 utterance {u}")


def test_fp8_batch_independence_and_graph(orc):
    """Per-row scales keep utterances independent: one utterance solved alone is
    bit-identical to its row of a 16-utterance batch; graph == eager."""
    w = synth.dit_weights(3, n_layers=4)
    n_utt, fm_len = 16, 60
    fc, fu = synth.fm_history(13, n_utt, fm_len, w)
    z0 = synth.normal(13, "z0", (n_utt, 4, 128), 1.0)
    eng = dtts.DiT(w, n_layers=4, dtype=dtts.DTYPE_FP8)
    full = eng.solve(fc, fu, z0, None, nfe=4)
    eager = eng.solve(fc, fu, z0, None, nfe=4, use_graph=False)
    assert np.array_equal(full, eager)
    for u in (0, 11):
        one = eng.solve(fc[u:u + 1], fu[u:u + 1], z0[u:u + 1], None, nfe=4)
        assert np.array_equal(one[0], full[u])
    eng.close()
