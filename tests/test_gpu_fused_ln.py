"""The LayerNorm + adaLN modulation fused into the residual GEMMs' epilogue
(EPI_RESID_GATED_LN: LN2 inside the O projection, the next block's LN1 inside
FFN2; dtts_dit_set_fused_ln) against the standalone LayerNorm kernels
(include/dit_manual.h:158-168 of the reference, checked against the reference
itself by the velocity tests).  Both paths run the same per-row arithmetic, so
the solves must be bit-identical, in bf16 and with e4m3 block weights, at batch
shapes whose 128-token blocks take one wave of the persistent GEMM, two (the
benchmark), several, a ragged last block, and with 128-wide tiles (8 tiles per
block instead of 4).  A second fused solve checks that the per-block arrival
counters are re-armed."""
import numpy as np
import pytest

import dtts
import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def w18():
    return synth.dit_weights(1, n_layers=18)


# (utterances, FM history length, O / FFN2 tile width); L = history + 4 tokens
CASES = [
    (2, 60, 256),     # 256 tokens: 2 blocks, one wave
    (64, 60, 256),    # 8192 tokens (the benchmark): 64 blocks, two waves
    (160, 60, 256),   # 20480 tokens: 160 blocks, five waves
    (3, 45, 256),     # 294 tokens: the last block holds 38 rows
    (64, 60, 128),    # 8 tiles of 128 columns per block
]


@pytest.mark.parametrize("dtype", [dtts.DTYPE_BF16, dtts.DTYPE_FP8], ids=["bf16", "e4m3"])
@pytest.mark.parametrize("n_utt,fm_len,bn", CASES)
def test_fused_layernorm_is_bit_identical(w18, dtype, n_utt, fm_len, bn):
    eng = dtts.DiT(w18, n_layers=18, dtype=dtype)
    try:
        eng.tune("o", bn, 4, 1)
        eng.tune("ffn2", bn, 4, 1)
        fc, fu = synth.fm_history(21, n_utt, fm_len, w18)
        z0 = synth.normal(21, "z0", (n_utt, 4, 128), 1.0)
        spk = synth.normal(21, "spk", (n_utt, 512), 1.0 / np.sqrt(512.0))
        eng.set_fused_ln(True)
        fused = eng.solve(fc, fu, z0, spk, nfe=3, cfg_scale=2.0)
        again = eng.solve(fc, fu, z0, spk, nfe=3, cfg_scale=2.0)
        eng.set_fused_ln(False)
        apart = eng.solve(fc, fu, z0, spk, nfe=3, cfg_scale=2.0)
        assert np.all(np.isfinite(fused))
        assert np.array_equal(fused, again)
        assert np.array_equal(fused, apart)
        assert not np.array_equal(fused, z0)
    finally:
        eng.close()


def test_fused_layernorm_launch_count(w18):
    """With the fusion, a forward launches one standalone LayerNorm (block 0's
    LN1) instead of two per block; the default is the standalone form."""
    eng = dtts.DiT(w18, n_layers=18)
    try:
        fc, fu = synth.fm_history(22, 2, 60, w18)
        z0 = synth.normal(22, "z0", (2, 4, 128), 1.0)
        eng.solve(fc, fu, z0, None, nfe=2, use_graph=False)
        default = eng.last_launch_count()
        eng.set_fused_ln(True)
        eng.solve(fc, fu, z0, None, nfe=2, use_graph=False)
        fused = eng.last_launch_count()
        eng.set_fused_ln(False)
        eng.solve(fc, fu, z0, None, nfe=2, use_graph=False)
        assert eng.last_launch_count() - fused == 2 * (2 * 18 - 1)
        assert eng.last_launch_count() == default
    finally:
        eng.close()
