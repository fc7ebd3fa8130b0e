"""The oracle's e4m3 arithmetic (the FP8 weight path's quantisation recipe,
which has no counterpart in the fp32 reference) pinned against PyTorch's
float8_e4m3fn conversion, and the library's host-side weight quantiser
checked against it."""
import numpy as np
import pytest

import dtts
import oracle as O
import synth
from helpers import cos, rel


@pytest.fixture(scope="module")
def codes(orc):
    c = np.arange(256, dtype=np.uint8)
    return c, orc.e4m3_decode(c)


def test_e4m3_format(orc, codes):
    c, d = codes
    fin = np.isfinite(d)
    assert fin.sum() == 254                      # 0x7f and 0xff are NaN
    assert d[0x7e] == 448.0 and d[0x01] == 2.0 ** -9 and d[0x08] == 2.0 ** -6
    nz = fin & (d != 0)
    assert np.array_equal(orc.e4m3_encode(d[nz]), c[nz])   # every finite code round-trips
    assert orc.e4m3_encode([448.5, 464.0, 1e30, -1e30, np.inf]).tolist() == [0x7E, 0x7E, 0x7E, 0xFE, 0x7E]


def test_e4m3_matches_torch(orc, codes):
    torch = pytest.importorskip("torch")
    _, d = codes
    pos = np.sort(d[np.isfinite(d) & (d >= 0)])
    ties = (pos[:-1] + pos[1:]) / 2                        # exact midpoints: round to even
    rng = np.random.default_rng(0)
    x = rng.standard_normal(20000) * np.exp(rng.uniform(-13, 6, 20000))
    x = np.concatenate([x, ties, -ties]).astype(np.float32)
    x = x[np.abs(x) < 448]
    mine = orc.e4m3_decode(orc.e4m3_encode(x))
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).to(torch.float32).numpy()
    assert np.array_equal(mine, ref)


def test_library_weight_quantiser_matches_oracle(orc, dtts_mod):
    w = synth.normal(3, "q.w", (64, 256), 0.02)
    w[5] = 0.0
    w[7, 3] = 1e3
    q, sc = dtts.fp8_quantize_rows(w)
    amax = np.abs(w).max(axis=1)
    assert sc[5] == 0 and np.all(q[5] == 0)
    ok = amax > 0
    assert np.array_equal(sc[ok], (amax[ok] / np.float32(448)).astype(np.float32))
    inv = (np.float32(448) / amax[ok]).astype(np.float32)
    want = orc.e4m3_encode((w[ok] * inv[:, None]).astype(np.float32)).reshape(-1, 256)
    assert np.array_equal(q[ok], want)


def test_fp8_block_recipe_close_to_fp32(orc):
    """Size of the FP8 recipe's own error on one block (oracle against oracle):
    the bar the engine's FP8 path is held to against the fp32 reference."""
    w = synth.dit_weights(1, n_layers=1, ada_bias_std=0.5)
    L = 32
    h = synth.normal(4, "h", (L, 1024), 1.0)
    cond = synth.normal(4, "c", (1024,), 1.0)
    a = orc.dit_block(w, 0, h, cond)
    orc.set_dit_fp8(1)
    try:
        b = orc.dit_block(w, 0, h, cond)
    finally:
        orc.set_dit_fp8(0)
    assert 1e-3 < rel(b - h, a - h) < 0.1 and cos(b - h, a - h) > 0.995
