"""The vocoder oracle (oracle/voc_oracle.c, the fp32 restatement of
src/modules/vocoder/bigvgan_cpp.cpp and lstm.cpp) pinned against the
reference's own bigvgan_decode: the committed golden vectors
(tests/golden/make_voc_golden.py, from the reference built into oracle/_ref)
and, where oracle/_ref is present, a live run on other inputs.  Also the
Kaiser-sinc filter restatement against the 12 taps the reference hard-codes,
and known answers of the anti-aliased SnakeBeta activation."""
import os
import sys

import numpy as np
import pytest

import oracle as O
import synth
from helpers import rel

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_voc_golden as G  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "voc_ref_small.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_aa_filter_restatement_matches_reference_taps(golden):
    f = O.aa_filter()
    assert np.abs(f - golden["aa_filter"]).max() <= 1e-7
    assert abs(float(f.sum()) - 1.0) < 1e-6 and np.allclose(f, f[::-1])


def test_oracle_decode_matches_reference_golden(orc, golden):
    w, lat = G.inputs()
    got = orc.voc_decode(w, lat, aa=golden["aa_filter"])
    assert got.shape == golden["audio"].shape == (G.N_FRAMES * 1920,)
    assert rel(got, golden["audio"]) <= 2e-5


def test_oracle_decode_matches_reference_live(orc, ref):
    w = synth.voc_weights(7, aa_filter=O.aa_filter())
    lat = synth.normal(7, "voc.live", (1, 128), 1.5)
    want = ref.voc_decode(w, lat)
    got = orc.voc_decode(w, lat)
    assert rel(got, want) <= 2e-5


def test_activation_known_answers(orc):
    """Constant input c: once the 12 up-taps are all inside the signal
    (t >= 6) u = c (each parity class of the symmetric filter sums to 1/2,
    times the ratio 2), so the output settles to snake(c) = c + sin^2(a c)/b
    from t = 11 on; and the activation is causal."""
    f = O.aa_filter()
    ch, L = 5, 40
    c = np.linspace(-1.5, 2.0, ch).astype(np.float32)
    x = np.tile(c, (L, 1))
    alpha = np.linspace(-0.3, 0.4, ch).astype(np.float32)
    beta = np.linspace(0.2, -0.5, ch).astype(np.float32)
    y = orc.voc_activation(x, alpha, beta, f, f)
    a, b = np.exp(alpha), np.exp(beta)
    want = c + np.sin(a * c) ** 2 / (b + 1e-9)
    assert np.abs(y[11:] - want).max() <= 1e-5
    x2 = x.copy()
    x2[25:] += 3.0
    y2 = orc.voc_activation(x2, alpha, beta, f, f)
    assert np.array_equal(y[:25], y2[:25]) and not np.array_equal(y[25:], y2[25:])


def test_activation_per_channel_filters(orc):
    """fch = ch filters equal to the shared filter give the shared result."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((33, 6)).astype(np.float32)
    al, be = rng.normal(0, 0.1, 6).astype(np.float32), rng.normal(0, 0.1, 6).astype(np.float32)
    f = O.aa_filter()
    y1 = orc.voc_activation(x, al, be, f, f)
    y2 = orc.voc_activation(x, al, be, np.tile(f, (6, 1)), np.tile(f, (6, 1)))
    assert np.array_equal(y1, y2)
