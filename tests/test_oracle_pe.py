"""PatchEncoder oracle (restatement of src/modules/backbone/patchenc.cpp; ggml
is not vendored, so its rope/rms_norm/silu numerics are restated from ggml's
published definitions).  Checked here through properties of the algorithm."""
import numpy as np

import oracle as O
import synth
from helpers import rel


def _w(n_layers=1, seed=21):
    return synth.pe_weights(seed, n_layers=n_layers)


def test_conv_taps_and_in_proj(orc):
    """0 layers: output = out_proj(pairs(in_proj(conv(x)))) with taps 2t-1, 2t
    (patchenc.cpp:19-39) -- recomputed in numpy."""
    w = _w()
    fr = synth.normal(3, "fr", (8, 128), 1.0)
    out, h = orc.pe_forward(w, 0, fr, want_hidden=True)
    cw, cb = w["patch_encoder.ds_proj.weight"].astype(np.float64), w["patch_encoder.ds_proj.bias"]
    T = 4
    xc = np.zeros((T, 128))
    for t in range(T):
        prev = fr[2 * t - 1] if t > 0 else np.zeros(128)
        xc[t] = cb + cw[:, :, 0] @ prev + cw[:, :, 1] @ fr[2 * t]
    hh = xc @ w["patch_encoder.in_proj.weight"].T.astype(np.float64) + w["patch_encoder.in_proj.bias"]
    assert rel(h, hh) < 1e-5
    cat = hh.reshape(2, 2048)
    want = cat @ w["patch_encoder.out_proj.weight"].T.astype(np.float64) + w["patch_encoder.out_proj.bias"]
    assert rel(out, want) < 1e-5


def test_causal_prefix_invariance(orc):
    """Attention and conv are causal: outputs for the first k patches do not
    depend on later frames (the basis of the streaming decode)."""
    w = _w(n_layers=2)
    fr = synth.normal(4, "fr", (16, 128), 1.0)
    full = orc.pe_forward(w, 2, fr)
    fr2 = fr.copy()
    fr2[9:] = synth.normal(5, "fr2", (7, 128), 1.0)
    part = orc.pe_forward(w, 2, fr2)
    assert rel(full[:2], part[:2]) < 1e-6
    assert np.abs(full[2:] - part[2:]).max() > 1e-3
    prefix = orc.pe_forward(w, 2, fr[:8])
    assert rel(prefix, full[:2]) < 1e-6


def test_pairing_as_written(orc):
    """patchenc.cpp:230-232 reshape/permute/reshape: output q half s takes token
    2*((2q+s) % n) + (2q+s) // n; identical to adjacent pairing for one patch."""
    w = _w()
    fr = synth.normal(6, "fr", (12, 128), 1.0)
    adj, h = orc.pe_forward(w, 1, fr, O.PAIR_ADJACENT, want_hidden=True)
    asw = orc.pe_forward(w, 1, fr, O.PAIR_AS_WRITTEN)
    n = 3
    cat = np.zeros((n, 2048))
    for q in range(n):
        for s in range(2):
            g = 2 * q + s
            cat[q, s * 1024:(s + 1) * 1024] = h[2 * (g % n) + g // n]
    want = cat @ w["patch_encoder.out_proj.weight"].T.astype(np.float64) + w["patch_encoder.out_proj.bias"]
    assert rel(asw, want) < 1e-5
    assert rel(adj[0], asw[0]) > 1e-3            # q = 0 pairs tokens (0, 2) as written, (0, 1) adjacent
    one = fr[:4]
    assert rel(orc.pe_forward(w, 1, one, O.PAIR_ADJACENT), orc.pe_forward(w, 1, one, O.PAIR_AS_WRITTEN)) == 0.0
