"""FM history on the device (dtts_fm_*): the v4 pipeline's buffer assembly
(src/e2e_pipeline_v4.cpp:324-340, 551-588) and EOS head (:598-619), checked
against the oracle's fp32 projections and EOS restatement, and the solve on
the device-resident history against the solve on host buffers (bit-identical)
and against the oracle (bf16 bar)."""
import numpy as np
import pytest

import dtts
import synth
from helpers import F32_REL, assert_bf16_close, rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    w = synth.dit_weights(31, n_layers=2, ada_bias_std=0.5)
    eng = dtts.DiT(w, n_layers=2)
    yield w, eng
    eng.close()


def test_fm_history_rows_and_eos(model, orc):
    w, eng = model
    n = 3
    fm = dtts.FMHistory(eng, n_utt=n, capacity=16)
    h0 = synth.normal(31, "fm.h0", (n, 1536), 1.0)
    z = synth.normal(31, "fm.z", (n, 4, 128), 1.0)
    h1 = synth.normal(31, "fm.h1", (n, 1536), 1.0)
    fm.start(h0)
    fm.append_latents(z)
    p = fm.append_hidden(h1)
    p_as = None
    assert fm.length() == 6
    cond, uncond = fm.read()
    hp = lambda x: orc.linear_rows(x, w["hidden_proj.weight"], w["hidden_proj.bias"])
    lp = lambda x: orc.linear_rows(x, w["latent_proj.weight"], w["latent_proj.bias"])
    want_c = np.concatenate([hp(h0)[:, None], lp(z.reshape(-1, 128)).reshape(n, 4, 1024), hp(h1)[:, None]], 1)
    null = np.broadcast_to(w["hidden_proj.bias"], (n, 1, 1024))
    want_u = np.concatenate([null, lp(z.reshape(-1, 128)).reshape(n, 4, 1024), null], 1)
    assert rel(cond, want_c) <= 1e-5 and rel(uncond, want_u) <= 1e-5
    assert np.abs(p - orc.eos_prob(w, h1, False)).max() < 1e-5
    fm2 = dtts.FMHistory(eng, n_utt=n, capacity=2)
    fm2.start(h0)
    p_as = fm2.append_hidden(h1, eos_act=dtts.EOS_AS_WRITTEN)
    assert np.abs(p_as - orc.eos_prob(w, h1, True)).max() < 1e-5
    with pytest.raises(dtts.DttsError):
        fm2.append_hidden(h1)          # capacity 2 reached
    fm.close()
    fm2.close()


def test_solve_on_device_history(model, orc):
    """A few AR steps driven entirely through the device history: each solve
    equals the engine's solve of the same rows passed from the host (bitwise),
    and the oracle's solve of those rows (bf16 bar)."""
    w, eng = model
    n, patch = 2, 4
    fm = dtts.FMHistory(eng, n_utt=n, capacity=64)
    fm.start(synth.normal(32, "ar.h0", (n, 1536), 1.0))
    spk = synth.normal(32, "ar.spk", (n, 512), 1.0 / np.sqrt(512))
    for step in range(3):
        z0 = synth.normal(32, f"ar.z0.{step}", (n, patch, 128), 1.0)
        got = fm.solve(z0, spk, nfe=3)
        cond, uncond = fm.read()
        host = eng.solve(cond, uncond, z0, spk, nfe=3)
        assert np.array_equal(got, host)
        if step == 2:
            want = orc.euler_solve(w, 2, cond, uncond, z0, spk, 1.5, nfe=3, cfg_scale=2.0)
            assert_bf16_close(got - z0, want - z0, "solve on the device FM history")
        fm.append_latents(got)
        fm.append_hidden(synth.normal(32, f"ar.h.{step}", (n, 1536), 1.0), eos=False)
    assert fm.length() == 1 + 3 * (patch + 1)
    fm.close()
