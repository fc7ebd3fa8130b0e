"""Engines created from safetensors checkpoints, the way a pipeline loads the
model (dtts_dit_create_from_safetensors / dtts_pe_create_from_safetensors in
place of load_dit_weights, src/utils/dit_loader.cpp:15, and
load_patchenc_weights, src/utils/patchenc_loader.cpp:14): checkpoints written
with the reference's tensor names (dit_loader.cpp:47-115,
patchenc_loader.cpp:36-69) in BF16 and in F16.  An engine created from the
file must compute exactly what an engine created from the same values, rounded
the same way and passed as arrays, computes: bit for bit."""
import numpy as np
import pytest

import dtts
import synth
from helpers import assert_bf16_close, bf16, bf16_bits, f16_bits, write_safetensors

pytestmark = pytest.mark.gpu

ENC = {
    "BF16": (bf16_bits, bf16),
    "F16": (f16_bits, lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32)),
}


def _write(path, w, dtype):
    bits, _ = ENC[dtype]
    write_safetensors(path, {k: (dtype, bits(v)) for k, v in w.items()}, metadata={"format": "pt"})


def _rounded(w, dtype):
    _, rnd = ENC[dtype]
    return {k: rnd(v) for k, v in w.items()}


@pytest.mark.parametrize("dtype", ["BF16", "F16"])
def test_dit_from_checkpoint_equals_arrays(tmp_path, orc, dtype):
    n_layers = 2
    w = synth.dit_weights(17, n_layers=n_layers, ada_bias_std=0.3)
    path = str(tmp_path / f"dit_{dtype}.safetensors")
    _write(path, w, dtype)
    a = dtts.DiT.from_safetensors(path, n_layers=n_layers)
    b = dtts.DiT(_rounded(w, dtype), n_layers=n_layers)
    L, rows = 24, 4
    x = synth.normal(17, "ck.x", (rows, L, 1024), 1.0)
    cond = synth.normal(17, "ck.c", (rows, 1024), 1.0)
    mask, pos = orc.fm_mask(L, L - 4, 4), orc.fm_pos(L, L - 4, 4)
    assert np.array_equal(a.velocity(x, cond, mask, pos), b.velocity(x, cond, mask, pos))
    spk = synth.normal(17, "ck.spk", (512,), 1.0 / np.sqrt(512.0))
    assert np.array_equal(a.cond(0.4, spk, 1.5), b.cond(0.4, spk, 1.5))
    fc, fu = synth.fm_history(17, 2, 12, w)
    z0 = synth.normal(17, "ck.z0", (2, 4, 128), 1.0)
    assert np.array_equal(a.solve(fc, fu, z0, None, nfe=4), b.solve(fc, fu, z0, None, nfe=4))
    a.close()
    b.close()


@pytest.mark.parametrize("dtype", ["BF16", "F16"])
def test_pe_from_checkpoint_equals_arrays(tmp_path, dtype):
    n_layers = 2
    w = synth.pe_weights(18, n_layers=n_layers)
    path = str(tmp_path / f"pe_{dtype}.safetensors")
    _write(path, w, dtype)
    a = dtts.PatchEncoder.from_safetensors(path, n_layers=n_layers, max_batch=2, max_tokens=320)
    b = dtts.PatchEncoder(_rounded(w, dtype), n_layers=n_layers, max_batch=2, max_tokens=320)
    # 2 x 300 tokens: calls of more than 256 tokens sum every K in a fixed order,
    # so the two engines must agree bit for bit
    fr = synth.normal(18, "ck.fr", (2, 604, 128), 1.0)
    assert np.array_equal(a.forward(fr[:, :600]), b.forward(fr[:, :600]))
    a.reset(2)
    b.reset(2)
    assert np.array_equal(a.decode(fr[:, :600]), b.decode(fr[:, :600]))
    # a one-patch decode step (4 tokens) splits its GEMMs along K and reduce-adds
    # the parts in arrival order; a last-bit difference of an fp32 sum can move a
    # bf16 rounding of the next layer's input, so two runs agree at the bf16 bar
    assert_bf16_close(a.decode(fr[:, 600:]), b.decode(fr[:, 600:]), "decode step")
    a.close()
    b.close()


def test_checkpoint_missing_required_tensor(tmp_path):
    w = synth.pe_weights(18, n_layers=1)
    del w["patch_encoder.in_proj.weight"]
    path = str(tmp_path / "pe_bad.safetensors")
    _write(path, w, "BF16")
    with pytest.raises(dtts.DttsError) as e:
        dtts.PatchEncoder.from_safetensors(path, n_layers=1, max_batch=1, max_tokens=8)
    assert e.value.status == dtts.ERR_IO
