"""The BigVGAN decoder on the device (dtts_voc_*) against the reference's own
bigvgan_decode (golden vectors from oracle/_ref) and the fp32 oracle
(oracle/voc_oracle.c).  Convolutions run in bf16 on the tensor cores with
fp32 accumulation and an fp32 residual stream; the LSTM bottleneck and the
activations are fp32.  Bar for the waveform (after tanh x 1.92): max
relative error <= VOC_REL and cosine >= VOC_COS (helpers.py); the activation
kernel alone: <= 1e-5."""
import os
import sys

import numpy as np
import pytest

import dtts
import oracle as O
import synth
from helpers import VOC_COS, VOC_REL, cos, rel

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_voc_golden as G  # noqa: E402

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "voc_ref_small.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="module")
def voc():
    w, _ = G.inputs()
    v = dtts.Vocoder(w, max_frames=16)
    yield v
    v.close()


def test_engine_filter_matches_reference_taps(golden):
    assert np.abs(dtts.voc_aa_filter() - golden["aa_filter"]).max() <= 1e-7


@pytest.mark.parametrize("per_channel", [False, True])
def test_activation_kernel_vs_oracle(orc, per_channel):
    rng = np.random.default_rng(11 + per_channel)
    L, ch = 300, 40
    x = rng.standard_normal((L, ch)).astype(np.float32)
    x[17, 3] = np.nan   # a non-finite input gives 0 after the snake, as in the reference
    al = rng.normal(0, 0.3, ch).astype(np.float32)
    be = rng.normal(0, 0.3, ch).astype(np.float32)
    f = O.aa_filter()
    fu = f + rng.normal(0, 1e-3, (ch, 12)).astype(np.float32) if per_channel else f
    fd = f + rng.normal(0, 1e-3, (ch, 12)).astype(np.float32) if per_channel else f
    got = dtts.selftest_voc_activation(x, al, be, fu, fd)
    want = orc.voc_activation(x, al, be, fu, fd)
    assert np.isfinite(got).all()
    assert rel(got, want) <= 1e-5


def test_decode_matches_reference_golden(voc, golden):
    _, lat = G.inputs()
    got = voc.decode(lat)
    want = golden["audio"]
    assert rel(got, want) <= VOC_REL and cos(got, want) >= VOC_COS, (rel(got, want), cos(got, want))


def test_decode_matches_oracle_longer(orc):
    w = synth.voc_weights(9, aa_filter=O.aa_filter())
    lat = synth.normal(9, "voc.long", (7, 128), 1.0)
    v = dtts.Vocoder(w, max_frames=8)
    got = v.decode(lat)
    again = v.decode(lat)
    v.close()
    want = orc.voc_decode(w, lat)
    assert np.array_equal(got, again)                      # no split reductions: repeatable
    assert rel(got, want) <= VOC_REL and cos(got, want) >= VOC_COS, (rel(got, want), cos(got, want))


def test_decode_is_causal_up_to_the_centred_conv(voc):
    """conv_pre looks two frames ahead and every later layer is causal, so a
    change of the last frame leaves the audio of frames 0 .. n-4 untouched."""
    _, lat = G.inputs()
    lat = np.concatenate([lat, synth.normal(5, "voc.more", (4, 128), 1.0)])   # 6 frames
    a = voc.decode(lat)
    lat2 = lat.copy()
    lat2[-1] += 1.0
    b = voc.decode(lat2)
    n = lat.shape[0]
    assert np.array_equal(a[:(n - 3) * 1920], b[:(n - 3) * 1920])
    assert not np.array_equal(a[(n - 3) * 1920:], b[(n - 3) * 1920:])


def test_decode_device_buffers(voc):
    import torch
    _, lat = G.inputs()
    want = voc.decode(lat)
    d_lat = torch.from_numpy(lat).cuda()
    d_out = torch.empty(lat.shape[0] * 1920, device="cuda")
    voc.decode(d_lat, out=d_out, mem=dtts.MEM_DEVICE)
    torch.cuda.synchronize()
    assert np.array_equal(d_out.cpu().numpy(), want)


def test_decode_rejects_bad_arguments(voc):
    with pytest.raises(dtts.DttsError):
        voc.decode(np.zeros((17, 128), np.float32))   # beyond max_frames
