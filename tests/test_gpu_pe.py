"""PatchEncoder through the C ABI: prefill against the CPU oracle
(restatement of src/modules/backbone/patchenc.cpp), the reference's
output pairing as written, and the new streaming decode against the
stateless forward over the whole prefix (the incremental == full pattern of
the reference's test/test_kv_cache_correctness.cpp)."""
import numpy as np
import pytest

import dtts
import oracle as O
import synth
from helpers import assert_bf16_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def w24():
    return synth.pe_weights(2, n_layers=24)


@pytest.fixture(scope="module")
def pe24(w24):
    p = dtts.PatchEncoder(w24, n_layers=24, max_batch=32, max_tokens=512)
    yield p
    p.close()


def test_prefill_500_frames_24_layers(w24, pe24, orc):
    fr = synth.normal(2, "pe.frames", (2, 500, 128), 1.0)
    got = pe24.forward(fr)
    want = orc.pe_forward(w24, 24, fr[0])
    assert_bf16_close(got[0], want, "PE prefill 500 frames")


@pytest.mark.parametrize("pair_mode", [dtts.PAIR_ADJACENT, dtts.PAIR_AS_WRITTEN])
def test_prefill_pairing_small(orc, pair_mode):
    w = synth.pe_weights(5, n_layers=2)
    p = dtts.PatchEncoder(w, n_layers=2, max_batch=4, max_tokens=64)
    fr = synth.normal(5, "fr", (3, 36, 128), 1.0)
    got = p.forward(fr, pair_mode)
    want = np.stack([orc.pe_forward(w, 2, fr[i], pair_mode) for i in range(3)])
    assert_bf16_close(got, want, f"PE pairing {pair_mode}")
    p.close()


def test_decode_equals_full_forward(w24, pe24):
    """Prefill 40 frames, then 15 one-patch decode steps: every output equals
    the stateless forward over the whole prefix (bf16 tolerance; the same
    kernels, only the split of the sequence into calls differs)."""
    B = 4
    fr = synth.normal(7, "pe.stream", (B, 100, 128), 1.0)
    full = pe24.forward(fr)
    pe24.reset(B)
    outs = [pe24.decode(fr[:, :40])]
    for s in range(40, 100, 4):
        outs.append(pe24.decode(fr[:, s:s + 4]))
    inc = np.concatenate(outs, axis=1)
    assert pe24.length() == 50
    assert_bf16_close(inc, full, "decode vs full")


def test_decode_batch_of_32_against_oracle(w24, pe24, orc):
    B = 32
    fr = synth.normal(8, "pe.b32", (B, 16, 128), 1.0)
    pe24.reset(B)
    a = pe24.decode(fr[:, :8])
    b = pe24.decode(fr[:, 8:12])
    c = pe24.decode(fr[:, 12:16])
    got = np.concatenate([a, b, c], 1)
    for i in (0, 31):
        assert_bf16_close(got[i], orc.pe_forward(w24, 24, fr[i]), f"stream {i}")


def test_prefill_against_reference_patchenc(w24, pe24, ref):
    """The engine's prefill with the as-written pairing against the reference's own
    patchenc_forward (src/modules/backbone/patchenc.cpp:146-239, compiled in
    oracle/_ref over the eager ggml stand-in): 500 frames, 24 layers."""
    fr = synth.normal(3, "pe.ref", (1, 500, 128), 1.0)
    got = pe24.forward(fr, dtts.PAIR_AS_WRITTEN)
    assert_bf16_close(got[0], ref.pe_forward(w24, 24, fr[0]), "PE prefill vs the reference's patchenc_forward")


def test_decode_at_benchmark_depth(w24, pe24, orc):
    """Config 4 as benchmarked: 32 streams, a 500-frame prefill (250 tokens), then
    125 one-patch decode steps, filling the cache to 500 tokens.  Outputs of
    steps 1, 60 and 125 for streams 0 and 31 against the oracle's stateless
    forward over the whole 1000 frames (causal, so its output for patch q is
    the output over the prefix ending there; the incremental == full pattern of
    the reference's test/test_kv_cache_correctness.cpp)."""
    B, pre, steps = 32, 500, 125
    fr = synth.normal(9, "pe.deep", (B, pre + 4 * steps, 128), 1.0)
    pe24.reset(B)
    first = pe24.decode(fr[:, :pre])
    got = {}
    for s in range(1, steps + 1):
        o = pe24.decode(fr[:, pre + 4 * (s - 1):pre + 4 * s])
        if s in (1, 60, 125):
            got[s] = o[:, 0]
    assert pe24.length() == (pre + 4 * steps) // 2
    for i in (0, 31):
        want = orc.pe_forward(w24, 24, fr[i])
        assert_bf16_close(first[i], want[:pre // 4], f"stream {i} prefill")
        for s, o in got.items():
            assert_bf16_close(o[i], want[pre // 4 + s - 1], f"stream {i} step {s}")


def test_cache_capacity_and_batch_errors(w24):
    p = dtts.PatchEncoder(w24, n_layers=24, max_batch=2, max_tokens=8)
    p.reset(2)
    p.decode(np.zeros((2, 16, 128), np.float32))
    with pytest.raises(dtts.DttsError) as e:
        p.decode(np.zeros((2, 4, 128), np.float32))
    assert e.value.status == dtts.ERR_ARG
    with pytest.raises(dtts.DttsError):
        p.reset(3)
    with pytest.raises(dtts.DttsError):
        p.forward(np.zeros((2, 6, 128), np.float32))
    p.close()
