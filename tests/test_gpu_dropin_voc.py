"""The vocoder drop-in (dots.tts.cpp_b200/dropin/dtts_dropin_voc.cpp) called as
the reference's pipelines call it: tests/cpp/dropin_voc_test.cpp fills the
reference's BigVGANDecoder (include/bigvgan_cpp.h) with bigvgan_load from a
safetensors checkpoint, runs bigvgan_decode twice (the second call must reuse
the engine and repeat the result bit for bit) and bigvgan_free; the audio is
compared with the fp32 oracle at the vocoder bar."""
import os
import subprocess

import numpy as np
import pytest

import oracle as O
import synth
from helpers import VOC_COS, VOC_REL, cos, rel, write_safetensors

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tests", "cpp", "_bin", "dropin_voc_test")


def test_bigvgan_dropin_matches_oracle(tmp_path, orc):
    if not os.path.exists(BIN):
        pytest.skip("tests/cpp/_bin/dropin_voc_test is built by __graft_entry__.build() where the reference headers exist")
    w = synth.voc_weights(21, aa_filter=O.aa_filter())
    n = 3
    lat = synth.normal(21, "dropin.voc", (n, 128), 1.0)
    write_safetensors(str(tmp_path / "voc.safetensors"), {k: ("F32", v) for k, v in w.items()})
    lat.tofile(str(tmp_path / "lat.bin"))
    r = subprocess.run([BIN, str(tmp_path / "voc.safetensors"), str(tmp_path / "lat.bin"), str(tmp_path / "out.bin"),
                        str(n)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    got = np.fromfile(str(tmp_path / "out.bin"), np.float32)
    want = orc.voc_decode(w, lat)
    assert got.shape == want.shape
    assert rel(got, want) <= VOC_REL and cos(got, want) >= VOC_COS, (rel(got, want), cos(got, want))
