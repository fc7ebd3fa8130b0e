"""The LLM restatement (oracle/llm_oracle.py, numpy fp32 after
src/llm_manual.cpp) pinned against the reference's own llm_kv_cache_init /
llm_kv_cache_step: the committed golden vectors (tests/golden/make_llm_golden.py,
from the reference built into oracle/_ref) and, where oracle/_ref is present, a
live run on other inputs.  Plus the cache properties the reference relies on:
a step equals the last row of the longer prefill, and a one-token prompt."""
import os
import sys

import numpy as np
import pytest

import llm_oracle as LO
import synth
from helpers import rel

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_llm_golden as G  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "llm_ref_small.npz")
# fp32 restatement against fp32 reference loops: summation order only
BAR = 1e-4


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="module")
def w2():
    return G.weights()


@pytest.mark.parametrize("case", range(len(G.CASES)))
def test_restatement_matches_reference_golden(golden, w2, case):
    p, s = G.inputs(case)
    ph, sh = LO.run(w2, G.N_LAYERS, p, s)
    assert ph.shape == golden[f"prompt_hidden{case}"].shape
    assert sh.shape == golden[f"step_hidden{case}"].shape
    assert rel(ph, golden[f"prompt_hidden{case}"]) <= BAR
    assert rel(sh, golden[f"step_hidden{case}"]) <= BAR


def test_restatement_matches_reference_live(ref):
    w = synth.llm_weights(23, n_layers=3)
    p = synth.normal(23, "llm.live_p", (6, 1536), 1.5)
    s = synth.normal(23, "llm.live_s", (5, 1536), 1.5)
    want_p, want_s = ref.llm_run(w, 3, p, s)
    got_p, got_s = LO.run(w, 3, p, s)
    assert rel(got_p, want_p) <= BAR
    assert rel(got_s, want_s) <= BAR


def test_step_equals_longer_prefill(w2):
    p = synth.normal(31, "llm.prop", (8, 1536), 1.0)
    full = LO.LLMOracle(w2, G.N_LAYERS).prefill(p)
    o = LO.LLMOracle(w2, G.N_LAYERS)
    o.prefill(p[:5])
    stepped = np.stack([o.step(p[t]) for t in range(5, 8)])
    assert o.length == 8
    assert rel(stepped, full[5:]) <= 1e-5


def test_rope_tables_known_answers():
    cs, sn = LO.rope_tables(np.array([0.0, 1.0]))
    assert np.all(cs[0] == 1.0) and np.all(sn[0] == 0.0)
    # frequency 0 rotates by the position itself; the last by 1e6^(-63/64) per position
    assert abs(float(cs[1, 0]) - np.cos(1.0)) < 1e-6 and abs(float(sn[1, 0]) - np.sin(1.0)) < 1e-6
    assert abs(float(sn[1, 63]) - 1e6 ** (-63 / 64)) < 1e-8
