"""The LLM decoder step (dtts_llm_*) against the reference's own
src/llm_manual.cpp (llm_kv_cache_init, llm_kv_cache_step), built from the
reference tree into oracle/_ref: a 2-layer decoder with seeded N(0, 0.02)
weights, several sequences prefilled together and stepped together; bf16 bar
on the final-normed hidden states."""
import numpy as np
import pytest

import dtts
import synth
from helpers import assert_bf16_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def weights():
    return synth.llm_weights(3, n_layers=2)


def test_prefill_and_steps_match_reference(weights, ref):
    B, n_tok, steps = 3, 13, 4
    prompts = synth.normal(5, "llm.prompt", (B, n_tok, 1536), 1.0)
    step_emb = synth.normal(5, "llm.steps", (steps, B, 1536), 1.0)
    llm = dtts.LLM(weights, n_layers=2, max_batch=4, max_seq=64)
    got_p = llm.prefill(prompts)
    got_s = np.stack([llm.step(step_emb[s]) for s in range(steps)], axis=1)   # [B][steps][1536]
    assert llm.length() == n_tok + steps
    llm.close()
    for b in range(B):
        want_p, want_s = ref.llm_run(weights, 2, prompts[b], step_emb[:, b])
        assert_bf16_close(got_p[b], want_p, f"prefill hidden, sequence {b}")
        assert_bf16_close(got_s[b], want_s, f"step hidden, sequence {b}")


def test_step_equals_longer_prefill(weights):
    """Causality of the cache: stepping one embedding after a prefill gives the
    hidden state that prefilling the longer prompt gives for that token."""
    B, n_tok = 2, 9
    prompts = synth.normal(6, "llm.p2", (B, n_tok + 1, 1536), 1.0)
    llm = dtts.LLM(weights, n_layers=2, max_batch=2, max_seq=32)
    full = llm.prefill(prompts)
    llm.prefill(prompts[:, :n_tok])
    stepped = llm.step(prompts[:, n_tok])
    llm.close()
    assert_bf16_close(stepped, full[:, n_tok], "step vs longer prefill")


def test_cache_capacity_is_checked(weights):
    llm = dtts.LLM(weights, n_layers=2, max_batch=1, max_seq=4)
    llm.prefill(synth.normal(7, "llm.c", (1, 4, 1536), 1.0))
    with pytest.raises(dtts.DttsError):
        llm.step(synth.normal(7, "llm.c2", (1, 1536), 1.0))
    llm.close()
