"""Config 1: one DiT self-attention sublayer, fp32, X ~ N(0,1) [B=2, L=64,
1024] (seed 0), Wq/k/v/o ~ N(0,0.02) with zero bias, qk-norm gains 1+N(0,0.02),
16 heads of 64, bidirectional, RoPE on positions 0..63 -- against the
reference's own manual_attention (include/dit_manual.h:88-146, compiled in
oracle/_ref).  Bar: fp32 max relative error <= 1e-3; the bf16 variant of the
same sublayer is held to the bf16 bar."""
import numpy as np
import pytest

import dtts
import synth
from helpers import F32_REL, assert_bf16_close, rel

pytestmark = pytest.mark.gpu


def _config1():
    w = synth.dit_weights(0, n_layers=1)
    p = "velocity_field_predictor.blocks.0."
    W = [w[p + n] for n in ("attn.q_proj.weight", "attn.k_proj.weight", "attn.v_proj.weight", "attn.o_proj.weight")]
    bo = np.zeros(1024, np.float32)
    return W, bo, w[p + "attn.q_norm.weight"], w[p + "attn.k_norm.weight"]


@pytest.fixture(scope="module")
def config1(ref):
    W, bo, qn, kn = _config1()
    x = synth.normal(0, "c1.x", (2, 64, 1024), 1.0)
    want = np.stack([ref.manual_attention(x[i], *W, bo, qn, kn) for i in range(2)])
    return W, bo, qn, kn, x, want


def test_config1_fp32_matches_reference(config1):
    W, bo, qn, kn, x, want = config1
    a = dtts.Attention(*W, bo, qn, kn, dtype=dtts.DTYPE_F32)
    got = a.forward(x)
    assert rel(got, want) <= F32_REL
    a.close()


def test_config1_bf16(config1):
    W, bo, qn, kn, x, want = config1
    a = dtts.Attention(*W, bo, qn, kn, dtype=dtts.DTYPE_BF16)
    assert_bf16_close(a.forward(x), want, "bf16 attention sublayer")
    a.close()


def test_sublayer_mask_and_pos_ids(ref, orc):
    W, _, qn, kn = _config1()
    bo = synth.normal(0, "c1.bo", (1024,), 0.02)
    L = 24
    x = synth.normal(1, "c1.x2", (1, L, 1024), 1.0)
    mask, pos = orc.fm_mask(L, L - 4, 4), orc.fm_pos(L, L - 4, 4)
    want = ref.manual_attention(x[0], *W, bo, qn, kn, mask=mask, pos=pos)[None]
    a = dtts.Attention(*W, bo, qn, kn, dtype=dtts.DTYPE_F32)
    assert rel(a.forward(x, mask, pos), want) <= F32_REL
    a.close()
