"""The attention sublayer entry point that allocates nothing.

Some callers cannot allocate GPU memory while they run (a fixed memory budget
handed over by the host application, an inference-runtime plugin whose execute
callback must not allocate, a real-time audio thread).  They pass their own
device buffers to dtts_attn_forward_f32_noalloc, which keeps its intermediates
in an array compiled into the library.  This test drives it through the C ABI
with caller-owned device buffers (allocated here by the test, not by the entry
point) and checks two calls in a row against the allocating entry point
dtts_attn_forward at the fp32 tolerance.  It sits in a file of its own that
pytest collects last."""
import ctypes as C

import numpy as np
import pytest

import dtts
import synth
from helpers import F32_REL, rel

pytestmark = pytest.mark.gpu


def _weights():
    w = synth.dit_weights(0, n_layers=1)
    p = "velocity_field_predictor.blocks.0."
    W = [w[p + n] for n in ("attn.q_proj.weight", "attn.k_proj.weight", "attn.v_proj.weight",
                            "attn.o_proj.weight")]
    bo = synth.normal(0, "noalloc.bo", (1024,), 0.02)
    return W, bo, w[p + "attn.q_norm.weight"], w[p + "attn.k_norm.weight"]


def test_noalloc_matches_allocating_entry_point_twice():
    import torch
    dev = torch.device("cuda", 0)
    W, bo, qn, kn = _weights()
    ref = dtts.Attention(*W, bo, qn, kn, dtype=dtts.DTYPE_F32)
    d_w = [torch.from_numpy(a).to(dev) for a in (*W, bo, qn, kn)]
    lib = dtts.lib()
    rows, L = 2, 64
    for call, seed in enumerate((21, 22)):
        x = synth.normal(seed, "noalloc.x", (rows, L, 1024), 1.0)
        mask = pos = d_mask = d_pos = None
        if call == 1:   # second call: v4 mask and position ids
            import oracle as O
            orc = O.Oracle()
            mask, pos = orc.fm_mask(L, L - 4, 4), orc.fm_pos(L, L - 4, 4)
            d_mask = torch.from_numpy(mask).to(dev)
            d_pos = torch.from_numpy(pos).to(dev)
        want = ref.forward(x, mask, pos)
        d_x = torch.from_numpy(x).to(dev)
        d_out = torch.full_like(d_x, float("nan"))
        torch.cuda.synchronize()
        st = lib.dtts_attn_forward_f32_noalloc(
            d_x.data_ptr(), *[t.data_ptr() for t in d_w],
            None if d_mask is None else d_mask.data_ptr(), None if d_pos is None else d_pos.data_ptr(),
            rows, L, d_out.data_ptr(), None)
        assert st == dtts.OK, lib.dtts_last_error().decode()
        torch.cuda.synchronize()
        got = d_out.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert rel(got, want) <= F32_REL, f"call {call}: max rel {rel(got, want):.3e}"
    ref.close()


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = dtts.lib()
    p = C.c_void_p(16)   # never dereferenced: the size check comes first
    st = lib.dtts_attn_forward_f32_noalloc(p, p, p, p, p, None, None, None, None, None, 5, 64, p, None)
    assert st == dtts.ERR_ARG
    assert b"exceeds" in lib.dtts_last_error()
