"""The attention sublayer entry point that allocates nothing.

Some callers cannot allocate GPU memory while they run (a fixed memory budget
handed over by the host application, an inference-runtime plugin whose execute
callback must not allocate, a real-time audio thread).  They pass their own
device buffers to dtts_attn_forward_f32_noalloc, which keeps its intermediates
in an array compiled into the library.  These tests drive it through the C ABI
with caller-owned device buffers (allocated here by the test, not by the entry
point) and check:
  * two calls in a row against the allocating entry point dtts_attn_forward
    and against the reference's own manual_attention (include/dit_manual.h:88,
    built in oracle/_ref), at the fp32 tolerance;
  * the largest shapes its array holds (rows * L = 256 tokens, L up to 256);
  * that the device's free memory is the same before and after the calls;
  * that larger shapes are refused before anything runs.
The file sits on its own and pytest collects it last."""
import ctypes as C

import numpy as np
import pytest

import dtts
import oracle as O
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


# (rows, L, mask): the v4 mask and position ids on the odd cases
CASES = [(2, 64, False), (2, 64, True), (1, 256, True), (4, 64, False), (16, 16, True)]


def test_noalloc_matches_allocating_entry_point_and_reference():
    import torch
    dev = torch.device("cuda", 0)
    W, bo, qn, kn = _weights()
    alloc = dtts.Attention(*W, bo, qn, kn, dtype=dtts.DTYPE_F32)
    ref = O.Reference() if O.Reference.available() else None
    orc = O.Oracle()
    lib = dtts.lib()
    d_w = [torch.from_numpy(a).to(dev) for a in (*W, bo, qn, kn)]
    # every device buffer the calls use exists before the first measurement
    bufs = []
    for i, (rows, L, with_mask) in enumerate(CASES):
        x = synth.normal(21 + i, "noalloc.x", (rows, L, 1024), 1.0)
        mask = orc.fm_mask(L, L - 4, 4) if with_mask else None
        pos = orc.fm_pos(L, L - 4, 4) if with_mask else None
        bufs.append(dict(x=x, mask=mask, pos=pos, d_x=torch.from_numpy(x).to(dev),
                         d_mask=None if mask is None else torch.from_numpy(mask).to(dev),
                         d_pos=None if pos is None else torch.from_numpy(pos).to(dev),
                         d_out=torch.full((rows, L, 1024), float("nan"), device=dev)))

    def call(b):
        rows, L = b["x"].shape[0], b["x"].shape[1]
        st = lib.dtts_attn_forward_f32_noalloc(
            b["d_x"].data_ptr(), *[t.data_ptr() for t in d_w],
            None if b["d_mask"] is None else b["d_mask"].data_ptr(),
            None if b["d_pos"] is None else b["d_pos"].data_ptr(), rows, L, b["d_out"].data_ptr(), None)
        assert st == dtts.OK, lib.dtts_last_error().decode()

    call(bufs[0])   # the first call on a device does the set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(dev)
    for b in bufs:
        b["d_out"].fill_(float("nan"))
        torch.cuda.synchronize()
        call(b)
        torch.cuda.synchronize()
        b["got"] = b["d_out"].cpu().numpy()
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
    for i, b in enumerate(bufs):
        got = b["got"]
        assert np.all(np.isfinite(got)), i
        want = alloc.forward(b["x"], b["mask"], b["pos"])
        assert rel(got, want) <= F32_REL, f"case {CASES[i]}: vs dtts_attn_forward max rel {rel(got, want):.3e}"
        if ref is not None and b["x"].shape[0] <= 2:
            for r in range(b["x"].shape[0]):
                want_r = ref.manual_attention(b["x"][r], *W, bo, qn, kn, b["mask"], b["pos"])
                assert rel(got[r], want_r) <= F32_REL, f"case {CASES[i]} row {r}: vs manual_attention"
    alloc.close()


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = dtts.lib()
    p = C.c_void_p(16)   # never dereferenced: the size checks come first
    st = lib.dtts_attn_forward_f32_noalloc(p, p, p, p, p, None, None, None, None, None, 5, 64, p, None)
    assert st == dtts.ERR_ARG
    assert b"exceeds" in lib.dtts_last_error()
    st = lib.dtts_attn_forward_f32_noalloc(p, p, p, p, p, None, None, None, None, None, 1, 257, p, None)
    assert st == dtts.ERR_ARG
    assert b"exceeds" in lib.dtts_last_error()
