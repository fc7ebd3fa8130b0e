"""The C++ drop-in layer (dots.tts.cpp_b200/dropin/dtts_dropin.cpp) called the
way a reference program calls it: tests/cpp/dropin_test.cpp builds the
reference's own structs (dit_model, dit_block, patch_encoder from
include/dit.h and include/patchenc.h) over ggml_tensor views of a safetensors
checkpoint, calls manual_attention, manual_dit_block, dit_forward_raw,
patchenc_forward, patchenc_stream_* and the manual_* host helpers by their
reference names, and writes every output; each is compared here with the CPU
oracle (bf16 tolerance for the bf16 engines, fp32 tolerance for the fp32
attention sublayer and the host helpers)."""
import os
import subprocess

import numpy as np
import pytest

import oracle as O
import synth
from helpers import F32_REL, assert_bf16_close, rel, write_safetensors

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tests", "cpp", "_bin", "dropin_test")
LA, LR, NP = 24, 20, 9          # attention/block tokens, dit_forward_raw tokens, PE patches
T_VAL = 0.37


@pytest.fixture(scope="module")
def case(tmp_path_factory, orc):
    if not os.path.exists(BIN):
        pytest.skip("tests/cpp/_bin/dropin_test is built by __graft_entry__.build() where the reference headers exist")
    d = tmp_path_factory.mktemp("dropin")
    wd = synth.dit_weights(11, n_layers=2, ada_bias_std=0.5)
    wp = synth.pe_weights(12, n_layers=2)
    write_safetensors(str(d / "w.safetensors"), {k: ("F32", v) for k, v in {**wd, **wp}.items()})
    x = synth.normal(13, "dropin.x", (LA, 1024), 1.0)
    mask = orc.fm_mask(LA, 20, 4)
    pos = orc.fm_pos(LA, 20, 4)
    cond = synth.normal(13, "dropin.cond", (1024,), 1.0)
    x_raw = synth.normal(13, "dropin.x_raw", (LR, 1024), 1.0)
    spk = synth.normal(13, "dropin.spk", (512,), 1.0)
    frames = synth.normal(13, "dropin.frames", (4 * NP, 128), 1.0)
    blob = np.concatenate([x.ravel(), mask.astype(np.float32).ravel(), pos, cond, x_raw.ravel(),
                           np.array([T_VAL], np.float32), spk, frames.ravel()]).astype(np.float32)
    blob.tofile(str(d / "in.bin"))
    r = subprocess.run([BIN, str(d / "w.safetensors"), str(d / "in.bin"), str(d / "out.bin"),
                        str(LA), str(LR), str(NP)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    out = np.fromfile(str(d / "out.bin"), np.float32)
    sizes = [("att_mask", (LA, 1024)), ("att_default", (LA, 1024)), ("blocks", (LA, 1024)),
             ("block0", (LA, 1024)), ("raw", (LR, 128)), ("pe", (NP, 1536)), ("stream", (NP, 1536)),
             ("ln", (1024,)), ("rms", (64,)), ("lin", (128,)), ("softmax", (LA,)), ("rope_q", (LA, 64)),
             ("rope_k", (LA, 64))]
    got, off = {}, 0
    for name, shape in sizes:
        n = int(np.prod(shape))
        got[name] = out[off:off + n].reshape(shape)
        off += n
    assert off == out.size
    return dict(wd=wd, wp=wp, x=x, mask=mask, pos=pos, cond=cond, x_raw=x_raw, spk=spk, frames=frames, got=got)


def _blk(w, i):
    p = f"velocity_field_predictor.blocks.{i}."
    return [w[p + n] for n in ("attn.q_proj.weight", "attn.k_proj.weight", "attn.v_proj.weight",
                               "attn.o_proj.weight", "attn.o_proj.bias", "attn.q_norm.weight",
                               "attn.k_norm.weight")]


def test_manual_attention(case, orc):
    wq, wk, wv, wo, bo, qn, kn = _blk(case["wd"], 0)
    want = orc.attention(case["x"], wq, wk, wv, wo, bo, qn, kn, case["mask"], case["pos"])
    r = rel(case["got"]["att_mask"], want)
    assert r <= F32_REL, f"manual_attention with mask/pos: max rel {r:.3e}"
    want = orc.attention(case["x"], wq, wk, wv, wo, bo, qn, kn)
    r = rel(case["got"]["att_default"], want)
    assert r <= F32_REL, f"manual_attention with default arguments: max rel {r:.3e}"


def test_manual_dit_block_chain_and_reuse(case, orc):
    wd, x, cond, mask, pos = case["wd"], case["x"], case["cond"], case["mask"], case["pos"]
    h0 = orc.dit_block(wd, 0, x, cond, mask, pos)
    h1 = orc.dit_block(wd, 1, h0, cond, mask, pos)
    assert_bf16_close(case["got"]["blocks"], h1, "manual_dit_block x2")
    assert_bf16_close(case["got"]["block0"], h0, "manual_dit_block (cached engine)")


def test_dit_forward_raw(case, orc):
    wd = case["wd"]
    orc.set_dit_rope(O.ROPE_ADJACENT)
    try:
        c = orc.compute_cond(wd, T_VAL, case["spk"], 1.0, n_layers=2)
        want = orc.dit_velocity(wd, 2, case["x_raw"], c)
    finally:
        orc.set_dit_rope(O.ROPE_HALF)
    assert_bf16_close(case["got"]["raw"], want, "dit_forward_raw")


def test_patchenc_forward_and_stream(case, orc):
    wp, fr = case["wp"], case["frames"]
    assert_bf16_close(case["got"]["pe"], orc.pe_forward(wp, 2, fr, O.PAIR_AS_WRITTEN), "patchenc_forward")
    assert_bf16_close(case["got"]["stream"], orc.pe_forward(wp, 2, fr, O.PAIR_ADJACENT), "patchenc_decode_step")


def test_host_helpers(case):
    """manual_layernorm / rms_norm / linear / softmax / rope keep the reference's
    fp32 host arithmetic (include/dit_manual.h:16-86)."""
    x, g = case["got"], case["x"]
    x0 = g[0].astype(np.float64)
    ln = (x0 - x0.mean()) / np.sqrt(x0.var() + 1e-5)
    assert rel(x["ln"], ln) <= 1e-5
    qn = case["wd"]["velocity_field_predictor.blocks.0.attn.q_norm.weight"].astype(np.float64)
    v = x0[:64]
    assert rel(x["rms"], v / np.sqrt((v * v).mean() + 1e-6) * qn) <= 1e-5
    w = case["wd"]["velocity_field_predictor.output_layer.linear.weight"].astype(np.float64)
    b = case["wd"]["velocity_field_predictor.output_layer.linear.bias"].astype(np.float64)
    assert rel(x["lin"], w @ x0 + b) <= 1e-5
    p = case["pos"].astype(np.float64)
    e = np.exp(p - p.max())
    assert rel(x["softmax"], e / e.sum()) <= 1e-5
    flat = g.ravel().astype(np.float64)
    q, k = flat[:LA * 64].reshape(LA, 64), flat[LA * 64:LA * 128].reshape(LA, 64)
    th = 10000.0 ** (-2.0 * np.arange(32) / 64.0)
    ang = np.arange(LA)[:, None] * th[None, :]
    cs, sn = np.cos(ang), np.sin(ang)

    def rope(a):
        lo, hi = a[:, :32], a[:, 32:]
        return np.concatenate([lo * cs - hi * sn, hi * cs + lo * sn], axis=1)
    assert rel(x["rope_q"], rope(q)) <= 1e-4
    assert rel(x["rope_k"], rope(k)) <= 1e-4
