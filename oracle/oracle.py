"""ctypes binding for the CPU oracle (oracle.c) and the reference build
(_ref/libdtts_ref.so, the reference's include/dit_manual.h compiled in place).

TEST INFRASTRUCTURE ONLY.  tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference legs load this module, as the checker or as the CPU
timing baseline; the CUDA engine never routes through it.

Weights are passed as dicts of float32 numpy arrays named exactly as in the
reference's safetensors checkpoint (src/utils/dit_loader.cpp:47-115,
src/utils/patchenc_loader.cpp:175-208)."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libdtts_ref.so")

FFN_PER_TOKEN = 0
FFN_AS_WRITTEN = 1
PAIR_ADJACENT = 0
PAIR_AS_WRITTEN = 1
ROPE_HALF = 0       # (d, d+32) pairs: manual_attention, include/dit_manual.h:111-128
ROPE_ADJACENT = 1   # (2i, 2i+1) pairs: ggml_rope mode 0 behind dit_forward_raw

_fp = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)


class DitBlock(C.Structure):
    _fields_ = [(n, _fp) for n in ("wq", "wk", "wv", "wo", "bo", "qn", "kn", "w1", "b1",
                                   "w2", "b2", "ada_w", "ada_b")]


class Dit(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("blocks", C.POINTER(DitBlock))] + [
        (n, _fp) for n in ("t_w1", "t_b1", "t_w2", "t_b2", "spk_w1", "spk_b1", "spk_ln_w",
                           "spk_ln_b", "oada_w", "oada_b", "out_w", "out_b", "in_w", "in_b",
                           "hid_w", "hid_b", "lat_w", "lat_b", "coord_w", "coord_b")]


class PeLayer(C.Structure):
    _fields_ = [(n, _fp) for n in ("attn_norm_w", "wq", "wk", "wv", "wo", "bo", "ffn_norm_w",
                                   "w1", "b1", "w2", "b2")]


class Pe(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("layers", C.POINTER(PeLayer))] + [
        (n, _fp) for n in ("conv_w", "conv_b", "in_w", "in_b", "out_w", "out_b")]


_fp3 = _fp * 3
_fp6 = _fp * 6


class Voc(C.Structure):
    """orc_voc (oracle.h) and ref_voc (ref_voc.cpp): BigVGAN decoder weights."""
    _fields_ = [(n, _fp) for n in ("post_proj_w", "post_proj_b", "mi_w1", "mi_b1", "mi_w2", "mi_b2")] + [
        (n, _fp * 4) for n in ("lstm_w_ih", "lstm_w_hh", "lstm_b_ih", "lstm_b_hh")] + [
        ("conv_pre_w", _fp), ("conv_pre_b", _fp), ("ups_w", _fp * 6), ("ups_b", _fp * 6)] + [
        (n, _fp3 * 18) for n in ("c1_w", "c1_b", "c2_w", "c2_b")] + [
        (n, _fp6 * 18) for n in ("alpha", "beta")] + [
        (n, _fp) for n in ("post_alpha", "post_beta", "post_filt_up", "post_filt_down", "conv_post_w")]


def aa_filter(cutoff=0.25, half_width=0.3, kernel_size=12):
    """The AMP activations' low-pass filter: BigVGAN's kaiser_sinc_filter1d
    (alias-free activation, published with BigVGAN) restated in float64 and
    rounded to float32.  The reference hard-codes its values
    (src/modules/vocoder/bigvgan_cpp.cpp:27-31, "kaiser_sinc_filter1d(cutoff=0.25,
    half_width=0.3, K=12)"); tests/golden/voc_aa_filter.npz pins them.
    Kaiser window of length K with beta from the attenuation
    A = 2.285 (K/2 - 1) pi (4 half_width) + 7.95; an even K samples the sinc at
    half-integer times; the taps are normalised to sum 1."""
    half = kernel_size // 2
    A = 2.285 * (half - 1) * np.pi * (4.0 * half_width) + 7.95
    if A > 50.0:
        beta = 0.1102 * (A - 8.7)
    elif A >= 21.0:
        beta = 0.5842 * (A - 21.0) ** 0.4 + 0.07886 * (A - 21.0)
    else:
        beta = 0.0
    n = np.arange(kernel_size, dtype=np.float64)
    window = np.i0(beta * np.sqrt(1.0 - (2.0 * n / (kernel_size - 1) - 1.0) ** 2)) / np.i0(beta)
    if kernel_size % 2 == 0:
        t = np.arange(-half, half, dtype=np.float64) + 0.5
    else:
        t = np.arange(kernel_size, dtype=np.float64) - half
    f = 2.0 * cutoff * window * np.sinc(2.0 * cutoff * t)
    f /= f.sum()
    return f.astype(np.float32)


def make_voc_struct(w: dict):
    """Voc struct over the checkpoint-named arrays of w (synth.voc_shapes)."""
    keep = []

    def P(name):
        a = np.ascontiguousarray(w[name], np.float32)
        keep.append(a)
        return _ptr(a)

    v = Voc()
    v.post_proj_w, v.post_proj_b = P("post_proj.weight"), P("post_proj.bias")
    v.mi_w1, v.mi_b1 = P("dec_mi_layer.0.weight"), P("dec_mi_layer.0.bias")
    v.mi_w2, v.mi_b2 = P("dec_mi_layer.2.weight"), P("dec_mi_layer.2.bias")
    for l in range(4):
        v.lstm_w_ih[l] = P(f"dec_mi_layer.1.lstm.weight_ih_l{l}")
        v.lstm_w_hh[l] = P(f"dec_mi_layer.1.lstm.weight_hh_l{l}")
        v.lstm_b_ih[l] = P(f"dec_mi_layer.1.lstm.bias_ih_l{l}")
        v.lstm_b_hh[l] = P(f"dec_mi_layer.1.lstm.bias_hh_l{l}")
    v.conv_pre_w, v.conv_pre_b = P("decoder.conv_pre.weight"), P("decoder.conv_pre.bias")
    for i in range(6):
        v.ups_w[i], v.ups_b[i] = P(f"decoder.ups.{i}.0.weight"), P(f"decoder.ups.{i}.0.bias")
    for rb in range(18):
        p = f"decoder.resblocks.{rb}."
        for j in range(3):
            v.c1_w[rb][j], v.c1_b[rb][j] = P(p + f"convs1.{j}.weight"), P(p + f"convs1.{j}.bias")
            v.c2_w[rb][j], v.c2_b[rb][j] = P(p + f"convs2.{j}.weight"), P(p + f"convs2.{j}.bias")
        for a in range(6):
            v.alpha[rb][a] = P(p + f"activations.{a}.act.alpha")
            v.beta[rb][a] = P(p + f"activations.{a}.act.beta")
    v.post_alpha = P("decoder.activation_post.act.alpha")
    v.post_beta = P("decoder.activation_post.act.beta")
    v.post_filt_up = P("decoder.activation_post.upsample.filter")
    v.post_filt_down = P("decoder.activation_post.downsample.lowpass.filter")
    v.conv_post_w = P("decoder.conv_post.weight")
    return v, keep


def _ptr(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous, "float32 C-contiguous expected"
    return a.ctypes.data_as(_fp)


def _u8(a):
    if a is None:
        return None
    a = np.ascontiguousarray(a, dtype=np.uint8)
    return a.ctypes.data_as(_u8p), a


DIT_BLOCK_NAMES = {
    "wq": "attn.q_proj.weight", "wk": "attn.k_proj.weight", "wv": "attn.v_proj.weight",
    "wo": "attn.o_proj.weight", "bo": "attn.o_proj.bias", "qn": "attn.q_norm.weight",
    "kn": "attn.k_norm.weight", "w1": "ffn.fc1.weight", "b1": "ffn.fc1.bias",
    "w2": "ffn.fc2.weight", "b2": "ffn.fc2.bias", "ada_w": "adaLN_modulation.1.weight",
    "ada_b": "adaLN_modulation.1.bias",
}
DIT_GLOBAL_NAMES = {
    "t_w1": "velocity_field_predictor.time_embedder.mlp.0.weight",
    "t_b1": "velocity_field_predictor.time_embedder.mlp.0.bias",
    "t_w2": "velocity_field_predictor.time_embedder.mlp.2.weight",
    "t_b2": "velocity_field_predictor.time_embedder.mlp.2.bias",
    "spk_w1": "xvec_proj.0.weight", "spk_b1": "xvec_proj.0.bias",
    "spk_ln_w": "xvec_proj.1.weight", "spk_ln_b": "xvec_proj.1.bias",
    "oada_w": "velocity_field_predictor.output_layer.adaLN_modulation.1.weight",
    "oada_b": "velocity_field_predictor.output_layer.adaLN_modulation.1.bias",
    "out_w": "velocity_field_predictor.output_layer.linear.weight",
    "out_b": "velocity_field_predictor.output_layer.linear.bias",
    "in_w": "velocity_field_predictor.input_layer.weight",
    "in_b": "velocity_field_predictor.input_layer.bias",
    "hid_w": "hidden_proj.weight", "hid_b": "hidden_proj.bias",
    "lat_w": "latent_proj.weight", "lat_b": "latent_proj.bias",
    "coord_w": "coordinate_proj.weight", "coord_b": "coordinate_proj.bias",
}
PE_LAYER_NAMES = {
    "attn_norm_w": "attn_norm.weight", "wq": "attn.q_proj.weight", "wk": "attn.k_proj.weight",
    "wv": "attn.v_proj.weight", "wo": "attn.o_proj.weight", "bo": "attn.o_proj.bias",
    "ffn_norm_w": "ffn_norm.weight", "w1": "ffn.fc1.weight", "b1": "ffn.fc1.bias",
    "w2": "ffn.fc2.weight", "b2": "ffn.fc2.bias",
}
PE_GLOBAL_NAMES = {
    "conv_w": "patch_encoder.ds_proj.weight", "conv_b": "patch_encoder.ds_proj.bias",
    "in_w": "patch_encoder.in_proj.weight", "in_b": "patch_encoder.in_proj.bias",
    "out_w": "patch_encoder.out_proj.weight", "out_b": "patch_encoder.out_proj.bias",
}


def dit_block_prefix(i):
    return f"velocity_field_predictor.blocks.{i}."


def pe_layer_prefix(i):
    return f"patch_encoder.encoder.layers.{i}."


class _Keep:
    """Holds the ctypes structs and the arrays they point into."""

    def __init__(self):
        self.refs = []


def make_block_struct(w: dict, i: int, keep: _Keep) -> DitBlock:
    b = DitBlock()
    pre = dit_block_prefix(i)
    for f, n in DIT_BLOCK_NAMES.items():
        a = w.get(pre + n)
        keep.refs.append(a)
        setattr(b, f, _ptr(a))
    return b


def make_dit_struct(w: dict, n_layers: int):
    keep = _Keep()
    arr = (DitBlock * n_layers)()
    for i in range(n_layers):
        arr[i] = make_block_struct(w, i, keep)
    m = Dit()
    m.n_layers = n_layers
    m.blocks = arr
    keep.refs.append(arr)
    for f, n in DIT_GLOBAL_NAMES.items():
        a = w.get(n)
        keep.refs.append(a)
        setattr(m, f, _ptr(a))
    return m, keep


def make_pe_struct(w: dict, n_layers: int):
    keep = _Keep()
    arr = (PeLayer * n_layers)()
    for i in range(n_layers):
        pre = pe_layer_prefix(i)
        for f, n in PE_LAYER_NAMES.items():
            a = w.get(pre + n)
            keep.refs.append(a)
            setattr(arr[i], f, _ptr(a))
    m = Pe()
    m.n_layers = n_layers
    m.layers = arr
    keep.refs.append(arr)
    for f, n in PE_GLOBAL_NAMES.items():
        a = w.get(n)
        keep.refs.append(a)
        setattr(m, f, _ptr(a))
    return m, keep


class Oracle:
    """The fp32 C restatement (liboracle.so)."""

    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        self.lib = C.CDLL(path)
        L = self.lib
        L.orc_num_threads.restype = C.c_int
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_set_dit_rope.argtypes = [C.c_int]
        L.orc_set_dit_fp8.argtypes = [C.c_int]
        L.orc_eos_prob.argtypes = [_fp, _fp, _fp, _fp, _fp, C.c_int]
        L.orc_eos_prob.restype = C.c_float
        L.orc_e4m3_encode.argtypes = [C.c_float]
        L.orc_e4m3_encode.restype = C.c_uint8
        L.orc_e4m3_decode.argtypes = [C.c_uint8]
        L.orc_e4m3_decode.restype = C.c_float
        L.orc_sinusoid.argtypes = [C.c_float, _fp]
        L.orc_compute_cond.argtypes = [C.POINTER(Dit), C.c_float, _fp, C.c_float, _fp]
        L.orc_attention.argtypes = [_fp, _fp, C.c_int] + [_fp] * 7 + [_u8p, _fp]
        L.orc_dit_block_fwd.argtypes = [_fp, _fp, _fp, C.POINTER(DitBlock), C.c_int, _u8p, _fp, C.c_int]
        L.orc_dit_velocity.argtypes = [C.POINTER(Dit), _fp, C.c_int, _fp, _u8p, _fp, C.c_int, C.c_int, _fp]
        L.orc_build_fm_mask.argtypes = [_u8p, C.c_int, C.c_int, C.c_int, C.c_int]
        L.orc_build_fm_pos.argtypes = [_fp, C.c_int, C.c_int, C.c_int]
        L.orc_euler_solve.argtypes = [C.POINTER(Dit), C.c_int, C.c_int, C.c_int, _fp, _fp, _fp, _fp,
                                      C.c_float, C.c_int, C.c_float, C.c_int, C.c_int, C.c_int, _fp]
        L.orc_pe_forward.argtypes = [C.POINTER(Pe), _fp, C.c_int, C.c_int, _fp, _fp]
        L.orc_pe_conv.argtypes = [_fp, _fp, C.c_int, _fp, _fp]
        L.orc_pe_causal_attention.argtypes = [_fp, _fp, _fp, _fp, C.c_int]
        L.orc_linear_rows.argtypes = [_fp, _fp, C.c_int, _fp, _fp, C.c_int, C.c_int]
        L.orc_voc_decode.argtypes = [C.POINTER(Voc), _fp, _fp, C.c_int, _fp]
        L.orc_voc_activation.argtypes = [_fp, C.c_int, C.c_int, _fp, _fp, _fp, _fp, C.c_int]
        L.orc_voc_bottleneck.argtypes = [C.POINTER(Voc), _fp, C.c_int, _fp]

    def voc_decode(self, w, latent, aa=None):
        """BigVGAN decoder on latent [n_frames][128] -> audio [n_frames * 1920]."""
        v, keep = make_voc_struct(w)
        lat = np.ascontiguousarray(latent, np.float32)
        f = np.ascontiguousarray(aa_filter() if aa is None else aa, np.float32)
        out = np.zeros(lat.shape[0] * 1920, np.float32)
        self.lib.orc_voc_decode(C.byref(v), _ptr(f), _ptr(lat), lat.shape[0], _ptr(out))
        return out

    def voc_activation(self, x, alpha, beta, filt_up, filt_down):
        """Activation1d on x [len][ch] (returns a new array); filters [12] or [ch][12]."""
        x = np.array(x, np.float32, copy=True, order="C")
        fu = np.ascontiguousarray(filt_up, np.float32)
        fd = np.ascontiguousarray(filt_down, np.float32)
        fch = 1 if fu.size == 12 else x.shape[1]
        self.lib.orc_voc_activation(_ptr(x), x.shape[0], x.shape[1], _ptr(np.ascontiguousarray(alpha, np.float32)),
                                    _ptr(np.ascontiguousarray(beta, np.float32)), _ptr(fu), _ptr(fd), fch)
        return x

    def voc_bottleneck(self, w, latent):
        v, keep = make_voc_struct(w)
        lat = np.ascontiguousarray(latent, np.float32)
        out = np.zeros((lat.shape[0], 128), np.float32)
        self.lib.orc_voc_bottleneck(C.byref(v), _ptr(lat), lat.shape[0], _ptr(out))
        return out

    def set_threads(self, n):
        self.lib.orc_set_threads(int(n))

    def set_dit_rope(self, mode):
        """0: half-split (manual_attention), 1: adjacent pairs (ggml mode 0, dit_forward_raw)."""
        self.lib.orc_set_dit_rope(int(mode))

    def num_threads(self):
        return self.lib.orc_num_threads()

    def set_dit_fp8(self, on):
        """1: DiT blocks use the engine's FP8 (e4m3) recipe; 0: fp32."""
        self.lib.orc_set_dit_fp8(int(on))

    def eos_prob(self, w, h, as_written=False):
        """EOS head probability for each row of h [n][1536]."""
        h = np.ascontiguousarray(h, np.float32)
        a = [np.ascontiguousarray(w[n], np.float32) for n in
             ("eos_proj.0.weight", "eos_proj.0.bias", "eos_proj.2.weight", "eos_proj.2.bias")]
        return np.array([self.lib.orc_eos_prob(*[_ptr(x) for x in a], _ptr(h[i]), int(as_written))
                         for i in range(h.shape[0])], np.float32)

    def e4m3_encode(self, x):
        x = np.ascontiguousarray(x, np.float32).ravel()
        return np.array([self.lib.orc_e4m3_encode(C.c_float(float(v))) for v in x], np.uint8)

    def e4m3_decode(self, b):
        b = np.ascontiguousarray(b, np.uint8).ravel()
        return np.array([self.lib.orc_e4m3_decode(C.c_uint8(int(v))) for v in b], np.float32)

    def sinusoid(self, t):
        se = np.zeros(256, np.float32)
        self.lib.orc_sinusoid(C.c_float(t), _ptr(se))
        return se

    def compute_cond(self, w, t, spk=None, spk_scale=1.0, n_layers=0):
        m, keep = make_dit_struct(w, n_layers)
        out = np.zeros(1024, np.float32)
        spk = None if spk is None else np.ascontiguousarray(spk, np.float32)
        self.lib.orc_compute_cond(C.byref(m), C.c_float(t), _ptr(spk), C.c_float(spk_scale), _ptr(out))
        return out

    def attention(self, x, wq, wk, wv, wo, bo=None, qn=None, kn=None, mask=None, pos=None):
        x = np.ascontiguousarray(x, np.float32)
        L = x.shape[0]
        out = np.zeros((L, 1024), np.float32)
        mk = _u8(mask)
        pos = None if pos is None else np.ascontiguousarray(pos, np.float32)
        self.lib.orc_attention(_ptr(out), _ptr(x), L, _ptr(wq), _ptr(wk), _ptr(wv), _ptr(wo), _ptr(bo),
                               _ptr(qn), _ptr(kn), mk[0] if mk else None, _ptr(pos))
        return out

    def dit_block(self, w, i, x, cond, mask=None, pos=None, ffn_mode=FFN_PER_TOKEN):
        keep = _Keep()
        b = make_block_struct(w, i, keep)
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        mk = _u8(mask)
        pos = None if pos is None else np.ascontiguousarray(pos, np.float32)
        cond = np.ascontiguousarray(cond, np.float32)
        self.lib.orc_dit_block_fwd(_ptr(out), _ptr(x), _ptr(cond), C.byref(b), x.shape[0],
                                   mk[0] if mk else None, _ptr(pos), ffn_mode)
        return out

    def dit_velocity(self, w, n_layers, x_in, cond, mask=None, pos=None, ffn_mode=FFN_PER_TOKEN, n_out=None):
        m, keep = make_dit_struct(w, n_layers)
        x_in = np.ascontiguousarray(x_in, np.float32)
        L = x_in.shape[0]
        n_out = L if n_out is None else n_out
        out = np.zeros((n_out, 128), np.float32)
        mk = _u8(mask)
        pos = None if pos is None else np.ascontiguousarray(pos, np.float32)
        cond = np.ascontiguousarray(cond, np.float32)
        self.lib.orc_dit_velocity(C.byref(m), _ptr(x_in), L, _ptr(cond), mk[0] if mk else None, _ptr(pos),
                                  ffn_mode, n_out, _ptr(out))
        return out

    def fm_mask(self, total, fm_len, patch, hidden_patch=1):
        m = np.zeros((total, total), np.uint8)
        self.lib.orc_build_fm_mask(m.ctypes.data_as(_u8p), total, fm_len, patch, hidden_patch)
        return m

    def fm_pos(self, total, fm_len, patch):
        p = np.zeros(total, np.float32)
        self.lib.orc_build_fm_pos(_ptr(p), total, fm_len, patch)
        return p

    def euler_solve(self, w, n_layers, fm_cond, fm_uncond, z0, spk=None, spk_scale=1.5, nfe=10,
                    cfg_scale=2.0, cfg_form=0, layout=0, ffn_mode=FFN_PER_TOKEN):
        m, keep = make_dit_struct(w, n_layers)
        fm_cond = np.ascontiguousarray(fm_cond, np.float32)
        fm_uncond = np.ascontiguousarray(fm_uncond, np.float32)
        z0 = np.ascontiguousarray(z0, np.float32)
        n_utt, fm_len = fm_cond.shape[0], fm_cond.shape[1]
        patch = z0.shape[1]
        out = np.zeros_like(z0)
        spk = None if spk is None else np.ascontiguousarray(spk, np.float32)
        self.lib.orc_euler_solve(C.byref(m), n_utt, fm_len, patch, _ptr(fm_cond), _ptr(fm_uncond), _ptr(z0),
                                 _ptr(spk), C.c_float(spk_scale), nfe, C.c_float(cfg_scale), cfg_form,
                                 layout, ffn_mode, _ptr(out))
        return out

    def pe_forward(self, w, n_layers, frames, pair_mode=PAIR_ADJACENT, want_hidden=False):
        m, keep = make_pe_struct(w, n_layers)
        frames = np.ascontiguousarray(frames, np.float32)
        n_patches = frames.shape[0] // 4
        out = np.zeros((n_patches, 1536), np.float32)
        h = np.zeros((n_patches * 2, 1024), np.float32) if want_hidden else None
        self.lib.orc_pe_forward(C.byref(m), _ptr(frames), n_patches, pair_mode, _ptr(out), _ptr(h))
        return (out, h) if want_hidden else out

    def pe_conv(self, x, wc, bc=None):
        """Causal stride-2 conv (patchenc.cpp:19-39): x [T][128] -> [T // 2][128]."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros((x.shape[0] // 2, 128), np.float32)
        self.lib.orc_pe_conv(_ptr(out), _ptr(x), x.shape[0], _ptr(np.ascontiguousarray(wc, np.float32)),
                             _ptr(None if bc is None else np.ascontiguousarray(bc, np.float32)))
        return out

    def pe_causal_attention(self, q, k, v):
        """Causal per-head attention (patchenc.cpp:59-101): [T][1024] each -> [T][1024]."""
        q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
        out = np.zeros_like(q)
        self.lib.orc_pe_causal_attention(_ptr(out), _ptr(q), _ptr(k), _ptr(v), q.shape[0])
        return out

    def linear_rows(self, x, w, b=None):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros((x.shape[0], w.shape[0]), np.float32)
        self.lib.orc_linear_rows(_ptr(out), _ptr(x), x.shape[0], _ptr(w), _ptr(b), w.shape[1], w.shape[0])
        return out


class _RefLLMLayer(C.Structure):
    _fields_ = [(n, _fp) for n in ("an", "fn", "qw", "qb", "kw", "kb", "vw", "vb", "ow", "ob", "gw", "uw", "dw")]


class Reference:
    """The reference's own include/dit_manual.h, compiled in place (_ref/)."""

    def __init__(self, path: str = REF_PATH):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle REF=<reference tree>`")
        self.lib = C.CDLL(path)
        L = self.lib
        L.ref_num_threads.restype = C.c_int
        L.ref_set_threads.argtypes = [C.c_int]
        L.ref_manual_attention.argtypes = [_fp, _fp, C.c_int] + [_fp] * 7 + [_u8p, _fp]
        L.ref_dit_block.argtypes = [_fp, _fp, _fp, C.POINTER(DitBlock), C.c_int, _u8p, _fp, C.c_int]
        L.ref_dit_velocity.argtypes = [C.POINTER(Dit), _fp, C.c_int, _fp, _u8p, _fp, C.c_int, C.c_int, _fp]
        L.ref_llm_run.argtypes = [C.c_int, C.POINTER(_RefLLMLayer), _fp, _fp, C.c_int, _fp, C.c_int, _fp, _fp]
        L.ref_voc_decode.argtypes = [C.POINTER(Voc), _fp, C.c_int, _fp]
        L.ref_voc_decode.restype = C.c_int
        # pieces of src/e2e_pipeline_v4.cpp and src/modules/backbone/patchenc.cpp (ref_pipeline.cpp)
        L.ref_gen_ranges.restype = C.c_char_p
        L.ref_set_solve_ffn.argtypes = [C.c_int]
        L.ref_compute_cond.argtypes = [C.POINTER(Dit), C.c_float, _fp, C.c_float, _fp]
        L.ref_compute_cond_raw.argtypes = [C.POINTER(Dit), C.c_float, _fp, _fp]
        L.ref_fm_mask.argtypes = [_u8p, C.c_int, C.c_int, C.c_int, C.c_int]
        L.ref_fm_pos.argtypes = [_fp, C.c_int, C.c_int, C.c_int]
        L.ref_latent_proj.argtypes = [C.POINTER(Dit), _fp, C.c_int, _fp]
        L.ref_hidden_proj.argtypes = [C.POINTER(Dit), _fp, _fp]
        L.ref_coord_proj.argtypes = [C.POINTER(Dit), _fp, _fp]
        L.ref_eos_prob.argtypes = [_fp, _fp, _fp, _fp, _fp]
        L.ref_eos_prob.restype = C.c_float
        L.ref_solve_patch.argtypes = [C.POINTER(Dit), _fp, _fp, C.c_int, _fp, C.c_int, C.c_float, C.c_int]
        L.ref_pe_forward.argtypes = [C.POINTER(Pe), _fp, C.c_int, _fp]
        L.ref_pe_conv.argtypes = [_fp, C.c_int, _fp, _fp, _fp]
        L.ref_pe_causal_attention.argtypes = [_fp, _fp, _fp, _fp, C.c_int]

    def gen_ranges(self):
        """{piece: (first, last)}: where the verbatim pieces of src/e2e_pipeline_v4.cpp
        sit in the reference file the library was built from."""
        out = {}
        for part in self.lib.ref_gen_ranges().decode().split(";"):
            name, rng = part.strip().rsplit(" ", 1)
            a, b = rng.split("-")
            out[name] = (int(a), int(b))
        return out

    def compute_cond(self, w, t, spk=None, spk_scale=1.0):
        """compute_cond (src/e2e_pipeline_v4.cpp:57-71) -> c [1024]."""
        m, keep = make_dit_struct(w, 0)
        out = np.zeros(1024, np.float32)
        spk = None if spk is None else np.ascontiguousarray(spk, np.float32)
        self.lib.ref_compute_cond(C.byref(m), C.c_float(t), _ptr(spk), C.c_float(spk_scale), _ptr(out))
        return out

    def compute_cond_raw(self, w, t, spk=None):
        """compute_cond of the ggml DiT path (src/modules/backbone/dit_forward.cpp:22-36)."""
        m, keep = make_dit_struct(w, 0)
        out = np.zeros(1024, np.float32)
        spk = None if spk is None else np.ascontiguousarray(spk, np.float32)
        self.lib.ref_compute_cond_raw(C.byref(m), C.c_float(t), _ptr(spk), _ptr(out))
        return out

    def fm_mask(self, total, fm_len, patch, hidden_patch=1):
        """build_fm_attn_mask (:120-146) as uint8 [total][total]."""
        m = np.zeros((total, total), np.uint8)
        self.lib.ref_fm_mask(m.ctypes.data_as(_u8p), total, fm_len, patch, hidden_patch)
        return m

    def fm_pos(self, total, fm_len, patch):
        """build_fm_pos_ids (:149-155)."""
        p = np.zeros(total, np.float32)
        self.lib.ref_fm_pos(_ptr(p), total, fm_len, patch)
        return p

    def latent_proj(self, w, z):
        """apply_latent_proj (:81-91): z [P][128] -> [P][1024]."""
        m, keep = make_dit_struct(w, 0)
        z = np.ascontiguousarray(z, np.float32)
        out = np.zeros((z.shape[0], 1024), np.float32)
        self.lib.ref_latent_proj(C.byref(m), _ptr(z), z.shape[0], _ptr(out))
        return out

    def hidden_proj(self, w, h):
        """apply_hidden_proj (:94-102): h [1536] -> [1024]."""
        m, keep = make_dit_struct(w, 0)
        h = np.ascontiguousarray(h, np.float32)
        out = np.zeros(1024, np.float32)
        self.lib.ref_hidden_proj(C.byref(m), _ptr(h), _ptr(out))
        return out

    def coord_proj(self, w, z):
        """apply_coord_proj (:105-113): z [128] -> [1024]."""
        m, keep = make_dit_struct(w, 0)
        z = np.ascontiguousarray(z, np.float32)
        out = np.zeros(1024, np.float32)
        self.lib.ref_coord_proj(C.byref(m), _ptr(z), _ptr(out))
        return out

    def eos_prob(self, w, h):
        """The EOS head as written (:599-619) on each row of h [n][1536]."""
        h = np.ascontiguousarray(h, np.float32)
        a = [np.ascontiguousarray(w[n], np.float32) for n in
             ("eos_proj.0.weight", "eos_proj.0.bias", "eos_proj.2.weight", "eos_proj.2.bias")]
        return np.array([self.lib.ref_eos_prob(*[_ptr(x) for x in a], _ptr(h[i])) for i in range(h.shape[0])],
                        np.float32)

    def solve_patch(self, w, n_layers, fm_cond, fm_uncond, z0, nfe=10, cfg_scale=2.0, fast=False,
                    ffn_mode=FFN_PER_TOKEN):
        """One patch of the decode loop's Euler + CFG solve (:381-400, :410-533) for one
        utterance: histories [fm_len][1024], z0 [4][128] -> z [4][128].  No speaker
        (the pipeline passes none); ffn_mode picks the block the loop calls."""
        m, keep = make_dit_struct(w, n_layers)
        fc = np.ascontiguousarray(fm_cond, np.float32)
        fu = np.ascontiguousarray(fm_uncond, np.float32)
        z = np.array(z0, np.float32, copy=True, order="C")
        assert z.shape == (4, 128)
        self.lib.ref_set_solve_ffn(int(ffn_mode))
        try:
            self.lib.ref_solve_patch(C.byref(m), _ptr(fc), _ptr(fu), fc.shape[0], _ptr(z), int(nfe),
                                     C.c_float(cfg_scale), int(fast))
        finally:
            self.lib.ref_set_solve_ffn(FFN_PER_TOKEN)
        return z

    def pe_forward(self, w, n_layers, frames):
        """patchenc_forward (src/modules/backbone/patchenc.cpp:146-239) as written, ggml
        operators from the eager stand-in: frames [4 n][128] -> [n][1536]."""
        m, keep = make_pe_struct(w, n_layers)
        frames = np.ascontiguousarray(frames, np.float32)
        n_patches = frames.shape[0] // 4
        out = np.zeros((n_patches, 1536), np.float32)
        self.lib.ref_pe_forward(C.byref(m), _ptr(frames), n_patches, _ptr(out))
        return out

    def pe_conv(self, x, wc, bc=None):
        """causal_conv1d_stride2 (patchenc.cpp:19-39): x [T][128] -> [T // 2][128]."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros((x.shape[0] // 2, 128), np.float32)
        self.lib.ref_pe_conv(_ptr(x), x.shape[0], _ptr(np.ascontiguousarray(wc, np.float32)),
                             _ptr(None if bc is None else np.ascontiguousarray(bc, np.float32)), _ptr(out))
        return out

    def pe_causal_attention(self, q, k, v):
        """per_head_attention_cpu (patchenc.cpp:59-101): [T][1024] each -> [T][1024]."""
        q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
        out = np.zeros_like(q)
        self.lib.ref_pe_causal_attention(_ptr(out), _ptr(q), _ptr(k), _ptr(v), q.shape[0])
        return out

    def voc_decode(self, w, latent):
        """The reference's own bigvgan_decode (src/modules/vocoder/bigvgan_cpp.cpp:325)."""
        v, keep = make_voc_struct(w)
        lat = np.ascontiguousarray(latent, np.float32)
        out = np.zeros(lat.shape[0] * 1920, np.float32)
        n = self.lib.ref_voc_decode(C.byref(v), _ptr(lat), lat.shape[0], _ptr(out))
        assert n == out.size, (n, out.size)
        return out

    @staticmethod
    def available(path: str = REF_PATH) -> bool:
        return os.path.exists(path)

    def num_threads(self):
        return self.lib.ref_num_threads()

    def set_threads(self, n):
        self.lib.ref_set_threads(int(n))

    def manual_attention(self, x, wq, wk, wv, wo, bo=None, qn=None, kn=None, mask=None, pos=None):
        x = np.ascontiguousarray(x, np.float32)
        L = x.shape[0]
        out = np.zeros((L, 1024), np.float32)
        mk = _u8(mask)
        pos = None if pos is None else np.ascontiguousarray(pos, np.float32)
        self.lib.ref_manual_attention(_ptr(out), _ptr(x), L, _ptr(wq), _ptr(wk), _ptr(wv), _ptr(wo), _ptr(bo),
                                      _ptr(qn), _ptr(kn), mk[0] if mk else None, _ptr(pos))
        return out

    def dit_block(self, w, i, x, cond, mask=None, pos=None, ffn_mode=FFN_PER_TOKEN):
        keep = _Keep()
        b = make_block_struct(w, i, keep)
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        mk = _u8(mask)
        pos = None if pos is None else np.ascontiguousarray(pos, np.float32)
        cond = np.ascontiguousarray(cond, np.float32)
        self.lib.ref_dit_block(_ptr(out), _ptr(x), _ptr(cond), C.byref(b), x.shape[0],
                               mk[0] if mk else None, _ptr(pos), ffn_mode)
        return out

    def llm_run(self, w, n_layers, prompt_emb, step_emb):
        """The reference's llm_kv_cache_init on prompt_emb [n_tok][1536] then one
        llm_kv_cache_step per row of step_emb [n_steps][1536]; returns the
        prompt's hidden states and the steps' hidden states."""
        names = ["input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
                 "self_attn.q_proj.bias", "self_attn.k_proj.weight", "self_attn.k_proj.bias",
                 "self_attn.v_proj.weight", "self_attn.v_proj.bias", "self_attn.o_proj.weight", None,
                 "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"]
        keep = []
        arr = (_RefLLMLayer * n_layers)()
        for i in range(n_layers):
            vals = []
            for n in names:
                a = None if n is None else np.ascontiguousarray(w[f"llm.model.layers.{i}." + n], np.float32)
                keep.append(a)
                vals.append(_ptr(a))
            arr[i] = _RefLLMLayer(*vals)
        fn = np.ascontiguousarray(w["llm.model.norm.weight"], np.float32)
        pe = np.ascontiguousarray(prompt_emb, np.float32)
        se = np.ascontiguousarray(step_emb, np.float32)
        ph = np.zeros_like(pe)
        sh = np.zeros_like(se)
        self.lib.ref_llm_run(n_layers, arr, _ptr(fn), _ptr(pe), pe.shape[0], _ptr(se), se.shape[0], _ptr(ph), _ptr(sh))
        return ph, sh

    def dit_velocity(self, w, n_layers, x_in, cond, mask=None, pos=None, ffn_mode=FFN_PER_TOKEN, n_out=None):
        m, keep = make_dit_struct(w, n_layers)
        x_in = np.ascontiguousarray(x_in, np.float32)
        L = x_in.shape[0]
        n_out = L if n_out is None else n_out
        out = np.zeros((n_out, 128), np.float32)
        mk = _u8(mask)
        pos = None if pos is None else np.ascontiguousarray(pos, np.float32)
        cond = np.ascontiguousarray(cond, np.float32)
        self.lib.ref_dit_velocity(C.byref(m), _ptr(x_in), L, _ptr(cond), mk[0] if mk else None, _ptr(pos),
                                  ffn_mode, n_out, _ptr(out))
        return out
