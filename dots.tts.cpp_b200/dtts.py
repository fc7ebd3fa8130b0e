"""ctypes binding of libdtts.so (include/dtts.h) for tests and the benchmark.

Loads the in-tree library built by build.py and fails loudly if it is
missing: there is no CPU fallback.  Weights are dicts of float32 numpy arrays
keyed by the reference's safetensors tensor names (see synth.py)."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdtts.so")

OK, ERR_ARG, ERR_CUDA, ERR_OOM, ERR_TIMEOUT, ERR_NONFINITE, ERR_UNSUPPORTED, ERR_IO, ERR_NO_DEVICE = \
    0, -1, -2, -3, -4, -5, -6, -7, -8
DTYPE_BF16, DTYPE_FP8, DTYPE_F32 = 0, 1, 2
MEM_HOST, MEM_DEVICE = 0, 1
CFG_V4, CFG_V3 = 0, 1
LAYOUT_FM_MASK, LAYOUT_FULL = 0, 1
PAIR_ADJACENT, PAIR_AS_WRITTEN = 0, 1
ROPE_HALF, ROPE_ADJACENT = 0, 1

_fp = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_vp = C.c_void_p


class DitBlockW(C.Structure):
    _fields_ = [(n, _fp) for n in ("wq", "wk", "wv", "wo", "bo", "qn", "kn", "w1", "b1", "w2", "b2",
                                   "ada_w", "ada_b")]


class DitW(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("blocks", C.POINTER(DitBlockW))] + [
        (n, _fp) for n in ("t_w1", "t_b1", "t_w2", "t_b2", "spk_w1", "spk_b1", "spk_ln_w", "spk_ln_b",
                           "oada_w", "oada_b", "out_w", "out_b", "in_w", "in_b", "hid_w", "hid_b", "lat_w",
                           "lat_b", "coord_w", "coord_b", "eos_w1", "eos_b1", "eos_w2", "eos_b2")]


class AttnW(C.Structure):
    _fields_ = [(n, _fp) for n in ("wq", "wk", "wv", "wo", "bo", "qn", "kn")]


class PeLayerW(C.Structure):
    _fields_ = [(n, _fp) for n in ("attn_norm_w", "wq", "wk", "wv", "wo", "bo", "ffn_norm_w", "w1", "b1",
                                   "w2", "b2")]


class PeW(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("layers", C.POINTER(PeLayerW))] + [
        (n, _fp) for n in ("conv_w", "conv_b", "in_w", "in_b", "out_w", "out_b")]


class SolveArgs(C.Structure):
    _fields_ = [("n_utt", C.c_int), ("fm_len", C.c_int), ("patch", C.c_int),
                ("fm_cond", _vp), ("fm_uncond", _vp), ("z0", _vp), ("spk", _vp),
                ("spk_scale", C.c_float), ("nfe", C.c_int), ("cfg_scale", C.c_float), ("cfg_form", C.c_int),
                ("layout", C.c_int), ("z_out", _vp), ("mem", C.c_int), ("use_graph", C.c_int)]


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
    "eos_w1": "eos_proj.0.weight", "eos_b1": "eos_proj.0.bias",
    "eos_w2": "eos_proj.2.weight", "eos_b2": "eos_proj.2.bias",
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

# launch kinds of dtts_dit_solve_timeline (DTTS_TL_*)
TL_NAMES = ["gemm_qkv", "gemm_o", "gemm_ffn1", "gemm_ffn2", "attention", "ln_modulate", "gemm_adaln", "gemm_input",
            "out_head", "cfg_euler", "conditioning"]
TL_KINDS = len(TL_NAMES)

# every symbol include/dtts.h declares (checked against the library by the CPU tests)
EXPORTS = [
    "dtts_version", "dtts_status_string", "dtts_last_error", "dtts_device_count",
    "dtts_dit_create", "dtts_dit_create_from_safetensors", "dtts_dit_destroy", "dtts_dit_set_stream",
    "dtts_dit_sync", "dtts_dit_velocity", "dtts_dit_blocks", "dtts_dit_cond", "dtts_dit_set_rope", "dtts_dit_euler_solve", "dtts_dit_solve_timeline",
    "dtts_dit_profile_kernel",
    "dtts_dit_last_launch_count", "dtts_dit_tune", "dtts_dit_set_fused_ln", "dtts_fm_create", "dtts_fm_destroy", "dtts_fm_start",
    "dtts_fm_append_latents", "dtts_fm_append_hidden", "dtts_fm_length", "dtts_fm_read", "dtts_fm_solve", "dtts_fm_layout",
    "dtts_llm_create", "dtts_llm_destroy", "dtts_llm_set_stream", "dtts_llm_prefill", "dtts_llm_step", "dtts_llm_length",
    "dtts_voc_create", "dtts_voc_destroy", "dtts_voc_set_stream", "dtts_voc_decode", "dtts_voc_aa_filter",
    "dtts_selftest_voc_activation", "dtts_selftest_wait_limit", "dtts_selftest_conv", "dtts_attn_create", "dtts_attn_destroy", "dtts_attn_forward",
    "dtts_attn_profile_core", "dtts_attn_forward_f32_noalloc", "dtts_pe_create", "dtts_pe_create_from_safetensors", "dtts_pe_destroy",
    "dtts_pe_set_stream", "dtts_pe_sync", "dtts_pe_forward", "dtts_pe_stream_reset", "dtts_pe_decode",
    "dtts_pe_stream_length", "dtts_selftest_gemm", "dtts_selftest_attention", "dtts_selftest_e4m3",
    "dtts_selftest_gemm_e4m3",
    "dtts_fp8_quantize_rows", "dtts_st_open",
    "dtts_st_close", "dtts_st_count", "dtts_st_shape", "dtts_st_read_f32",
]


_fp3 = _fp * 3
_fp6 = _fp * 6


class VocW(C.Structure):
    """dtts_voc_weights (include/dtts.h)."""
    _fields_ = [(n, _fp) for n in ("post_proj_w", "post_proj_b", "mi_w1", "mi_b1", "mi_w2", "mi_b2")] + [
        (n, _fp * 4) for n in ("lstm_w_ih", "lstm_w_hh", "lstm_b_ih", "lstm_b_hh")] + [
        ("conv_pre_w", _fp), ("conv_pre_b", _fp), ("ups_w", _fp * 6), ("ups_b", _fp * 6)] + [
        (n, _fp3 * 18) for n in ("c1_w", "c1_b", "c2_w", "c2_b")] + [
        (n, _fp6 * 18) for n in ("alpha", "beta")] + [
        (n, _fp) for n in ("post_alpha", "post_beta", "post_filt_up", "post_filt_down", "conv_post_w")]


class DttsError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"dtts status {status}: {msg}")
        self.status = status


def _ptr(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous, "float32 C-contiguous expected"
    return a.ctypes.data_as(_fp)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


_LIB = None


def lib(path: str = LIB_PATH):
    """The loaded libdtts.so (raises if it was not built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is missing: run `python {os.path.join(HERE, 'build.py')}`")
    L = C.CDLL(path)
    L.dtts_version.restype = C.c_char_p
    L.dtts_version.argtypes = []
    L.dtts_status_string.restype = C.c_char_p
    L.dtts_status_string.argtypes = [C.c_int]
    L.dtts_last_error.restype = C.c_char_p
    L.dtts_last_error.argtypes = []
    L.dtts_device_count.argtypes = [C.POINTER(C.c_int)]
    L.dtts_dit_create.argtypes = [C.POINTER(DitW), C.c_int, C.c_int, C.POINTER(_vp)]
    L.dtts_dit_create_from_safetensors.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]
    L.dtts_dit_destroy.argtypes = [_vp]
    L.dtts_dit_set_stream.argtypes = [_vp, _vp]
    L.dtts_dit_sync.argtypes = [_vp]
    L.dtts_dit_velocity.argtypes = [_vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, C.c_int]
    L.dtts_dit_euler_solve.argtypes = [_vp, C.POINTER(SolveArgs)]
    L.dtts_dit_blocks.argtypes = [_vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int, _vp, C.c_int]
    L.dtts_dit_cond.argtypes = [_vp, C.c_float, _vp, C.c_float, _vp]
    L.dtts_dit_set_rope.argtypes = [_vp, C.c_int]
    L.dtts_dit_profile_kernel.argtypes = [_vp, C.c_int, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_double),
                                          C.POINTER(C.c_double)]
    L.dtts_dit_last_launch_count.argtypes = [_vp, C.POINTER(C.c_int)]
    L.dtts_dit_tune.argtypes = [_vp, C.c_char_p, C.c_int, C.c_int, C.c_int]
    L.dtts_dit_set_fused_ln.argtypes = [_vp, C.c_int]
    L.dtts_attn_create.argtypes = [C.POINTER(AttnW), C.c_int, C.c_int, C.POINTER(_vp)]
    L.dtts_attn_destroy.argtypes = [_vp]
    L.dtts_attn_forward.argtypes = [_vp, _fp, C.c_int, C.c_int, _u8p, _fp, _fp]
    L.dtts_attn_profile_core.argtypes = [_vp, C.c_int, C.POINTER(C.c_float)]
    L.dtts_attn_forward_f32_noalloc.argtypes = [_vp] * 10 + [C.c_int, C.c_int, _vp, _vp]
    L.dtts_pe_create.argtypes = [C.POINTER(PeW), C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]
    L.dtts_pe_create_from_safetensors.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                                  C.POINTER(_vp)]
    L.dtts_pe_destroy.argtypes = [_vp]
    L.dtts_pe_set_stream.argtypes = [_vp, _vp]
    L.dtts_pe_sync.argtypes = [_vp]
    L.dtts_pe_forward.argtypes = [_vp, _vp, C.c_int, C.c_int, C.c_int, _vp, C.c_int]
    L.dtts_pe_stream_reset.argtypes = [_vp, C.c_int]
    L.dtts_pe_decode.argtypes = [_vp, _vp, C.c_int, C.c_int, _vp, C.c_int]
    L.dtts_pe_stream_length.argtypes = [_vp, C.POINTER(C.c_int)]
    L.dtts_selftest_gemm.argtypes = [_fp, _fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
    L.dtts_selftest_attention.argtypes = [_fp, _fp, _fp, _fp, C.c_int, C.c_int, C.c_int, _u8p, C.c_int,
                                          C.c_int, C.c_int, C.c_int]
    L.dtts_st_open.argtypes = [C.c_char_p, C.POINTER(_vp)]
    L.dtts_st_close.argtypes = [_vp]
    L.dtts_st_count.argtypes = [_vp, C.POINTER(C.c_int)]
    L.dtts_st_shape.argtypes = [_vp, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int64)]
    L.dtts_st_read_f32.argtypes = [_vp, C.c_char_p, _fp, C.c_size_t]
    L.dtts_dit_solve_timeline.argtypes = [_vp, C.POINTER(SolveArgs), C.c_int, C.POINTER(C.c_float),
                                          C.POINTER(C.c_int)]
    L.dtts_fm_create.argtypes = [_vp, C.c_int, C.c_int, C.POINTER(_vp)]
    L.dtts_fm_destroy.argtypes = [_vp]
    L.dtts_fm_start.argtypes = [_vp, _vp, C.c_int]
    L.dtts_fm_append_latents.argtypes = [_vp, _vp, C.c_int, C.c_int]
    L.dtts_fm_append_hidden.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int]
    L.dtts_fm_length.argtypes = [_vp, C.POINTER(C.c_int)]
    L.dtts_fm_read.argtypes = [_vp, _vp, _vp]
    L.dtts_fm_solve.argtypes = [_vp, C.POINTER(SolveArgs)]
    L.dtts_llm_create.argtypes = [C.POINTER(LLMW), C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]
    L.dtts_llm_destroy.argtypes = [_vp]
    L.dtts_llm_set_stream.argtypes = [_vp, _vp]
    L.dtts_llm_prefill.argtypes = [_vp, _vp, C.c_int, C.c_int, _vp, C.c_int]
    L.dtts_llm_step.argtypes = [_vp, _vp, C.c_int, _vp, C.c_int]
    L.dtts_llm_length.argtypes = [_vp, C.POINTER(C.c_int)]
    L.dtts_voc_create.argtypes = [C.POINTER(VocW), C.c_int, C.c_int, C.POINTER(_vp)]
    L.dtts_voc_destroy.argtypes = [_vp]
    L.dtts_voc_set_stream.argtypes = [_vp, _vp]
    L.dtts_voc_decode.argtypes = [_vp, _vp, C.c_int, _vp, C.c_int]
    L.dtts_voc_aa_filter.argtypes = [_fp]
    L.dtts_selftest_voc_activation.argtypes = [_fp, C.c_int, C.c_int, _fp, _fp, _fp, _fp, C.c_int, _fp]
    L.dtts_selftest_wait_limit.argtypes = [C.c_int, C.POINTER(C.c_int)]
    L.dtts_selftest_conv.argtypes = [_fp, C.c_int, C.c_int, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                     _fp, C.c_int]
    L.dtts_selftest_e4m3.argtypes = [_fp, _u8p, C.c_int, C.c_int]
    L.dtts_selftest_gemm_e4m3.argtypes = [_u8p, _fp, _u8p, _fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                          C.c_int]
    L.dtts_fp8_quantize_rows.argtypes = [_fp, C.c_int, C.c_int, _u8p, _fp]
    L.dtts_fm_layout.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, _u8p, _fp]
    _LIB = L
    return L


def check(status):
    if status != OK:
        raise DttsError(status, lib().dtts_last_error().decode())
    return status


def device_count():
    n = C.c_int(0)
    check(lib().dtts_device_count(C.byref(n)))
    return n.value


# ------------------------------------------------------------------ weights -> structs
class _Keep:
    def __init__(self):
        self.refs = []


def dit_struct(w: dict, n_layers: int):
    keep = _Keep()
    arr = (DitBlockW * n_layers)()
    for i in range(n_layers):
        pre = f"velocity_field_predictor.blocks.{i}."
        for f, n in DIT_BLOCK_NAMES.items():
            a = _f32(w.get(pre + n))
            keep.refs.append(a)
            setattr(arr[i], f, _ptr(a))
    s = DitW()
    s.n_layers = n_layers
    s.blocks = arr
    keep.refs.append(arr)
    for f, n in DIT_GLOBAL_NAMES.items():
        a = _f32(w.get(n))
        keep.refs.append(a)
        setattr(s, f, _ptr(a))
    return s, keep


def pe_struct(w: dict, n_layers: int):
    keep = _Keep()
    arr = (PeLayerW * n_layers)()
    for i in range(n_layers):
        pre = f"patch_encoder.encoder.layers.{i}."
        for f, n in PE_LAYER_NAMES.items():
            a = _f32(w.get(pre + n))
            keep.refs.append(a)
            setattr(arr[i], f, _ptr(a))
    s = PeW()
    s.n_layers = n_layers
    s.layers = arr
    keep.refs.append(arr)
    for f, n in PE_GLOBAL_NAMES.items():
        a = _f32(w.get(n))
        keep.refs.append(a)
        setattr(s, f, _ptr(a))
    return s, keep


def _addr(a):
    """Host numpy array -> pointer; anything with data_ptr() (device tensor) -> its address."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


# ------------------------------------------------------------------ engines
class DiT:
    """The velocity head on one device."""

    def __init__(self, weights: dict, n_layers: int = 18, dtype=DTYPE_BF16, device=0):
        s, keep = dit_struct(weights, n_layers)
        h = _vp()
        check(lib().dtts_dit_create(C.byref(s), dtype, device, C.byref(h)))
        self.h = h
        self.n_layers = n_layers

    @classmethod
    def from_safetensors(cls, path, n_layers=18, dtype=DTYPE_BF16, device=0):
        self = cls.__new__(cls)
        h = _vp()
        check(lib().dtts_dit_create_from_safetensors(path.encode(), n_layers, dtype, device, C.byref(h)))
        self.h = h
        self.n_layers = n_layers
        return self

    def close(self):
        if getattr(self, "h", None):
            lib().dtts_dit_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_ptr):
        check(lib().dtts_dit_set_stream(self.h, stream_ptr))

    def sync(self):
        check(lib().dtts_dit_sync(self.h))

    def velocity(self, x_in, cond, mask=None, pos=None, n_out=None):
        x_in = _f32(x_in)
        rows, L = x_in.shape[0], x_in.shape[1]
        n_out = L if n_out is None else n_out
        cond = _f32(cond)
        mask = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        pos = _f32(pos)
        out = np.zeros((rows, n_out, 128), np.float32)
        check(lib().dtts_dit_velocity(self.h, _addr(x_in), _addr(cond), _addr(mask), _addr(pos), rows, L, n_out,
                                      _addr(out), MEM_HOST))
        return out

    def blocks(self, h_in, cond, mask=None, pos=None):
        h_in = _f32(h_in)
        rows, L = h_in.shape[0], h_in.shape[1]
        cond = _f32(cond)
        mask = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        pos = _f32(pos)
        out = np.zeros_like(h_in)
        check(lib().dtts_dit_blocks(self.h, _addr(h_in), _addr(cond), _addr(mask), _addr(pos), rows, L, _addr(out),
                                    MEM_HOST))
        return out

    def set_rope(self, mode):
        check(lib().dtts_dit_set_rope(self.h, mode))

    def cond(self, t, spk=None, spk_scale=1.5):
        spk = _f32(spk)
        out = np.zeros(1024, np.float32)
        check(lib().dtts_dit_cond(self.h, C.c_float(t), _addr(spk), C.c_float(spk_scale), _addr(out)))
        return out

    def solve(self, fm_cond, fm_uncond, z0, spk=None, spk_scale=1.5, nfe=10, cfg_scale=2.0, cfg_form=CFG_V4,
              layout=LAYOUT_FM_MASK, use_graph=True, z_out=None, mem=MEM_HOST):
        """Euler + CFG solve.  With mem=MEM_DEVICE every buffer is a device
        tensor (anything with data_ptr()) and the call only enqueues."""
        if mem == MEM_HOST:
            fm_cond, fm_uncond, z0, spk = _f32(fm_cond), _f32(fm_uncond), _f32(z0), _f32(spk)
            if z_out is None:
                z_out = np.zeros_like(z0)
        a = SolveArgs()
        a.n_utt, a.fm_len, a.patch = z0.shape[0], fm_cond.shape[1], z0.shape[1]
        a.fm_cond, a.fm_uncond, a.z0, a.spk = _addr(fm_cond), _addr(fm_uncond), _addr(z0), _addr(spk)
        a.spk_scale, a.nfe, a.cfg_scale, a.cfg_form = spk_scale, nfe, cfg_scale, cfg_form
        a.layout, a.z_out, a.mem, a.use_graph = layout, _addr(z_out), mem, int(use_graph)
        check(lib().dtts_dit_euler_solve(self.h, C.byref(a)))
        return z_out

    def solve_timeline(self, fm_cond, fm_uncond, z0, z_out, spk=None, spk_scale=1.5, nfe=10, cfg_scale=2.0,
                       cfg_form=CFG_V4, layout=LAYOUT_FM_MASK, reps=3):
        """Device time of every launch kind in one solve (device buffers), measured
        in place with events around each launch of the captured solve.  Returns
        {kind name: (summed us per solve, launches per solve)}."""
        a = SolveArgs()
        a.n_utt, a.fm_len, a.patch = z0.shape[0], fm_cond.shape[1], z0.shape[1]
        a.fm_cond, a.fm_uncond, a.z0, a.spk = _addr(fm_cond), _addr(fm_uncond), _addr(z0), _addr(spk)
        a.spk_scale, a.nfe, a.cfg_scale, a.cfg_form = spk_scale, nfe, cfg_scale, cfg_form
        a.layout, a.z_out, a.mem, a.use_graph = layout, _addr(z_out), MEM_DEVICE, 1
        us = (C.c_float * TL_KINDS)()
        n = (C.c_int * TL_KINDS)()
        check(lib().dtts_dit_solve_timeline(self.h, C.byref(a), reps, us, n))
        return {TL_NAMES[k]: (us[k], n[k]) for k in range(TL_KINDS)}

    def profile(self, kind, iters=20):
        us, fl, by = C.c_float(), C.c_double(), C.c_double()
        check(lib().dtts_dit_profile_kernel(self.h, kind, iters, C.byref(us), C.byref(fl), C.byref(by)))
        return us.value, fl.value, by.value

    def tune(self, gemm, bn, epi_warps=4, ksplit=1):
        check(lib().dtts_dit_tune(self.h, gemm.encode(), bn, epi_warps, ksplit))

    def set_fused_ln(self, on):
        """LayerNorm + modulation in the residual GEMMs' epilogue (True) or as separate kernels."""
        check(lib().dtts_dit_set_fused_ln(self.h, 1 if on else 0))

    def last_launch_count(self):
        n = C.c_int()
        check(lib().dtts_dit_last_launch_count(self.h, C.byref(n)))
        return n.value


EOS_SILU, EOS_AS_WRITTEN = 0, 1


class FMHistory:
    """The autoregressive loop's FM buffers on the device (dtts_fm_*)."""

    def __init__(self, dit, n_utt, capacity):
        h = _vp()
        check(lib().dtts_fm_create(dit.h, n_utt, capacity, C.byref(h)))
        self.h, self.dit, self.n_utt = h, dit, n_utt

    def close(self):
        if getattr(self, "h", None):
            lib().dtts_fm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def start(self, hidden0):
        check(lib().dtts_fm_start(self.h, _addr(_f32(hidden0)), MEM_HOST))

    def append_latents(self, z):
        z = _f32(z)
        check(lib().dtts_fm_append_latents(self.h, _addr(z), z.shape[1], MEM_HOST))

    def append_hidden(self, h, eos=True, eos_act=EOS_SILU):
        h = _f32(h)
        p = np.zeros(h.shape[0], np.float32) if eos else None
        check(lib().dtts_fm_append_hidden(self.h, _addr(h), _addr(p), eos_act, MEM_HOST))
        return p

    def length(self):
        n = C.c_int()
        check(lib().dtts_fm_length(self.h, C.byref(n)))
        return n.value

    def read(self):
        L = self.length()
        c = np.zeros((self.n_utt, L, 1024), np.float32)
        u = np.zeros_like(c)
        check(lib().dtts_fm_read(self.h, _addr(c), _addr(u)))
        return c, u

    def solve(self, z0, spk=None, spk_scale=1.5, nfe=10, cfg_scale=2.0, cfg_form=CFG_V4, layout=LAYOUT_FM_MASK,
              use_graph=True):
        z0, spk = _f32(z0), _f32(spk)
        z_out = np.zeros_like(z0)
        a = SolveArgs()
        a.n_utt, a.fm_len, a.patch = z0.shape[0], 0, z0.shape[1]
        a.fm_cond, a.fm_uncond, a.z0, a.spk = None, None, _addr(z0), _addr(spk)
        a.spk_scale, a.nfe, a.cfg_scale, a.cfg_form = spk_scale, nfe, cfg_scale, cfg_form
        a.layout, a.z_out, a.mem, a.use_graph = layout, _addr(z_out), MEM_HOST, int(use_graph)
        check(lib().dtts_fm_solve(self.h, C.byref(a)))
        return z_out


class LLMLayerW(C.Structure):
    _fields_ = [(n, _fp) for n in ("an", "fn", "qw", "qb", "kw", "kb", "vw", "vb", "ow", "ob", "gw", "uw", "dw")]


class LLMW(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("layers", C.POINTER(LLMLayerW)), ("final_norm", _fp)]


LLM_LAYER_NAMES = {
    "an": "input_layernorm.weight", "fn": "post_attention_layernorm.weight",
    "qw": "self_attn.q_proj.weight", "qb": "self_attn.q_proj.bias",
    "kw": "self_attn.k_proj.weight", "kb": "self_attn.k_proj.bias",
    "vw": "self_attn.v_proj.weight", "vb": "self_attn.v_proj.bias",
    "ow": "self_attn.o_proj.weight", "ob": "self_attn.o_proj.bias",
    "gw": "mlp.gate_proj.weight", "uw": "mlp.up_proj.weight", "dw": "mlp.down_proj.weight",
}


class LLM:
    """The LLM decoder step (dtts_llm_*), names as the checkpoint's llm.model.* tensors."""

    def __init__(self, weights: dict, n_layers=28, max_batch=64, max_seq=512, device=0):
        keep = _Keep()
        arr = (LLMLayerW * n_layers)()
        for i in range(n_layers):
            for f, n in LLM_LAYER_NAMES.items():
                a = _f32(weights.get(f"llm.model.layers.{i}." + n))
                keep.refs.append(a)
                setattr(arr[i], f, _ptr(a))
        fn = _f32(weights["llm.model.norm.weight"])
        keep.refs.append(fn)
        s = LLMW(n_layers, arr, _ptr(fn))
        h = _vp()
        check(lib().dtts_llm_create(C.byref(s), device, max_batch, max_seq, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().dtts_llm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_ptr):
        check(lib().dtts_llm_set_stream(self.h, stream_ptr))

    def prefill(self, emb, out=None, mem=MEM_HOST):
        """mem=MEM_DEVICE: emb and out are device tensors and the call only enqueues."""
        if mem == MEM_HOST:
            emb = _f32(emb)
            out = np.zeros_like(emb) if out is None else out
        check(lib().dtts_llm_prefill(self.h, _addr(emb), emb.shape[0], emb.shape[1], _addr(out), mem))
        return out

    def step(self, emb, out=None, mem=MEM_HOST):
        if mem == MEM_HOST:
            emb = _f32(emb)
            out = np.zeros_like(emb) if out is None else out
        check(lib().dtts_llm_step(self.h, _addr(emb), emb.shape[0], _addr(out), mem))
        return out

    def length(self):
        n = C.c_int()
        check(lib().dtts_llm_length(self.h, C.byref(n)))
        return n.value


def voc_struct(w: dict):
    """VocW over the checkpoint-named arrays of w (bigvgan_load's names)."""
    keep = []

    def P(name):
        a = _f32(w.get(name))
        keep.append(a)
        return _ptr(a)

    v = VocW()
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


class Vocoder:
    """The BigVGAN decoder (dtts_voc_*): latents [n_frames][128] -> audio [n_frames * 1920]."""

    HOP = 1920

    def __init__(self, weights: dict, max_frames=256, device=0):
        v, keep = voc_struct(weights)
        h = _vp()
        check(lib().dtts_voc_create(C.byref(v), device, max_frames, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().dtts_voc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_ptr):
        check(lib().dtts_voc_set_stream(self.h, stream_ptr))

    def decode(self, latent, out=None, mem=MEM_HOST):
        """mem=MEM_DEVICE: latent and out are device tensors and the call only enqueues."""
        if mem == MEM_HOST:
            latent = _f32(latent)
            out = np.zeros(latent.shape[0] * self.HOP, np.float32) if out is None else out
        check(lib().dtts_voc_decode(self.h, _addr(latent), latent.shape[0], _addr(out), mem))
        return out


def selftest_wait_limit(device=0):
    """(status, code): a kernel wait that nothing completes must give up with
    DTTS_ERR_TIMEOUT and its code in the error word, leaving the context usable."""
    code = C.c_int()
    st = lib().dtts_selftest_wait_limit(device, C.byref(code))
    return st, code.value


def selftest_conv(x, w, bias=None, dil=1, pad_left=None, bn=64, device=0):
    """Time convolution through the GEMM over taps: x [T][C], w [N][C][K];
    pad_left defaults to the causal dil (K - 1)."""
    x, w, bias = _f32(x), _f32(w), _f32(bias)
    T, Cc = x.shape
    N, _, K = w.shape
    pad = dil * (K - 1) if pad_left is None else pad_left
    out = np.zeros((T, N), np.float32)
    check(lib().dtts_selftest_conv(_ptr(x), T, Cc, _ptr(w), _ptr(bias), N, K, dil, pad, bn, _ptr(out), device))
    return out


def voc_aa_filter():
    f = np.zeros(12, np.float32)
    check(lib().dtts_voc_aa_filter(_ptr(f)))
    return f


def selftest_voc_activation(x, alpha, beta, filt_up, filt_down):
    x = _f32(x)
    fu, fd = _f32(filt_up), _f32(filt_down)
    fch = 1 if fu.size == 12 else x.shape[1]
    out = np.zeros_like(x)
    check(lib().dtts_selftest_voc_activation(_ptr(x), x.shape[0], x.shape[1], _ptr(_f32(alpha)), _ptr(_f32(beta)),
                                             _ptr(fu), _ptr(fd), fch, _ptr(out)))
    return out


class Attention:
    """The DiT attention sublayer alone (manual_attention)."""

    def __init__(self, wq, wk, wv, wo, bo=None, qn=None, kn=None, dtype=DTYPE_F32, device=0):
        self._keep = [_f32(a) for a in (wq, wk, wv, wo, bo, qn, kn)]
        s = AttnW(*[_ptr(a) for a in self._keep])
        h = _vp()
        check(lib().dtts_attn_create(C.byref(s), dtype, device, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().dtts_attn_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, x, mask=None, pos=None):
        x = _f32(x)
        rows, L = x.shape[0], x.shape[1]
        out = np.zeros_like(x)
        mk = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
        pos = _f32(pos)
        check(lib().dtts_attn_forward(self.h, _ptr(x), rows, L, None if mk is None else mk.ctypes.data_as(_u8p),
                                      _ptr(pos), _ptr(out)))
        return out

    def profile_core(self, iters=50):
        us = C.c_float()
        check(lib().dtts_attn_profile_core(self.h, iters, C.byref(us)))
        return us.value


class PatchEncoder:
    def __init__(self, weights: dict, n_layers=24, max_batch=32, max_tokens=512, dtype=DTYPE_BF16, device=0):
        s, keep = pe_struct(weights, n_layers)
        h = _vp()
        check(lib().dtts_pe_create(C.byref(s), dtype, device, max_batch, max_tokens, C.byref(h)))
        self.h = h

    @classmethod
    def from_safetensors(cls, path, n_layers=24, max_batch=32, max_tokens=512, dtype=DTYPE_BF16, device=0):
        self = cls.__new__(cls)
        h = _vp()
        check(lib().dtts_pe_create_from_safetensors(path.encode(), n_layers, dtype, device, max_batch, max_tokens,
                                                    C.byref(h)))
        self.h = h
        return self

    def close(self):
        if getattr(self, "h", None):
            lib().dtts_pe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_ptr):
        check(lib().dtts_pe_set_stream(self.h, stream_ptr))

    def sync(self):
        check(lib().dtts_pe_sync(self.h))

    def forward(self, frames, pair_mode=PAIR_ADJACENT):
        frames = _f32(frames)
        B, n = frames.shape[0], frames.shape[1]
        out = np.zeros((B, n // 4, 1536), np.float32)
        check(lib().dtts_pe_forward(self.h, _addr(frames), B, n, pair_mode, _addr(out), MEM_HOST))
        return out

    def reset(self, B):
        check(lib().dtts_pe_stream_reset(self.h, B))

    def decode(self, frames, out=None, mem=MEM_HOST):
        if mem == MEM_HOST:
            frames = _f32(frames)
        B, n = frames.shape[0], frames.shape[1]
        if out is None:
            out = np.zeros((B, n // 4, 1536), np.float32)
        check(lib().dtts_pe_decode(self.h, _addr(frames), B, n, _addr(out), mem))
        return out

    def length(self):
        n = C.c_int()
        check(lib().dtts_pe_stream_length(self.h, C.byref(n)))
        return n.value


def selftest_gemm(A, B, bias=None, bn=256, device=0):
    A, B, bias = _f32(A), _f32(B), _f32(bias)
    M, K = A.shape
    N = B.shape[0]
    Cm = np.zeros((M, N), np.float32)
    check(lib().dtts_selftest_gemm(_ptr(A), _ptr(B), _ptr(bias), _ptr(Cm), M, N, K, bn, device))
    return Cm


def selftest_attention(q, k, v, mask=None, causal=False, q_pos0=0, use_f32=False, device=0):
    q, k, v = _f32(q), _f32(k), _f32(v)
    rows, Tq, kv = q.shape[0], q.shape[1], k.shape[1]
    out = np.zeros_like(q)
    mk = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
    check(lib().dtts_selftest_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), rows, Tq, kv,
                                        None if mk is None else mk.ctypes.data_as(_u8p), int(causal), q_pos0,
                                        int(use_f32), device))
    return out


def selftest_e4m3(x, device=0):
    """Device e4m3 conversion (round to nearest even, saturating) of x."""
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.zeros(x.size, np.uint8)
    check(lib().dtts_selftest_e4m3(_ptr(x), out.ctypes.data_as(_u8p), x.size, device))
    return out


def selftest_gemm_e4m3(A, a_scale, B, b_scale, bias=None, bn=128, device=0):
    """C = diag(a_scale) (A B^T) diag(b_scale) + bias with e4m3 byte matrices
    A [M][K], B [N][K] on the tcgen05 kind::f8f6f4 GEMM."""
    A, B = np.ascontiguousarray(A, np.uint8), np.ascontiguousarray(B, np.uint8)
    a_scale, b_scale, bias = _f32(a_scale), _f32(b_scale), _f32(bias)
    M, K = A.shape
    N = B.shape[0]
    C_ = np.zeros((M, N), np.float32)
    check(lib().dtts_selftest_gemm_e4m3(A.ctypes.data_as(_u8p), _ptr(a_scale), B.ctypes.data_as(_u8p),
                                        _ptr(b_scale), _ptr(bias), _ptr(C_), M, N, K, bn, device))
    return C_


def fp8_quantize_rows(w):
    """The FP8 engine's per-output-channel weight quantisation (host only):
    returns (e4m3 bytes [rows][cols], scale [rows])."""
    w = np.ascontiguousarray(w, np.float32)
    q = np.zeros(w.shape, np.uint8)
    sc = np.zeros(w.shape[0], np.float32)
    check(lib().dtts_fp8_quantize_rows(_ptr(w), w.shape[0], w.shape[1], q.ctypes.data_as(_u8p), _ptr(sc)))
    return q, sc


def fm_layout(total, fm_len, patch, hidden_patch=1):
    """The attention mask (uint8 [total][total]) and position ids ([total]) a solve
    builds for fm_len history rows and `patch` noise rows (host only)."""
    m = np.zeros((total, total), np.uint8)
    p = np.zeros(total, np.float32)
    check(lib().dtts_fm_layout(total, fm_len, patch, hidden_patch, m.ctypes.data_as(_u8p), _ptr(p)))
    return m, p


class SafeTensors:
    def __init__(self, path):
        h = _vp()
        check(lib().dtts_st_open(path.encode(), C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().dtts_st_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def count(self):
        n = C.c_int()
        check(lib().dtts_st_count(self.h, C.byref(n)))
        return n.value

    def shape(self, name):
        nd = C.c_int()
        shp = (C.c_int64 * 8)()
        check(lib().dtts_st_shape(self.h, name.encode(), C.byref(nd), shp))
        return tuple(shp[i] for i in range(nd.value))

    def read(self, name):
        shp = self.shape(name)
        out = np.zeros(shp, np.float32)
        check(lib().dtts_st_read_f32(self.h, name.encode(), _ptr(out), out.size))
        return out
