"""Host-side checks of the C ABI that need no GPU: the library loads, exports
every symbol include/dtts.h declares, validates arguments before touching a
device, and its safetensors reader (F32/F16/BF16, the reference's format,
include/safetensors.h) parses files and rejects malformed ones."""
import ctypes as C
import os
import re
import struct

import numpy as np
import pytest

import dtts
from helpers import bf16_bits, f16_bits, write_safetensors

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "dtts.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dtts_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(dtts.LIB_PATH)
    names = _declared()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert sorted(names) == sorted(dtts.EXPORTS)


def test_every_export_has_a_ctypes_signature(dtts_mod):
    """Without argtypes ctypes would pass a 64-bit pointer as a C int."""
    L = dtts.lib()
    missing = [n for n in dtts.EXPORTS if getattr(L, n).argtypes is None]
    assert not missing, missing


def test_version_and_status_strings(dtts_mod):
    L = dtts_mod.lib()
    assert b"sm_100a" in L.dtts_version()
    for s in range(0, -9, -1):
        assert L.dtts_status_string(s)


def test_argument_validation_without_device(dtts_mod):
    L = dtts_mod.lib()
    h = C.c_void_p()
    assert L.dtts_dit_create(None, 0, 0, C.byref(h)) == dtts.ERR_ARG
    assert L.dtts_dit_velocity(None, None, None, None, None, 1, 1, 1, None, 0) == dtts.ERR_ARG
    assert L.dtts_pe_decode(None, None, 1, 4, None, 0) == dtts.ERR_ARG
    assert L.dtts_dit_euler_solve(None, None) == dtts.ERR_ARG
    assert L.dtts_dit_set_fused_ln(None, 1) == dtts.ERR_ARG
    assert L.dtts_dit_tune(None, b"o", 256, 8, 1) == dtts.ERR_ARG
    w = dtts.DitW()
    w.n_layers = 0
    assert L.dtts_dit_create(C.byref(w), 0, 0, C.byref(h)) == dtts.ERR_ARG
    assert b"n_layers" in L.dtts_last_error()


def test_no_device_is_an_error_not_a_fallback(dtts_mod):
    if dtts_mod.device_count() > 0:
        pytest.skip("a device is visible here")
    import synth
    w = synth.dit_weights(1, n_layers=1)
    with pytest.raises(dtts.DttsError) as e:
        dtts.DiT(w, n_layers=1)
    assert e.value.status == dtts.ERR_NO_DEVICE




def test_safetensors_reader_dtypes(tmp_path, dtts_mod):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 5), dtype=np.float32)
    b = rng.standard_normal((7,), dtype=np.float32)
    c = rng.standard_normal((2, 2, 2), dtype=np.float32)
    p = str(tmp_path / "t.safetensors")
    write_safetensors(p, {"a.weight": ("F32", a), "b": ("F16", f16_bits(b)), "c": ("BF16", bf16_bits(c))},
                      metadata={"format": "pt"})
    st = dtts.SafeTensors(p)
    assert st.count() == 3
    assert st.shape("a.weight") == (3, 5)
    np.testing.assert_array_equal(st.read("a.weight"), a)
    np.testing.assert_array_equal(st.read("b"), b.astype(np.float16).astype(np.float32))
    from helpers import bf16
    np.testing.assert_array_equal(st.read("c"), bf16(c))
    with pytest.raises(dtts.DttsError) as e:
        st.read("missing")
    assert e.value.status == dtts.ERR_IO
    st.close()


def test_safetensors_reader_rejects_malformed(tmp_path, dtts_mod):
    p = str(tmp_path / "bad.safetensors")
    a = np.ones((4,), np.float32)
    write_safetensors(p, {"x": ("F32", a)})
    raw = open(p, "rb").read()
    open(p, "wb").write(raw[:-4])                      # truncated data
    with pytest.raises(dtts.DttsError) as e:
        dtts.SafeTensors(p)
    assert e.value.status == dtts.ERR_IO
    open(p, "wb").write(struct.pack("<Q", 10) + b"not json!!")
    with pytest.raises(dtts.DttsError):
        dtts.SafeTensors(p)
    with pytest.raises(dtts.DttsError):
        dtts.SafeTensors(str(tmp_path / "absent.safetensors"))
    write_safetensors(p, {"x": ("I64", np.ones(2, np.int64))})
    st = dtts.SafeTensors(p)
    with pytest.raises(dtts.DttsError) as e:
        st.read("x")
    assert e.value.status == dtts.ERR_UNSUPPORTED


def test_checkpoint_loader_reports_missing_tensor(tmp_path, dtts_mod):
    p = str(tmp_path / "partial.safetensors")
    write_safetensors(p, {"velocity_field_predictor.blocks.0.attn.q_proj.weight": ("F32", np.zeros((2, 2), np.float32))})
    h = C.c_void_p()
    st = dtts_mod.lib().dtts_dit_create_from_safetensors(p.encode(), 1, 0, 0, C.byref(h))
    assert st in (dtts.ERR_IO, dtts.ERR_ARG)
