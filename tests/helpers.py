"""Comparison helpers.  Tolerances follow the parity bar of this path:
  bf16 paths      max relative error <= 2e-2 and cosine >= 0.999
  fp32 attention  max relative error <= 1e-3
  vocoder audio   max relative error <= 5e-2 and cosine >= 0.998
where max relative error = max|got - ref| / max|ref| over the whole tensor."""
import json
import struct

import numpy as np

BF16_REL, BF16_COS = 2e-2, 0.999
F32_REL = 1e-3
# vocoder waveform (bf16 convolutions through 6 stages, 54 AMP layers)
VOC_REL, VOC_COS = 5e-2, 0.998


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(1e-30, np.abs(b).max()))


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


def bf16(a):
    """Round-to-nearest-even to bf16, returned as float32."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def assert_bf16_close(got, want, what=""):
    r, c = rel(got, want), cos(got, want)
    assert r <= BF16_REL and c >= BF16_COS, f"{what}: max rel {r:.3e} (<= {BF16_REL}), cos {c:.6f} (>= {BF16_COS})"


def f16_bits(a):
    """IEEE half bit patterns of a (round to nearest even), as uint16."""
    return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def bf16_bits(a):
    """bf16 bit patterns of a (round to nearest even), as uint16."""
    u = np.asarray(a, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def write_safetensors(path, tensors, metadata=None):
    """Minimal writer of the safetensors layout: u64 header length, JSON header,
    raw little-endian data."""
    hdr, blobs, off = {}, [], 0
    if metadata:
        hdr["__metadata__"] = metadata
    for name, (dtype, arr) in tensors.items():
        raw = np.ascontiguousarray(arr).tobytes()
        hdr[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(hdr).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


# FP8 (e4m3) path against the fp32 reference: the quantisation itself moves the
# velocity by a few percent (3.8% max relative error, cosine 0.9993 on a
# 2-layer model), so this bar is wider; against the oracle's restatement of the
# same FP8 recipe the engine meets the bf16 bar above.
FP8_REL, FP8_COS = 1e-1, 0.995
# FP8 engine against the oracle's restatement of the same recipe: tiny
# upstream differences (bf16 intermediates) flip single e4m3 roundings, each a
# whole quantum (6-12%), so the two agree to cosine 0.999 but not element-wise
# to the bf16 bar.  The GEMM itself is pinned tightly by the e4m3 GEMM test.
FP8_ORACLE_REL, FP8_ORACLE_COS = 5e-2, 0.999
# A whole Euler solve (18 layers, CFG scale 2 amplifies velocity differences
# threefold): the recipe's own displacement error against fp32 is 14% max
# relative, cosine 0.993, and the engine is held to the same order.
FP8_SOLVE_REL, FP8_SOLVE_COS = 2.5e-1, 0.985


def assert_fp8_close(got, want, what=""):
    r, c = rel(got, want), cos(got, want)
    assert r <= FP8_REL and c >= FP8_COS, f"{what}: max rel {r:.3e} (<= {FP8_REL}), cos {c:.6f} (>= {FP8_COS})"


def assert_fp8_recipe_close(got, want, what=""):
    r, c = rel(got, want), cos(got, want)
    assert r <= FP8_ORACLE_REL and c >= FP8_ORACLE_COS, \
        f"{what}: max rel {r:.3e} (<= {FP8_ORACLE_REL}), cos {c:.6f} (>= {FP8_ORACLE_COS})"


def assert_fp8_solve_close(got, want, what=""):
    r, c = rel(got, want), cos(got, want)
    assert r <= FP8_SOLVE_REL and c >= FP8_SOLVE_COS, \
        f"{what}: max rel {r:.3e} (<= {FP8_SOLVE_REL}), cos {c:.6f} (>= {FP8_SOLVE_COS})"


def assert_no_worse_than_recipe(got, recipe, exact, what=""):
    """The engine's distance from the fp32 result is of the order of the FP8
    recipe's own: 1 - cos(got, exact) <= 1.5 (1 - cos(recipe, exact)) + 1e-4."""
    e_got, e_rec = 1.0 - cos(got, exact), 1.0 - cos(recipe, exact)
    assert e_got <= 1.5 * e_rec + 1e-4, f"{what}: 1-cos {e_got:.3e} against the recipe's {e_rec:.3e}"
