"""Comparison helpers.  Tolerances follow the parity bar of this path:
  bf16 paths      max relative error <= 2e-2 and cosine >= 0.999
  fp32 attention  max relative error <= 1e-3
where max relative error = max|got - ref| / max|ref| over the whole tensor."""
import json
import struct

import numpy as np

BF16_REL, BF16_COS = 2e-2, 0.999
F32_REL = 1e-3


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
