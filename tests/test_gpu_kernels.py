"""Engine kernels in isolation through the C ABI self-test entry points,
against float64 numpy on the same bf16-rounded inputs."""
import numpy as np
import pytest

import dtts
from helpers import bf16, rel

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,bn", [
    (128, 256, 64, 256), (128, 128, 64, 128), (1, 256, 128, 256), (200, 512, 1024, 256),
    (1000, 1024, 4096, 256), (8192, 3072, 1024, 256), (64, 1536, 2048, 256), (333, 384, 192, 128),
    (333, 384, 192, 64), (700, 576, 512, 192),
])
def test_tcgen05_gemm(M, N, K, bn):
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((M, K), dtype=np.float32)
    B = rng.standard_normal((N, K), dtype=np.float32)
    bias = rng.standard_normal(N, dtype=np.float32)
    got = dtts.selftest_gemm(A, B, bias, bn=bn)
    want = bf16(A).astype(np.float64) @ bf16(B).astype(np.float64).T + bias
    assert rel(got, want) < 1e-5


def test_gemm_rejects_bad_shapes():
    A = np.zeros((4, 100), np.float32)
    B = np.zeros((256, 100), np.float32)
    with pytest.raises(dtts.DttsError) as e:
        dtts.selftest_gemm(A, B)
    assert e.value.status == dtts.ERR_ARG


def _attn_ref(q, k, v, mask=None, causal=False, q0=0):
    q, k, v = (np.asarray(a, np.float64) for a in (q, k, v))
    rows, Tq, kv = q.shape[0], q.shape[1], k.shape[1]
    out = np.zeros_like(q)
    for h in range(16):
        sl = slice(64 * h, 64 * h + 64)
        s = np.einsum("rid,rjd->rij", q[..., sl], k[..., sl]) * 0.125
        if causal:
            s = np.where(np.arange(kv)[None, None] <= (q0 + np.arange(Tq))[None, :, None], s, -np.inf)
        if mask is not None:
            s = np.where(mask[None] != 0, s, -np.inf)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        out[..., sl] = np.einsum("rij,rjd->rid", p, v[..., sl])
    return out


@pytest.mark.parametrize("rows,Tq,kv,causal,q0,use_mask", [
    (2, 64, 64, False, 0, False), (2, 64, 64, False, 0, True), (3, 250, 250, True, 0, False),
    (4, 2, 130, True, 128, False), (2, 100, 100, False, 0, True), (1, 16, 16, False, 0, False),
    (2, 256, 256, False, 0, False),
    # 64 < L <= 256 bidirectional on the tensor cores (whole key range in TMEM):
    # 128- and 256-key tiles, a second query tile, L not a multiple of 32 or 128
    (3, 256, 256, False, 0, True), (2, 130, 130, False, 0, True), (1, 65, 65, False, 0, False),
    (5, 200, 200, False, 0, True), (2, 128, 128, False, 0, True), (3, 97, 97, False, 0, False),
    # L = 64 on the tensor cores, an odd number of sequences (the last pair half empty)
    (3, 64, 64, False, 0, True), (5, 64, 64, False, 0, False),
    # decode shapes (a few queries against a long cache)
    (3, 1, 500, False, 0, False), (2, 8, 1000, True, 992, False), (1, 5, 67, True, 62, False),
])
@pytest.mark.parametrize("use_f32", [False, True])
def test_attention(rows, Tq, kv, causal, q0, use_mask, use_f32):
    if use_f32 and kv > 400:
        pytest.skip("the fp32 kernel holds K and V of one head in 200 KB of shared memory: kv_len <= 400")
    rng = np.random.default_rng(rows * 1000 + Tq + kv)
    q = rng.standard_normal((rows, Tq, 1024), dtype=np.float32)
    k = rng.standard_normal((rows, kv, 1024), dtype=np.float32)
    v = rng.standard_normal((rows, kv, 1024), dtype=np.float32)
    mask = None
    if use_mask:
        mask = (rng.random((Tq, kv)) < 0.6).astype(np.uint8)
        np.fill_diagonal(mask, 1)
    got = dtts.selftest_attention(q, k, v, mask, causal, q0, use_f32=use_f32)
    if use_f32:
        want = _attn_ref(q, k, v, mask, causal, q0)
        assert rel(got, want) < 1e-5
    else:
        want = _attn_ref(bf16(q), bf16(k), bf16(v), mask, causal, q0)
        assert rel(got, want) < 1e-2


def _conv_ref(x, w, bias, dil, pad):
    T, N, K = x.shape[0], w.shape[0], w.shape[2]
    xb, wb = bf16(x).astype(np.float64), bf16(w).astype(np.float64)
    out = np.zeros((T, N)) + (0 if bias is None else bias)
    for k in range(K):
        sh = k * dil - pad
        src = np.zeros_like(xb)
        lo, hi = max(0, -sh), min(T, T - sh)
        if hi > lo:
            src[lo:hi] = xb[lo + sh:hi + sh]
        out += src @ wb[:, :, k].T
    return out


@pytest.mark.parametrize("T,C,N,K,dil,pad,bn", [
    (300, 64, 64, 11, 5, 50, 64),      # causal dilated (AMP c1, 64-channel stages)
    (200, 128, 128, 7, 1, 6, 128),     # causal, two channel blocks per tap
    (150, 192, 192, 3, 3, 6, 192),     # 192-wide tiles
    (77, 128, 256, 5, 1, 2, 128),      # centred K = 5 (conv_pre), rows past T read as zero
    (130, 64, 128, 2, 1, 0, 64),       # taps x[q], x[q+1]; pad 0
])
def test_conv_over_taps(T, C, N, K, dil, pad, bn):
    rng = np.random.default_rng(T + C + N + K)
    x = rng.standard_normal((T, C), dtype=np.float32)
    w = rng.standard_normal((N, C, K), dtype=np.float32)
    bias = rng.standard_normal(N, dtype=np.float32)
    got = dtts.selftest_conv(x, w, bias, dil=dil, pad_left=pad, bn=bn)
    assert rel(got, _conv_ref(x, w, bias, dil, pad)) < 1e-5
