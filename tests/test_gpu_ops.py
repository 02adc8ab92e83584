"""Isolated operators on the GPU: the int8 GEMV sweep (the five projection
shapes of the model) and split-KV GQA attention at 128..32768 positions,
FP32 and F16 KV, against the CPU oracle; RMSNorm, RoPE and argmax against
the reference's known answers."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import dcb, oracle

pytestmark = pytest.mark.gpu

GEMV_SHAPES = [(1152, 896, True), (896, 896, False), (9728, 896, False), (896, 4864, False), (151936, 896, False),
               (9, 148, False), (33, 4860, True)]


@pytest.mark.parametrize("rows,cols,bias", GEMV_SHAPES)
def test_gemv_i8_matches_oracle(rows, cols, bias):
    import torch
    rng = np.random.default_rng(rows * 7 + cols)
    w = rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)
    s = rng.uniform(1e-4, 1e-3, size=rows).astype(np.float32)
    x = rng.standard_normal(cols, dtype=np.float32)
    b = rng.standard_normal(rows, dtype=np.float32) if bias else None
    dw, ds, dx = (torch.from_numpy(a).cuda() for a in (w, s, x))
    dy = torch.zeros(rows, dtype=torch.float32, device="cuda")
    db = torch.from_numpy(b).cuda() if bias else None
    dcb.gemv_i8(dw.data_ptr(), ds.data_ptr(), db.data_ptr() if bias else None, dx.data_ptr(), dy.data_ptr(), rows,
                cols)
    torch.cuda.synchronize()
    got = dy.cpu().numpy()
    exp = oracle.matvec(w, s, x, threads=8) + (b if bias else 0)
    # FP32 sums in another order: bounded by a few ulps of sum_j |w_j x_j| * scale
    mag = (np.abs(w.astype(np.float64)) @ np.abs(x.astype(np.float64))) * s
    assert np.all(np.abs(got - exp) <= 2e-6 * mag + 1e-6)


@pytest.mark.parametrize("length", [1, 63, 128, 1024, 4096, 32768])
@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_attention_matches_oracle(length, kv):
    import torch
    heads, kvh, dim, theta = 14, 2, 64, 1e6
    rng = np.random.default_rng(length)
    q = rng.standard_normal(heads * dim, dtype=np.float32)
    k = rng.standard_normal((length, kvh * dim), dtype=np.float32)
    v = rng.standard_normal((length, kvh * dim), dtype=np.float32)
    if kv == "f16":
        k, v = oracle.f16_round(k), oracle.f16_round(v)
    tdt = torch.float16 if kv == "f16" else torch.float32
    dq = torch.from_numpy(q).cuda()
    dk = torch.from_numpy(k).cuda().to(tdt)
    dv = torch.from_numpy(v).cuda().to(tdt)
    out = torch.zeros(heads * dim, device="cuda")
    dcb.attention(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv, out.data_ptr(), length, heads, kvh, dim, theta)
    torch.cuda.synchronize()
    qr = oracle.rope_cached(q, heads, dim, length - 1, theta)
    exp = oracle.attention(qr, k, v, length, heads, kvh, dim, threads=8)
    np.testing.assert_allclose(out.cpu().numpy(), exp, atol=2e-5, rtol=1e-4)


def test_attention_known_answer_without_rope():
    import torch
    heads, kvh, dim, length = 4, 2, 4, 3
    q = (np.arange(heads * dim) % 5).astype(np.float32) - 2
    idx = np.arange(length * kvh * dim)
    keys = (idx % 7).astype(np.float32) * np.float32(0.1)
    values = (idx % 11).astype(np.float32) - 4
    out = torch.zeros(heads * dim, device="cuda")
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, keys, values))
    dcb.attention(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), "f32", out.data_ptr(), length, heads, kvh, dim, 0.0)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), oracle.attention(q, keys, values, length, heads, kvh, dim),
                               atol=2e-6)


def test_rmsnorm_rope_argmax():
    import torch
    x = torch.tensor([1, -2, 3, -4], dtype=torch.float32, device="cuda")
    w = torch.tensor([1, 0.5, -1, 2], dtype=torch.float32, device="cuda")
    out = torch.zeros(4, device="cuda")
    dcb.rmsnorm(x.data_ptr(), w.data_ptr(), out.data_ptr(), 4, 1e-6)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), (x * w).cpu().numpy() / np.sqrt(7.5 + 1e-6), atol=1e-6)
    r = np.array([1, 2, 3, 4, -2, 3, -4, 5], np.float32)
    for direct in (True, False):
        dr = torch.from_numpy(r).cuda()
        dcb.rope(dr.data_ptr(), 2, 4, 7, 10000.0, direct)
        torch.cuda.synchronize()
        exp = oracle.rope_direct(r, 2, 4, 7, 10000.0) if direct else oracle.rope_cached(r, 2, 4, 7, 10000.0)
        np.testing.assert_allclose(dr.cpu().numpy(), exp, atol=3e-6)
    rng = np.random.default_rng(0)
    for n in (1, 7, 151936):
        v = rng.standard_normal(n).astype(np.float32)
        v[n // 2] = v.max() + 1
        if n > 2:
            v[n - 1] = v[n // 2]  # tie: the first index wins
        dv = torch.from_numpy(v).cuda()
        o = torch.zeros(1, dtype=torch.int32, device="cuda")
        dcb.argmax(dv.data_ptr(), n, o.data_ptr())
        torch.cuda.synchronize()
        assert int(o.item()) == oracle.argmax(v)


def test_read_bandwidth_probe_sweeps_the_whole_array():
    """The HBM read probe (tools/bandwidth.cpp's sweep on the GPU): the XOR of
    all words of the i*6364136223846793005+1 pattern matches numpy, every sample
    is a positive rate, and sizes out of range are refused with the reference's
    message."""
    mib = 64
    r = dcb.read_bandwidth(mib=mib, passes=2, repeats=3)
    n = (mib << 20) // 8
    words = np.arange(n, dtype=np.uint64) * np.uint64(6364136223846793005) + np.uint64(1)
    assert r["checksum"] == int(np.bitwise_xor.reduce(words))
    assert len(r["samples"]) == 3 and all(s["GB_per_s"] > 0 for s in r["samples"])
    with pytest.raises(ValueError, match="invalid sweep parameters"):
        dcb.read_bandwidth(mib=16)
