"""The CPU oracle and the model writer, pinned to the reference's own outputs.

Golden vectors in tests/golden/ were produced by the reference itself, built
from its sources (tests/golden/make_golden.py). Known-answer inputs restate
tests/native.cpp:42-113 of the reference."""
from __future__ import annotations

import hashlib
import json
import math
from pathlib import Path

import numpy as np
import pytest

from conftest import ODD, SMALL, oracle, synthetic

GOLDEN = Path(__file__).resolve().parent / "golden"
REF = np.load(GOLDEN / "reference_outputs.npz")
META = json.loads((GOLDEN / "reference_outputs.json").read_text())
TOKENS = META["tokens"]


def _sha(p: Path) -> str:
    return hashlib.sha256(p.read_bytes()).hexdigest()


def test_int8_writer_is_byte_identical_to_reference_quantizer(tiny_int8, small_int8, odd_int8):
    assert _sha(tiny_int8 / "model.safetensors") == META["models"]["tiny"]["int8_sha256"]
    assert _sha(small_int8 / "model.safetensors") == META["models"]["small"]["int8_sha256"]
    assert _sha(odd_int8 / "model.safetensors") == META["models"]["odd"]["int8_sha256"]


@pytest.mark.parametrize("name", ["tiny", "small", "odd"])
@pytest.mark.parametrize("rope", ["cached", "direct"])
def test_oracle_step_matches_reference_engine(name, rope, tiny_int8, small_int8, odd_int8):
    model = {"tiny": tiny_int8, "small": small_int8, "odd": odd_int8}[name]
    orc = oracle.Oracle(model, 16, cached_rope=(rope == "cached"))
    got = np.stack([orc.step(t).copy() for t in TOKENS])
    # bit-exact with the reference's scalar kernel (same operation order)
    np.testing.assert_array_equal(got, REF[f"{name}_scalar_{rope}"])
    # the AVX-512 kernel only reorders the sums
    np.testing.assert_allclose(got, REF[f"{name}_simd512x4_{rope}"], atol=1e-5, rtol=0)


def test_rmsnorm_known_answer():
    # tests/native.cpp:43-45
    x = np.array([1, -2, 3, -4], np.float32)
    w = np.array([1, 0.5, -1, 2], np.float32)
    out = oracle.rmsnorm(x, w, 1e-6)
    np.testing.assert_allclose(out, x * w / math.sqrt(7.5 + 1e-6), atol=1e-6)


def test_rope_known_answer():
    # tests/native.cpp:46-53: split-half rotation at position 7, theta 1e4
    x = np.array([1, 2, 3, 4, -2, 3, -4, 5], np.float32)
    got = oracle.rope_direct(x, 2, 4, 7, 10000.0)
    for h in range(2):
        for j in range(2):
            a = 7 / 10000.0 ** (2 * j / 4)
            first, second = x[4 * h + j], x[4 * h + j + 2]
            assert abs(got[4 * h + j] - (first * math.cos(a) - second * math.sin(a))) <= 3e-6
            assert abs(got[4 * h + j + 2] - (first * math.sin(a) + second * math.cos(a))) <= 3e-6
    cached = oracle.rope_cached(x, 2, 4, 7, 10000.0)
    np.testing.assert_allclose(cached, got, atol=3e-6)


def test_quantize_row_known_answer():
    # tests/native.cpp:54-69: 9x147 matrix with an all-zero first row
    q, s = REF["kat_matrix_q"], REF["kat_matrix_scales"]
    rows, cols = q.shape
    j = np.arange(rows * cols, dtype=np.float32)
    m = (np.sin(j * np.float32(0.7)).astype(np.float32) * np.float32(0.4)).reshape(rows, cols)
    m[0] = 0
    mq, ms = synthetic.quantize_rows(m)
    np.testing.assert_array_equal(mq, q)
    np.testing.assert_array_equal(ms, s)
    assert s[0] == 1.0
    assert np.all(np.abs(q.astype(np.float32) * s[:, None] - m) <= s[:, None] * 0.501 + 1e-7)


def test_quantizer_rounds_half_away_from_zero():
    w = np.array([[127.0, 0.5, -0.5, 1.5, -2.5, 63.5]], np.float32)
    q, s = synthetic.quantize_rows(w)
    assert s[0] == 1.0
    assert q.tolist() == [[127, 1, -1, 2, -3, 64]]
    with pytest.raises(ValueError):
        synthetic.quantize_rows(np.array([[np.nan, 1.0]], np.float32))


def test_matvec_known_answer_and_tail():
    # tests/native.cpp:70-86: 147 columns exercise every tail path; tolerance 3e-6
    q, s = REF["kat_matrix_q"], REF["kat_matrix_scales"]
    x = np.cos(np.arange(q.shape[1], dtype=np.float32) * np.float32(0.3)).astype(np.float32)
    exact = (q.astype(np.float64) @ x.astype(np.float64)) * s
    got = oracle.matvec(q, s, x)
    np.testing.assert_array_equal(got, REF["kat_matvec_scalar"])
    np.testing.assert_allclose(got, exact, atol=3e-6)
    np.testing.assert_allclose(REF["kat_matvec_simd512x4"], exact, atol=3e-6)


def test_attention_known_answer():
    # tests/native.cpp:91-111: 4 heads over 2 KV heads, length 3
    heads, kvh, dim, length = 4, 2, 4, 3
    q = (np.arange(heads * dim) % 5).astype(np.float32) - 2
    idx = np.arange(length * kvh * dim)
    keys = (idx % 7).astype(np.float32) * np.float32(0.1)
    values = (idx % 11).astype(np.float32) - 4
    got = oracle.attention(q, keys, values, length, heads, kvh, dim)
    np.testing.assert_array_equal(got, REF["kat_attention"])
    for h in range(heads):
        p = np.array([math.exp(sum(float(q[h * dim + j]) * float(keys[t * kvh * dim + (h // 2) * dim + j])
                                   for j in range(dim)) / 2) for t in range(length)])
        p /= p.sum()
        for j in range(dim):
            exp = sum(p[t] * values[t * kvh * dim + (h // 2) * dim + j] for t in range(length))
            assert abs(got[h * dim + j] - exp) <= 2e-6
    with pytest.raises(RuntimeError):
        oracle.attention(q, keys, values, 0, heads, kvh, dim)


def test_argmax_first_index_wins():
    x = np.array([1.0, 3.0, -2.0, 3.0, 3.0], np.float32)
    assert oracle.argmax(x) == 1
    assert oracle.argmax(np.full(7, -np.inf, np.float32)) == 0


def test_oracle_kv_f16_rounds_cache(small_int8):
    a = oracle.Oracle(small_int8, 8, kv_f16=False)
    b = oracle.Oracle(small_int8, 8, kv_f16=True)
    for t in TOKENS[:5]:
        la, lb = a.step(t).copy(), b.step(t).copy()
    kb, vb = b.kv_view()
    np.testing.assert_array_equal(kb[:, :5], oracle.f16_round(kb[:, :5]))
    assert np.abs(la - lb).max() < 5e-2


@pytest.mark.skipif(not oracle.ref_available(), reason="reference build not present")
def test_oracle_against_live_reference_engine(small_int8):
    ref = oracle.RefEngine(small_int8, 32, "scalar", 2, True)
    orc = oracle.Oracle(small_int8, 32, threads=2)
    for t in [5, 17, 999, 0, 123, 456]:
        np.testing.assert_array_equal(orc.step(t), ref.step(t))
    ref.rewind(3)
    orc.rewind(3)
    np.testing.assert_array_equal(orc.step(42), ref.step(42))
    _, prof = ref.step_profiled(7)
    assert prof["steps"] == 1 and prof["head_steps"] == 1
