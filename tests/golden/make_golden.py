"""Regenerate the golden vectors in this directory from the reference itself.

Runs only where the reference sources are present: it builds the reference's
own engine from them (oracle/Makefile -> oracle/_ref/) and records
  * the SHA-256 of the int8 model files written by the reference's quantiser
    for the tiny test model (tests/native.cpp:114-148) and a small random model,
  * reference-engine logits for fixed token sequences (scalar and simd512x4,
    cached and direct RoPE),
  * reference matvec / attention outputs on the known-answer inputs of
    tests/native.cpp:54-111.
Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from conftest import SMALL, ODD, synthetic  # noqa: E402
import oracle  # noqa: E402

TOKENS = [1, 4, 2, 5, 3, 7, 0, 9, 10, 6]


def sha(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def katt_inputs():
    """Inputs of the reference's numeric known-answer tests (tests/native.cpp:54-95)."""
    rows, cols = 9, 147
    j = np.arange(rows * cols, dtype=np.float32)
    matrix = (np.sin(j * np.float32(0.7)).astype(np.float32) * np.float32(0.4)).astype(np.float32)
    matrix[:cols] = 0
    x = np.cos(np.arange(cols, dtype=np.float32) * np.float32(0.3)).astype(np.float32)
    heads, kvh, dim, length = 4, 2, 4, 3
    q = (np.arange(heads * dim) % 5).astype(np.float32) - 2
    idx = np.arange(length * kvh * dim)
    keys = (idx % 7).astype(np.float32) * np.float32(0.1)
    values = (idx % 11).astype(np.float32) - 4
    return matrix.reshape(rows, cols), x, q, keys, values


def main() -> None:
    oracle.build(reference=True)
    out: dict = {"tokens": TOKENS, "models": {}}
    arrays: dict[str, np.ndarray] = {}
    with tempfile.TemporaryDirectory() as td:
        td = Path(td)
        # tiny fixture: BF16 written like the reference test, quantised by the reference
        synthetic.write_bf16_model(td / "tiny_bf16", synthetic.TINY, synthetic.tiny_values())
        oracle.ref_quantize_model(td / "tiny_bf16", td / "tiny")
        synthetic.write_bf16_model(td / "small_bf16", SMALL, synthetic.random_values(3))
        oracle.ref_quantize_model(td / "small_bf16", td / "small")
        synthetic.write_bf16_model(td / "odd_bf16", ODD, synthetic.random_values(5))
        oracle.ref_quantize_model(td / "odd_bf16", td / "odd")
        for name in ("tiny", "small", "odd"):
            out["models"][name] = {"int8_sha256": sha(td / name / "model.safetensors")}
            for kernel in ("scalar", "simd512x4"):
                for cached in (True, False):
                    eng = oracle.RefEngine(td / name, 16, kernel, 1, cached)
                    logits = np.stack([eng.step(t).copy() for t in TOKENS])
                    arrays[f"{name}_{kernel}_{'cached' if cached else 'direct'}"] = logits
                    eng.close()
    matrix, x, q, keys, values = katt_inputs()
    qm = np.zeros(matrix.shape, np.int8)
    sc = np.zeros(matrix.shape[0], np.float32)
    import ctypes as C
    for r in range(matrix.shape[0]):
        s = C.c_float()
        oracle.ref_lib().ref_quantize_row(np.ascontiguousarray(matrix[r]), matrix.shape[1], qm[r], C.byref(s))
        sc[r] = s.value
    arrays["kat_matrix_q"] = qm
    arrays["kat_matrix_scales"] = sc
    arrays["kat_matvec_scalar"] = oracle.ref_matvec(qm, sc, x, "scalar")
    arrays["kat_matvec_simd512x4"] = oracle.ref_matvec(qm, sc, x, "simd512x4")
    arrays["kat_attention"] = oracle.ref_attention(q, keys, values, 3, 4, 2, 4)
    np.savez_compressed(HERE / "reference_outputs.npz", **arrays)
    (HERE / "reference_outputs.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", HERE / "reference_outputs.npz")


if __name__ == "__main__":
    main()
