"""The quantiser on the GPU (dcb_quantize_model, dcb_quantize_rows_bf16)
against the reference's own quantiser (src/model.cpp:354-417,
src/kernels.cpp:121-131): the SHA-256 of the files it wrote for the test
models (tests/golden, made by the reference itself), and row by row against
the reference's quantize_row on awkward values."""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from conftest import SMALL, ODD, dcb, oracle, synthetic

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "reference_outputs.json").read_text())


@pytest.mark.parametrize("name", ["tiny", "small", "odd"])
def test_device_quantiser_writes_the_reference_file(name, tmp_path):
    dims = {"tiny": synthetic.TINY, "small": SMALL, "odd": ODD}[name]
    values = {"tiny": synthetic.tiny_values, "small": lambda: synthetic.random_values(3),
              "odd": lambda: synthetic.random_values(5)}[name]()
    src = synthetic.write_bf16_model(tmp_path / "bf16", dims, values)
    dcb.quantize_model(src, tmp_path / "int8")
    got = hashlib.sha256((tmp_path / "int8" / "model.safetensors").read_bytes()).hexdigest()
    assert got == META["models"][name]["int8_sha256"]
    assert (tmp_path / "int8" / "config.json").read_text() == (src / "config.json").read_text()


def test_device_rows_match_the_reference_rule():
    rng = np.random.default_rng(9)
    rows = [rng.standard_normal(300).astype(np.float32) * 0.02,
            np.zeros(300, np.float32),                                   # all zero: scale 1
            np.full(300, -3.0, np.float32),
            (np.arange(300, dtype=np.float32) - 150) * 127 / 150,        # exact multiples of the scale
            (np.arange(300, dtype=np.float32) - 149.5) * (127 / 149.5),  # halves
            rng.standard_normal(300).astype(np.float32) * 1e-30,         # tiny magnitudes
            rng.standard_normal(300).astype(np.float32) * 1e30]
    m = np.stack(rows)
    bits = (m.view(np.uint32) >> 16).astype(np.uint16)  # BF16 truncation of each value
    q, sc = dcb.quantize_rows_bf16(bits)
    as_f32 = (bits.astype(np.uint32) << 16).view(np.float32)
    if oracle.ref_available():
        import ctypes as C
        for r in range(m.shape[0]):
            eq = np.zeros(m.shape[1], np.int8)
            es = C.c_float()
            assert oracle.ref_lib().ref_quantize_row(np.ascontiguousarray(as_f32[r]), m.shape[1], eq, C.byref(es)) == 0
            np.testing.assert_array_equal(q[r], eq)
            assert sc[r] == np.float32(es.value)
    eq, es = synthetic.quantize_rows(as_f32)
    np.testing.assert_array_equal(q, eq)
    np.testing.assert_array_equal(sc, es)


def test_device_quantiser_rejects_nonfinite():
    bits = np.zeros((2, 8), np.uint16)
    bits[1, 3] = 0x7FC0  # NaN
    with pytest.raises(ValueError, match="nonfinite model weight"):
        dcb.quantize_rows_bf16(bits)
