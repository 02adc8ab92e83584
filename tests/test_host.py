"""Host-side checks that need no GPU: the C ABI library loads and exports every
declared symbol, and the model loader rejects what the reference rejects
(tests/native.cpp:233-263 of the reference) with the same messages. The loader
validates before it touches the device, so these run on CPU."""
from __future__ import annotations

import json
import re
import shutil
import struct
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT, cuda_available, dcb, synthetic


def declared_symbols() -> set[str]:
    text = (ROOT / "include" / "decode_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(dcb_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    lib = dcb.lib()
    declared = declared_symbols()
    assert declared == set(dcb.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name


def _open(path, capacity=4):
    import ctypes as C
    h = C.c_void_p()
    rc = dcb.lib().dcb_create_from_dir(str(path).encode(), capacity, 0, 1, 0, C.byref(h))
    msg = dcb.lib().dcb_last_error().decode()
    if rc == 0:
        dcb.lib().dcb_destroy(h)
    return rc, msg


def _header_file(path: Path, header: dict, payload: bytes = b"\0" * 8) -> None:
    enc = json.dumps(header).encode()
    enc += b" " * (-len(enc) % 8)
    path.write_bytes(struct.pack("<Q", len(enc)) + enc + payload)


@pytest.fixture()
def bad_dir(tmp_path, tiny_int8):
    d = tmp_path / "bad"
    d.mkdir()
    shutil.copy(tiny_int8 / "config.json", d / "config.json")
    return d


def test_missing_model_rejected(tmp_path):
    rc, msg = _open(tmp_path / "missing")
    assert rc != 0 and "cannot open" in msg


def test_truncated_and_oversize_header_rejected(bad_dir):
    (bad_dir / "model.safetensors").write_bytes(b"bad")
    rc, msg = _open(bad_dir)
    assert rc != 0 and msg == "invalid safetensors file"
    (bad_dir / "model.safetensors").write_bytes(struct.pack("<Q", 1000000))
    rc, msg = _open(bad_dir)
    assert rc != 0 and msg == "invalid safetensors header length"


@pytest.mark.parametrize("header,expected", [
    ({"x": {"dtype": "F16", "shape": [1], "data_offsets": [0, 2]}}, "unsupported tensor dtype: F16"),
    ({"x": {"dtype": "BF16", "shape": [-1], "data_offsets": [0, 2]}}, "invalid tensor shape"),
    ({"x": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 100]}}, "tensor bounds/alignment mismatch: x"),
    ({"x": {"dtype": "F32", "shape": [1], "data_offsets": [1, 5]}}, "tensor bounds/alignment mismatch: x"),
    ({"x": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]},
      "y": {"dtype": "BF16", "shape": [2], "data_offsets": [2, 6]}}, "gapped or overlapping safetensors payload"),
    ({"x": {"dtype": "BF16", "shape": [1], "data_offsets": [2, 4]}}, "gapped or overlapping safetensors payload"),
    ({"x": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 2]}}, "unindexed safetensors payload"),
    ({"x": {"dtype": "BF16", "shape": [1, 1, 1], "data_offsets": [0, 2]}}, "expected vector or matrix tensor"),
])
def test_malformed_safetensors_rejected(bad_dir, header, expected):
    _header_file(bad_dir / "model.safetensors", header)
    rc, msg = _open(bad_dir)
    assert rc != 0 and msg == expected


@pytest.mark.parametrize("change,expected", [
    ({"num_attention_heads": 3}, "invalid Qwen dimensions or constants"),
    ({"model_type": "llama"}, "requires tied-head Qwen2 architecture"),
    ({"tie_word_embeddings": False}, "requires tied-head Qwen2 architecture"),
    ({"rope_scaling": {"type": "yarn"}}, "scaled RoPE is not supported"),
    ({"hidden_act": "gelu"}, "requires SiLU"),
    ({"vocab_size": 0}, "invalid config: vocab_size"),
    ({"head_dim": 5}, "incompatible head_dim"),
])
def test_invalid_architecture_rejected(tmp_path, tiny_int8, change, expected):
    d = tmp_path / "arch"
    shutil.copytree(tiny_int8, d)
    cfg = json.loads((d / "config.json").read_text())
    cfg.update(change)
    (d / "config.json").write_text(json.dumps(cfg))
    rc, msg = _open(d)
    assert rc != 0 and msg == expected


def test_capacity_checked_against_max_positions(tiny_int8):
    rc, msg = _open(tiny_int8, capacity=33)
    assert rc != 0 and msg == "invalid thread count or context capacity"
    rc, msg = _open(tiny_int8, capacity=0)
    assert rc != 0 and msg == "invalid thread count or context capacity"


def test_bf16_model_needs_quantization(tmp_path):
    d = synthetic.write_bf16_model(tmp_path / "bf16", synthetic.TINY, synthetic.tiny_values())
    rc, msg = _open(d)
    assert rc != 0 and "int8" in msg


def test_missing_tensor_and_bad_scales_rejected(tmp_path, tiny_int8):
    t = synthetic.load_safetensors(tiny_int8 / "model.safetensors")
    for drop, expected in (("model.norm.weight", "missing tensor: model.norm.weight"),):
        items = [(n, {"I8": "I8"}.get(str(a.dtype), None), a) for n, a in t.items() if n != drop]
        out = []
        for n, _, a in sorted(items):
            dt = "I8" if a.dtype == np.int8 else "F32"
            out.append((n, dt, a.shape, np.ascontiguousarray(a)))
        d = tmp_path / "drop"
        d.mkdir()
        synthetic.write_safetensors(d / "model.safetensors", out, synthetic.QUANT_METADATA)
        shutil.copy(tiny_int8 / "config.json", d / "config.json")
        rc, msg = _open(d)
        assert rc != 0 and msg == expected
    out = []
    for n, a in sorted(t.items()):
        a = np.array(a)
        if n == "model.embed_tokens.weight.scales":
            a[3] = 0.0
        out.append((n, "I8" if a.dtype == np.int8 else "F32", a.shape, a))
    d = tmp_path / "scales"
    d.mkdir()
    synthetic.write_safetensors(d / "model.safetensors", out, synthetic.QUANT_METADATA)
    shutil.copy(tiny_int8 / "config.json", d / "config.json")
    rc, msg = _open(d)
    assert rc != 0 and msg == "invalid quantization scale"


@pytest.mark.skipif(cuda_available(), reason="checks the no-GPU failure path")
def test_engine_fails_loudly_without_a_gpu(tiny_int8):
    rc, msg = _open(tiny_int8)
    assert rc != 0 and msg  # a CUDA error, never a silent CPU path


def _sum_word(v: float) -> int:
    """One contribution to a step-kernel sum word: 2^56 + (rint(v * 2^26) + 2^47),
    the integer clamped to |q| < 2^47 (the encoding of dacc_add in
    csrc/step_kernel.cuh)."""
    bias = 1 << 47
    q = int(np.rint(np.float64(v) * 2.0 ** 26))
    q = max(1 - bias, min(bias - 1, q))
    return (1 << 56) + q + bias


def _decode(w: int) -> tuple[int, float]:
    count = w >> 56
    q = (w & ((1 << 56) - 1)) - count * (1 << 47)
    return count, q / 2.0 ** 26


def test_sum_words_are_exact_order_free_and_self_counting():
    """The O and down projections' outputs are summed over blocks as 64-bit
    integer additions into L2 words that count their own contributions: the
    sum must not depend on the order of the additions, the count field must
    equal the number of contributors, and no carry may reach it."""
    rng = np.random.default_rng(7)
    mask = (1 << 64) - 1
    for n, scale in ((148, 1e-2), (148, 3.0), (14, 40.0), (255, 2.0 ** 21 - 1)):
        v = rng.uniform(-scale, scale, n)
        words = [_sum_word(x) for x in v]
        w1 = sum(words) & mask
        w2 = sum(words[i] for i in rng.permutation(n)) & mask
        assert w1 == w2
        count, total = _decode(w1)
        assert count == n
        exact = sum(int(np.rint(x * 2.0 ** 26)) for x in v) / 2.0 ** 26
        assert total == exact
        assert abs(total - float(np.sum(v))) <= n * 2.0 ** -27 + 1e-9 * abs(float(np.sum(v)))
    # The largest magnitudes from 255 contributors stay below the count field.
    top = sum(_sum_word(2.0 ** 21) for _ in range(255)) & mask
    assert _decode(top)[0] == 255
    bottom = sum(_sum_word(-2.0 ** 21) for _ in range(255)) & mask
    assert _decode(bottom)[0] == 255


@pytest.mark.parametrize("mib,passes,repeats", [(16, 1, 1), (65537, 1, 1), (64, 0, 1), (64, 1, 0)])
def test_read_bandwidth_probe_rejects_invalid_sweeps(mib, passes, repeats):
    """The HBM read probe checks its sizes before touching a device, with the
    reference's message (tools/bandwidth.cpp:72-73)."""
    with pytest.raises(ValueError, match="invalid sweep parameters"):
        dcb.read_bandwidth(mib=mib, passes=passes, repeats=repeats)
