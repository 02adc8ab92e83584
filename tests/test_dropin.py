"""The drop-in check: the reference's own CLI (its unchanged src/main.cpp)
linked against this repository's libdecode_b200.so instead of its CPU engine
(oracle/_ref/cpu-decode-b200, built by oracle/Makefile's `dropin` target),
run side by side with the reference CLI built from the same sources
(oracle/_ref/cpu-decode). The commands and outputs compared are the ones
src/main.cpp:93-178 defines: `logits` (PREFIX.bin + PREFIX.json) and `bench`
(JSON with per-sample bytes_per_token and the engine's metadata)."""
from __future__ import annotations

import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT, synthetic

DROPIN = ROOT / "oracle" / "_ref" / "cpu-decode-b200"
REFCLI = ROOT / "oracle" / "_ref" / "cpu-decode"
need_dropin = pytest.mark.skipif(not DROPIN.exists(), reason="drop-in CLI not built (needs the reference sources)")


def run(binary: Path, *args: str, check: bool = True) -> subprocess.CompletedProcess:
    return subprocess.run([str(binary), *args], capture_output=True, text=True, check=check, timeout=900)


@need_dropin
def test_cli_smoke():
    # The reference's CTest smoke (CMakeLists.txt:68-70): --help passes, a
    # malformed token list fails with the CLI's error prefix and exit code 1.
    assert run(DROPIN, "--help").returncode == 0
    bad = run(DROPIN, "logits", "--model", "nowhere", "--tokens", "1,x", "--output", "o", check=False)
    assert bad.returncode == 1 and bad.stderr.startswith("cpu-decode: ")


@pytest.mark.gpu
@need_dropin
@pytest.mark.skipif(not REFCLI.exists(), reason="reference CLI not built")
def test_reference_cli_on_the_b200_engine(qwen05_int8, tmp_path):
    tokens = synthetic.random_tokens(32, synthetic.QWEN05.vocab, seed=11)
    tok_arg = ",".join(map(str, tokens))
    threads = "8"
    # logits: teacher-forced, one row of vocab floats per prompt position.
    run(DROPIN, "logits", "--model", str(qwen05_int8), "--tokens", tok_arg, "--output", str(tmp_path / "b200"),
        "--threads", threads, "--kernel", "simd512x4")
    run(REFCLI, "logits", "--model", str(qwen05_int8), "--tokens", tok_arg, "--output", str(tmp_path / "ref"),
        "--threads", threads, "--kernel", "simd512x4")
    meta_b = json.loads((tmp_path / "b200.json").read_text())
    meta_r = json.loads((tmp_path / "ref.json").read_text())
    shape = tuple(meta_r["shape"])
    assert tuple(meta_b["shape"]) == shape
    got = np.fromfile(tmp_path / "b200.bin", dtype="<f4").reshape(shape)
    exp = np.fromfile(tmp_path / "ref.bin", dtype="<f4").reshape(shape)
    assert float(np.abs(got - exp).max()) < 1e-3
    assert meta_b["argmax"] == meta_r["argmax"]
    # bench: the same byte model per token, and the metadata keys the
    # reference's tools read (tools/summarize.py:38,80-82).
    bench_args = ["bench", "--model", str(qwen05_int8), "--tokens", tok_arg, "--context", "128", "--steps", "16",
                  "--repeats", "1", "--threads", threads, "--kernel", "simd512x4"]
    b = json.loads(run(DROPIN, *bench_args).stdout)
    r = json.loads(run(REFCLI, *bench_args).stdout)
    for key in ("kernel", "weight_dtype", "rope", "threads", "context", "kv_capacity"):
        assert key in b, key
        assert b[key] == r[key], key
    bb, rb = b["samples"][0]["bytes_per_token"], r["samples"][0]["bytes_per_token"]
    assert bb["total_min"] == rb["total_min"]
    assert bb["kv_read_min"] == rb["kv_read_min"]
    assert b["samples"][0]["generated_tokens"] == r["samples"][0]["generated_tokens"]
    assert b["samples"][0]["operation_seconds"]["device_step"] > 0
