"""Helpers shared by the GPU tests: the CPU checker for full-size runs."""
from __future__ import annotations

import os
import shutil
import json
from pathlib import Path

import numpy as np

from conftest import oracle


def host_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def has_avx512() -> bool:
    try:
        return "avx512bw" in Path("/proc/cpuinfo").read_text()
    except OSError:
        return False


class Checker:
    """The reference engine built from its sources when present, else the C
    restatement of its step; both on all host threads."""

    def __init__(self, model, capacity: int, cached_rope: bool = True):
        if oracle.ref_available():
            kernel = "simd512x4" if has_avx512() else "simd256"
            self.impl = oracle.RefEngine(model, capacity, kernel, host_threads(), cached_rope)
            self.kind = "reference"
        else:
            self.impl = oracle.Oracle(model, capacity, cached_rope=cached_rope, threads=host_threads())
            self.kind = "port"

    def step(self, token: int, head: bool = True) -> np.ndarray:
        return self.impl.step(token, head)


def with_max_positions(model: Path, dst: Path, max_positions: int) -> Path:
    """The same weights under a config that allows longer contexts."""
    dst.mkdir(parents=True, exist_ok=True)
    cfg = json.loads((model / "config.json").read_text())
    cfg["max_position_embeddings"] = max_positions
    (dst / "config.json").write_text(json.dumps(cfg))
    link = dst / "model.safetensors"
    if not link.exists():
        link.symlink_to((model / "model.safetensors").resolve())
    return dst
