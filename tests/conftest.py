"""Shared fixtures. GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
from __future__ import annotations

import importlib.util
import os
import tempfile
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def load_package():
    """Import the product package (its directory name is not an identifier)."""
    if "cpu_decode_b200" in sys.modules:
        return sys.modules["cpu_decode_b200"]
    pkg = ROOT / "cpu-decode_b200"
    spec = importlib.util.spec_from_file_location("cpu_decode_b200", pkg / "__init__.py",
                                                  submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["cpu_decode_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


dcb = load_package()
import cpu_decode_b200.synthetic as synthetic  # noqa: E402
import oracle  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 and the built CUDA library")


MODEL_CACHE = Path(os.environ.get("DCB_MODEL_CACHE", str(Path(tempfile.gettempdir()) / "dcb_models")))


@pytest.fixture(scope="session")
def tiny_int8(tmp_path_factory) -> Path:
    """The reference test suite's tiny Qwen (tests/native.cpp:114-148), int8."""
    d = tmp_path_factory.mktemp("tiny")
    bf16 = synthetic.write_bf16_model(d / "bf16", synthetic.TINY, synthetic.tiny_values())
    src = synthetic.load_safetensors(bf16 / "model.safetensors")
    synthetic.write_int8_model(d / "int8", synthetic.TINY,
                               lambda n, s: (src[n].astype(np.uint32) << 16).view(np.float32))
    return d / "int8"


SMALL = synthetic.Dims(hidden=128, intermediate=320, layers=2, heads=4, kv_heads=2, vocab=1000, max_positions=512,
                       epsilon=1e-6, theta=1e6)
# Row lengths that are multiples of 4 but not of 16 (the reference only needs 4).
ODD = synthetic.Dims(hidden=72, intermediate=100, layers=2, heads=6, kv_heads=2, vocab=333, max_positions=128,
                     epsilon=1e-6, theta=10000.0)

# head_dim 64 with 7 and 2 query heads per KV head: the batched engine's TMA
# attention path (the Qwen shape's head geometry at a small width).
G64 = synthetic.Dims(hidden=448, intermediate=512, layers=2, heads=7, kv_heads=1, vocab=1000, max_positions=4096,
                     epsilon=1e-6, theta=1e6)
G64B = synthetic.Dims(hidden=256, intermediate=384, layers=2, heads=4, kv_heads=2, vocab=777, max_positions=4096,
                      epsilon=1e-6, theta=1e6)


@pytest.fixture(scope="session")
def g64_int8(tmp_path_factory) -> Path:
    return synthetic.write_int8_model(tmp_path_factory.mktemp("g64") / "int8", G64, synthetic.random_values(17))


@pytest.fixture(scope="session")
def g64b_int8(tmp_path_factory) -> Path:
    return synthetic.write_int8_model(tmp_path_factory.mktemp("g64b") / "int8", G64B, synthetic.random_values(19))


@pytest.fixture(scope="session")
def small_int8(tmp_path_factory) -> Path:
    return synthetic.write_int8_model(tmp_path_factory.mktemp("small") / "int8", SMALL, synthetic.random_values(3))


@pytest.fixture(scope="session")
def odd_int8(tmp_path_factory) -> Path:
    return synthetic.write_int8_model(tmp_path_factory.mktemp("odd") / "int8", ODD, synthetic.random_values(5))


@pytest.fixture(scope="session")
def qwen05_int8() -> Path:
    """The seeded Qwen2.5-0.5B-shape int8 model (about 500 MB, built once)."""
    return synthetic.ensure_random_model(MODEL_CACHE / "qwen05_seed0", synthetic.QWEN05, seed=0)


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
