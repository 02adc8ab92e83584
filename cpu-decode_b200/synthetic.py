"""Seeded synthetic models in the reference's on-disk format.

The engine loads a directory holding ``config.json`` and ``model.safetensors``,
the layout the reference writes in ``quantize_model`` (src/model.cpp:354-417):
tensors in byte order of their names, every matrix stored as I8 followed by its
``<name>.scales`` F32 row scales, every vector as F32, a compact JSON header
padded with spaces to a multiple of 8, and a ``__metadata__`` entry. The
per-row quantiser restates ``quantize_row`` (src/kernels.cpp:121-131):
``scale = max|w| / 127`` (1 for an all-zero row) and
``q = clamp(round_half_away(w / scale), -127, 127)``, all in FP32.

No real checkpoint is available offline, so every benchmark model is
random-initialised from a seed: matrices N(0, 0.02) rounded to BF16, RMSNorm
gains 1.0, QKV biases N(0, 0.02) rounded to BF16.
"""
from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass, asdict
from pathlib import Path

import numpy as np


@dataclass(frozen=True)
class Dims:
    hidden: int = 896
    intermediate: int = 4864
    layers: int = 24
    heads: int = 14
    kv_heads: int = 2
    vocab: int = 151936
    max_positions: int = 32768
    epsilon: float = 1e-6
    theta: float = 1e6

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def config_json(self) -> dict:
        return {
            "model_type": "qwen2", "tie_word_embeddings": True, "hidden_act": "silu",
            "hidden_size": self.hidden, "intermediate_size": self.intermediate,
            "num_hidden_layers": self.layers, "num_attention_heads": self.heads,
            "num_key_value_heads": self.kv_heads, "vocab_size": self.vocab,
            "max_position_embeddings": self.max_positions,
            "rms_norm_eps": self.epsilon, "rope_theta": self.theta,
        }


QWEN05 = Dims()
# The reference's own tiny test model (tests/native.cpp:118-123).
TINY = Dims(hidden=8, intermediate=12, layers=1, heads=2, kv_heads=1, vocab=11,
            max_positions=32, epsilon=1e-6, theta=10000.0)


def tensor_shapes(d: Dims) -> dict[str, tuple[int, ...]]:
    """Every tensor of a tied-head Qwen2 checkpoint (src/model.cpp:192-217)."""
    s: dict[str, tuple[int, ...]] = {
        "model.embed_tokens.weight": (d.vocab, d.hidden),
        "model.norm.weight": (d.hidden,),
    }
    for l in range(d.layers):
        b = f"model.layers.{l}."
        s[b + "input_layernorm.weight"] = (d.hidden,)
        s[b + "post_attention_layernorm.weight"] = (d.hidden,)
        s[b + "self_attn.q_proj.weight"] = (d.hidden, d.hidden)
        s[b + "self_attn.q_proj.bias"] = (d.hidden,)
        s[b + "self_attn.k_proj.weight"] = (d.kv_dim, d.hidden)
        s[b + "self_attn.k_proj.bias"] = (d.kv_dim,)
        s[b + "self_attn.v_proj.weight"] = (d.kv_dim, d.hidden)
        s[b + "self_attn.v_proj.bias"] = (d.kv_dim,)
        s[b + "self_attn.o_proj.weight"] = (d.hidden, d.hidden)
        s[b + "mlp.gate_proj.weight"] = (d.intermediate, d.hidden)
        s[b + "mlp.up_proj.weight"] = (d.intermediate, d.hidden)
        s[b + "mlp.down_proj.weight"] = (d.hidden, d.intermediate)
    return s


def is_norm(name: str) -> bool:
    return name.endswith("layernorm.weight") or name == "model.norm.weight"


def bf16_round(x: np.ndarray) -> np.ndarray:
    """FP32 -> BF16 (round to nearest even, as torch does) -> FP32, finite inputs."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bits = bits + (np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1)))
    bits &= np.uint32(0xFFFF0000)
    return bits.view(np.float32)


def bf16_truncate(x: np.ndarray) -> np.ndarray:
    """FP32 -> BF16 by dropping the low half, as tests/native.cpp:30-33 does."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return (bits & np.uint32(0xFFFF0000)).view(np.float32)


def quantize_rows(w: np.ndarray, block: int = 8192) -> tuple[np.ndarray, np.ndarray]:
    """Per-row symmetric int8, restating src/kernels.cpp:121-131 in FP32."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows = w.shape[0]
    q = np.empty(w.shape, np.int8)
    scale = np.empty(rows, np.float32)
    for a in range(0, rows, block):
        blk = w[a:a + block]
        if not np.isfinite(blk).all():
            raise ValueError("nonfinite model weight")
        maximum = np.abs(blk).max(axis=1)
        sc = np.where(maximum == 0, np.float32(1.0), maximum / np.float32(127.0)).astype(np.float32)
        r = (blk / sc[:, None]).astype(np.float64)  # exact widening of the FP32 quotient
        r = np.copysign(np.floor(np.abs(r) + 0.5), r)  # std::round: half away from zero
        q[a:a + block] = np.clip(r, -127, 127).astype(np.int8)
        scale[a:a + block] = sc
    return q, scale


def _header_bytes(entries: list[tuple[str, str, tuple[int, ...], int]], metadata: dict | None) -> bytes:
    header: dict = {}
    offset = 0
    for name, dtype, shape, nbytes in entries:
        header[name] = {"data_offsets": [offset, offset + nbytes], "dtype": dtype, "shape": list(shape)}
        offset += nbytes
    if metadata is not None:
        header["__metadata__"] = metadata
    enc = json.dumps(header, sort_keys=True, separators=(",", ":")).encode()
    enc += b" " * (-len(enc) % 8)
    return len(enc).to_bytes(8, "little") + enc


def write_safetensors(path: Path, tensors: list[tuple[str, str, tuple[int, ...], bytes | np.ndarray]],
                      metadata: dict | None = None) -> None:
    """Write tensors in the given order (callers pass them sorted by name)."""
    entries = [(n, dt, sh, (b.nbytes if isinstance(b, np.ndarray) else len(b))) for n, dt, sh, b in tensors]
    tmp = Path(str(path) + ".partial")
    with open(tmp, "wb") as f:
        f.write(_header_bytes(entries, metadata))
        for _, _, _, b in tensors:
            f.write(b.tobytes() if isinstance(b, np.ndarray) else b)
    os.replace(tmp, path)


QUANT_METADATA = {"format": "pt", "quantization": "symmetric-per-row-int8"}


def write_int8_model(directory: Path | str, d: Dims, values) -> Path:
    """Write an int8 model whose FP32 source tensors come from ``values(name, shape)``."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    shapes = tensor_shapes(d)
    out: list = []
    for name in sorted(shapes):
        shape = shapes[name]
        w = np.asarray(values(name, shape), dtype=np.float32).reshape(shape)
        if len(shape) == 2:
            if (shape[0] * shape[1]) % 4:
                raise ValueError("int8 matrices must contain a multiple of four elements")
            q, s = quantize_rows(w)
            out.append((name, "I8", shape, q))
            out.append((name + ".scales", "F32", (shape[0],), s))
        else:
            out.append((name, "F32", shape, w.astype(np.float32)))
    write_safetensors(directory / "model.safetensors", out, QUANT_METADATA)
    (directory / "config.json").write_text(json.dumps(d.config_json()))
    return directory


def write_bf16_model(directory: Path | str, d: Dims, values) -> Path:
    """Write an unquantised BF16 checkpoint (the reference quantiser's input)."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    shapes = tensor_shapes(d)
    out = []
    for name in sorted(shapes):
        w = np.asarray(values(name, shapes[name]), dtype=np.float32).reshape(shapes[name])
        bits = (np.ascontiguousarray(w).view(np.uint32) >> 16).astype(np.uint16)
        out.append((name, "BF16", shapes[name], bits))
    write_safetensors(directory / "model.safetensors", out, None)
    (directory / "config.json").write_text(json.dumps(d.config_json()))
    return directory


def random_values(seed: int):
    """N(0, 0.02) matrices and biases rounded to BF16; norm gains 1.0.

    Each tensor draws from its own generator seeded by (seed, tensor name), so a
    tensor's values do not depend on which other tensors exist."""
    import zlib

    def values(name: str, shape: tuple[int, ...]) -> np.ndarray:
        if is_norm(name):
            return np.ones(shape, dtype=np.float32)
        rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
        x = rng.standard_normal(size=shape, dtype=np.float32) * np.float32(0.02)
        return bf16_round(x)
    return values


def tiny_values():
    """The reference test fixture's values (tests/native.cpp:143-148): norms
    1 + 0.05 sin(j), everything else 0.15 sin(j + 17 k) with k the number of
    tensors added before it, in float, truncated to BF16."""
    libm = ctypes.CDLL("libm.so.6")
    libm.sinf.restype = ctypes.c_float
    libm.sinf.argtypes = [ctypes.c_float]
    order = ["model.embed_tokens.weight", "model.norm.weight",
             "model.layers.0.input_layernorm.weight", "model.layers.0.post_attention_layernorm.weight",
             "model.layers.0.self_attn.q_proj.weight", "model.layers.0.self_attn.q_proj.bias",
             "model.layers.0.self_attn.k_proj.weight", "model.layers.0.self_attn.k_proj.bias",
             "model.layers.0.self_attn.v_proj.weight", "model.layers.0.self_attn.v_proj.bias",
             "model.layers.0.self_attn.o_proj.weight", "model.layers.0.mlp.gate_proj.weight",
             "model.layers.0.mlp.up_proj.weight", "model.layers.0.mlp.down_proj.weight"]
    added = {n: i for i, n in enumerate(order)}

    def values(name: str, shape: tuple[int, ...]) -> np.ndarray:
        n = int(np.prod(shape))
        k = added[name]
        out = np.empty(n, dtype=np.float32)
        for j in range(n):
            if is_norm(name):
                v = np.float32(1) + np.float32(0.05) * np.float32(libm.sinf(float(np.float32(j))))
            else:
                v = np.float32(0.15) * np.float32(libm.sinf(float(np.float32(j + k * 17))))
            out[j] = v
        return bf16_truncate(out)
    return values


def load_safetensors(path: Path | str) -> dict[str, np.ndarray]:
    """Read-only views of every tensor in a safetensors file."""
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    n = int.from_bytes(bytes(raw[:8]), "little")
    header = json.loads(bytes(raw[8:8 + n]))
    origin = 8 + n
    kinds = {"I8": np.int8, "F32": np.float32, "BF16": np.uint16}
    out = {}
    for name, e in header.items():
        if name == "__metadata__":
            continue
        a, b = e["data_offsets"]
        out[name] = raw[origin + a: origin + b].view(kinds[e["dtype"]]).reshape(e["shape"])
    return out


def load_model(directory: Path | str) -> tuple[Dims, dict[str, np.ndarray]]:
    directory = Path(directory)
    c = json.loads((directory / "config.json").read_text())
    d = Dims(hidden=c["hidden_size"], intermediate=c["intermediate_size"], layers=c["num_hidden_layers"],
             heads=c["num_attention_heads"], kv_heads=c["num_key_value_heads"], vocab=c["vocab_size"],
             max_positions=c["max_position_embeddings"], epsilon=float(c["rms_norm_eps"]),
             theta=float(c["rope_theta"]))
    return d, load_safetensors(directory / "model.safetensors")


def ensure_random_model(directory: Path | str, d: Dims = QWEN05, seed: int = 0) -> Path:
    """Create the seeded int8 model once; reuse it when its stamp matches."""
    directory = Path(directory)
    stamp = directory / "synthetic.json"
    want = {"seed": seed, "dims": asdict(d), "format": 1}
    if stamp.exists() and (directory / "model.safetensors").exists():
        try:
            if json.loads(stamp.read_text()) == want:
                return directory
        except ValueError:
            pass
    write_int8_model(directory, d, random_values(seed))
    stamp.write_text(json.dumps(want))
    return directory


def random_tokens(n: int, vocab: int, seed: int) -> list[int]:
    rng = np.random.default_rng([seed, 7])
    return [int(t) for t in rng.integers(0, vocab, size=n)]
