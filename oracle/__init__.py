"""Test infrastructure only: Python access to the CPU checkers.

* ``Oracle`` wraps ``liboracle.so``, the plain-C restatement of the reference's
  decode step (oracle.c), with a caller-owned KV cache.
* ``RefEngine`` / ``ref_*`` wrap ``_ref/libdecode_ref.so``: the reference's own
  ``src/kernels.cpp`` and ``src/model.cpp`` compiled in place, reached through
  the C shim in ref_shim.cpp.

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use this package; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
# The reference checkout whose sources the Makefile compiles into _ref/ (a
# build-time input only; nothing reads it when the tests or the bench run).
REFERENCE_SOURCES = Path(os.environ.get("DCB_REFERENCE", "/root/reference"))
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")


def build(reference: bool = True) -> None:
    """Compile liboracle.so, and the reference binaries when its sources exist."""
    targets = ["oracle"]
    if reference and (REFERENCE_SOURCES / "src" / "model.cpp").exists():
        targets.append("ref")
        if (HERE.parent / "cpu-decode_b200" / "libdecode_b200.so").exists():
            targets.append("dropin")
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF={REFERENCE_SOURCES}", *targets], check=True)


def _lib() -> C.CDLL:
    path = HERE / "liboracle.so"
    if not path.exists():
        build(reference=False)
    lib = C.CDLL(str(path))
    lib.orc_matvec_i8.argtypes = [_i8p, _f32p, C.c_size_t, C.c_size_t, _f32p, _f32p, C.c_int]
    lib.orc_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_size_t, C.c_float]
    lib.orc_inverse_frequency.argtypes = [_f32p, C.c_size_t, C.c_float]
    lib.orc_rope_direct.argtypes = [_f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float]
    lib.orc_rope_cached.argtypes = [_f32p, C.c_size_t, C.c_size_t, C.c_size_t, _f32p]
    lib.orc_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, C.c_size_t, C.c_size_t,
                                  C.c_size_t, C.c_size_t, C.c_int]
    lib.orc_argmax.argtypes = [_f32p, C.c_size_t]
    lib.orc_argmax.restype = C.c_int
    lib.orc_f16_round_array.argtypes = [_f32p, C.c_size_t]
    lib.orc_silu_mul.argtypes = [_f32p, _f32p, C.c_size_t]
    lib.orc_quantize_row.argtypes = [_f32p, C.c_size_t, _i8p, C.POINTER(C.c_float)]
    lib.orc_step.argtypes = [C.c_void_p, _f32p, _f32p, C.c_size_t, C.c_int, C.c_size_t, C.c_int,
                             C.c_int, C.c_int, _f32p, C.c_int]
    return lib


_LIB = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = _lib()
    return _LIB


class _Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "q", "k", "v", "o", "gate", "up", "down",
        "q_scales", "k_scales", "v_scales", "o_scales", "gate_scales", "up_scales", "down_scales",
        "input_norm", "post_norm", "q_bias", "k_bias", "v_bias")]


class _Model(C.Structure):
    _fields_ = [("hidden", C.c_size_t), ("intermediate", C.c_size_t), ("layers", C.c_size_t),
                ("heads", C.c_size_t), ("kv_heads", C.c_size_t), ("dim", C.c_size_t),
                ("vocab", C.c_size_t), ("epsilon", C.c_float), ("theta", C.c_float),
                ("embed", C.c_void_p), ("embed_scales", C.c_void_p), ("final_norm", C.c_void_p),
                ("layer", C.POINTER(_Layer))]


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ---- free functions (restatement) ------------------------------------------------
def matvec(w: np.ndarray, scales: np.ndarray, x: np.ndarray, threads: int = 1) -> np.ndarray:
    w = np.ascontiguousarray(w, np.int8)
    y = np.zeros(w.shape[0], np.float32)
    lib().orc_matvec_i8(w, np.ascontiguousarray(scales, np.float32), w.shape[0], w.shape[1],
                        np.ascontiguousarray(x, np.float32), y, threads)
    return y


def rmsnorm(x, w, eps: float) -> np.ndarray:
    out = np.zeros(len(x), np.float32)
    lib().orc_rmsnorm(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w, np.float32), out, len(x), eps)
    return out


def inverse_frequency(dim: int, theta: float) -> np.ndarray:
    inv = np.zeros(dim // 2, np.float32)
    lib().orc_inverse_frequency(inv, dim, theta)
    return inv


def rope_cached(x: np.ndarray, heads: int, dim: int, pos: int, theta: float) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    lib().orc_rope_cached(x, heads, dim, pos, inverse_frequency(dim, theta))
    return x


def rope_direct(x: np.ndarray, heads: int, dim: int, pos: int, theta: float) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    lib().orc_rope_direct(x, heads, dim, pos, theta)
    return x


def attention(q, keys, values, length: int, heads: int, kv_heads: int, dim: int, threads: int = 1) -> np.ndarray:
    out = np.zeros(heads * dim, np.float32)
    scores = np.zeros(heads * length, np.float32)
    rc = lib().orc_attention(np.ascontiguousarray(q, np.float32), np.ascontiguousarray(keys, np.float32),
                             np.ascontiguousarray(values, np.float32), out, scores, length, heads,
                             kv_heads, dim, threads)
    if rc:
        raise RuntimeError("invalid attention dimensions")
    return out


def argmax(x: np.ndarray) -> int:
    return int(lib().orc_argmax(np.ascontiguousarray(x, np.float32), len(x)))


def f16_round(x: np.ndarray) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    lib().orc_f16_round_array(x, x.size)
    return x


def _synthetic():
    """The model-format module of the product package (file I/O only)."""
    import importlib.util
    import sys
    if "cpu_decode_b200.synthetic" in sys.modules:
        return sys.modules["cpu_decode_b200.synthetic"]
    path = Path(__file__).resolve().parent.parent / "cpu-decode_b200" / "synthetic.py"
    spec = importlib.util.spec_from_file_location("_oracle_synthetic", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["_oracle_synthetic"] = mod
    spec.loader.exec_module(mod)
    return mod


# ---- full step ------------------------------------------------------------------
class Oracle:
    """The restated decode step over a model directory and an owned KV cache."""

    def __init__(self, directory, capacity: int, kv_f16: bool = False, cached_rope: bool = True,
                 threads: int = 1):
        self.dims, self.t = _synthetic().load_model(directory)
        d = self.dims
        self.capacity, self.kv_f16, self.cached_rope, self.threads = capacity, kv_f16, cached_rope, threads
        kvd = d.kv_dim
        self.kcache = np.zeros(d.layers * capacity * kvd, np.float32)
        self.vcache = np.zeros(d.layers * capacity * kvd, np.float32)
        self.logits = np.zeros(d.vocab, np.float32)
        self.pos = 0
        t = self.t
        self._keep = []

        def f(name):
            a = np.ascontiguousarray(t[name])
            self._keep.append(a)
            return _ptr(a)
        layers = (_Layer * d.layers)()
        for l in range(d.layers):
            b = f"model.layers.{l}."
            L = layers[l]
            for fld, nm in (("q", "self_attn.q_proj"), ("k", "self_attn.k_proj"), ("v", "self_attn.v_proj"),
                            ("o", "self_attn.o_proj"), ("gate", "mlp.gate_proj"), ("up", "mlp.up_proj"),
                            ("down", "mlp.down_proj")):
                setattr(L, fld, f(b + nm + ".weight"))
                setattr(L, fld + "_scales", f(b + nm + ".weight.scales"))
            L.input_norm = f(b + "input_layernorm.weight")
            L.post_norm = f(b + "post_attention_layernorm.weight")
            L.q_bias = f(b + "self_attn.q_proj.bias")
            L.k_bias = f(b + "self_attn.k_proj.bias")
            L.v_bias = f(b + "self_attn.v_proj.bias")
        self._layers = layers
        self.model = _Model(d.hidden, d.intermediate, d.layers, d.heads, d.kv_heads, d.head_dim, d.vocab,
                            d.epsilon, d.theta, f("model.embed_tokens.weight"),
                            f("model.embed_tokens.weight.scales"), f("model.norm.weight"), layers)

    def step(self, token: int, head: bool = True) -> np.ndarray:
        rc = lib().orc_step(C.addressof(self.model), self.kcache, self.vcache, self.capacity,
                            int(self.kv_f16), self.pos, token, int(head), int(self.cached_rope),
                            self.logits, self.threads)
        if rc == 2:
            raise RuntimeError("token ID outside vocabulary")
        if rc == 3:
            raise RuntimeError("context capacity exceeded")
        if rc:
            raise RuntimeError(f"oracle step failed ({rc})")
        self.pos += 1
        return self.logits

    def rewind(self, pos: int) -> None:
        if pos > self.pos:
            raise RuntimeError("cannot rewind forward")
        self.pos = pos

    def kv_view(self):
        d = self.dims
        shape = (d.layers, self.capacity, d.kv_dim)
        return self.kcache.reshape(shape), self.vcache.reshape(shape)


# ---- the reference itself, built from its sources --------------------------------
def ref_available() -> bool:
    return (REF_DIR / "libdecode_ref.so").exists()


_REF = None


def ref_lib() -> C.CDLL:
    global _REF
    if _REF is None:
        lib = C.CDLL(str(REF_DIR / "libdecode_ref.so"))
        lib.ref_last_error.restype = C.c_char_p
        lib.ref_matvec.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_int, _f32p, _f32p,
                                   C.c_int, C.c_int]
        lib.ref_quantize_row.argtypes = [_f32p, C.c_size_t, _i8p, C.POINTER(C.c_float)]
        lib.ref_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_size_t, C.c_float]
        lib.ref_rope.argtypes = [_f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float]
        lib.ref_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, C.c_size_t, C.c_size_t, C.c_size_t,
                                      C.c_size_t, C.c_int]
        lib.ref_quantize_model.argtypes = [C.c_char_p, C.c_char_p]
        lib.ref_engine_create.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_size_t, C.c_int,
                                          C.POINTER(C.c_void_p)]
        lib.ref_engine_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t]
        lib.ref_engine_step_profiled.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                                                 C.POINTER(C.c_ulonglong)]
        lib.ref_engine_rewind.argtypes = [C.c_void_p, C.c_size_t]
        lib.ref_engine_reset.argtypes = [C.c_void_p]
        lib.ref_engine_position.argtypes = [C.c_void_p]
        lib.ref_engine_position.restype = C.c_size_t
        lib.ref_engine_destroy.argtypes = [C.c_void_p]
        _REF = lib
    return _REF


def _check(rc: int) -> None:
    if rc:
        raise RuntimeError(ref_lib().ref_last_error().decode())


KERNELS = {"scalar": 0, "simd256": 1, "simd512": 2, "simd512x4": 3}
PROFILE_KEYS = ("matrix_weight_bytes", "scale_bytes", "norm_bias_bytes", "embedding_bytes", "kv_write_bytes",
                "kv_read_min_bytes", "kv_read_logical_bytes", "lm_head_weight_bytes", "lm_head_scale_bytes",
                "steps", "head_steps")


class RefEngine:
    """``decode::Engine`` of the reference, in-process."""

    def __init__(self, directory, capacity: int, kernel: str = "scalar", threads: int = 1,
                 cached_rope: bool = True, vocab: int | None = None):
        h = C.c_void_p()
        _check(ref_lib().ref_engine_create(str(directory).encode(), KERNELS[kernel], threads, capacity,
                                           int(cached_rope), C.byref(h)))
        self.h = h
        if vocab is None:
            import json
            vocab = json.loads((Path(directory) / "config.json").read_text())["vocab_size"]
        self.logits = np.zeros(vocab, np.float32)

    def step(self, token: int, head: bool = True) -> np.ndarray:
        _check(ref_lib().ref_engine_step(self.h, token, int(head), self.logits.ctypes.data, len(self.logits)))
        return self.logits

    def step_profiled(self, token: int, head: bool = True):
        c = (C.c_ulonglong * 11)()
        _check(ref_lib().ref_engine_step_profiled(self.h, token, int(head), self.logits.ctypes.data,
                                                  len(self.logits), c))
        return self.logits, dict(zip(PROFILE_KEYS, list(c)))

    def rewind(self, pos: int) -> None:
        _check(ref_lib().ref_engine_rewind(self.h, pos))

    def reset(self) -> None:
        _check(ref_lib().ref_engine_reset(self.h))

    @property
    def position(self) -> int:
        return int(ref_lib().ref_engine_position(self.h))

    def close(self) -> None:
        if self.h:
            ref_lib().ref_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ref_matvec(w: np.ndarray, scales: np.ndarray, x: np.ndarray, kernel: str = "scalar", threads: int = 1):
    w = np.ascontiguousarray(w, np.int8)
    s = np.ascontiguousarray(scales, np.float32)
    y = np.zeros(w.shape[0], np.float32)
    _check(ref_lib().ref_matvec(w.ctypes.data, s.ctypes.data, w.shape[0], w.shape[1], 2,
                                np.ascontiguousarray(x, np.float32), y, KERNELS[kernel], threads))
    return y


def ref_attention(q, keys, values, length, heads, kv_heads, dim, threads: int = 1):
    out = np.zeros(heads * dim, np.float32)
    scores = np.zeros(heads * length, np.float32)
    _check(ref_lib().ref_attention(np.ascontiguousarray(q, np.float32), np.ascontiguousarray(keys, np.float32),
                                   np.ascontiguousarray(values, np.float32), out, scores, length, heads, kv_heads,
                                   dim, threads))
    return out


def ref_quantize_model(src, dst) -> None:
    _check(ref_lib().ref_quantize_model(str(src).encode(), str(dst).encode()))
