"""Python access to the B200 decode engine (libdecode_b200.so) through its C ABI.

The engine is the reference's ``decode::Engine`` (include/decode.hpp:41-58 of
mottopanikeiku/cpu-decode) rebuilt on sm_100a: ``Engine(directory, capacity)``
loads the per-row int8 safetensors model, ``step(token, head)`` runs one token
and returns the logits, ``rewind``/``reset``/``position`` keep the reference's
cache semantics. Isolated operators (int8 GEMV, split-KV attention, RMSNorm,
RoPE, argmax) take device pointers, e.g. ``tensor.data_ptr()`` of CUDA tensors.

There is no CPU path: importing works anywhere, but every call loads the CUDA
library and fails loudly when it is missing or no GPU is present.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libdecode_b200.so"

KV_F32, KV_F16 = 0, 1
KV_DTYPES = {"f32": KV_F32, "f16": KV_F16}

ERRORS = {1: ValueError, 2: ValueError, 3: RuntimeError, 4: RuntimeError, 5: RuntimeError, 6: TimeoutError,
          7: NotImplementedError}

# Every symbol include/decode_b200.h declares.
EXPORTS = (
    "dcb_last_error", "dcb_set_error", "dcb_create", "dcb_create_from_dir", "dcb_destroy", "dcb_step",
    "dcb_step_async", "dcb_synchronize", "dcb_rewind", "dcb_reset", "dcb_position", "dcb_set_stream", "dcb_stream",
    "dcb_logits_device", "dcb_kv_write", "dcb_kv_read", "dcb_set_position", "dcb_launch_info", "dcb_launch_count",
    "dcb_gemv_i8", "dcb_attention", "dcb_attention_noalloc", "dcb_rmsnorm", "dcb_rope", "dcb_argmax",
    "dcb_read_bandwidth", "dcb_quantize_rows_bf16", "dcb_quantize_model",
    "dcb_trace_enable", "dcb_trace_read", "dcb_exchange_buffer", "dcb_ipc_handle", "dcb_ipc_open", "dcb_ipc_close",
    "dcb_set_kv_shard", "dcb_batch_create", "dcb_batch_destroy", "dcb_batch_info", "dcb_batch_set_position",
    "dcb_batch_position", "dcb_batch_kv_write", "dcb_batch_kv_read", "dcb_batch_step", "dcb_batch_step_greedy", "dcb_prefill", "dcb_prefill_logits",
    "dcb_batch_read", "dcb_batch_stream", "dcb_batch_kernels_per_step",
)


def build(force: bool = False) -> Path:
    """Compile libdecode_b200.so in-tree for sm_100a (nvcc cross-compiles without a GPU)."""
    if force or not LIB_PATH.exists():
        subprocess.run(["make", "-s", "-C", str(HERE), "-j4"], check=True)
    return LIB_PATH


_LIB: C.CDLL | None = None


def lib() -> C.CDLL:
    """The loaded CUDA library. Raises when it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH.name} is not built; run `make -C {HERE}` (needs nvcc)")
    L = C.CDLL(str(LIB_PATH))
    vp, sz, i32 = C.c_void_p, C.c_size_t, C.c_int
    L.dcb_last_error.restype = C.c_char_p
    L.dcb_set_error.argtypes = [C.c_char_p]
    L.dcb_create_from_dir.argtypes = [C.c_char_p, sz, i32, i32, i32, C.POINTER(vp)]
    L.dcb_destroy.argtypes = [vp]
    L.dcb_step.argtypes = [vp, i32, i32, vp, vp]
    L.dcb_step_async.argtypes = [vp, i32, vp, i32, vp]
    L.dcb_synchronize.argtypes = [vp]
    L.dcb_rewind.argtypes = [vp, sz]
    L.dcb_reset.argtypes = [vp]
    L.dcb_position.argtypes = [vp]
    L.dcb_position.restype = sz
    L.dcb_set_stream.argtypes = [vp, vp]
    L.dcb_stream.argtypes = [vp]
    L.dcb_stream.restype = vp
    L.dcb_logits_device.argtypes = [vp]
    L.dcb_logits_device.restype = vp
    L.dcb_kv_write.argtypes = [vp, i32, sz, sz, vp, vp]
    L.dcb_kv_read.argtypes = [vp, i32, sz, sz, vp, vp]
    L.dcb_set_position.argtypes = [vp, sz]
    L.dcb_launch_info.argtypes = [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32), C.POINTER(i32)]
    L.dcb_launch_count.argtypes = [vp]
    L.dcb_launch_count.restype = C.c_uint64
    L.dcb_gemv_i8.argtypes = [vp, vp, vp, vp, vp, i32, i32, vp]
    L.dcb_attention.argtypes = [vp, vp, vp, i32, vp, i32, i32, i32, i32, C.c_float, vp]
    L.dcb_attention_noalloc.argtypes = [vp, vp, vp, i32, vp, i32, i32, i32, i32, C.c_float, vp]
    L.dcb_rmsnorm.argtypes = [vp, vp, vp, i32, C.c_float, vp]
    L.dcb_rope.argtypes = [vp, i32, i32, i32, C.c_float, i32, vp]
    L.dcb_argmax.argtypes = [vp, i32, vp, vp]
    L.dcb_read_bandwidth.argtypes = [i32, C.c_size_t, i32, i32, C.POINTER(C.c_double), C.POINTER(C.c_uint64)]
    L.dcb_quantize_rows_bf16.argtypes = [vp, C.c_size_t, C.c_size_t, vp, vp, i32]
    L.dcb_quantize_model.argtypes = [C.c_char_p, C.c_char_p, i32]
    L.dcb_trace_enable.argtypes = [vp, i32]
    L.dcb_trace_read.argtypes = [vp, vp, vp, C.POINTER(i32)]
    L.dcb_exchange_buffer.argtypes = [vp, C.POINTER(vp), C.POINTER(sz)]
    L.dcb_ipc_handle.argtypes = [vp, vp]
    L.dcb_ipc_open.argtypes = [vp, C.POINTER(vp)]
    L.dcb_ipc_close.argtypes = [vp]
    L.dcb_set_kv_shard.argtypes = [vp, i32, i32, sz, sz, vp]
    L.dcb_batch_create.argtypes = [vp, i32, sz, i32, C.POINTER(vp)]
    L.dcb_batch_destroy.argtypes = [vp]
    L.dcb_batch_info.argtypes = [vp, C.POINTER(i32), C.POINTER(sz), C.POINTER(i32)]
    L.dcb_batch_set_position.argtypes = [vp, i32, sz]
    L.dcb_batch_position.argtypes = [vp, i32]
    L.dcb_batch_position.restype = sz
    L.dcb_batch_kv_write.argtypes = [vp, i32, i32, sz, sz, vp, vp]
    L.dcb_batch_kv_read.argtypes = [vp, i32, i32, sz, sz, vp, vp]
    L.dcb_batch_step.argtypes = [vp, i32, vp, vp, vp]
    L.dcb_prefill.argtypes = [vp, vp, i32, vp, vp]
    L.dcb_prefill_logits.argtypes = [vp, vp, i32, vp, vp]
    L.dcb_batch_step_greedy.argtypes = [vp, i32, i32]
    L.dcb_batch_read.argtypes = [vp, i32, vp, vp]
    L.dcb_batch_stream.argtypes = [vp]
    L.dcb_batch_stream.restype = vp
    L.dcb_batch_kernels_per_step.argtypes = [vp, i32]
    L.dcb_batch_kernels_per_step.restype = C.c_uint64
    _LIB = L
    return L


def _check(rc: int) -> None:
    if rc:
        msg = lib().dcb_last_error().decode()
        raise ERRORS.get(rc, RuntimeError)(msg)


class Engine:
    """One model on one GPU with its own KV cache (the reference's Engine)."""

    def __init__(self, directory, capacity: int, kv_dtype: str = "f32", cached_rope: bool = True, device: int = 0):
        h = C.c_void_p()
        _check(lib().dcb_create_from_dir(str(directory).encode(), int(capacity), KV_DTYPES[kv_dtype],
                                         int(bool(cached_rope)), int(device), C.byref(h)))
        self._h = h
        import json
        cfg = json.loads((Path(directory) / "config.json").read_text())
        self.vocab = int(cfg["vocab_size"])
        self.layers = int(cfg["num_hidden_layers"])
        self.kv_dim = int(cfg["num_key_value_heads"]) * (int(cfg["hidden_size"]) // int(cfg["num_attention_heads"]))
        self.capacity = int(capacity)
        self.logits = np.zeros(self.vocab, np.float32)
        self._argmax = C.c_int(0)

    # -- the reference API -------------------------------------------------------
    def step(self, token: int, head: bool = True, logits: bool = True):
        """Run one token. Returns (logits or None, argmax or None)."""
        want = head and logits
        _check(lib().dcb_step(self._h, int(token), int(bool(head)),
                              self.logits.ctypes.data if want else None,
                              C.addressof(self._argmax) if head else None))
        return (self.logits if want else None), (int(self._argmax.value) if head else None)

    def prefill(self, tokens, logits: bool = True):
        """All prompt tokens in batched form (dcb_prefill): the engine ends at
        position + len(tokens) with their K/V rows written. Returns (the last
        token's logits or None, its argmax)."""
        t = np.ascontiguousarray(tokens, np.int32)
        _check(lib().dcb_prefill(self._h, t.ctypes.data, int(t.shape[0]),
                                 self.logits.ctypes.data if logits else None, C.addressof(self._argmax)))
        return (self.logits if logits else None), int(self._argmax.value)

    def prefill_logits(self, tokens):
        """Prefill with every position's logits (dcb_prefill_logits): returns
        (logits [n][vocab], argmax [n])."""
        t = np.ascontiguousarray(tokens, np.int32)
        n = int(t.shape[0])
        out = np.zeros((n, self.vocab), np.float32)
        best = np.zeros(n, np.int32)
        _check(lib().dcb_prefill_logits(self._h, t.ctypes.data, n, out.ctypes.data, best.ctypes.data))
        return out, best

    def rewind(self, position: int) -> None:
        _check(lib().dcb_rewind(self._h, int(position)))

    def reset(self) -> None:
        _check(lib().dcb_reset(self._h))

    @property
    def position(self) -> int:
        return int(lib().dcb_position(self._h))

    # -- device-resident stepping --------------------------------------------------
    def step_async(self, token: int = 0, token_dev: int | None = None, head: bool = True,
                   argmax_dev: int | None = None) -> None:
        _check(lib().dcb_step_async(self._h, int(token), token_dev, int(bool(head)), argmax_dev))

    def synchronize(self) -> None:
        _check(lib().dcb_synchronize(self._h))

    def set_stream(self, stream_handle: int | None) -> None:
        _check(lib().dcb_set_stream(self._h, stream_handle))

    @property
    def stream(self) -> int:
        return int(lib().dcb_stream(self._h) or 0)

    @property
    def logits_device(self) -> int:
        return int(lib().dcb_logits_device(self._h))

    def set_position(self, position: int) -> None:
        _check(lib().dcb_set_position(self._h, int(position)))

    def kv_write(self, layer: int, start: int, keys: np.ndarray, values: np.ndarray) -> None:
        k = np.ascontiguousarray(keys, np.float32).reshape(-1, self.kv_dim)
        v = np.ascontiguousarray(values, np.float32).reshape(-1, self.kv_dim)
        assert k.shape == v.shape
        _check(lib().dcb_kv_write(self._h, int(layer), int(start), k.shape[0], k.ctypes.data, v.ctypes.data))

    def kv_read(self, layer: int, start: int, count: int):
        k = np.zeros((count, self.kv_dim), np.float32)
        v = np.zeros((count, self.kv_dim), np.float32)
        _check(lib().dcb_kv_read(self._h, int(layer), int(start), int(count), k.ctypes.data, v.ctypes.data))
        return k, v

    def launch_info(self) -> dict:
        b, t, s, m = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        _check(lib().dcb_launch_info(self._h, C.byref(b), C.byref(t), C.byref(s), C.byref(m)))
        return {"blocks": b.value, "threads": t.value, "smem_bytes": s.value, "sms": m.value}

    def trace(self, on: bool = True) -> None:
        _check(lib().dcb_trace_enable(self._h, int(bool(on))))

    def trace_read(self) -> dict:
        """Per-phase timing of the last step, in microseconds from the kernel
        start: for each phase, when the last block finished it (`done`), and over
        the blocks that had work in it, the mean and max of ready->done."""
        blocks = self.launch_info()["blocks"]
        n = C.c_int()
        ready = np.zeros(512 * blocks, np.uint64)
        done = np.zeros(512 * blocks, np.uint64)
        _check(lib().dcb_trace_read(self._h, ready.ctypes.data, done.ctypes.data, C.byref(n)))
        k = n.value
        ready = ready[:k * blocks].reshape(k, blocks).astype(np.int64)
        done = done[:k * blocks].reshape(k, blocks).astype(np.int64)
        t0 = done[0].min()
        last_done = (done.max(axis=1) - t0) / 1000.0
        work = np.where(ready > 0, done - ready, 0) / 1000.0
        busy = (ready > 0).sum(axis=1)
        mean_work = np.where(busy > 0, work.sum(axis=1) / np.maximum(busy, 1), 0.0)
        first_ready = np.where(busy > 0, (np.where(ready > 0, ready, np.iinfo(np.int64).max).min(axis=1) - t0) / 1000.0, 0.0)
        last_ready = np.where(busy > 0, (ready.max(axis=1) - t0) / 1000.0, 0.0)
        return {"phases": k, "done_us": last_done, "mean_work_us": mean_work, "max_work_us": work.max(axis=1),
                "busy_blocks": busy, "first_ready_us": first_ready, "last_ready_us": last_ready}

    @property
    def launch_count(self) -> int:
        return int(lib().dcb_launch_count(self._h))

    def exchange_buffer(self) -> int:
        """Device pointer of the buffer peers write this engine's share of a
        KV-split attention into."""
        ptr, size = C.c_void_p(), C.c_size_t()
        _check(lib().dcb_exchange_buffer(self._h, C.byref(ptr), C.byref(size)))
        return int(ptr.value)

    def set_kv_shard(self, rank: int, world: int, begin: int, end: int | None, peers: list[int]) -> None:
        """Keep KV positions [begin, end) (end None: open) as rank `rank` of
        `world` engines; peers[q] is rank q's exchange buffer opened here."""
        arr = (C.c_void_p * max(1, world))(*[C.c_void_p(int(p) or None) for p in peers])
        _check(lib().dcb_set_kv_shard(self._h, int(rank), int(world), int(begin),
                                      SIZE_MAX if end is None else int(end), arr))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().dcb_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Batch:
    """Up to 64 independent sequences stepping together on one GPU, sharing
    `model`'s weights; sequence s has its own KV cache and position. The
    reference has no batch API: per sequence this is Engine.step."""

    def __init__(self, model: Engine, max_seqs: int, capacity: int, kv_dtype: str = "f32"):
        self.model = model  # the weights stay alive with the batch
        h = C.c_void_p()
        _check(lib().dcb_batch_create(model._h, int(max_seqs), int(capacity), KV_DTYPES[kv_dtype], C.byref(h)))
        self._h = h
        slots, cap, split = C.c_int(), C.c_size_t(), C.c_int()
        _check(lib().dcb_batch_info(h, C.byref(slots), C.byref(cap), C.byref(split)))
        self.slots, self.capacity, self.split_len = slots.value, cap.value, split.value
        self.vocab, self.layers, self.kv_dim = model.vocab, model.layers, model.kv_dim
        self._argmax = np.zeros(self.slots, np.int32)

    def set_position(self, seq: int, position: int) -> None:
        _check(lib().dcb_batch_set_position(self._h, int(seq), int(position)))

    def position(self, seq: int) -> int:
        return int(lib().dcb_batch_position(self._h, int(seq)))

    def kv_write(self, seq: int, layer: int, start: int, keys, values, count: int | None = None) -> None:
        """Rows [start, start+count) of `layer`: numpy float32 [count][kv_dim],
        or device pointers (ints) with `count` given."""
        if isinstance(keys, int):
            _check(lib().dcb_batch_kv_write(self._h, int(seq), int(layer), int(start), int(count), keys, values))
            return
        k = np.ascontiguousarray(keys, np.float32)
        v = np.ascontiguousarray(values, np.float32)
        _check(lib().dcb_batch_kv_write(self._h, int(seq), int(layer), int(start), k.shape[0],
                                        k.ctypes.data, v.ctypes.data))

    def kv_read(self, seq: int, layer: int, start: int, count: int):
        k = np.zeros((count, self.kv_dim), np.float32)
        v = np.zeros((count, self.kv_dim), np.float32)
        _check(lib().dcb_batch_kv_read(self._h, int(seq), int(layer), int(start), int(count),
                                       k.ctypes.data, v.ctypes.data))
        return k, v

    def step(self, tokens=None, n: int | None = None, logits: bool = True):
        """One step of sequences 0..n-1 (n = len(tokens)); tokens None: each
        sequence's previous argmax. Returns (logits [n][vocab] or None, argmax [n])."""
        if tokens is not None:
            t = np.ascontiguousarray(tokens, np.int32)
            n = t.shape[0]
        if n is None:
            raise ValueError("n is needed without tokens")
        out = np.zeros((n, self.vocab), np.float32) if logits else None
        _check(lib().dcb_batch_step(self._h, int(n), t.ctypes.data if tokens is not None else None,
                                    out.ctypes.data if logits else None, self._argmax.ctypes.data))
        return out, self._argmax[:n].copy()

    def step_greedy(self, n: int, steps: int) -> None:
        _check(lib().dcb_batch_step_greedy(self._h, int(n), int(steps)))

    def read(self, n: int, logits: bool = False):
        toks = np.zeros(n, np.int32)
        out = np.zeros((n, self.vocab), np.float32) if logits else None
        _check(lib().dcb_batch_read(self._h, int(n), toks.ctypes.data, out.ctypes.data if logits else None))
        return toks, out

    @property
    def stream(self) -> int:
        return int(lib().dcb_batch_stream(self._h) or 0)

    def kernels_per_step(self, n: int) -> int:
        return int(lib().dcb_batch_kernels_per_step(self._h, int(n)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().dcb_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- one stream over several GPUs (KV sequence split) -------------------------------
SIZE_MAX = (1 << 64) - 1
IPC_HANDLE_BYTES = 64


def ipc_handle(device_ptr: int) -> bytes:
    buf = C.create_string_buffer(IPC_HANDLE_BYTES)
    _check(lib().dcb_ipc_handle(device_ptr, buf))
    return buf.raw


def ipc_open(handle: bytes) -> int:
    ptr = C.c_void_p()
    buf = C.create_string_buffer(bytes(handle), IPC_HANDLE_BYTES)
    _check(lib().dcb_ipc_open(buf, C.byref(ptr)))
    return int(ptr.value)


def ipc_close(device_ptr: int) -> None:
    _check(lib().dcb_ipc_close(device_ptr))


def kv_shard_ranges(total: int, world: int) -> list[tuple[int, int | None]]:
    """Contiguous KV ranges of `total` cached positions over `world` engines;
    the last range is open (it also keeps the positions generated later)."""
    bounds = [total * r // world for r in range(world + 1)]
    return [(bounds[r], bounds[r + 1] if r + 1 < world else None) for r in range(world)]


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """All ranks' IPC handles, indexed by rank (torch.distributed plumbing)."""
    import torch.distributed as dist
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    return [bytes(h) for h in out]


def split_kv(engine: "Engine", begin: int, end: int | None, group=None) -> list[int]:
    """Join the engines of all ranks of `group` into one KV-split stream: this
    rank keeps [begin, end). Returns the peer buffers opened here (close them
    with ipc_close after the engines are done)."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    handles = exchange_handles(ipc_handle(engine.exchange_buffer()), group)
    peers = [0 if q == rank else ipc_open(h) for q, h in enumerate(handles)]
    engine.set_kv_shard(rank, world, begin, end, peers)
    return [p for p in peers if p]


# ---- isolated operators on device pointers ------------------------------------------
def gemv_i8(w: int, scales: int, bias: int | None, x: int, y: int, rows: int, cols: int, stream: int | None = None):
    _check(lib().dcb_gemv_i8(w, scales, bias, x, y, rows, cols, stream))


def attention(q: int, keys: int, values: int, kv_dtype: str, out: int, length: int, heads: int, kv_heads: int,
              dim: int, rope_theta: float = 0.0, stream: int | None = None):
    _check(lib().dcb_attention(q, keys, values, KV_DTYPES[kv_dtype], out, length, heads, kv_heads, dim,
                               float(rope_theta), stream))


def rmsnorm(x: int, w: int, out: int, n: int, eps: float, stream: int | None = None):
    _check(lib().dcb_rmsnorm(x, w, out, n, float(eps), stream))


def rope(x: int, heads: int, dim: int, pos: int, theta: float, direct: bool, stream: int | None = None):
    _check(lib().dcb_rope(x, heads, dim, pos, float(theta), int(bool(direct)), stream))


def argmax(x: int, n: int, out: int, stream: int | None = None):
    _check(lib().dcb_argmax(x, n, out, stream))


def quantize_model(source, output, device: int = 0) -> None:
    """BF16 checkpoint directory -> per-row int8 checkpoint, the per-row rule
    on the GPU (dcb_quantize_model): the reference quantiser's file byte for byte."""
    _check(lib().dcb_quantize_model(str(source).encode(), str(output).encode(), int(device)))


def quantize_rows_bf16(weights: np.ndarray, device: int = 0):
    """One BF16 matrix (uint16 bits, rows x cols) -> (int8 rows, float32 scales) on the GPU."""
    w = np.ascontiguousarray(weights, np.uint16)
    rows, cols = w.shape
    q = np.zeros((rows, cols), np.int8)
    sc = np.zeros(rows, np.float32)
    _check(lib().dcb_quantize_rows_bf16(w.ctypes.data, rows, cols, q.ctypes.data, sc.ctypes.data, int(device)))
    return q, sc


def read_bandwidth(mib: int = 1024, passes: int = 8, repeats: int = 5, device: int = 0) -> dict:
    """HBM read bandwidth of `device` from a read-only sweep of an mib-MiB array
    (the reference's tools/bandwidth.cpp, on the GPU), in the reference's record
    format: {"kind": "read_bandwidth", ..., "samples": [{"seconds", "GB_per_s"}],
    "checksum"}."""
    gbs = (C.c_double * repeats)()
    cs = C.c_uint64()
    _check(lib().dcb_read_bandwidth(int(device), int(mib), int(passes), int(repeats), gbs, C.byref(cs)))
    nbytes = int(mib) << 20
    return {"kind": "read_bandwidth", "kernel": "ld.global.nc.v4", "device": int(device), "array_bytes": nbytes,
            "passes": int(passes),
            "samples": [{"seconds": nbytes * passes / (g * 1e9), "GB_per_s": g} for g in gbs],
            "checksum": int(cs.value)}
