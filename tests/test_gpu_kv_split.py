"""One decode stream with its KV cache split over two GPUs: two processes,
one engine each, KV positions [0, 150) and [150, ...) of a 300-position
pre-filled context; 8 greedy steps through the C ABI. Rank 0 then runs the
same steps on one unsplit engine and compares logits and tokens. Needs two
GPUs (skipped otherwise)."""
from __future__ import annotations

import json
import socket

import numpy as np
import pytest

from conftest import dcb, synthetic, SMALL

pytestmark = pytest.mark.gpu

CTX, STEPS = 300, 8


def _gpu_count() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _kv(d):
    rng = np.random.default_rng(300)
    return [(rng.standard_normal((CTX, d.kv_dim), dtype=np.float32),
             rng.standard_normal((CTX, d.kv_dim), dtype=np.float32)) for _ in range(d.layers)]


def _run(engine, first_token):
    tok, logits = first_token, []
    for _ in range(STEPS):
        lg, tok = engine.step(tok)
        logits.append(lg.copy())
    return np.stack(logits)


def _rank_main(rank: int, world: int, port: int, model: str, out: str) -> None:
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    d = SMALL
    kv = _kv(d)
    begin, end = dcb.kv_shard_ranges(CTX, world)[rank]
    cap = (end if end is not None else CTX + STEPS + 2) - begin
    eng = dcb.Engine(model, cap, device=rank)
    peers = dcb.split_kv(eng, begin, end)
    for l, (k, v) in enumerate(kv):
        top = CTX if end is None else end
        eng.kv_write(l, begin, k[begin:top], v[begin:top])
    eng.set_position(CTX)
    dist.barrier()
    split = _run(eng, 7)
    dist.barrier()
    eng.close()
    for p in peers:
        dcb.ipc_close(p)
    if rank == 0:
        ref = dcb.Engine(model, CTX + STEPS + 2, device=0)
        for l, (k, v) in enumerate(kv):
            ref.kv_write(l, 0, k, v)
        ref.set_position(CTX)
        whole = _run(ref, 7)
        ref.close()
        np.save(out + ".split.npy", split)
        np.save(out + ".whole.npy", whole)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_kv_split_over_two_gpus_matches_one_engine(small_int8, tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "kv")
    mp.start_processes(_rank_main, args=(2, _free_port(), str(small_int8), out), nprocs=2, start_method="spawn")
    split, whole = np.load(out + ".split.npy"), np.load(out + ".whole.npy")
    assert split.shape == (STEPS, SMALL.vocab)
    np.testing.assert_allclose(split, whole, atol=1e-4, rtol=1e-4)
    assert (split.argmax(axis=1) == whole.argmax(axis=1)).all()
