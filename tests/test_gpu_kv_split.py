"""One decode stream with its KV cache split over two GPUs: two processes,
one engine each, KV positions [0, ctx/2) and [ctx/2, ...) of a pre-filled
context; 8 greedy steps through the C ABI. Rank 0 then runs the same steps on
one unsplit engine and compares logits and tokens. Two cases: a 300-position
context (attention units per query head) and a 2304-position one with
head_dim 64 (units per KV group on every rank). Needs two GPUs (skipped
otherwise)."""
from __future__ import annotations

import json
import socket

import numpy as np
import pytest

from conftest import dcb, synthetic, SMALL, G64

pytestmark = pytest.mark.gpu

STEPS = 8
CASES = {"small": (SMALL, 300), "g64": (G64, 2304)}


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


def _kv(d, ctx):
    rng = np.random.default_rng(ctx)
    return [(rng.standard_normal((ctx, d.kv_dim), dtype=np.float32),
             rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)) for _ in range(d.layers)]


def _run(engine, first_token):
    tok, logits = first_token, []
    for _ in range(STEPS):
        lg, tok = engine.step(tok)
        logits.append(lg.copy())
    return np.stack(logits)


def _rank_main(rank: int, world: int, port: int, model: str, out: str, case: str) -> None:
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    d, CTX = CASES[case]
    kv = _kv(d, CTX)
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
@pytest.mark.parametrize("case", ["small", "g64"])
def test_kv_split_over_two_gpus_matches_one_engine(case, small_int8, g64_int8, tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "kv")
    model = small_int8 if case == "small" else g64_int8
    mp.start_processes(_rank_main, args=(2, _free_port(), str(model), out, case), nprocs=2, start_method="spawn")
    split, whole = np.load(out + ".split.npy"), np.load(out + ".whole.npy")
    assert split.shape == (STEPS, CASES[case][0].vocab)
    np.testing.assert_allclose(split, whole, atol=1e-4, rtol=1e-4)
    assert (split.argmax(axis=1) == whole.argmax(axis=1)).all()
