"""Host side of the KV-sequence split over GPUs, on CPU: the position ranges
and the exchange of IPC handles between two gloo ranks."""
from __future__ import annotations

import os
import socket

import pytest

from conftest import dcb


def test_kv_shard_ranges_cover_every_position_once():
    for total, world in [(32768, 2), (32768, 8), (300, 3), (7, 7)]:
        ranges = dcb.kv_shard_ranges(total, world)
        assert len(ranges) == world and ranges[0][0] == 0 and ranges[-1][1] is None
        for (b0, e0), (b1, _) in zip(ranges, ranges[1:]):
            assert e0 == b1 and b0 < e0
        assert ranges[-1][0] < total


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out: str) -> None:
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    handle = bytes([rank + 1]) * dcb.IPC_HANDLE_BYTES
    got = dcb.exchange_handles(handle)
    with open(f"{out}.{rank}", "w") as f:
        f.write(",".join(str(h[0]) + ":" + str(len(h)) for h in got))
    dist.destroy_process_group()


def test_exchange_handles_gloo_world2(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "handles")
    mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    for r in range(2):
        assert open(f"{out}.{r}").read() == "1:64,2:64"
