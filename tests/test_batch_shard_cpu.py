"""Multi-rank host logic of the batch sharding (gloo, world size 2, CPU).

Each rank computes its contiguous shard of a C3-shaped attention batch with the
CPU oracle and the shards are all-gathered; rank 0 checks the gathered batch
against the unsharded computation. A second case makes one rank leave before
the collective and checks that the survivor gets an error within the process
group timeout instead of hanging.
"""
from __future__ import annotations

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for _p in (REPO, os.path.join(REPO, "vla-kernels_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

from kernels.batch_shard import gather, shard  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(B: int):
    rng = np.random.default_rng(7)
    q = rng.standard_normal((B, 50, 15, 64)).astype(np.float32)
    k = rng.standard_normal((B, 291, 5, 64)).astype(np.float32)
    v = rng.standard_normal((B, 291, 5, 64)).astype(np.float32)
    return q, k, v


def _rank_main(rank: int, world: int, port: int, B: int, result_path: str, mode: str):
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "vla-kernels_b200"))
    from oracle import gqa_attention

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        if mode == "leave" and rank == 1:
            return  # leaves between steps, before the collective
        q, k, v = _inputs(B)
        lo, hi = shard(B, rank, world)
        local = torch.from_numpy(gqa_attention(q[lo:hi], k[lo:hi], v[lo:hi], 241, 0, 0, 0.125))
        try:
            full = gather(local, B)
        except Exception as e:  # the survivor of "leave" ends up here
            if rank == 0:
                with open(result_path, "w") as f:
                    f.write(f"error {type(e).__name__}")
            return
        if rank == 0:
            ref = gqa_attention(q, k, v, 241, 0, 0, 0.125)
            err = float(np.abs(full.numpy() - ref).max())
            with open(result_path, "w") as f:
                f.write(f"ok {err}")
    finally:
        if mode != "leave":
            dist.destroy_process_group()


@pytest.mark.parametrize("B,world", [(0, 3), (1, 2), (5, 2), (2048, 8), (2047, 8), (7, 4)])
def test_shards_cover_batch(B, world):
    got = [shard(B, r, world) for r in range(world)]
    assert got[0][0] == 0 and got[-1][1] == B
    for (l0, h0), (l1, h1) in zip(got, got[1:]):
        assert h0 == l1
    sizes = [h - l for l, h in got]
    assert max(sizes) - min(sizes) <= (1 if B else 0)


def test_shard_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard(8, 2, 2)


def test_gather_two_ranks_uneven(tmp_path):
    path = str(tmp_path / "res.txt")
    mp.start_processes(_rank_main, args=(2, _free_port(), 5, path, "ok"), nprocs=2,
                       start_method="spawn", join=True)
    status, val = open(path).read().split()
    assert status == "ok"
    assert float(val) == 0.0  # shards are bit-identical to the unsharded rows


def test_rank_leaving_does_not_hang(tmp_path):
    path = str(tmp_path / "res.txt")
    mp.start_processes(_rank_main, args=(2, _free_port(), 4, path, "leave"), nprocs=2,
                       start_method="spawn", join=True)
    assert open(path).read().startswith("error")
