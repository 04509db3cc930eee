"""Batch-sharded parity on several GPUs of one node (NCCL, one process per GPU).

The C5 workload shards the policy queries of a batch contiguously over the
GPUs, each rank runs the op on its shard and one NCCL all-gather assembles the
batch. Here every visible GPU (up to 8) takes a shard of a C3/C5-shaped
attention batch and of a wide bf16 softmax, and rank 0 checks the gathered
result against the same op run on the whole batch on one GPU (bit-identical:
each batch element and row is computed independently of the others) and the
attention against the CPU oracle (atol 1e-2, rtol 1.6e-2). Shards keep at
least 30 queries per GPU, so no rank takes the small-batch key-split path.
Skipped with fewer than two GPUs.
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

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs"),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, B: int, result_path: str):
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "vla-kernels_b200"))
    from kernels import workloads as wl
    from kernels.attention import fused_attention_gqa_v4
    from kernels.batch_shard import gather, shard
    from kernels.softmax import softmax
    from oracle import gqa_attention

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        s = wl.expert_shape(B)
        q, k, v = wl.attn_inputs(s, device="cpu", seed=21)  # same inputs on every rank
        x = wl.softmax_c2(4 * B, 4096, device="cpu", seed=22)
        lo, hi = shard(B, rank, world)
        dev = torch.device("cuda", rank)
        o_local = fused_attention_gqa_v4(q[lo:hi].to(dev), k[lo:hi].to(dev), v[lo:hi].to(dev),
                                         scale=0.125, prefix_len=s.P)
        o = gather(o_local, B)
        rlo, rhi = shard(4 * B, rank, world)
        y = gather(softmax(x[rlo:rhi].to(dev), "auto"), 4 * B)
        if rank == 0:
            o_one = fused_attention_gqa_v4(q.to(dev), k.to(dev), v.to(dev), scale=0.125,
                                           prefix_len=s.P)
            y_one = softmax(x.to(dev), "auto")
            n = 8  # oracle cost: the first and last batch elements
            idx = list(range(n // 2)) + list(range(B - n // 2, B))
            ref = gqa_attention(q[idx].float().numpy(), k[idx].float().numpy(),
                                v[idx].float().numpy(), s.P, 0, 0, 0.125)
            got = o[idx].float().cpu().numpy()
            within = bool((np.abs(got - ref) <= 1e-2 + 1.6e-2 * np.abs(ref)).all())
            with open(result_path, "w") as f:
                f.write(f"{int(torch.equal(o, o_one))} {int(torch.equal(y, y_one))} "
                        f"{int(within)} {float(np.abs(got - ref).max())}")
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [256, 253])
def test_sharded_batch_matches_one_gpu(B, tmp_path, monkeypatch):
    world = min(torch.cuda.device_count(), 8)
    path = str(tmp_path / "res.txt")
    # the spawned ranks inherit it: plain peer transfers, no NVLink multicast
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_rank_main, args=(world, _free_port(), B, path), nprocs=world,
                       start_method="spawn", join=True)
    same_attn, same_softmax, within, err = open(path).read().split()
    assert same_attn == "1", "gathered attention differs from the one-GPU call"
    assert same_softmax == "1", "gathered softmax differs from the one-GPU call"
    assert within == "1", f"attention vs oracle: max abs err {err}"
