"""Multi-rank host logic on CPU: 2 gloo ranks shard a batch, run the per-rank work, take the max
time over ranks and gather results; rank 0 checks the gathered shards against the unsharded
oracle result.  (The GPU path runs the same code with NCCL, one process per GPU.)"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from my_own_cnn_b200.shard import checksum, gather_tensors, max_over_ranks, shard_range


def test_shard_range_partitions():
    for total in (0, 1, 7, 512, 513):
        for world in (1, 2, 3, 8):
            parts = [shard_range(total, r, world) for r in range(world)]
            assert sum(c for _, c in parts) == total
            pos = 0
            for s, c in parts:
                assert s == pos
                pos += c
            assert max(c for _, c in parts) - min(c for _, c in parts) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle

        n, h, w, c, k = 6, 9, 8, 16, 8
        rng = np.random.default_rng(0)  # same full batch on every rank
        x = rng.integers(-127, 128, size=(n, h, w, c)).astype(np.int8)
        wt = rng.integers(-127, 128, size=(k, 3, 3, c)).astype(np.int8)
        start, count = shard_range(n, rank, world)
        part = oracle.conv_s8(oracle.conv_args(count, h, w, c, 3, 3, k), x[start:start + count], wt)
        t = max_over_ranks([1.0 + rank, 5.0 - rank])
        parts = gather_tensors(torch.from_numpy(part))
        sums = gather_tensors(checksum(torch.from_numpy(part)))
        if rank == 0:
            full = oracle.conv_s8(oracle.conv_args(n, h, w, c, 3, 3, k), x, wt)
            ok = np.array_equal(np.concatenate([p.numpy() for p in parts]), full)
            ok = ok and t == [float(world), 5.0]
            ok = ok and int(sum(s.item() for s in sums)) == int(checksum(torch.from_numpy(full)).item())
            with open(result_path, "w") as f:
                f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_gather(tmp_path):
    result = tmp_path / "result.txt"
    mp.spawn(_worker, args=(2, _free_port(), str(result)), nprocs=2, join=True)
    assert result.read_text() == "ok"
