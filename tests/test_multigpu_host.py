"""Host logic of the image sharding: contiguous ranges and the rank-0 gather, run as two `gloo` ranks on
CPU (the layout the GPU ranks use, without the GPUs)."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from foidfinder_b200.multigpu import gather_rows, shard_range, shard_sizes


@pytest.mark.parametrize("n,world", [(64, 1), (64, 2), (64, 8), (65, 8), (3, 8), (0, 4), (1025, 3)])
def test_shard_range_partitions(n, world):
    got = [shard_range(n, world, r) for r in range(world)]
    assert got[0][0] == 0 and got[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
    sizes = shard_sizes(n, world)
    assert sum(sizes) == n and max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)
    with pytest.raises(ValueError):
        shard_range(8, 0, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, n: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = shard_range(n, world, rank)
        # Each rank's "results": rows derived from the global image index, as an engine's would be.
        idx = torch.arange(lo, hi, dtype=torch.int32)[:, None] * 100 + torch.arange(5, dtype=torch.int32)
        val = torch.arange(lo, hi, dtype=torch.float32)[:, None].expand(-1, 5).contiguous()
        gi = gather_rows(idx, n)
        gv = gather_rows(val, n)
        if rank == 0:
            q.put((gi.tolist(), gv.tolist()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [8, 7, 1])
def test_gather_rows_two_ranks(n):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n, q)) for r in range(2)]
    for p in procs:
        p.start()
    gi, gv = q.get(timeout=120)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    want_i = (torch.arange(n, dtype=torch.int32)[:, None] * 100 + torch.arange(5, dtype=torch.int32)).tolist()
    assert gi == want_i
    assert gv == torch.arange(n, dtype=torch.float32)[:, None].expand(-1, 5).tolist()
