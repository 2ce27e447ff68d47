"""Image sharding over several B200s (no counterpart in the reference, which runs one GPU).

Images are independent, so a batch is split contiguously by index — device g of G takes images
[g*B//G, (g+1)*B//G) — and every device runs its own engine and CUDA graph on its shard with the weights
replicated. Nothing crosses between GPUs on the hot path; results are gathered on the host in image order
(the result shaping of foidfinder/tagging.py:39-57 then runs per image as before).

Two forms:
- `ShardedEngine`: one process drives the local GPUs, one host thread per device;
- `gather_rows`: one process per GPU (torchrun), rank 0 collects each rank's rows after its stream has
  finished; with the `gloo` group this is a host-side gather, with `nccl` it runs once after the timed work.
"""

from __future__ import annotations

import concurrent.futures as cf

import torch
import torch.distributed as dist

from .config import ModelConfig


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) of `n` images for `rank` of `world`; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return n * rank // world, n * (rank + 1) // world


def shard_sizes(n: int, world: int) -> list[int]:
    return [hi - lo for lo, hi in (shard_range(n, world, r) for r in range(world))]


def gather_rows(rows: torch.Tensor, n_total: int, group=None) -> torch.Tensor | None:
    """Each rank's [n_rank, ...] rows (its `shard_range` of n_total) -> rank 0 gets [n_total, ...] in image
    order, other ranks None. Shards may be uneven or empty; rows are padded to the largest shard for the
    gather and trimmed after."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    sizes = shard_sizes(n_total, world)
    if rows.shape[0] != sizes[rank]:
        raise ValueError(f"rank {rank} holds {rows.shape[0]} rows, its shard is {sizes[rank]}")
    cap = max(sizes)
    pad = torch.zeros((cap,) + tuple(rows.shape[1:]), dtype=rows.dtype, device=rows.device)
    pad[: rows.shape[0]] = rows
    bucket = [torch.empty_like(pad) for _ in range(world)] if rank == 0 else None
    dist.gather(pad, bucket, dst=0, group=group)
    if rank != 0:
        return None
    return torch.cat([b[:s] for b, s in zip(bucket, sizes)])


class ShardedEngine:
    """One `Engine` per local device; `forward(images)` splits the batch, runs the shards concurrently
    (one host thread per device, each on its own device's current stream) and concatenates results."""

    def __init__(self, cfg: ModelConfig, devices: list[int] | None = None, *, seed: int = 0, weights=None):
        from .engine import Engine

        self.cfg = cfg
        self.devices = list(range(torch.cuda.device_count())) if devices is None else list(devices)
        if not self.devices:
            raise RuntimeError("no CUDA devices")
        self.engines = [Engine(cfg, weights, device=d, seed=seed) for d in self.devices]
        self._pool = cf.ThreadPoolExecutor(max_workers=len(self.devices))

    def _run(self, i: int, images: torch.Tensor, topk: bool):
        e = self.engines[i]
        with torch.cuda.device(e.device):
            logits, idx, val = e.forward(images, topk=topk)
            torch.cuda.current_stream(e.device).synchronize()
        return logits, idx, val

    @torch.no_grad()
    def forward(self, images: torch.Tensor, *, topk: bool = True):
        """images [B, S, S, 3] uint8 (host or any device) -> (logits [B, tags], idx [B, k], val [B, k]) on the
        host, in image order."""
        n, G = images.shape[0], len(self.engines)
        jobs = []
        for i in range(G):
            lo, hi = shard_range(n, G, i)
            if hi > lo:
                jobs.append(self._pool.submit(self._run, i, images[lo:hi], topk))
        parts = [j.result() for j in jobs]
        logits = torch.cat([p[0].cpu() for p in parts])
        if not topk:
            return logits, None, None
        return logits, torch.cat([p[1].cpu() for p in parts]), torch.cat([p[2].cpu() for p in parts])

    def close(self) -> None:
        self._pool.shutdown()
        for e in self.engines:
            e.close()
