#!/usr/bin/env python
"""Throughput of the EVA02-L/448 int8 forward on 1..8 B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

One step = one forward of a global batch of B seeded 448x448 uint8 images (default 64),
split contiguously over the N ranks (rank r takes `multigpu.shard_range(B, N, r)`; no collective on the
data path; `scaling` is strong: the job's work is fixed as N grows). `value` is images/s of the whole job
with inputs resident in HBM (CUDA-graph replays timed with CUDA events, max over ranks); `e2e` is the same
metric through the public `Engine.forward` API with, every step, the host->device copy of each rank's
images from pinned memory, the device->host copy of its logits, and the gather of every rank's top-50 to
rank 0 (`multigpu.gather_rows`) and its copy to the host; the input copies run on a copy stream one step
ahead of the forward (two device buffers), as a serving loop overlaps them, and all K steps' copies lie
inside the timed region. `weak` repeats the device-timed measurement
with B images per GPU (the per-GPU batch fixed as N grows). The roofline entry covers the dominant kernel
(the tcgen05 int8 GEMM, all four block GEMMs) from a live per-launch CUDA-event profile of one rank's
shard.

`--impl reference` times the reference's CPU path instead: the fp32 PyTorch forward of the same model
(the oracle restatement of foidfinder/backends/cuda/reference.py:109-131 with the EVA02 block), on all
host threads, one image per step; under torchrun only rank 0 runs it.

`--config pixai-1008` runs the reference's own `cuda` workload instead (PixAI Tagger v1.0: 1008 px, 5184
window-ordered tokens, 32 blocks, GELU 4736, attention-pool head; default batch 16), with the same keys.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "images/sec (1/2/4/8 B200) EVA02-L int8 bs64"
UNIT = "images/s"
DEFAULT_BATCH = {"pixai": 16, "eva02": 64}


def metric_for(cfg, B: int) -> str:
    if cfg.name == "eva02-l-448" and B == 64:
        return METRIC
    return f"images/sec (1/2/4/8 B200) {cfg.name} int8 bs{B}"


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=None,
                    help="global images per step, split over the GPUs (default 64; pixai-1008: 16)")
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", default="eva02-l-448")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--latency-reps", type=int, default=200)
    return ap.parse_args()


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while running (read-only)."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
        "clocks_event_reasons.sw_power_cap"
    )
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(self.NAMES, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        loaded = [s for s in sm if s > 0.5 * mx] if mx else sm
        return {
            "sm_mhz": statistics.median(loaded) if loaded else None,
            "sm_max_mhz": mx or None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return {"bf16": d.get("bf16_tflops"), "bf16_sustained": d.get("bf16_tflops_sustained"), "hbm": d.get("hbm_gbs"),
                "source": "measured"}
    return {"bf16": 1590.0, "bf16_sustained": 1400.0, "hbm": 6650.0, "source": "fallback"}


PROFILES = {("eva02-l-448", 64): "launches_eva02l_bs64.md", ("pixai-1008", 16): "launches_pixai1008_bs16.md"}


def profiled_traffic(kernel: str, cfg_name: str, B: int) -> int | None:
    """DRAM bytes per launch of `kernel` from the committed ncu launch-list summary of this workload."""
    name = PROFILES.get((cfg_name, B))
    if name is None:
        return None
    f = ROOT / "profiles" / name
    if not f.is_file():
        return None
    for line in f.read_text().splitlines():
        if line.startswith(f"traffic_bytes_per_launch[{kernel}]"):
            return int(line.split("=")[1])
    return None


def cpu_forward_timing(cfg, n_images: int, warmup: int = 1) -> tuple[float, int, str]:
    """Seconds per image of the fp32 CPU forward (oracle restatement), all host threads."""
    from foidfinder_b200.weights import pixai_random_raw, random_raw

    if cfg.arch == "pixai":
        from oracle.pixai import forward_fp32

        raw = pixai_random_raw(cfg, seed=0, device="cpu")
    else:
        from oracle.eva02 import forward_fp32

        raw = random_raw(cfg, seed=0, device="cpu")
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(1234)
    imgs = torch.randint(0, 256, (n_images + warmup, cfg.image_size, cfg.image_size, 3), generator=g, dtype=torch.uint8)
    with torch.no_grad():
        for i in range(warmup):
            forward_fp32(raw, cfg, imgs[i : i + 1])
        times = []
        for i in range(warmup, warmup + n_images):
            t0 = time.perf_counter()
            forward_fp32(raw, cfg, imgs[i : i + 1])
            times.append(time.perf_counter() - t0)
    return statistics.median(times), torch.get_num_threads(), f"{n_images} images of the fp32 CPU forward, batch 1"


def workload(cfg, B: int, world: int) -> dict:
    """B: the global batch of one step, split over `world` GPUs."""
    if cfg.arch == "pixai":
        desc = (f"{cfg.name} int8 forward (the reference's PixAICuda workload): {cfg.image_size}px, {cfg.tokens} "
                f"window-ordered tokens, {cfg.depth} blocks ({cfg.window}x{cfg.window} windows, global blocks "
                f"{list(cfg.global_blocks)}), dim {cfg.dim}, GELU {cfg.mlp_hidden}, attention-pool head, "
                f"{cfg.num_tags} tags, top-{cfg.topk}")
    else:
        which = "BASELINE config 4" if cfg.head == "tree" else "BASELINE config 3"
        desc = (f"{cfg.name} int8 forward ({which}): {cfg.image_size}px, {cfg.tokens} tokens, "
                f"{cfg.depth} blocks, dim {cfg.dim}, SwiGLU {cfg.mlp_hidden}, {cfg.num_tags} tags, top-{cfg.topk}")
    from foidfinder_b200.multigpu import shard_sizes

    return {
        "workload": desc,
        "global_batch": B,
        "batch_per_gpu": shard_sizes(B, world),
        "parallelism": f"dp{world} (one global batch split contiguously by rank; no collective on the data path, "
                       "top-50 gathered to rank 0 in the e2e step)",
        "l2_policy": "no flush: each step streams > 1 GB of weights and activations, far above the 126 MB L2",
        "weights": "random-init N(0, 0.02), seed 0",
    }


def run_reference(args) -> None:
    rank, _, world = dist_env()
    if rank != 0:
        return
    from foidfinder_b200.config import CONFIGS

    cfg = CONFIGS[args.config]
    B = args.batch or DEFAULT_BATCH[cfg.arch]
    sec, cores, _ = cpu_forward_timing(cfg, n_images=max(1, args.steps), warmup=max(1, min(args.warmup, 2)))
    value = 1.0 / sec
    line = {
        "impl": "reference",
        "metric": metric_for(cfg, B),
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": sec * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded uint8 images U[0,255], random-init N(0,0.02) weights",
        "config": workload(cfg, B, world),
        "cpu_baseline": {
            "value": value,
            "unit": UNIT,
            "cores": cores,
            "kind": "port",
            "sample": f"{args.steps} steps of 1 image each (a bounded sample of the {B}-image step): fp32 "
            "PyTorch CPU forward (oracle restatement of the reference's PixAITorch forward"
            + ("" if cfg.arch == "pixai" else " with the EVA02 block") + "), median step, on rank 0 only",
        },
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        # The communicator set-up may print a version banner on the process's stdout (seen on the GPU hosts);
        # stdout is reserved for the one JSON result line, so the C-level stdout points at stderr until the
        # first collective has created the communicator.
        import ctypes

        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
            dist.barrier()
        finally:
            ctypes.CDLL(None).fflush(None)  # C stdio buffers still hold what was printed in the window
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)
    from foidfinder_b200.config import CONFIGS
    from foidfinder_b200.engine import Engine
    from foidfinder_b200.multigpu import gather_rows, shard_range

    cfg = CONFIGS[args.config]
    BG, K, W = args.batch or DEFAULT_BATCH[cfg.arch], args.steps, max(args.warmup, 3)
    if BG < world:
        raise SystemExit(f"global batch {BG} is smaller than the {world} GPUs")
    lo, hi = shard_range(BG, world, rank)
    B = hi - lo  # this rank's images of the global batch
    eng = Engine(cfg, device=local, seed=0)
    # One seeded global batch, identical on every rank; each rank keeps its contiguous shard.
    g = torch.Generator(device=dev).manual_seed(1000)
    batch = torch.randint(0, 256, (BG, cfg.image_size, cfg.image_size, 3), generator=g, dtype=torch.uint8, device=dev)
    imgs = batch[lo:hi].contiguous()
    del batch
    logits = torch.empty(B, cfg.num_tags, device=dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed_replays(x: torch.Tensor, out: torch.Tensor) -> float:
        for _ in range(W):
            eng.forward(x, logits=out)
        barrier()
        start.record(stream)
        for _ in range(K):
            eng.forward(x, logits=out)
        end.record(stream)
        barrier()
        return max_over_ranks(start.elapsed_time(end))

    with ClockSampler(local) as clocks:
        dev_ms = timed_replays(imgs, logits)

        # end to end through the public API, host buffers: H2D of this rank's images, forward, D2H of its
        # logits, gather of every rank's top-50 to rank 0 and its D2H there
        # (the input copies run on a copy stream into two device buffers, one step ahead of the forward, as a
        # serving loop overlaps them; every copy of the K steps is inside the timed region)
        host_in = imgs.cpu().pin_memory()
        host_logits = torch.empty(B, cfg.num_tags, pin_memory=True)
        host_idx = torch.empty(BG, cfg.topk, dtype=torch.int32, pin_memory=True)
        host_val = torch.empty(BG, cfg.topk, pin_memory=True)
        dev_in = [torch.empty_like(imgs), torch.empty_like(imgs)]
        copy_stream = torch.cuda.Stream(device=dev)
        copied = [torch.cuda.Event(), torch.cuda.Event()]
        used = [torch.cuda.Event(), torch.cuda.Event()]

        def issue_copy(k):  # the H2D of step k into buffer k % 2, after the forward that last read it
            b = k % 2
            copy_stream.wait_event(used[b])
            with torch.cuda.stream(copy_stream):
                dev_in[b].copy_(host_in, non_blocking=True)
                copied[b].record(copy_stream)

        def e2e_step(k):
            b = k % 2
            stream.wait_event(copied[b])
            lg, ix, vl = eng.forward(dev_in[b], logits=logits)
            used[b].record(stream)
            host_logits.copy_(lg, non_blocking=True)
            if world > 1:
                ix, vl = gather_rows(ix, BG), gather_rows(vl, BG)
            if rank == 0:
                host_idx.copy_(ix, non_blocking=True)
                host_val.copy_(vl, non_blocking=True)

        def e2e_run(n):
            for k in range(min(2, n)):
                issue_copy(k)
            for k in range(n):
                e2e_step(k)
                if k + 2 < n:
                    issue_copy(k + 2)

        for ev in used:
            ev.record(stream)
        e2e_run(W)
        torch.cuda.synchronize()
        barrier()
        start.record(stream)
        copy_stream.wait_event(start)
        e2e_run(K)
        end.record(stream)
        barrier()
        e2e_ms = max_over_ranks(start.elapsed_time(end))

        # weak scaling for context: the full batch on every GPU
        if world > 1:
            weak_imgs = imgs.repeat((BG + B - 1) // B, 1, 1, 1)[:BG].contiguous()
            weak_logits = torch.empty(BG, cfg.num_tags, device=dev)
            weak_ms = timed_replays(weak_imgs, weak_logits)
            del weak_imgs, weak_logits
    h2d = BG * cfg.image_size * cfg.image_size * 3  # every rank's shard, summed over the job
    d2h = BG * cfg.num_tags * 4 + 2 * BG * cfg.topk * 4  # every rank's logits + the gathered top-50 on rank 0

    # batch-1 latency: p50 over individually timed graph replays
    one = imgs[:1].contiguous()
    l1 = torch.empty(1, cfg.num_tags, device=dev)
    for _ in range(5):
        eng.forward(one, logits=l1)
    lat = []
    for _ in range(args.latency_reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        eng.forward(one, logits=l1)
        e.record(stream)
        e.synchronize()
        lat.append(s.elapsed_time(e))
    lat_p50 = max_over_ranks(statistics.median(lat))

    prof = eng.profile(imgs, iters=2)
    from foidfinder_b200 import ops as _ops

    int8_peak = max(_ops.int8_mma_peak(local) for _ in range(2))  # TOPS, measured on this GPU now
    err = eng.device_error()
    if err:
        raise RuntimeError(f"a kernel reported device error {err}")
    gemm_ms = sum(prof[k][0] for k in ("gemm_qkv", "gemm_proj", "gemm_fc1", "gemm_fc2"))
    gemm_launches = sum(prof[k][1] for k in ("gemm_qkv", "gemm_proj", "gemm_fc1", "gemm_fc2"))
    gemm_ops = cfg.gemm_ops_per_image() * B
    achieved = gemm_ops / (gemm_ms * 1e-3) / 1e12
    peaks = measured_peaks()
    peak = 2.0 * peaks["bf16_sustained"]
    attn_tflops = cfg.attention_flops_per_image() * B / (prof["attention"][0] * 1e-3) / 1e12

    total = BG * K
    line = {
        "metric": metric_for(cfg, BG),
        "value": total / (dev_ms * 1e-3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": dev_ms / K,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic: seeded uint8 images U[0,255], random-init N(0,0.02) weights",
        "config": workload(cfg, BG, world),
        "e2e": {"value": total / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "latency_bs1_p50_ms": lat_p50,
        "gpu_launches": eng.launches_per_forward * K,
        "roofline": {
            "bound": "tensor",
            "kernel": "gemm_tc_kernel (tcgen05 kind::i8; qkv, proj, " + ("fc1" if cfg.arch == "pixai" else "gate|up")
            + ", down)",
            "achieved": achieved,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": achieved / peak,
            "traffic": profiled_traffic("gemm_tc_kernel int8", cfg.name, B),
            "traffic_source": (
                f"ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, averaged over the int8 GEMM launches "
                f"of one forward (profiles/{PROFILES[(cfg.name, B)]}); algorithmic A + W + output bytes per launch "
                f"average {427 if cfg.arch == 'eva02' else 667} MB"
                if (cfg.name, B) in PROFILES else "not captured for this workload"),
            "peak_source": f"2 x bf16_tflops_sustained of MEASURED_PEAKS.json ({peaks['source']}): dense int8 runs "
            "at twice the dense bf16 rate on B200; int8 ops counted as 2 per multiply-add",
            "frac_of_nominal_4500": achieved / 4500.0,
            "measured_int8_peak": int8_peak,
            "frac_of_measured_int8_peak": achieved / int8_peak,
            "measured_int8_peak_source": "ops.int8_mma_peak: one CTA per SM issuing back-to-back tcgen05 kind::i8 "
            "M128 N256 K32 MMAs on resident operands for ~50 ms, CUDA events, best of 2, after the timed region",
            "launches_per_forward": gemm_launches,
            "ms_per_forward": gemm_ms,
        },
        "breakdown_ms_per_forward": {k: round(v[0], 4) for k, v in prof.items()},
        "breakdown_batch": B,
        "attention_tflops": attn_tflops,
        "clocks": clocks.summary(),
    }
    if world > 1:
        line["weak"] = {"value": world * BG * K / (weak_ms * 1e-3), "unit": UNIT, "batch_per_gpu": BG,
                        "ms_per_step": weak_ms / K, "scaling": "weak"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sec, cores, sample = cpu_forward_timing(cfg, n_images=1 if cfg.arch == "pixai" else 3)
        line["cpu_baseline"] = {"value": 1.0 / sec, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
    eng.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def main() -> None:
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
