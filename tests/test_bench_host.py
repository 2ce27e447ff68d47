"""bench.py's host-side pieces without a GPU: metric names, workload descriptions, the ncu traffic lookup,
and the reference-kernel build recipe's behaviour where the reference tree is absent."""

from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402

from foidfinder_b200.config import CONFIGS  # noqa: E402


def test_metric_names():
    assert bench.metric_for(CONFIGS["eva02-l-448"], 64) == bench.METRIC
    assert bench.metric_for(CONFIGS["pixai-1008"], 16) == "images/sec (1/2/4/8 B200) pixai-1008 int8 bs16"


def test_workload_descriptions():
    w = bench.workload(CONFIGS["eva02-l-448"], 64, 2)
    assert w["global_batch"] == 64 and w["batch_per_gpu"] == [32, 32]
    assert "1025 tokens" in w["workload"] and w["parallelism"].startswith("dp2")
    assert bench.workload(CONFIGS["eva02-l-448"], 64, 8)["batch_per_gpu"] == [8] * 8
    assert bench.workload(CONFIGS["eva02-l-448"], 10, 4)["batch_per_gpu"] == [2, 3, 2, 3]
    w = bench.workload(CONFIGS["pixai-1008"], 16, 1)
    assert "5184 window-ordered tokens" in w["workload"] and "global blocks [7, 15, 23, 31]" in w["workload"]


def test_profiled_traffic_comes_from_the_committed_launch_lists():
    eva = bench.profiled_traffic("gemm_tc_kernel int8", "eva02-l-448", 64)
    pix = bench.profiled_traffic("gemm_tc_kernel int8", "pixai-1008", 16)
    assert eva is not None and 2e8 < eva < 6e8
    assert pix is not None and 3e8 < pix < 9e8
    assert bench.profiled_traffic("gemm_tc_kernel int8", "eva02-l-448", 8) is None


def test_reference_kernel_recipe_without_reference_tree(tmp_path):
    from oracle import build_ref

    assert build_ref.build(tmp_path / "no-reference-here") is None
