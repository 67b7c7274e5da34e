"""bench.py's command line and JSON-line contract, checked on CPU (no kernels run).

Every workload must parse, name itself in ``config`` with the dtype the line reports,
and choose the CPU leg of the same math (the reference arm and ``cpu_baseline``).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

WORKLOADS = ("parakeet", "parakeet_long", "zipformer", "zipformer_fused", "ragged")


def parse(argv):
    old = sys.argv
    sys.argv = ["bench.py", *argv]
    try:
        return bench.parse_args()
    finally:
        sys.argv = old


def test_defaults_are_config2_on_one_gpu():
    args = parse([])
    assert (args.gpus, args.workload, args.batch, args.impl) == (1, "parakeet", 256, "ours")
    assert args.warmup >= 3


@pytest.mark.parametrize("workload", WORKLOADS)
def test_every_workload_has_a_config(workload):
    args = parse(["--workload", workload, "--gpus", "2"])
    cfg = bench.workload_config(args)
    assert cfg["workload"] and cfg["dtype"] in ("f16", "bf16", "f16+bf16")
    assert cfg["parallelism"] == "dp2"
    assert "l2" in cfg
    assert args.batch == (16 if workload == "parakeet_long" else 256)


def test_cpu_leg_follows_the_math_of_the_workload():
    assert bench.cpu_leg(parse(["--workload", "parakeet"])) is bench.cpu_parakeet
    for w in ("zipformer", "zipformer_fused"):
        assert bench.cpu_leg(parse(["--workload", w])) is bench.cpu_zipformer


def test_fused_config_says_it_is_not_the_drop_in_path():
    cfg = bench.workload_config(parse(["--workload", "zipformer_fused"]))
    assert "drop-in" in cfg["workload"]
    assert cfg["stacks_T"] == bench.workload_config(parse(["--workload", "zipformer"]))["stacks_T"]
