"""The reference arm of ``bench.py`` (the reference's CPU path timed on the
host cores) keeps the benchmark's JSON contract; runs on CPU."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
        "cpu_baseline", "e2e"}


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                           "--warmup", "0"], cwd=REPO, env=env, capture_output=True, text=True,
                          timeout=600)


def test_reference_arm_prints_one_contract_line():
    res = _run({})
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["unit"] == "ms" and d["higher_is_better"] is False
    assert d["value"] > 0 and d["value"] == d["ms_per_step"] == d["cpu_baseline"]["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "ms", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    # the repo arm's default workload (configs[4], global batch 64, bf16), and
    # the driver's --steps / --warmup honoured
    assert d["config"]["workload"].startswith("configs[4]")
    assert d["config"]["global_batch"] == 64 and d["dtype"] == "bf16"
    assert d["steps"] == 1 and d["warmup"] == 0 and d["scaling"] == "strong"


def test_both_arms_print_the_same_config():
    import bench

    for world in (1, 2, 8):
        for argv in ([], ["--workload", "b1"]):
            args = bench.parse_args(argv)
            cfg, scaling = bench.workload_config(args, world)
            assert cfg["parallelism"] == f"dp{world}"
            if args.workload == "sharded":
                assert (cfg["global_batch"], cfg["batch_per_gpu"]) == (64, 64 // world)
                assert scaling == "strong"
            else:
                assert (cfg["global_batch"], cfg["batch_per_gpu"]) == (world, 1)
                assert scaling == "weak"


def test_reference_arm_other_ranks_exit_quietly():
    res = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert res.returncode == 0, res.stderr[-2000:]
    assert not [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
