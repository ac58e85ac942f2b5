"""bench.py's reference arm on the host cores: one JSON line per workload with the keys the
benchmark contract names, on the same metric and config as the tideway arm."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from tests.conftest import ROOT

KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
        "cpu_baseline", "e2e"}


def run_bench(*args, env=None) -> list[dict]:
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0", *args], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]


@pytest.mark.parametrize("workload,metric_has,lines", [
    ("c2-decode", "MoE decode tokens/s + expert-weight HBM GB/s vs peak", 1),
    ("c3-prefill", "MoE prefill tokens/s", 1),
    ("c5-ep-decode", "expert-parallel MoE layer tokens/s (configs[4], decode)", 1),
])
def test_reference_arm_line(workload, metric_has, lines):
    import bench

    got = run_bench("--workload", workload)
    assert len(got) == lines
    line = got[0]
    assert KEYS <= set(line), KEYS - set(line)
    assert line["impl"] == "reference" and metric_has in line["metric"]
    assert line["value"] > 0 and line["ms_per_step"] > 0 and line["higher_is_better"] is True
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"],
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["value"] == line["value"] and cpu["cores"] >= 1
    assert cpu["sample"]
    assert line["config"]["workload"].startswith({"c2-decode": "configs[1]",
                                                  "c3-prefill": "configs[2]",
                                                  "c5-ep-decode": "configs[4]"}[workload])
    if workload == "c3-prefill":
        from tideway_b200.prefill import C3

        assert line["config"] == bench.prefill_config(C3)
        assert line["metric"] == bench.PREFILL_METRIC


def test_reference_arm_other_ranks_print_nothing():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    assert run_bench(env=env) == []
