"""The benchmark's output contract, checked on CPU through its reference arm.

`bench.py --impl reference` times the CPU baseline (no GPU needed) and must
print exactly one JSON line with the keys the driver reads; the same metric,
unit and config as the GPU arm.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_reference(*extra):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          *extra], capture_output=True, text=True, timeout=600, cwd=ROOT,
                         env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


@pytest.mark.parametrize("config", ["1"])       # the others generate GBs of rows
def test_reference_arm_prints_one_contract_line(config):
    d = run_reference("--config", config, "--steps", "2", "--warmup", "1", "--ref-sample", "4")
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1
    assert d["steps"] == 2 and d["warmup"] == 1
    assert d["unit"] == "queries/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["value"] == d["cpu_baseline"]["value"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["config_id"] == int(config) and "workload" in d["config"]
