"""`bench.py --impl reference` for the non-default workloads, on the CPU: one JSON line with
"impl": "reference", the CUDA arm's metric and unit, and the reference-arm keys."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("workload,extra,metric,unit", [
    ("qmatvec", [], "qmatvec HBM GB/s", "GB/s"),
    ("attention", [], "int8-KV decode attention HBM GB/s", "GB/s"),
    ("single", ["--prompt-len", "5", "--new-tokens", "3"], "batch-1 greedy decode tokens/s (prefill included)",
     "tokens/s"),
])
def test_reference_arm_line(workload, extra, metric, unit):
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", workload, *extra],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == metric and line["unit"] == unit
    assert line["value"] > 0 and line["ms_per_step"] > 0 and line["higher_is_better"] is True
    assert line["cpu_baseline"]["value"] == line["value"] and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
