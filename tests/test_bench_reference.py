"""The reference arm of bench.py keeps the bench line contract on the host
(no GPU): one JSON line with impl "reference", the arm's metric and unit, and
cpu_baseline / e2e objects; or an "unavailable" line when the reference build
is absent."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("workload,metric", [
    ("default", "decode attn KV-bytes GB/s"),
    ("qkv_append_bf16", "qkv projection + paged append TFLOP/s"),
    ("outproj_bf16", "output projection + residual TFLOP/s"),
])
def test_reference_arm_line(workload, metric):
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload",
                          workload, "--steps", "1", "--warmup", "3"], cwd=ROOT,
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    if "unavailable" in line:
        return
    unit = "GB/s" if metric.endswith("GB/s") else "TFLOP/s"
    assert line["metric"] == metric and line["unit"] == unit and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
