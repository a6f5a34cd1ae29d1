"""bench.py's two arms.  The reference arm (`--impl reference`) runs on the
host cores: it times the reference's CPU path (its own attention_reference
when staged, else the numpy restatement) on a bounded sample of the headline
workload and prints one JSON line with the same metric, unit and config as the
GPU arm, plus its cpu_baseline and e2e objects.  The GPU arm's line carries
the per-rank parity check."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps",
                        "1", "--warmup", "3"], capture_output=True, text=True, timeout=600,
                       cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = r.stdout.strip().splitlines()[-1]
    d = json.loads(line)
    assert d["impl"] == "reference"
    assert d["metric"].startswith("attn-fwd TFLOPS") and d["unit"] == "TFLOPS"
    assert d["higher_is_better"] is True and d["n_gpus"] == 1 and d["steps"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["unit"] == d["unit"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]


@pytest.mark.gpu
def test_bench_kernel_only_line_reports_parity():
    # the GPU arm on one batch element of the headline workload: one JSON
    # line whose per-rank parity check passes
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--kernel-only", "--batch", "1",
                        "--steps", "3", "--warmup", "3"], capture_output=True, text=True,
                       timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["parity"]["ok"] is True and d["value"] > 0
