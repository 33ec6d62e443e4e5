"""The benchmark's output contract, checked on its CPU arm (`--impl
reference`, which needs no GPU): exactly one JSON line on stdout with the
keys a driver reads, the reference-arm fields (`impl`, `cpu_baseline`, an
`e2e` with no transfers) and W >= 3 warm-up steps whatever is asked; and
library output written to file descriptor 1 kept off stdout."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"}


@pytest.mark.parametrize("workload", ["chain", "rmsnorm", "swiglu", "rope", "ce"])
def test_reference_arm_prints_one_contract_line(workload):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
         "--workload", workload, "--steps", "1", "--warmup", "1"],
        capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference"
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] >= 3
    assert "workload" in d["config"] and "model" not in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["unit"] == d["unit"] and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_library_output_on_fd1_does_not_reach_stdout():
    """Whatever a library writes to file descriptor 1 after the bench starts
    (NCCL prints its version banner there) goes to stderr; stdout keeps only
    the JSON lines the bench emits."""
    code = (
        "import os, sys; sys.path.insert(0, %r); import bench; "
        "bench._json_out(); os.write(1, b'NCCL version banner\\n'); print('chatter'); "
        "bench.emit({'metric': 'x', 'value': 1})" % ROOT)
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert lines == ['{"metric": "x", "value": 1}'], out.stdout
    assert "NCCL version banner" in out.stderr and "chatter" in out.stderr
