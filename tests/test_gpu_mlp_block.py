"""The end-to-end MLP block of ouroboros/e2e_block_bench.py:94-148 (RMSNorm
with residual -> gate/up GEMMs -> SwiGLU -> down GEMM, fp16) through the
benchmark's own mode: the b200k block's output must match the eager PyTorch
block before anything is timed (the reference's correctness gate,
e2e_block_bench.py:118-127), here on 1024 rows."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_mlp_block_is_gated_on_parity():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--workload",
                          "mlp_block", "--rows", "1024", "--steps", "3"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads([l for l in out.stdout.splitlines() if l.strip()][-1])
    assert line["correct_vs_eager"] is True, line
    assert line["config"]["rows"] == 1024
    assert line["speedup_vs_eager"] > 0 and line["value"] > 0
