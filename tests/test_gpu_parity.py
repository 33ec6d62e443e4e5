"""Parity of the CUDA kernels with the reference (golden vectors made by the
reference itself) and with the CPU oracle on the harness's case mix: the
deterministic stress cases, the bench shape and the adversarial random sweep
(ouroboros/harness.py:166-202).  Every call goes through the C ABI
(libb200k.so) via the b200k spec-signature functions."""
import zlib

import numpy as np
import pytest
import torch

import b200k
from b200k import _lib
from b200k.registry import ENTRY, OPS as B2K_OPS
from golden_io import golden_ops, load
from gpu_util import run_checked
from oracle import regimes

import os, sys
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_golden import build_case  # noqa: E402

pytestmark = pytest.mark.gpu

ALL_OPS = sorted(B2K_OPS)
BASE_OPS = [o for o in ALL_OPS if not o.endswith("_short")]


def _require(op):
    assert _lib.exported_symbols()[ENTRY[op]], f"{ENTRY[op]} not exported by libb200k.so"


@pytest.mark.parametrize("op", golden_ops())
def test_golden(op):
    _require(op)
    run = b200k.get_op(op)
    for rec, ref in load(op):
        ok, err, bad = run_checked(op, run, build_case(rec), ref)
        assert ok, f"{op} golden {rec['dt']} {rec['M']}x{rec['N']}: max err {err} ({bad} bad)"


@pytest.mark.parametrize("op", BASE_OPS)
def test_stress_and_random(op):
    _require(op)
    run = b200k.get_op(op)
    cases = regimes.stress_cases(op) + regimes.random_cases(op, 6, seed=zlib.crc32(op.encode()),
                                                            max_elems=1 << 20)
    for case in cases:
        ref = regimes.reference(op, case)
        ok, err, bad = run_checked(op, run, case, ref)
        M, N = case[0][0].shape
        assert ok, f"{op} {case[0][1]} {M}x{N}: max err {err} ({bad} bad)"


@pytest.mark.parametrize("op", ALL_OPS)
def test_bench_shape_sampled_rows(op):
    """The op's bench shape (8192x4096, 32768x128 for rope, 16384x2048 for
    *_short, 8x131072 for rmsnorm_wide) on the GPU, checked row-by-row on a
    sample of rows (row ops are row-independent)."""
    _require(op)
    run = b200k.get_op(op)
    case = regimes.bench_case(op)
    M = case[0][0].shape[0]
    rows = np.unique(np.r_[0, M - 1, np.random.default_rng(0).integers(0, M, 30)])
    sub = [(v[rows] if (v.ndim >= 1 and v.shape[0] == M and not (regimes.OPS[op].kind == "x_scale" and i == 1)) else v, t)
           for i, (v, t) in enumerate(case)]
    ref = regimes.reference(op, sub)
    ok, err, bad = run_checked(op, run, case, ref, rows=rows)
    assert ok, f"{op} bench shape: max err {err} ({bad} bad)"


def test_zz_no_pipeline_timeouts():
    """No bounded pipeline wait gave up during the parity runs above."""
    torch.cuda.synchronize()
    assert _lib.lib.b2k_pipeline_timeouts(1) == 0
