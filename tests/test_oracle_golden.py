"""Pins the CPU oracle (oracle/ops.py) to the reference: every golden vector
made by importing ouroboros/specs.py must be reproduced within the parity
tolerance, and the regenerated inputs must hash to what the reference saw."""
import numpy as np
import pytest

from golden_io import golden_ops, load
from oracle import regimes
from oracle.numerics import allclose_report, tol_for

import sys, os
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_golden import build_case, input_hash  # noqa: E402


@pytest.mark.parametrize("op", golden_ops())
def test_oracle_matches_reference_golden(op):
    for rec, ref in load(op):
        case = build_case(rec)
        assert input_hash(case) == rec["sha256"], f"{op}: regenerated inputs differ from golden"
        out = regimes.reference(op, case)
        rtol, atol = tol_for(op, rec["dt"])
        ok, err, bad = allclose_report(out, ref, rtol, atol)
        assert ok, f"{op} {rec}: max err {err} ({bad} bad)"


def test_op_table_covers_reference_suite():
    # 29 explicit + 75 chain ops (layernorm_gelu is explicit) + 14 _short = 118 specs
    assert len(regimes.OPS) == 118
    assert len([o for o in regimes.OPS if o.endswith("_short")]) == 14


def test_chain_grammar_count():
    # chains.py: 2 norms x 2 residual x 19 epilogues = 76 names (tests/test_cpu.py:61-64)
    from oracle.ops import ACTNAMES
    assert len(ACTNAMES) == 19
    names = {("add_" if r else "") + ("rmsnorm" if n == "rms" else "layernorm") + "_" + a
             for n in ("rms", "layer") for r in (False, True) for a in ACTNAMES}
    assert len(names) == 76
    assert names <= set(regimes.OPS)


def test_epilogues_finite_on_wide_range():
    # chains.py epilogues are finite on [-30, 30] (tests/test_cpu.py:74-79)
    from oracle.ops import act, ACTNAMES
    t = np.linspace(-30, 30, 257, dtype=np.float32)
    for a in ACTNAMES:
        assert np.isfinite(act(a, t)).all(), a
