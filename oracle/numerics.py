"""Storage-precision helpers for the oracle (TEST INFRASTRUCTURE ONLY).

Values are carried as numpy float32 arrays; a dtype tag ("f32", "f16",
"bf16") says which storage type they model.  `rnd(a, dt)` is the value after
a `.to(dtype)` in the reference (round to nearest even).  Nothing here is
used by the product path.
"""
from __future__ import annotations

import numpy as np

DTYPES = ("f16", "bf16", "f32")


def bf16_round(a: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bfloat16 value, returned as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.nan
    return out


def f16_round(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def rnd(a: np.ndarray, dt: str) -> np.ndarray:
    """Value of `a` after storage in dtype dt."""
    a = np.asarray(a, dtype=np.float32)
    if dt == "f32":
        return a
    if dt == "f16":
        return f16_round(a)
    if dt == "bf16":
        return bf16_round(a)
    raise ValueError(dt)


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """uint16 storage of values already representable in bfloat16."""
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# allclose tolerances (rtol, atol) used by the parity tests: the element-wise
# minimum of the harness tolerance (ouroboros/specs.py:41-45) and the
# tolerance the op suite is accepted at (fp16 1e-2, bf16 2e-2).
TOL = {"f32": (2e-4, 2e-5), "f16": (1e-2, 2e-3), "bf16": (2e-2, 8e-3)}


def tol_for(op: str, dt: str) -> tuple[float, float]:
    """Per-op overrides of specs.py:849 (cumsum fp32) and :859 (entropy fp32)."""
    if dt == "f32" and op == "cumsum":
        return (2e-4, 5e-3)
    if dt == "f32" and op == "entropy":
        return (2e-4, 2e-2)
    return TOL[dt]


def allclose_report(out: np.ndarray, ref: np.ndarray, rtol: float, atol: float):
    """(ok, max_abs_err, n_bad) with torch.allclose semantics (NaN != NaN)."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if out.shape != ref.shape:
        return False, float("inf"), -1
    with np.errstate(invalid="ignore"):
        d = np.abs(out - ref)
        bad = ~(d <= atol + rtol * np.abs(ref))
        # equal infinities are close (torch.allclose)
        same_inf = np.isinf(out) & np.isinf(ref) & (np.sign(out) == np.sign(ref))
        bad &= ~same_inf
    finite = d[np.isfinite(d)]
    err = float(finite.max()) if finite.size else 0.0
    if np.isnan(d).any():
        err = float("nan")
    return (not bad.any()), err, int(bad.sum())
