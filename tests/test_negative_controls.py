"""Negative controls of the reference's self-test (ouroboros/harness.py:326-345,
seed_kernels/*_wrong.py): plausible-but-wrong versions of the ops, planted
in the oracle on the CPU, must be REJECTED by the same golden vectors and
tolerances that the CUDA kernels pass.  This proves the parity checks
discriminate (a wrong kernel cannot pass by tolerance slack)."""
import numpy as np
import pytest

from golden_io import load
from oracle import ops as O
from oracle.numerics import allclose_report, rnd, tol_for

import os, sys
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_golden import build_case  # noqa: E402

F = np.float32


def _mean(a):
    return np.mean(a, axis=-1, keepdims=True, dtype=np.float32)


def _exp(a):
    with np.errstate(over="ignore", invalid="ignore"):
        return np.exp(a)


def w_rmsnorm(a, dt):            # no rsqrt: multiplies by the mean square
    x, w = a
    return rnd(rnd(x * _mean(x * x), dt) * w, dt)


def w_softmax(a, dt):            # no max subtraction
    e = _exp(a[0])
    with np.errstate(invalid="ignore"):
        return rnd(e / e.sum(-1, keepdims=True), dt)


def w_add_rmsnorm(a, dt):        # statistic from x alone, output (x + r)
    x, r, w = a
    h = x + r
    return rnd(rnd(h / np.sqrt(_mean(x * x) + F(1e-6)), dt) * w, dt)


def w_rope(a, dt):               # rotate_half without the negation
    x, c, s = a
    h = x.shape[-1] // 2
    return rnd(x * c + np.concatenate([x[..., h:], x[..., :h]], -1) * s, dt)


def w_layernorm(a, dt):          # no mean subtraction
    x, w, b = a
    return rnd(x / np.sqrt(_mean(x * x) + F(1e-5)) * w + b, dt)


def w_add_layernorm(a, dt):      # statistics from x alone
    x, r, w, b = a
    mu = _mean(x)
    var = _mean((x - mu) ** 2)
    return rnd((x + r - mu) / np.sqrt(var + F(1e-5)) * w + b, dt)


def w_geglu(a, dt):              # SiLU instead of GELU
    g, u = a
    return O.swiglu(g, u, dt)


def w_softcap(a, dt):            # no cap
    return w_softmax_stable(a[0], dt)


def w_softmax_stable(x, dt):
    return O.softmax(x, dt)


def w_gemma(a, dt):              # drops the +1
    x, w = a
    return rnd(x / np.sqrt(_mean(x * x) + F(1e-6)) * w, dt)


def w_glu(a, dt):                # silu instead of sigmoid
    return O.swiglu(a[0], a[1], dt)


def w_rope_inter(a, dt):         # drops the negation
    x, c, s = a
    out = np.empty_like(x)
    out[..., 0::2] = x[..., 0::2] * c + x[..., 1::2] * s
    out[..., 1::2] = x[..., 1::2] * c + x[..., 0::2] * s
    return rnd(out, dt)


def w_cross_entropy(a, dt):      # logsumexp without max subtraction
    x, t = a
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        lse = np.log(_exp(x).sum(-1))
    tt = np.where(t == -100, 0, t)
    loss = lse - np.take_along_axis(x, tt[:, None].astype(np.int64), -1)[:, 0]
    return rnd(np.where(t == -100, 0, loss), dt)


def w_cumsum(a, dt):             # no carry across blocks of 1024
    x = a[0].astype(np.float64)
    out = np.empty_like(x)
    for c0 in range(0, x.shape[-1], 1024):
        out[:, c0:c0 + 1024] = np.cumsum(x[:, c0:c0 + 1024], -1)
    return rnd(out, dt)


def w_entropy(a, dt):            # no max subtraction
    x = a[0]
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        s = _exp(x).sum(-1, keepdims=True)
        p = _exp(x) / s
        return rnd(np.log(s)[:, 0] - (x * p).sum(-1), dt)


def w_kl(a, dt):                 # second logsumexp not max-subtracted
    x, y = a
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        m = x.max(-1, keepdims=True)
        lx = x - (m + np.log(_exp(x - m).sum(-1, keepdims=True)))
        ly = y - np.log(_exp(y).sum(-1, keepdims=True))
        return rnd((np.exp(lx) * (lx - ly)).sum(-1), dt)


def w_qknorm_rope(a, dt):        # rms scale dropped on the rotated half
    x, w, c, s = a
    rs = 1 / np.sqrt(_mean(x * x) + F(1e-6))
    n = x * rs * w
    h = x.shape[-1] // 2
    raw = x * w
    rot = np.concatenate([-raw[..., h:], raw[..., :h]], -1)
    return rnd(n * c + rot * s, dt)


def w_relu2(a, dt):              # relu without the square
    return rnd(np.maximum(a[0], 0), dt)


def w_gelu(a, dt):               # silu instead of gelu
    return O.silu(a[0], dt)


def w_silu(a, dt):               # relu instead of silu
    return rnd(np.maximum(a[0], 0), dt)


WRONG = {
    "rmsnorm": w_rmsnorm, "softmax": w_softmax, "add_rmsnorm": w_add_rmsnorm, "rope": w_rope,
    "layernorm": w_layernorm, "add_layernorm": w_add_layernorm, "geglu": w_geglu,
    "softcap_softmax": w_softcap, "rmsnorm_gemma": w_gemma, "glu": w_glu,
    "rope_interleaved": w_rope_inter, "cross_entropy": w_cross_entropy, "cumsum": w_cumsum,
    "entropy": w_entropy, "kl_div": w_kl, "qknorm_rope": w_qknorm_rope, "relu2": w_relu2,
    "gelu": w_gelu, "silu": w_silu,
}


@pytest.mark.parametrize("op", sorted(WRONG))
def test_wrong_version_is_rejected(op):
    rejected = False
    for rec, ref in load(op):
        case = build_case(rec)
        vals = [v.astype(np.int64) if t == "i64" else v for v, t in case]
        out = WRONG[op](vals, rec["dt"])
        ok, _, _ = allclose_report(out, ref, *tol_for(op, rec["dt"]))
        rejected |= not ok
    assert rejected, f"the planted mistake in {op} passed every golden case"
