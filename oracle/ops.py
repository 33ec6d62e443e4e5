"""CPU oracle for the op suite — TEST INFRASTRUCTURE ONLY.

A numpy restatement of every op of ouroboros/specs.py (references at
specs.py:75-265) and the chain grammar ouroboros/chains.py:13-87, in float32
with explicit storage rounding (numerics.rnd) wherever the reference casts
with `.to(dtype)`.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg use it, as the checker; the product path (b200k) never imports
it.  Pinned against outputs of the reference itself: tests/golden/ holds
vectors produced by importing ouroboros/specs.py on CPU (make_golden.py).

Every function takes float32 arrays holding the exact input values plus the
storage dtype tag of the inputs, and returns float32 values already rounded
to the output dtype.
"""
from __future__ import annotations

import numpy as np

from .numerics import rnd

try:  # gelu_erf needs erf; scipy ships in the image
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover
    import math
    _erf = np.vectorize(math.erf, otypes=[np.float32])

F = np.float32
_GELU_C = F(0.7978845608028654)  # sqrt(2/pi), specs.py:123 / chains.py:10


def _f(a):
    return np.asarray(a, dtype=np.float32)


def _mean(a):
    return np.mean(a, axis=-1, keepdims=True, dtype=np.float32)


def _rsqrt(a):
    return (F(1.0) / np.sqrt(a)).astype(np.float32)


def _sigmoid(t):
    with np.errstate(over="ignore"):
        return (F(1.0) / (F(1.0) + np.exp(-t))).astype(np.float32)


def _gelu_tanh(t):
    return F(0.5) * t * (F(1.0) + np.tanh(_GELU_C * (t + F(0.044715) * t * t * t)))


def _softplus(t):  # chains.py:43 (threshold 20)
    with np.errstate(over="ignore"):
        return np.where(t > 20.0, t, np.log(F(1.0) + np.exp(np.minimum(t, F(20.0))))).astype(np.float32)


# epilogues, chains.py:13-53, in ACTNAMES order (chains.py:56-58)
ACTS = {
    "gelu": _gelu_tanh,
    "silu": lambda t: t * _sigmoid(t),
    "relu2": lambda t: np.maximum(t, F(0)) * np.maximum(t, F(0)),
    "tanh": np.tanh,
    "sigmoid": _sigmoid,
    "relu": lambda t: np.maximum(t, F(0)),
    "square": lambda t: t * t,
    "abs": np.abs,
    "softsign": lambda t: t / (F(1.0) + np.abs(t)),
    "hardsigmoid": lambda t: np.clip(t + F(3.0), F(0.0), F(6.0)) / F(6.0),
    "hardswish": lambda t: t * np.clip(t + F(3.0), F(0.0), F(6.0)) / F(6.0),
    "leaky_relu": lambda t: np.where(t > 0, t, F(0.01) * t),
    "relu6": lambda t: np.clip(t, F(0.0), F(6.0)),
    "hardtanh": lambda t: np.clip(t, F(-1.0), F(1.0)),
    "elu": lambda t: np.where(t > 0, t, np.exp(np.minimum(t, F(0.0))) - F(1.0)),
    "selu": lambda t: F(1.0507009873554805) * np.where(
        t > 0, t, F(1.6732632423543772) * (np.exp(np.minimum(t, F(0.0))) - F(1.0))),
    "softplus": _softplus,
    "mish": lambda t: t * np.tanh(_softplus(t)),
    "gelu_erf": lambda t: F(0.5) * t * (F(1.0) + _erf(t * F(0.7071067811865476)).astype(np.float32)),
}
ACTNAMES = ["gelu", "silu", "relu2", "tanh", "sigmoid", "relu", "square",
            "abs", "softsign", "hardsigmoid", "hardswish",
            "leaky_relu", "relu6", "hardtanh", "elu", "selu", "softplus", "mish", "gelu_erf"]


def act(name, t):
    with np.errstate(over="ignore", invalid="ignore"):
        return _f(ACTS[name](_f(t)))


# ---------------------------------------------------------------- norms
def rmsnorm(x, w, dt, eps=1e-6):
    """specs.py:75-78: (xf*rsqrt(mean(xf^2)+eps)).to(dt) * w  (product in dt)."""
    xf = _f(x)
    rs = _rsqrt(_mean(xf * xf) + F(eps))
    return rnd(rnd(xf * rs, dt) * _f(w), dt)


def add_rmsnorm(x, r, w, dt, eps=1e-6):
    """specs.py:90-93."""
    h = _f(x) + _f(r)
    rs = _rsqrt(_mean(h * h) + F(eps))
    return rnd(rnd(h * rs, dt) * _f(w), dt)


def _ln(h, w, b, eps):
    mu = _mean(h)
    hc = h - mu
    var = _mean(hc * hc)
    return hc * _rsqrt(var + F(eps)) * _f(w) + _f(b)


def layernorm(x, w, b, dt, eps=1e-5):
    """specs.py:105-112."""
    return rnd(_ln(_f(x), w, b, eps), dt)


def add_layernorm(x, r, w, b, dt, eps=1e-5):
    """specs.py:115-120."""
    return rnd(_ln(_f(x) + _f(r), w, b, eps), dt)


def l2norm(x, dt, eps=1e-6):
    """specs.py:171-173."""
    xf = _f(x)
    return rnd(xf * _rsqrt(np.sum(xf * xf, axis=-1, keepdims=True, dtype=np.float32) + F(eps)), dt)


def layernorm_gelu(x, w, b, dt, eps=1e-5):
    """specs.py:184-190."""
    return rnd(_gelu_tanh(_ln(_f(x), w, b, eps)), dt)


def rmsnorm_gemma(x, w, dt, eps=1e-6):
    """specs.py:216-220."""
    xf = _f(x)
    return rnd(xf * _rsqrt(_mean(xf * xf) + F(eps)) * (F(1.0) + _f(w)), dt)


def chain(norm, residual, actname, args, dt):
    """chains.py:69-87 (eps 1e-6 rms / 1e-5 layer), output in args[0]'s dtype."""
    if residual and norm == "rms":
        x, r, w = args; h = _f(x) + _f(r); b = None
    elif residual:
        x, r, w, b = args; h = _f(x) + _f(r)
    elif norm == "rms":
        x, w = args; h = _f(x); b = None
    else:
        x, w, b = args; h = _f(x)
    if norm == "rms":
        n = h * _rsqrt(_mean(h * h) + F(1e-6)) * _f(w)
    else:
        n = _ln(h, w, b, 1e-5)
    return rnd(act(actname, n), dt)


# ---------------------------------------------------------------- softmax family
def _softmax(t):
    m = np.max(t, axis=-1, keepdims=True)
    e = np.exp(t - m)
    return e / np.sum(e, axis=-1, keepdims=True, dtype=np.float32)


def softmax(x, dt):
    """specs.py:81-82."""
    return rnd(_softmax(_f(x)), dt)


def softcap_softmax(x, dt):
    """specs.py:210-213 (cap 30)."""
    t = F(30.0) * np.tanh(_f(x) / F(30.0))
    return rnd(_softmax(t), dt)


def log_softmax(x, dt):
    """specs.py:176-177."""
    t = _f(x)
    m = np.max(t, axis=-1, keepdims=True)
    lse = m + np.log(np.sum(np.exp(t - m), axis=-1, keepdims=True, dtype=np.float32))
    return rnd(t - lse, dt)


def softmax_scale(x, scale, dt):
    """specs.py:180-181: softmax(x * scale[0])."""
    return rnd(_softmax(_f(x) * _f(scale).reshape(-1)[0]), dt)


# ---------------------------------------------------------------- pointwise / gated
def swiglu(g, u, dt):
    """specs.py:85-87."""
    gf = _f(g)
    return rnd(gf * _sigmoid(gf) * _f(u), dt)


def glu(g, u, dt):
    """specs.py:223-225."""
    return rnd(_sigmoid(_f(g)) * _f(u), dt)


def geglu(g, u, dt):
    """specs.py:126-130."""
    return rnd(_gelu_tanh(_f(g)) * _f(u), dt)


def reglu(g, u, dt):
    """specs.py:167-168."""
    return rnd(np.maximum(_f(g), F(0)) * _f(u), dt)


def gelu(x, dt):
    """specs.py:147-149."""
    return rnd(_gelu_tanh(_f(x)), dt)


def silu(x, dt):
    """specs.py:152-154."""
    xf = _f(x)
    return rnd(xf * _sigmoid(xf), dt)


def relu2(x, dt):
    """specs.py:157-159."""
    r = np.maximum(_f(x), F(0))
    return rnd(r * r, dt)


def bias_gelu(x, bias, dt):
    """specs.py:162-164."""
    return rnd(_gelu_tanh(_f(x) + _f(bias)), dt)


def dequant_int8(q, scale, dt=None):
    """specs.py:201-203: (q.float() * scale.float()).to(float16)."""
    return rnd(_f(q) * _f(scale).reshape(-1, 1), "f16")


# ---------------------------------------------------------------- rope
def rope(x, cos, sin, dt):
    """specs.py:96-102: x*cos + cat(-x2, x1)*sin."""
    xf = _f(x)
    h = xf.shape[-1] // 2
    rot = np.concatenate([-xf[..., h:], xf[..., :h]], axis=-1)
    return rnd(xf * _f(cos) + rot * _f(sin), dt)


def rope_interleaved(x, cos, sin, dt):
    """specs.py:228-236."""
    xf = _f(x)
    x1, x2 = xf[..., 0::2], xf[..., 1::2]
    c, s = _f(cos), _f(sin)
    out = np.empty_like(xf)
    out[..., 0::2] = x1 * c - x2 * s
    out[..., 1::2] = x2 * c + x1 * s
    return rnd(out, dt)


def qknorm_rope(x, w, cos, sin, dt, eps=1e-6):
    """specs.py:133-143."""
    xf = _f(x)
    n = xf * _rsqrt(_mean(xf * xf) + F(eps)) * _f(w)
    h = n.shape[-1] // 2
    rot = np.concatenate([-n[..., h:], n[..., :h]], axis=-1)
    return rnd(n * _f(cos) + rot * _f(sin), dt)


def add_rmsnorm_rope(x, r, w, cos, sin, dt, eps=1e-6):
    """specs.py:193-198."""
    hs = _f(x) + _f(r)
    n = hs * _rsqrt(_mean(hs * hs) + F(eps)) * _f(w)
    h = n.shape[-1] // 2
    rot = np.concatenate([-n[..., h:], n[..., :h]], axis=-1)
    return rnd(n * _f(cos) + rot * _f(sin), dt)


def rope_qk_tables(q, k, cos_t, sin_t, dt, interleaved=False):
    """Attention-layout RoPE: q [B,S,H,D], k [B,S,Hk,D], tables [S,D/2];
    position s uses table row s (the rope / rope_interleaved math above)."""
    S, half = cos_t.shape
    def one(t):
        c = _f(cos_t)[None, :, None, :]
        s = _f(sin_t)[None, :, None, :]
        tf = _f(t)
        if interleaved:
            out = np.empty_like(tf)
            out[..., 0::2] = tf[..., 0::2] * c - tf[..., 1::2] * s
            out[..., 1::2] = tf[..., 1::2] * c + tf[..., 0::2] * s
            return rnd(out, dt)
        cc = np.concatenate([c, c], axis=-1)
        ss = np.concatenate([s, s], axis=-1)
        rot = np.concatenate([-tf[..., half:], tf[..., :half]], axis=-1)
        return rnd(tf * cc + rot * ss, dt)
    return one(q), one(k)


# ---------------------------------------------------------------- reductions
def cross_entropy(x, tgt, dt, ignore_index=-100):
    """specs.py:239-241: F.cross_entropy(x.float(), t, reduction='none').to(dt);
    rows whose target equals ignore_index (torch's default -100) give 0."""
    xf = _f(x)
    t = np.asarray(tgt, dtype=np.int64)
    m = np.max(xf, axis=-1)
    lse = m + np.log(np.sum(np.exp(xf - m[:, None]), axis=-1, dtype=np.float32))
    valid = t != ignore_index
    tt = np.where(valid, t, 0)
    picked = np.take_along_axis(xf, tt[:, None], axis=-1)[:, 0]
    loss = np.where(valid, lse - picked, F(0.0)).astype(np.float32)
    return rnd(loss, dt)


def cross_entropy_sum_count(x, tgt, ignore_index=-100):
    """(sum of fp32 per-row losses in fp64, number of valid rows)."""
    loss = cross_entropy(x, tgt, "f32", ignore_index)
    valid = np.asarray(tgt) != ignore_index
    return float(np.sum(loss[valid], dtype=np.float64)), int(valid.sum())


def cumsum(x, dt):
    """specs.py:245-248 (torch's CPU cumsum accumulates float in double)."""
    return rnd(np.cumsum(_f(x).astype(np.float64), axis=-1), dt)


def entropy(x, dt):
    """specs.py:251-256."""
    xf = _f(x)
    m = np.max(xf, axis=-1, keepdims=True)
    lse = m + np.log(np.sum(np.exp(xf - m), axis=-1, keepdims=True, dtype=np.float32))
    p = np.exp(xf - lse)
    return rnd(lse[:, 0] - np.sum(xf * p, axis=-1, dtype=np.float32), dt)


def kl_div(x, y, dt):
    """specs.py:259-265."""
    def lsm(t):
        m = np.max(t, axis=-1, keepdims=True)
        return t - (m + np.log(np.sum(np.exp(t - m), axis=-1, keepdims=True, dtype=np.float32)))
    lx, ly = lsm(_f(x)), lsm(_f(y))
    return rnd(np.sum(np.exp(lx) * (lx - ly), axis=-1, dtype=np.float32), dt)


def cross_entropy_grad(x, tgt, dt, grad_scale=1.0, ignore_index=-100):
    """d(grad_scale * mean over valid rows of cross_entropy(x, t)) / dx, the
    backward of specs.py:239-241 under a mean reduction: (softmax(x) -
    onehot(t)) * grad_scale / n_valid, 0 on rows whose target is ignore_index."""
    xf = _f(x)
    t = np.asarray(tgt, dtype=np.int64)
    valid = t != ignore_index
    n = max(int(valid.sum()), 1)
    m = np.max(xf, axis=-1, keepdims=True)
    e = np.exp(xf - m)
    p = e / np.sum(e, axis=-1, keepdims=True, dtype=np.float32)
    rows = np.nonzero(valid)[0]
    p[rows, t[rows]] -= F(1.0)
    p[~valid] = F(0.0)
    return rnd(p * F(grad_scale / n), dt)
