"""Op table and seeded input regimes of the suite — TEST INFRASTRUCTURE ONLY.

Restates, device-independently, what ouroboros/specs.py defines per op:
the input kind of each op (specs._grid_kind, specs.py:890-915), the
adversarial random regimes (_DTYPES/_SCALES/_ROWLEN/_NROWS/_HEADDIM,
specs.py:56-59,401; tall-skinny specs.py:544-548), the deterministic stress
cases (specs.py:291-315,413-476,562-597,615-641,655-658) and the bench
shapes (specs.py:321, :353-356, short variants :974-997).  The reference
builds its inputs with a CUDA torch.Generator; here every tensor comes from
numpy's PCG64 with the same shapes, dtypes and magnitudes, so the cases run
anywhere.  A case is a list of (values, tag) pairs: float inputs as float32
arrays of exactly representable values, tag in {f32, f16, bf16, i8, i64}.
"""
from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Callable

import numpy as np

from . import ops as O
from .numerics import rnd

_DTYPES = ["f16", "bf16", "f32"]
_SCALES = [1.0, 8.0, 64.0]
_ROWLEN = [128, 512, 1024, 4096, 4097, 8192]
_NROWS = [8, 64, 1000, 4096]
_HEADDIM = [64, 128, 256]
_TALL_M = [4, 8, 16, 32]
_WIDE_N = [16384, 32768, 65536, 131072]

ROPE_FAMILY = {"rope", "rope_interleaved", "qknorm_rope", "add_rmsnorm_rope"}


@dataclass
class OpInfo:
    name: str
    kind: str
    oracle: Callable  # (list of value arrays, dtype tag) -> output values
    base: str         # op whose semantics this is (name without _short)


def _chain_oracle(norm, residual, act):
    return lambda a, dt: O.chain(norm, residual, act, a, dt)


def _build_ops() -> dict[str, OpInfo]:
    e = {}

    def add(name, kind, fn):
        e[name] = OpInfo(name, kind, fn, name)

    add("rmsnorm", "rms", lambda a, dt: O.rmsnorm(a[0], a[1], dt))
    add("softmax", "x", lambda a, dt: O.softmax(a[0], dt))
    add("swiglu", "gate_up", lambda a, dt: O.swiglu(a[0], a[1], dt))
    add("add_rmsnorm", "add_rms", lambda a, dt: O.add_rmsnorm(a[0], a[1], a[2], dt))
    add("rope", "rope", lambda a, dt: O.rope(a[0], a[1], a[2], dt))
    add("layernorm", "ln", lambda a, dt: O.layernorm(a[0], a[1], a[2], dt))
    add("add_layernorm", "add_ln", lambda a, dt: O.add_layernorm(a[0], a[1], a[2], a[3], dt))
    add("geglu", "gate_up", lambda a, dt: O.geglu(a[0], a[1], dt))
    add("qknorm_rope", "qkr", lambda a, dt: O.qknorm_rope(a[0], a[1], a[2], a[3], dt))
    add("gelu", "x", lambda a, dt: O.gelu(a[0], dt))
    add("silu", "x", lambda a, dt: O.silu(a[0], dt))
    add("relu2", "x", lambda a, dt: O.relu2(a[0], dt))
    add("bias_gelu", "x_bias", lambda a, dt: O.bias_gelu(a[0], a[1], dt))
    add("reglu", "gate_up", lambda a, dt: O.reglu(a[0], a[1], dt))
    add("l2norm", "x", lambda a, dt: O.l2norm(a[0], dt))
    add("log_softmax", "x", lambda a, dt: O.log_softmax(a[0], dt))
    add("softmax_scale", "x_scale", lambda a, dt: O.softmax_scale(a[0], a[1], dt))
    add("layernorm_gelu", "ln", lambda a, dt: O.layernorm_gelu(a[0], a[1], a[2], dt))
    add("add_rmsnorm_rope", "arr", lambda a, dt: O.add_rmsnorm_rope(a[0], a[1], a[2], a[3], a[4], dt))
    add("dequant_int8", "int8", lambda a, dt: O.dequant_int8(a[0], a[1]))
    add("softcap_softmax", "x", lambda a, dt: O.softcap_softmax(a[0], dt))
    add("rmsnorm_gemma", "rms", lambda a, dt: O.rmsnorm_gemma(a[0], a[1], dt))
    add("glu", "gate_up", lambda a, dt: O.glu(a[0], a[1], dt))
    add("rope_interleaved", "rope_inter", lambda a, dt: O.rope_interleaved(a[0], a[1], a[2], dt))
    add("cross_entropy", "ce", lambda a, dt: O.cross_entropy(a[0], a[1], dt))
    add("cumsum", "x", lambda a, dt: O.cumsum(a[0], dt))
    add("entropy", "x", lambda a, dt: O.entropy(a[0], dt))
    add("kl_div", "xy", lambda a, dt: O.kl_div(a[0], a[1], dt))
    add("rmsnorm_wide", "rms_wide", lambda a, dt: O.rmsnorm(a[0], a[1], dt))
    # chain grammar, chains.py:172-181 (layernorm_gelu is explicit above)
    for norm in ("rms", "layer"):
        for residual in (False, True):
            for act in O.ACTNAMES:
                name = ("add_" if residual else "") + ("rmsnorm" if norm == "rms" else "layernorm") \
                    + "_" + act
                if name in e:
                    continue
                kind = ("add_" if residual else "") + ("rms" if norm == "rms" else "ln")
                add(name, kind, _chain_oracle(norm, residual, act))
    # short-row variants, specs.py:974-997: same op, bench pinned to 16384x2048
    for base in SHORT_BASES:
        b = e[base]
        e[base + "_short"] = OpInfo(base + "_short", b.kind, b.oracle, base)
    return e


SHORT_BASES = ["rmsnorm", "softmax", "layernorm_gelu", "add_layernorm_sigmoid",
               "add_layernorm_tanh", "add_layernorm_silu", "add_layernorm_gelu",
               "layernorm_sigmoid", "layernorm_tanh", "rmsnorm_silu", "add_rmsnorm_silu",
               "add_rmsnorm_sigmoid", "add_layernorm_square", "add_rmsnorm_gelu"]

OPS: dict[str, OpInfo] = _build_ops()


def reference(op: str, case) -> np.ndarray:
    """Oracle output of `op` on a case (list of (values, tag))."""
    info = OPS[op]
    vals = [v for v, _ in case]
    dt = case[0][1]
    if dt not in ("f16", "bf16", "f32"):
        dt = "f16"
    return info.oracle(vals, dt)


# ---------------------------------------------------------------- generators
def _randn(seed, shape, dt, scale):
    g = np.random.default_rng(seed)
    return rnd(g.standard_normal(shape, dtype=np.float32) * np.float32(scale), dt), dt


def _costab(seed, M, D, dt, full=True):
    g = np.random.default_rng(seed)
    ang = g.standard_normal((M, D // 2), dtype=np.float32)
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    if full:
        c, s = np.concatenate([c, c], -1), np.concatenate([s, s], -1)
    return (rnd(c, dt), dt), (rnd(s, dt), dt)


def make_case(kind: str, seed: int, M: int, N: int, dt: str, scale: float,
              aux_scale: float = 1.0, ignore_frac: float = 0.0):
    """Inputs of one case for an op of `kind`; N is the head dim for the rope
    kinds.  aux_scale is the magnitude of the second operand where the
    reference varies it (up/bias in the stress cases)."""
    s = seed * 16
    x = _randn(s, (M, N), dt, scale)
    if kind in ("x",):
        return [x]
    if kind in ("rms", "rms_wide"):
        return [x, _randn(s + 1, (N,), dt, 1.0)]
    if kind == "ln":
        return [x, _randn(s + 1, (N,), dt, 1.0), _randn(s + 2, (N,), dt, 1.0)]
    if kind == "add_rms":
        return [x, _randn(s + 3, (M, N), dt, scale), _randn(s + 1, (N,), dt, 1.0)]
    if kind == "add_ln":
        return [x, _randn(s + 3, (M, N), dt, scale), _randn(s + 1, (N,), dt, 1.0),
                _randn(s + 2, (N,), dt, 1.0)]
    if kind == "gate_up":
        return [x, _randn(s + 3, (M, N), dt, aux_scale)]
    if kind == "xy":
        return [x, _randn(s + 3, (M, N), dt, scale)]
    if kind == "x_bias":
        return [x, _randn(s + 1, (N,), dt, aux_scale)]
    if kind == "x_scale":
        g = np.random.default_rng(s + 1)
        return [x, (rnd(np.array([0.05 + g.random() * 1.5], dtype=np.float32), dt), dt)]
    if kind == "ce":
        g = np.random.default_rng(s + 4)
        t = g.integers(0, N, size=(M,), dtype=np.int64)
        if ignore_frac > 0:
            t[g.random(M) < ignore_frac] = -100
        return [x, (t, "i64")]
    if kind == "int8":
        g = np.random.default_rng(s)
        q = g.integers(-127, 127, size=(M, N), dtype=np.int64).astype(np.int8)
        g2 = np.random.default_rng(s + 1)
        sc = rnd((g2.random((M, 1), dtype=np.float32) * 0.05 + 0.005), "f16")
        return [(q.astype(np.float32), "i8"), (sc, "f16")]
    D = N
    if kind == "rope":
        c, sn = _costab(s + 5, M, D, dt)
        return [x, c, sn]
    if kind == "rope_inter":
        c, sn = _costab(s + 5, M, D, dt, full=False)
        return [x, c, sn]
    if kind == "qkr":
        c, sn = _costab(s + 5, M, D, dt)
        return [x, _randn(s + 1, (D,), dt, 1.0), c, sn]
    if kind == "arr":
        c, sn = _costab(s + 5, M, D, dt)
        return [x, _randn(s + 3, (M, D), dt, scale), _randn(s + 1, (D,), dt, 1.0), c, sn]
    raise KeyError(kind)


def stress_cases(op: str):
    """Deterministic hard cases (high magnitude, low precision, odd N)."""
    info = OPS[op]
    k = info.kind
    if k in ("rope", "rope_inter", "qkr", "arr"):
        dims = [(128, "f16"), (256, "bf16"), (64, "f16")] if k != "arr" else [(128, "f16"), (256, "bf16")]
        return [make_case(k, 700 + D, 37, D, dt, 64.0) for D, dt in dims]
    if k == "rms_wide":
        return [make_case(k, 90, 8, 131072, "f16", 64.0), make_case(k, 92, 5, 65537, "bf16", 32.0),
                make_case(k, 94, 16, 40000, "f16", 16.0)]
    if k == "int8":
        return [make_case(k, 71, 37, 4097, "f16", 1.0), make_case(k, 72, 3, 8192, "f16", 1.0)]
    aux = 8.0 if k == "gate_up" else (4.0 if k == "x_bias" else 1.0)
    out = [make_case(k, 91, 37, 4097, "f16", 64.0, aux), make_case(k, 92, 37, 4097, "bf16", 64.0, aux)]
    if k in ("x", "rms", "ce", "xy"):
        out.append(make_case(k, 93, 3, 8192, "f16", 32.0, aux))
    return out


def bench_shape(op: str):
    """(M, N) of the op's bench inputs."""
    info = OPS[op]
    if op.endswith("_short"):
        return 16384, 2048
    if info.kind in ("rope", "rope_inter", "qkr", "arr"):
        return 32768, 128
    if info.kind == "rms_wide":
        return 8, 131072
    return 8192, 4096


def bench_case(op: str, seed: int = 1):
    M, N = bench_shape(op)
    return make_case(OPS[op].kind, seed, M, N, "f16", 1.0)


def random_cases(op: str, n: int, seed: int = 0, max_elems: int | None = None):
    """n adversarial random cases (specs._mk_* regimes); max_elems caps M*N
    by shrinking M (row ops are row-independent, so fewer rows of the same
    width exercise the same code path)."""
    info = OPS[op]
    rng = random.Random(seed)
    out = []
    for i in range(n):
        k = info.kind
        if k in ("rope", "rope_inter", "qkr", "arr"):
            M, N = rng.choice(_NROWS), rng.choice(_HEADDIM)
        elif k == "rms_wide":
            M, N = rng.choice(_TALL_M), rng.choice(_WIDE_N)
        else:
            M, N = rng.choice(_NROWS), rng.choice(_ROWLEN)
        dt = rng.choice(_DTYPES) if k != "int8" else "f16"
        sc = rng.choice(_SCALES)
        if max_elems and M * N > max_elems:
            M = max(1, max_elems // N)
        out.append(make_case(k, rng.randrange(2 ** 31), M, N, dt, sc))
    return out
