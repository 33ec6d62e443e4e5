"""Op name -> `run` function, one entry per op of ouroboros/specs.py SPECS
(29 explicit ops, 75 chain ops registered at specs.py:1001-1017, and the 14
*_short variants of specs.py:974-997, which share their base op's `run`).

`get_op(name)` mirrors specs.get_spec (specs.py:875-878): unknown names raise
KeyError listing the known ones.
"""
from __future__ import annotations

from . import ops

ACTNAMES = ["gelu", "silu", "relu2", "tanh", "sigmoid", "relu", "square",
            "abs", "softsign", "hardsigmoid", "hardswish",
            "leaky_relu", "relu6", "hardtanh", "elu", "selu", "softplus", "mish", "gelu_erf"]

SHORT_BASES = ["rmsnorm", "softmax", "layernorm_gelu", "add_layernorm_sigmoid",
               "add_layernorm_tanh", "add_layernorm_silu", "add_layernorm_gelu",
               "layernorm_sigmoid", "layernorm_tanh", "rmsnorm_silu", "add_rmsnorm_silu",
               "add_rmsnorm_sigmoid", "add_layernorm_square", "add_rmsnorm_gelu"]

# which C-ABI entry point backs each explicit op
ENTRY = {
    "rmsnorm": "b2k_norm", "add_rmsnorm": "b2k_norm", "layernorm": "b2k_norm",
    "add_layernorm": "b2k_norm", "l2norm": "b2k_norm", "layernorm_gelu": "b2k_norm",
    "rmsnorm_gemma": "b2k_norm", "rmsnorm_wide": "b2k_norm",
    "softmax": "b2k_softmax", "softcap_softmax": "b2k_softmax", "log_softmax": "b2k_softmax",
    "softmax_scale": "b2k_softmax",
    "swiglu": "b2k_glu", "glu": "b2k_glu", "geglu": "b2k_glu", "reglu": "b2k_glu",
    "gelu": "b2k_act", "silu": "b2k_act", "relu2": "b2k_act", "bias_gelu": "b2k_act",
    "dequant_int8": "b2k_dequant_i8",
    "rope": "b2k_rope", "rope_interleaved": "b2k_rope",
    "qknorm_rope": "b2k_norm_rope", "add_rmsnorm_rope": "b2k_norm_rope",
    "cross_entropy": "b2k_cross_entropy",
    "cumsum": "b2k_cumsum", "entropy": "b2k_entropy", "kl_div": "b2k_kl_div",
}


def _build():
    table = {name: getattr(ops, name) for name in ENTRY}
    for norm in ("rms", "layer"):
        for residual in (False, True):
            for act in ACTNAMES:
                name = ("add_" if residual else "") + ("rmsnorm" if norm == "rms" else "layernorm") \
                    + "_" + act
                if name not in table:
                    table[name] = ops.make_chain(norm, residual, act)
                    ENTRY[name] = "b2k_norm"
    for base in SHORT_BASES:
        table[base + "_short"] = table[base]
        ENTRY[base + "_short"] = ENTRY[base]
    return table


OPS = _build()


def get_op(name: str):
    if name not in OPS:
        raise KeyError(f"unknown op {name!r}; have {sorted(OPS)}")
    return OPS[name]


def candidate_source(name: str, package_dir: str) -> str:
    """Source of a harness candidate for op `name`: a module defining
    `run(*inputs)` that forwards to b200k (ouroboros/harness.py:135-148
    imports such a source and calls its `run`)."""
    get_op(name)
    return (f"import sys as _sys\n"
            f"_sys.path.insert(0, {package_dir!r})\n"
            f"import b200k as _b2k\n"
            f"_run = _b2k.get_op({name!r})\n\n"
            f"def run(*inputs):\n"
            f"    return _run(*inputs)\n")
