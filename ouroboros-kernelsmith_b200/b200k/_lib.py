"""ctypes binding of libb200k.so (declared in include/b200k.h).

The library is loaded at import time from this package directory.  There is
no fallback: if the shared object is missing or fails to load, importing
b200k raises, so no op can silently run anywhere but the CUDA kernels.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_double, c_float, c_int, c_int64, c_void_p, POINTER

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libb200k.so")

# enum values mirrored from include/b200k.h
F32, F16, BF16, I8, I64 = 0, 1, 2, 3, 4
OK, EINVAL, EALIGN, ELAUNCH, EUNSUPPORTED = 0, 1, 2, 3, 4
NORM_RMS, NORM_L2, NORM_LN = 0, 1, 2
AFF_NONE, AFF_W_ROUNDED, AFF_W, AFF_ONE_PLUS_W, AFF_WB = 0, 1, 2, 3, 4
SOFTMAX, SOFTCAP, LOG_SOFTMAX, SOFTMAX_SCALE = 0, 1, 2, 3

# epilogue ids: the order of ouroboros/chains.py:56-58 (ACTNAMES), 0 = none
ACT_NAMES = ["none", "gelu", "silu", "relu2", "tanh", "sigmoid", "relu", "square",
             "abs", "softsign", "hardsigmoid", "hardswish", "leaky_relu", "relu6",
             "hardtanh", "elu", "selu", "softplus", "mish", "gelu_erf"]
ACT = {name: i for i, name in enumerate(ACT_NAMES)}

# name -> (restype, argtypes); every entry point of include/b200k.h
SIGNATURES = {
    "b2k_version": (c_int, []),
    "b2k_last_error": (ctypes.c_char_p, []),
    "b2k_pipeline_timeouts": (ctypes.c_uint, [c_int]),
    "b2k_selftest_bounded_wait": (c_int, [ctypes.c_ulonglong, c_void_p, c_void_p]),
    "b2k_norm": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                         c_int64, c_void_p, c_int64, c_int64, c_int64, c_int, c_int, c_int, c_int,
                         c_float, c_void_p]),
    "b2k_softmax": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int, c_int,
                            c_void_p, c_int, c_void_p]),
    "b2k_glu": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64,
                        c_int, c_int, c_void_p]),
    "b2k_act": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int,
                        c_int, c_void_p]),
    "b2k_dequant_i8": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_int64,
                               c_int64, c_int64, c_void_p]),
    "b2k_rope": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                         c_int64, c_int64, c_int, c_int, c_void_p]),
    "b2k_rope_qk": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                            c_int64, c_int64, c_int64, c_int64, c_int, c_int, c_void_p]),
    "b2k_norm_rope": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64,
                              c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int, c_float,
                              c_void_p]),
    "b2k_cross_entropy": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int,
                                  c_int, c_int64, c_void_p]),
    "b2k_ce_reduce": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "b2k_ce_mean": (c_int, [c_void_p, c_void_p, c_void_p]),
    "b2k_ce_exchange_bytes": (c_int64, [c_int]),
    "b2k_ce_exchange_alloc": (c_int, [c_int, c_void_p]),
    "b2k_ce_exchange_free": (c_int, [c_void_p]),
    "b2k_ipc_handle": (c_int, [c_void_p, c_void_p]),
    "b2k_ipc_open": (c_int, [c_void_p, c_void_p]),
    "b2k_ipc_close": (c_int, [c_void_p]),
    "b2k_ce_reduce_exchange_mean": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int,
                                            c_int, ctypes.c_ulonglong, c_void_p, c_void_p,
                                            c_void_p, c_void_p]),
    "b2k_exchange_pair": (c_int, [c_void_p, c_void_p, c_int, c_int, ctypes.c_ulonglong,
                                  c_void_p, c_void_p, c_void_p]),
    "b2k_ce_valid_count": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "b2k_cross_entropy_fwd_bwd": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int,
                                          c_int64, c_void_p, c_float, c_void_p, c_void_p,
                                          c_int64, c_void_p]),
    "b2k_cross_entropy_mean_noalloc": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64,
                                               c_int, c_int64, c_void_p, c_void_p]),
    "b2k_cumsum": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int,
                           c_void_p]),
    "b2k_entropy": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_void_p]),
    "b2k_kl_div": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int,
                           c_void_p]),
}


class B200KError(RuntimeError):
    """A libb200k entry point returned a non-zero status."""


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"b200k: {LIB_PATH} is missing; build it with `make -C "
            f"{os.path.join(os.path.dirname(_HERE), 'csrc')}` (no CPU fallback exists)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:  # reported by exported_symbols(); calling it raises
            continue
        fn.restype = res
        fn.argtypes = args
    return lib


def exported_symbols() -> dict:
    """{entry point: bool exported} for every name in SIGNATURES."""
    return {name: hasattr(lib, name) for name in SIGNATURES}


lib = _load()


def last_error() -> str:
    return (lib.b2k_last_error() or b"").decode("utf-8", "replace")


def check(status: int, what: str) -> None:
    if status != OK:
        raise B200KError(f"{what}: status {status}: {last_error()}")
