"""b200k — sm_100a (B200) CUDA kernels for the ouroboros-kernelsmith op suite.

Every op of ouroboros/specs.py and ouroboros/chains.py is available under its
spec name with the spec's `run` signature (see registry.OPS / get_op), plus
attention-layout RoPE (rope_qk), the fused residual-add+norm that also returns
the residual stream (fused_add_norm) and the reduced cross-entropy used for
training (cross_entropy_mean).  Importing the package loads libb200k.so; if
it is missing the import fails (there is no CPU fallback).
"""
from . import _lib
from ._lib import B200KError
from .ops import *  # noqa: F401,F403
from .ops import fused_add_norm, norm_chain, rope_qk, cross_entropy_mean, cross_entropy_fwd_bwd  # noqa: F401
from . import dist, host  # noqa: F401
from .registry import OPS, get_op, candidate_source  # noqa: F401

__all__ = ["OPS", "get_op", "candidate_source", "B200KError", "fused_add_norm", "rope_qk",
           "cross_entropy_mean", "cross_entropy_fwd_bwd", "dist", "host"]
__version__ = "0.1.0"
