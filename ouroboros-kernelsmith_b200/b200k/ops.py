"""Spec-signature ops: each function is a drop-in `run(*inputs) -> Tensor`
for the op of the same name in ouroboros/specs.py (SPECS, specs.py:666-872)
and the chain grammar (ouroboros/chains.py:69-87), backed by libb200k.so.

Contract (ouroboros/harness.py:166-202): inputs are CUDA tensors that are
never written; the result is a fresh tensor of the reference's shape and
dtype; the launch goes on the current CUDA stream and nothing synchronises
the host.  Unsupported inputs raise (TypeError / ValueError); a failed kernel
launch raises B200KError.  There is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import torch

from . import _lib as L

_DT = {torch.float32: L.F32, torch.float16: L.F16, torch.bfloat16: L.BF16}


# --------------------------------------------------------------------------
# plumbing
def _dtype_id(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"b200k: unsupported dtype {t.dtype}; expected float32/float16/bfloat16")


def _cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError("b200k: every operand must be a CUDA tensor (no CPU path exists)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"b200k: operands on different devices ({dev} vs {t.device})")
    return dev


def _same_dtype(x, *ts):
    for t in ts:
        if t is not None and t.dtype != x.dtype:
            raise TypeError(f"b200k: operand dtype {t.dtype} differs from {x.dtype}; the kernels "
                            "take one floating dtype per call")


def _rows(t: torch.Tensor, n: int):
    """View t as (rows, n) with unit inner stride; returns (2-D tensor, row stride)."""
    if t.dim() == 0:
        raise ValueError("b200k: expected at least one dimension")
    if t.shape[-1] != n:
        raise ValueError(f"b200k: last dimension {t.shape[-1]} != {n}")
    if t.dim() == 2 and (t.stride(1) == 1 or n <= 1):
        return t, (t.stride(0) if t.shape[0] > 1 else n)
    t2 = t.reshape(-1, n)
    if t2.stride(-1) != 1 and n > 1:
        t2 = t2.contiguous()
    return t2, (t2.stride(0) if t2.shape[0] > 1 else n)


def _vec(t: torch.Tensor, n: int, what: str) -> torch.Tensor:
    if t.numel() != n:
        raise ValueError(f"b200k: {what} has {t.numel()} elements, expected {n}")
    if t.dim() == 1 and (n <= 1 or t.stride(0) == 1):
        return t
    t = t.reshape(n)
    return t if t.is_contiguous() else t.contiguous()


# the raw cudaStream_t of a device's current stream without building a
# torch.cuda.Stream object (about 0.3 against 4 us per call)
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


class _dev:
    """Makes t's device current for the call (the library launches on the
    current device) and yields the raw current stream handle."""

    __slots__ = ("device", "guard")

    def __init__(self, device: torch.device):
        self.device = device
        self.guard = None

    def __enter__(self):
        idx = self.device.index
        if torch.cuda.current_device() != idx:
            self.guard = torch.cuda.device(self.device)
            self.guard.__enter__()
        if _raw_stream is not None:
            return _raw_stream(idx)
        return torch.cuda.current_stream(self.device).cuda_stream

    def __exit__(self, *exc):
        if self.guard is not None:
            self.guard.__exit__(*exc)
        return False


def _p(t):
    return None if t is None else t.data_ptr()


# --------------------------------------------------------------------------
# norm family (b2k_norm)
def norm_chain(x, residual, w, b, *, norm: int, affine: int, act: int, eps: float,
               want_h: bool = False):
    """[x + residual] -> norm -> affine -> act; returns y, or (h, y) with
    want_h (h = T(x + residual), the residual stream)."""
    dev = _cuda(x, residual, w, b)
    _same_dtype(x, residual, w, b)
    dt = _dtype_id(x)
    n = x.shape[-1]
    x2, ldx = _rows(x, n)
    m = x2.shape[0]
    if residual is not None:
        if residual.shape != x.shape:
            raise ValueError(f"b200k: residual shape {tuple(residual.shape)} != {tuple(x.shape)}")
        r2, ldr = _rows(residual, n)
    else:
        r2, ldr = None, 0
    w1 = _vec(w, n, "weight") if w is not None else None
    b1 = _vec(b, n, "bias") if b is not None else None
    y = torch.empty((m, n), dtype=x.dtype, device=dev)
    h = torch.empty((m, n), dtype=x.dtype, device=dev) if want_h else None
    with _dev(dev) as stream:
        st = L.lib.b2k_norm(_p(x2), ldx, _p(r2), ldr, _p(w1), _p(b1), _p(y), n, _p(h), n,
                            m, n, dt, norm, affine, act, eps, stream)
    L.check(st, "b2k_norm")
    if x.dim() != 2:
        y = y.view(x.shape)
        h = h.view(x.shape) if want_h else None
    return (h, y) if want_h else y


def rmsnorm(x, w):
    """specs.py:75-78 / :667-678: T(T(x*rsqrt(mean(x^2)+1e-6)) * w)."""
    return norm_chain(x, None, w, None, norm=L.NORM_RMS, affine=L.AFF_W_ROUNDED, act=0, eps=1e-6)


def add_rmsnorm(x, residual, w):
    """specs.py:90-93 / :701-712."""
    return norm_chain(x, residual, w, None, norm=L.NORM_RMS, affine=L.AFF_W_ROUNDED, act=0,
                      eps=1e-6)


def layernorm(x, w, b):
    """specs.py:105-112 / :725-736."""
    return norm_chain(x, None, w, b, norm=L.NORM_LN, affine=L.AFF_WB, act=0, eps=1e-5)


def add_layernorm(x, residual, w, b):
    """specs.py:115-120 / :737-748."""
    return norm_chain(x, residual, w, b, norm=L.NORM_LN, affine=L.AFF_WB, act=0, eps=1e-5)


def l2norm(x):
    """specs.py:171-173 / :788-790: x * rsqrt(sum(x^2) + 1e-6)."""
    return norm_chain(x, None, None, None, norm=L.NORM_L2, affine=L.AFF_NONE, act=0, eps=1e-6)


def layernorm_gelu(x, w, b):
    """specs.py:184-190 / :798-801: gelu_tanh(LayerNorm(x)*w + b)."""
    return norm_chain(x, None, w, b, norm=L.NORM_LN, affine=L.AFF_WB, act=L.ACT["gelu"],
                      eps=1e-5)


def rmsnorm_gemma(x, w):
    """specs.py:216-220 / :818-823: x*rsqrt(mean(x^2)+1e-6)*(1+w)."""
    return norm_chain(x, None, w, None, norm=L.NORM_RMS, affine=L.AFF_ONE_PLUS_W, act=0,
                      eps=1e-6)


def rmsnorm_wide(x, w):
    """specs.py:866-871: rmsnorm at tall-skinny shapes (M small, N huge)."""
    return rmsnorm(x, w)


def make_chain(norm: str, residual: bool, act: str):
    """The `run` of one chains.py grammar op (chains.py:69-87): [x + r] ->
    {rms (eps 1e-6) | layer (eps 1e-5)} -> *w (+b) -> act -> x.dtype."""
    a = L.ACT[act]
    if norm == "rms":
        if residual:
            def run(x, residual, w):
                return norm_chain(x, residual, w, None, norm=L.NORM_RMS, affine=L.AFF_W, act=a,
                                  eps=1e-6)
        else:
            def run(x, w):
                return norm_chain(x, None, w, None, norm=L.NORM_RMS, affine=L.AFF_W, act=a,
                                  eps=1e-6)
    else:
        if residual:
            def run(x, residual, w, b):
                return norm_chain(x, residual, w, b, norm=L.NORM_LN, affine=L.AFF_WB, act=a,
                                  eps=1e-5)
        else:
            def run(x, w, b):
                return norm_chain(x, None, w, b, norm=L.NORM_LN, affine=L.AFF_WB, act=a,
                                  eps=1e-5)
    run.__name__ = ("add_" if residual else "") + ("rmsnorm" if norm == "rms" else "layernorm") \
        + "_" + act
    run.__doc__ = f"chains.py:69-87 op {run.__name__}"
    return run


def fused_add_norm(x, residual, w, b=None, *, norm: str = "layer", act: str = "gelu",
                   eps: float | None = None):
    """Residual add + norm + epilogue that also returns the residual stream:
    (h, y) with h = T(x + residual), y = act(norm(h)*w (+b)).  The chain math
    of chains.py:69-87 with the sum written once for the next block."""
    if norm == "layer":
        return norm_chain(x, residual, w, b, norm=L.NORM_LN, affine=L.AFF_WB, act=L.ACT[act],
                          eps=1e-5 if eps is None else eps, want_h=True)
    if norm == "rms":
        return norm_chain(x, residual, w, None, norm=L.NORM_RMS, affine=L.AFF_W, act=L.ACT[act],
                          eps=1e-6 if eps is None else eps, want_h=True)
    raise ValueError(f"b200k: norm must be 'layer' or 'rms', got {norm!r}")


# --------------------------------------------------------------------------
# softmax family (b2k_softmax)
def _softmax_call(x, kind, scale=None):
    dev = _cuda(x, scale)
    dt = _dtype_id(x)
    n = x.shape[-1]
    x2, ldx = _rows(x, n)
    m = x2.shape[0]
    y = torch.empty((m, n), dtype=x.dtype, device=dev)
    sdt = 0
    if scale is not None:
        if scale.numel() < 1:
            raise ValueError("b200k: scale must hold one element")
        sdt = _dtype_id(scale)
        scale = scale.reshape(-1)[:1].contiguous()
    with _dev(dev) as stream:
        st = L.lib.b2k_softmax(_p(x2), ldx, _p(y), n, m, n, dt, kind, _p(scale), sdt, stream)
    L.check(st, "b2k_softmax")
    return y.view(x.shape)


def softmax(x):
    """specs.py:81-82 / :679-689."""
    return _softmax_call(x, L.SOFTMAX)


def softcap_softmax(x):
    """specs.py:210-213 / :813-817 (cap 30)."""
    return _softmax_call(x, L.SOFTCAP)


def log_softmax(x):
    """specs.py:176-177 / :791-793."""
    return _softmax_call(x, L.LOG_SOFTMAX)


def softmax_scale(x, scale):
    """specs.py:180-181 / :794-797; scale is a 1-element device tensor (read on
    the device, no host sync)."""
    return _softmax_call(x, L.SOFTMAX_SCALE, scale)


# --------------------------------------------------------------------------
# gated and pointwise (b2k_glu, b2k_act)
def _glu_call(gate, up, act):
    dev = _cuda(gate, up)
    _same_dtype(gate, up)
    if gate.shape != up.shape:
        raise ValueError(f"b200k: gate {tuple(gate.shape)} and up {tuple(up.shape)} differ")
    dt = _dtype_id(gate)
    n = gate.shape[-1]
    g2, ldg = _rows(gate, n)
    u2, ldu = _rows(up, n)
    m = g2.shape[0]
    y = torch.empty((m, n), dtype=gate.dtype, device=dev)
    with _dev(dev) as stream:
        st = L.lib.b2k_glu(_p(g2), ldg, _p(u2), ldu, _p(y), n, m, n, dt, act, stream)
    L.check(st, "b2k_glu")
    return y.view(gate.shape)


def swiglu(gate, up):
    """specs.py:85-87 / :690-700: silu(gate) * up."""
    return _glu_call(gate, up, L.ACT["silu"])


def glu(gate, up):
    """specs.py:223-225 / :824-826: sigmoid(gate) * up."""
    return _glu_call(gate, up, L.ACT["sigmoid"])


def geglu(gate, up):
    """specs.py:126-130 / :749-759: gelu_tanh(gate) * up."""
    return _glu_call(gate, up, L.ACT["gelu"])


def reglu(gate, up):
    """specs.py:167-168 / :785-787: relu(gate) * up."""
    return _glu_call(gate, up, L.ACT["relu"])


def _act_call(x, act, bias=None):
    dev = _cuda(x, bias)
    _same_dtype(x, bias)
    dt = _dtype_id(x)
    n = x.shape[-1]
    x2, ldx = _rows(x, n)
    m = x2.shape[0]
    b1 = _vec(bias, n, "bias") if bias is not None else None
    y = torch.empty((m, n), dtype=x.dtype, device=dev)
    with _dev(dev) as stream:
        st = L.lib.b2k_act(_p(x2), ldx, _p(b1), _p(y), n, m, n, dt, act, stream)
    L.check(st, "b2k_act")
    return y.view(x.shape)


def gelu(x):
    """specs.py:147-149 / :775."""
    return _act_call(x, L.ACT["gelu"])


def silu(x):
    """specs.py:152-154 / :778."""
    return _act_call(x, L.ACT["silu"])


def relu2(x):
    """specs.py:157-159 / :780."""
    return _act_call(x, L.ACT["relu2"])


def bias_gelu(x, bias):
    """specs.py:162-164 / :782: gelu_tanh(x + bias)."""
    return _act_call(x, L.ACT["gelu"], bias)


def dequant_int8(q, scale):
    """specs.py:201-203 / :808-811: (q.float() * scale.float()).to(float16)."""
    dev = _cuda(q, scale)
    if q.dtype != torch.int8:
        raise TypeError(f"b200k: dequant_int8 expects int8 q, got {q.dtype}")
    sdt = _dtype_id(scale)
    n = q.shape[-1]
    q2, ldq = _rows(q, n)
    m = q2.shape[0]
    if scale.numel() != m:
        raise ValueError(f"b200k: scale has {scale.numel()} elements for {m} rows")
    s2 = scale.reshape(m, 1)
    lds = s2.stride(0) if m > 1 else 1
    y = torch.empty((m, n), dtype=torch.float16, device=dev)
    with _dev(dev) as stream:
        st = L.lib.b2k_dequant_i8(_p(q2), ldq, _p(s2), lds, sdt, _p(y), n, m, n, stream)
    L.check(st, "b2k_dequant_i8")
    return y.view(q.shape)


# --------------------------------------------------------------------------
# rotary embeddings (b2k_rope, b2k_rope_qk, b2k_norm_rope)
def _rope_call(x, cos, sin, interleaved):
    dev = _cuda(x, cos, sin)
    _same_dtype(x, cos, sin)
    dt = _dtype_id(x)
    d = x.shape[-1]
    if d % 2:
        raise ValueError(f"b200k: head dim must be even, got {d}")
    tw = d // 2 if interleaved else d
    x2, ldx = _rows(x, d)
    c2, ldc = _rows(cos, tw)
    s2, lds = _rows(sin, tw)
    m = x2.shape[0]
    if c2.shape[0] != m or s2.shape[0] != m:
        raise ValueError("b200k: cos/sin must have one row per row of x")
    y = torch.empty((m, d), dtype=x.dtype, device=dev)
    with _dev(dev) as stream:
        st = L.lib.b2k_rope(_p(x2), ldx, _p(c2), ldc, _p(s2), lds, _p(y), d, m, d, dt,
                            1 if interleaved else 0, stream)
    L.check(st, "b2k_rope")
    return y.view(x.shape)


def rope(x, cos, sin):
    """specs.py:96-102 / :713-724: x*cos + rotate_half(x)*sin, tables (M,D)."""
    return _rope_call(x, cos, sin, False)


def rope_interleaved(x, cos, sin):
    """specs.py:228-236 / :827-832: GPT-J pairs, tables (M,D/2)."""
    return _rope_call(x, cos, sin, True)


def rope_qk(q, k, cos, sin, interleaved: bool = False):
    """RoPE of q [B,S,H,D] and k [B,S,Hk,D] in one launch from position tables
    cos, sin [S, D/2] (row s for position s); returns fresh (q_out, k_out).
    The attention-layout form of rope / rope_interleaved (specs.py:96-102,
    :228-236) with the half-split tables of a real model."""
    dev = _cuda(q, k, cos, sin)
    _same_dtype(q, k, cos, sin)
    dt = _dtype_id(q)
    if q.dim() != 4 or k.dim() != 4:
        raise ValueError("b200k: rope_qk expects q, k of shape [B, S, H, D]")
    B, S, H, D = q.shape
    if k.shape[0] != B or k.shape[1] != S or k.shape[3] != D:
        raise ValueError(f"b200k: k {tuple(k.shape)} does not match q {tuple(q.shape)}")
    if D % 2 or tuple(cos.shape) != (S, D // 2) or tuple(sin.shape) != (S, D // 2):
        raise ValueError(f"b200k: tables must be [S, D/2] = [{S}, {D // 2}]")
    q, k = q.contiguous(), k.contiguous()
    cos, sin = cos.contiguous(), sin.contiguous()
    qo = torch.empty_like(q)
    ko = torch.empty_like(k)
    with _dev(dev) as stream:
        st = L.lib.b2k_rope_qk(_p(q), _p(k), _p(cos), _p(sin), _p(qo), _p(ko), B, S, H,
                               k.shape[2], D, dt, 1 if interleaved else 0, stream)
    L.check(st, "b2k_rope_qk")
    return qo, ko


def _norm_rope_call(x, residual, w, cos, sin):
    dev = _cuda(x, residual, w, cos, sin)
    _same_dtype(x, residual, w, cos, sin)
    dt = _dtype_id(x)
    d = x.shape[-1]
    if d % 2:
        raise ValueError(f"b200k: head dim must be even, got {d}")
    x2, ldx = _rows(x, d)
    m = x2.shape[0]
    if residual is not None:
        if residual.shape != x.shape:
            raise ValueError("b200k: residual shape differs from x")
        r2, ldr = _rows(residual, d)
    else:
        r2, ldr = None, 0
    w1 = _vec(w, d, "weight")
    c2, ldc = _rows(cos, d)
    s2, lds = _rows(sin, d)
    if c2.shape[0] != m or s2.shape[0] != m:
        raise ValueError("b200k: cos/sin must have one row per row of x")
    y = torch.empty((m, d), dtype=x.dtype, device=dev)
    with _dev(dev) as stream:
        st = L.lib.b2k_norm_rope(_p(x2), ldx, _p(r2), ldr, _p(w1), _p(c2), ldc, _p(s2), lds,
                                 _p(y), d, m, d, dt, 1e-6, stream)
    L.check(st, "b2k_norm_rope")
    return y.view(x.shape)


def qknorm_rope(x, w, cos, sin):
    """specs.py:133-143 / :760-773: rmsnorm over D (*w) then rotate_half RoPE."""
    return _norm_rope_call(x, None, w, cos, sin)


def add_rmsnorm_rope(x, residual, w, cos, sin):
    """specs.py:193-198 / :802-807: residual add, rmsnorm, RoPE."""
    return _norm_rope_call(x, residual, w, cos, sin)


# --------------------------------------------------------------------------
# row reductions (b2k_cross_entropy, b2k_cumsum, b2k_entropy, b2k_kl_div)
def _check_tgt(tgt, m, dev):
    if tgt.dtype != torch.int64:
        raise TypeError(f"b200k: targets must be int64, got {tgt.dtype}")
    if tgt.numel() != m:
        raise ValueError(f"b200k: {tgt.numel()} targets for {m} rows")
    if tgt.device != dev:
        raise ValueError("b200k: targets on another device")
    return tgt.reshape(m).contiguous()


def cross_entropy(x, tgt, ignore_index: int = -100):
    """specs.py:239-241 / :833-838: per-row logsumexp(x) - x[tgt] in x.dtype;
    0 for rows whose target is ignore_index (torch's default -100)."""
    dev = _cuda(x, tgt)
    dt = _dtype_id(x)
    n = x.shape[-1]
    x2, ldx = _rows(x, n)
    m = x2.shape[0]
    t1 = _check_tgt(tgt, m, dev)
    out = torch.empty((m,), dtype=x.dtype, device=dev)
    with _dev(dev) as stream:
        st = L.lib.b2k_cross_entropy(_p(x2), ldx, _p(t1), _p(out), m, n, dt, dt, ignore_index,
                                     stream)
    L.check(st, "b2k_cross_entropy")
    return out.view(x.shape[:-1])


def cumsum(x):
    """specs.py:245-248 / :840-849: row-wise inclusive prefix sum."""
    dev = _cuda(x)
    dt = _dtype_id(x)
    n = x.shape[-1]
    x2, ldx = _rows(x, n)
    m = x2.shape[0]
    y = torch.empty((m, n), dtype=x.dtype, device=dev)
    with _dev(dev) as stream:
        st = L.lib.b2k_cumsum(_p(x2), ldx, _p(y), n, m, n, dt, stream)
    L.check(st, "b2k_cumsum")
    return y.view(x.shape)


def entropy(x):
    """specs.py:251-256 / :850-859: entropy of softmax(x) per row."""
    dev = _cuda(x)
    dt = _dtype_id(x)
    n = x.shape[-1]
    x2, ldx = _rows(x, n)
    m = x2.shape[0]
    out = torch.empty((m,), dtype=x.dtype, device=dev)
    with _dev(dev) as stream:
        st = L.lib.b2k_entropy(_p(x2), ldx, _p(out), m, n, dt, stream)
    L.check(st, "b2k_entropy")
    return out.view(x.shape[:-1])


def kl_div(x, y):
    """specs.py:259-265 / :860-864: KL(softmax(x) || softmax(y)) per row."""
    dev = _cuda(x, y)
    _same_dtype(x, y)
    if x.shape != y.shape:
        raise ValueError("b200k: x and y shapes differ")
    dt = _dtype_id(x)
    n = x.shape[-1]
    x2, ldx = _rows(x, n)
    y2, ldy = _rows(y, n)
    m = x2.shape[0]
    out = torch.empty((m,), dtype=x.dtype, device=dev)
    with _dev(dev) as stream:
        st = L.lib.b2k_kl_div(_p(x2), ldx, _p(y2), ldy, _p(out), m, n, dt, stream)
    L.check(st, "b2k_kl_div")
    return out.view(x.shape[:-1])


def cross_entropy_mean(logits, tgt, ignore_index: int = -100, group=None):
    """Mean cross-entropy over the rows whose target is not ignore_index, as a
    0-dim fp32 tensor on the logits' device.  With a process group, `logits`
    and `tgt` are this rank's row shard and the mean is over all ranks' rows
    (one NCCL all-reduce of [loss sum, valid count]).  Per-row losses are the
    spec op's (specs.py:239-241) in fp32; their sum is accumulated in fp64 in
    a fixed order."""
    from .dist import XCHG_LIMIT_NS, allreduce_sumcount, ce_exchange
    dev = _cuda(logits, tgt)
    dt = _dtype_id(logits)
    n = logits.shape[-1]
    x2, ldx = _rows(logits, n)
    m = x2.shape[0]
    t1 = _check_tgt(tgt, m, dev)
    row_loss = torch.empty((m,), dtype=torch.float32, device=dev)
    sumcount = torch.empty((2,), dtype=torch.float64, device=dev)
    out = torch.empty((), dtype=torch.float32, device=dev)
    xchg = ce_exchange(group, dev)
    with _dev(dev) as stream:
        st = L.lib.b2k_cross_entropy(_p(x2), ldx, _p(t1), _p(row_loss), m, n, dt, L.F32,
                                     ignore_index, stream)
        L.check(st, "b2k_cross_entropy")
        if xchg is not None:
            # reduce + exchange over peer memory + mean, one kernel; a failure
            # reported by an earlier call raises here (sticky on the device)
            xchg.raise_if_failed()
            L.check(L.lib.b2k_ce_reduce_exchange_mean(
                _p(row_loss), _p(t1), m, ignore_index, _p(xchg.peers), xchg.rank, xchg.world,
                XCHG_LIMIT_NS, _p(sumcount), _p(out), _p(xchg.status), stream),
                "b2k_ce_reduce_exchange_mean")
            xchg.after_launch()
            return out
        L.check(L.lib.b2k_ce_reduce(_p(row_loss), _p(t1), m, ignore_index, _p(sumcount), stream),
                "b2k_ce_reduce")
    allreduce_sumcount(sumcount, group)
    with _dev(dev) as stream:
        L.check(L.lib.b2k_ce_mean(_p(sumcount), _p(out), stream), "b2k_ce_mean")
    return out


def cross_entropy_fwd_bwd(logits, tgt, ignore_index: int = -100, group=None,
                          grad_scale: float = 1.0, inplace: bool = False):
    """Mean cross-entropy over valid rows AND its gradient w.r.t. the logits
    in one pass over the logits: returns (loss 0-dim fp32, dlogits) with
    dlogits = grad_scale * d(mean loss)/d logits in the logits' dtype
    (0 for ignored rows).  With a process group, logits/tgt are this rank's
    row shard; the valid count and the loss sum are summed over the ranks
    (over peer memory where the exchange is set up, else NCCL all-reduces)
    so the loss and gradient are those of the global mean.  inplace=True writes
    the gradient over the logits (the memory-saving form of fused CE)."""
    from .dist import XCHG_LIMIT_NS, allreduce_sumcount, ce_exchange
    dev = _cuda(logits, tgt)
    dt = _dtype_id(logits)
    n = logits.shape[-1]
    x2, ldx = _rows(logits, n)
    m = x2.shape[0]
    t1 = _check_tgt(tgt, m, dev)
    if inplace and not (x2.data_ptr() == logits.data_ptr() and logits.is_contiguous()):
        raise ValueError("b200k: inplace gradient needs contiguous logits")
    dx = x2 if inplace else torch.empty((m, n), dtype=logits.dtype, device=dev)
    lddx = ldx if inplace else n
    count = torch.empty((2,), dtype=torch.float64, device=dev)
    row_loss = torch.empty((m,), dtype=torch.float32, device=dev)
    sumcount = torch.empty((2,), dtype=torch.float64, device=dev)
    out = torch.empty((), dtype=torch.float32, device=dev)
    xchg = ce_exchange(group, dev)
    with _dev(dev) as stream:
        L.check(L.lib.b2k_ce_valid_count(_p(t1), m, ignore_index, _p(count), stream),
                "b2k_ce_valid_count")
    count[1:].zero_()
    if xchg is not None:
        # the global valid count and, after the kernel, the loss sum: both
        # over peer memory (no collective library on the step)
        xchg.raise_if_failed()
        count_g = torch.empty((2,), dtype=torch.float64, device=dev)
        with _dev(dev) as stream:
            L.check(L.lib.b2k_exchange_pair(_p(count), _p(xchg.peers), xchg.rank, xchg.world,
                                            XCHG_LIMIT_NS, _p(count_g), _p(xchg.status), stream),
                    "b2k_exchange_pair")
        count = count_g
    else:
        allreduce_sumcount(count, group)
    with _dev(dev) as stream:
        L.check(L.lib.b2k_cross_entropy_fwd_bwd(_p(x2), ldx, _p(t1), m, n, dt, ignore_index,
                                                _p(count), grad_scale, _p(row_loss), _p(dx),
                                                lddx, stream), "b2k_cross_entropy_fwd_bwd")
        if xchg is not None:
            L.check(L.lib.b2k_ce_reduce_exchange_mean(
                _p(row_loss), _p(t1), m, ignore_index, _p(xchg.peers), xchg.rank, xchg.world,
                XCHG_LIMIT_NS, _p(sumcount), _p(out), _p(xchg.status), stream),
                "b2k_ce_reduce_exchange_mean")
            xchg.after_launch()
            return out, dx.view(logits.shape)
        L.check(L.lib.b2k_ce_reduce(_p(row_loss), _p(t1), m, ignore_index, _p(sumcount), stream),
                "b2k_ce_reduce")
    allreduce_sumcount(sumcount, group)
    with _dev(dev) as stream:
        L.check(L.lib.b2k_ce_mean(_p(sumcount), _p(out), stream), "b2k_ce_mean")
    return out, dx.view(logits.shape)
