"""GPU parity beyond the spec cases: attention-layout RoPE, the reduced
cross-entropy, the fused residual-stream output, strided and misaligned
views (scalar kernel paths), edge shapes, long rows (streaming kernels),
and the harness import path of a generated candidate."""
import importlib.util
import os

import numpy as np
import pytest
import torch

import b200k
from b200k import _lib, registry
from gpu_util import TDT, to_cuda
from oracle import ops as O
from oracle import regimes
from oracle.numerics import allclose_report, rnd, tol_for

pytestmark = pytest.mark.gpu
DTS = ["f16", "bf16", "f32"]


def _close(out, ref, dt, op="x"):
    ok, err, bad = allclose_report(out.float().cpu().numpy(), ref, *tol_for(op, dt))
    assert ok, f"max err {err}, {bad} bad"


def _randn(shape, dt, scale, seed):
    g = np.random.default_rng(seed)
    return rnd(g.standard_normal(shape, dtype=np.float32) * np.float32(scale), dt)


def _t(a, dt):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().to(TDT[dt])


# ---------------------------------------------------------------- rope_qk
@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("inter", [False, True])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_rope_qk_small(dt, inter, D):
    B, S, H, Hk = 2, 33, 4, 2
    q = _randn((B, S, H, D), dt, 4.0, 1)
    k = _randn((B, S, Hk, D), dt, 4.0, 2)
    ang = np.arange(S, dtype=np.float32)[:, None] * (
        10000.0 ** (-np.arange(0, D, 2, dtype=np.float32) / D))[None, :]
    c, s = rnd(np.cos(ang), dt), rnd(np.sin(ang), dt)
    qo, ko = b200k.rope_qk(_t(q, dt), _t(k, dt), _t(c, dt), _t(s, dt), interleaved=inter)
    torch.cuda.synchronize()
    rq, rk = O.rope_qk_tables(q, k, c, s, dt, interleaved=inter)
    _close(qo, rq, dt)
    _close(ko, rk, dt)


@pytest.mark.parametrize("inter", [False, True])
def test_rope_qk_llama_shape_sampled(inter):
    """q [8,4096,32,128], k [8,4096,8,128] bf16; positions sampled."""
    B, S, H, Hk, D = 8, 4096, 32, 8, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn((B, S, H, D), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((B, S, Hk, D), generator=g, device="cuda").to(torch.bfloat16)
    inv = 10000.0 ** (-torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D)
    ang = torch.arange(S, device="cuda", dtype=torch.float32)[:, None] * inv[None, :]
    c, s = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    qo, ko = b200k.rope_qk(q, k, c, s, interleaved=inter)
    torch.cuda.synchronize()
    bs = [0, 3, 7]
    ss = [0, 1, 2047, 4095]
    for b in bs:
        qn = q[b, ss].float().cpu().numpy()[None]
        kn = k[b, ss].float().cpu().numpy()[None]
        rq, rk = O.rope_qk_tables(qn, kn, c[ss].float().cpu().numpy(), s[ss].float().cpu().numpy(),
                                  "bf16", interleaved=inter)
        _close(qo[b, ss][None], rq, "bf16")
        _close(ko[b, ss][None], rk, "bf16")


# ---------------------------------------------------------------- reduced CE
@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("shape", [(37, 4097), (256, 32000), (64, 128256)])
def test_cross_entropy_mean(dt, shape):
    M, V = shape
    case = regimes.make_case("ce", 11, M, V, dt, 3.0, ignore_frac=0.05)
    x, t = to_cuda(case)
    got = float(b200k.cross_entropy_mean(x, t))
    s, c = O.cross_entropy_sum_count(case[0][0], case[1][0].astype(np.int64))
    want = s / c
    assert abs(got - want) <= 1e-3 * abs(want), (got, want)


def test_cross_entropy_edge_targets():
    x = _t(_randn((4, 300), "f32", 3.0, 5), "f32")
    t = torch.tensor([5, -100, 299, 300], device="cuda", dtype=torch.int64)
    out = b200k.cross_entropy(x, t).cpu().numpy()
    ref = O.cross_entropy(x.cpu().numpy()[:3], t.cpu().numpy()[:3], "f32")
    assert np.allclose(out[:3], ref, rtol=2e-4, atol=2e-5)
    assert out[1] == 0.0
    assert np.isnan(out[3])  # target outside [0, V) and not ignore_index
    allign = torch.full((4,), -100, device="cuda", dtype=torch.int64)
    assert np.isnan(float(b200k.cross_entropy_mean(x, allign)))


# ---------------------------------------------------------------- residual stream
@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("norm", ["layer", "rms"])
@pytest.mark.parametrize("N", [8192, 4097, 1024])
def test_fused_add_norm(dt, norm, N):
    M = 19
    x, r = _randn((M, N), dt, 8.0, 1), _randn((M, N), dt, 8.0, 2)
    w, b = _randn((N,), dt, 1.0, 3), _randn((N,), dt, 1.0, 4)
    h, y = b200k.fused_add_norm(_t(x, dt), _t(r, dt), _t(w, dt), _t(b, dt), norm=norm,
                                act="gelu")
    torch.cuda.synchronize()
    assert np.array_equal(h.float().cpu().numpy(), rnd(x + r, dt))
    args = [x, r, w, b] if norm == "layer" else [x, r, w]
    _close(y, O.chain(norm, True, "gelu", args, dt), dt)


# ---------------------------------------------------------------- views
@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("op", ["rmsnorm", "add_layernorm_silu", "softmax", "log_softmax",
                                "swiglu", "gelu", "cross_entropy", "cumsum", "entropy", "kl_div",
                                "rope", "rope_interleaved"])
@pytest.mark.parametrize("view", ["strided", "offset"])
def test_non_contiguous_views(dt, op, view):
    """Row-strided views and bases shifted by one element (16-byte alignment
    lost) must give the same results through the scalar paths."""
    info = regimes.OPS[op]
    N = 64 if "rope" in op else 2048
    case = regimes.make_case(info.kind, 21, 9, N, dt, 8.0)
    base = to_cuda(case)
    args = []
    for (v, tag), t in zip(case, base):
        if t.dim() == 2 and t.shape[0] == 9 and t.is_floating_point():
            if view == "strided":
                big = torch.zeros((9, t.shape[1] + 24), dtype=t.dtype, device="cuda")
                big[:, 8:8 + t.shape[1]] = t
                t = big[:, 8:8 + t.shape[1]]
            else:
                flat = torch.zeros(t.numel() + 1, dtype=t.dtype, device="cuda")
                flat[1:] = t.reshape(-1)
                t = flat[1:].view(t.shape)
        args.append(t)
    out = b200k.get_op(op)(*args)
    torch.cuda.synchronize()
    _close(out, regimes.reference(op, case), dt, op)


# ---------------------------------------------------------------- shapes
@pytest.mark.parametrize("op", ["rmsnorm", "layernorm_gelu", "softmax", "softcap_softmax",
                                "entropy", "kl_div", "cumsum", "cross_entropy", "l2norm"])
@pytest.mark.parametrize("N", [1, 2, 3, 70000])
def test_edge_and_long_rows(op, N):
    info = regimes.OPS[op]
    dt = "bf16"
    case = regimes.make_case(info.kind, 31, 3, N, dt, 4.0)
    out = b200k.get_op(op)(*to_cuda(case))
    torch.cuda.synchronize()
    _close(out, regimes.reference(op, case), dt, op)


def test_empty_inputs():
    x = torch.empty((0, 64), device="cuda", dtype=torch.float16)
    w = torch.ones(64, device="cuda", dtype=torch.float16)
    assert b200k.rmsnorm(x, w).shape == (0, 64)
    assert b200k.softmax(x).shape == (0, 64)
    assert b200k.swiglu(x, x).shape == (0, 64)


# ---------------------------------------------------------------- drop-in
def test_candidate_imports_like_the_harness(tmp_path):
    """Write a generated candidate to a file and import it the way
    ouroboros/harness.py:135-148 does (preamble + source, `run` attribute),
    then apply the harness contract: fresh output, inputs untouched, and a
    poked input changes the next result (no memoisation)."""
    pkg = os.path.dirname(os.path.dirname(b200k.__file__))
    src = "import torch\n\n" + registry.candidate_source("softmax", pkg)
    path = tmp_path / "cand_softmax.py"
    path.write_text(src)
    spec = importlib.util.spec_from_file_location("cand_softmax", str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    case = regimes.stress_cases("softmax")[0]
    (x,) = to_cuda(case)
    clone = x.clone()
    y1 = mod.run(clone)
    assert torch.equal(clone, x) and y1.data_ptr() != clone.data_ptr()
    clone.view(-1)[0] = 1000.0  # dominates row 0 at any stress magnitude
    y2 = mod.run(clone)
    ref = O.softmax(clone.float().cpu().numpy(), "f16")
    _close(y2, ref, "f16")
    assert not torch.equal(y1, y2)
    torch.cuda.synchronize()
    assert _lib.lib.b2k_pipeline_timeouts(1) == 0


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_cross_entropy_nonfinite_logits_give_nan(dt):
    """A NaN or +inf logit anywhere in a row makes that row's loss NaN, as in
    F.cross_entropy (checked on CPU: all three rows NaN), in the first chunk of
    a row, a later one, and the last."""
    V = 40000  # long enough for the pipelined kernel
    x = torch.zeros(6, V, dtype=dt, device="cuda")
    x[0, 8] = float("nan")
    x[1, 20013] = float("nan")
    x[2, 16] = float("inf")
    x[3, V - 1] = float("nan")
    x[4, 39001] = float("inf")
    tgt = torch.tensor([1, 1, 1, 1, 1, 2], device="cuda")
    loss = b200k.cross_entropy(x, tgt).float().cpu()
    assert torch.isnan(loss[:5]).all(), loss
    assert abs(float(loss[5]) - float(np.log(V))) < 2e-2 * float(np.log(V))
    _, g = b200k.cross_entropy_fwd_bwd(x, tgt)
    assert torch.isnan(g[0].float()).any() and torch.isfinite(g[5].float()).all()


# ------------------------------------------------- fallback kernel mappings
@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("D", [96, 128])
def test_qknorm_rope_general_kernel(dt, D):
    """qknorm_rope / add_rmsnorm_rope through the general shared-memory kernel:
    rows with a stride of D + 1 elements (never 16-byte aligned), starting at
    element 0 or 1, and D = 96 (half a row is not a power-of-two number of
    vectors).  Contiguous power-of-two head dims (the per-lane both-halves
    kernel) are covered by the parity cases."""
    M = 77
    x = _randn((M, D + 1), dt, 3.0, 41)
    r = _randn((M, D + 1), dt, 3.0, 42)
    w = _randn((D,), dt, 1.0, 43)
    c = _randn((M, D), dt, 1.0, 44)
    s = _randn((M, D), dt, 1.0, 45)
    for off in (0, 1):  # off = 1: misaligned row starts
        xv, rv = x[:, off:off + D], r[:, off:off + D]
        got = b200k.qknorm_rope(_t(x, dt)[:, off:off + D], _t(w, dt), _t(c, dt), _t(s, dt))
        _close(got, O.qknorm_rope(xv, w, c, s, dt), dt, "qknorm_rope")
        got = b200k.add_rmsnorm_rope(_t(x, dt)[:, off:off + D], _t(r, dt)[:, off:off + D],
                                     _t(w, dt), _t(c, dt), _t(s, dt))
        _close(got, O.add_rmsnorm_rope(xv, rv, w, c, s, dt), dt, "add_rmsnorm_rope")


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_rope_qk_interleaved_8byte_tables(dt):
    """Interleaved q/k RoPE whose tables are 8- but not 16-byte aligned (a view
    offset by 4 entries) takes the split-vector mapping with 8-byte table
    loads; aligned tables take the adjacent-vector mapping.  Both against the
    oracle."""
    B, S, H, Hk, D = 2, 17, 3, 1, 128
    q = _randn((B, S, H, D), dt, 4.0, 51)
    k = _randn((B, S, Hk, D), dt, 4.0, 52)
    ang = np.arange(S, dtype=np.float32)[:, None] * (
        10000.0 ** (-np.arange(0, D, 2, dtype=np.float32) / D))[None, :]
    c, s = rnd(np.cos(ang), dt), rnd(np.sin(ang), dt)
    def shifted(a):  # contiguous, storage starting 4 entries (8 bytes) into a buffer
        flat = _t(np.concatenate([np.zeros(4, np.float32), a.ravel()]), dt)
        return flat[4:].view(a.shape)

    rq, rk = O.rope_qk_tables(q, k, c, s, dt, interleaved=True)
    for ct, st in ((_t(c, dt), _t(s, dt)), (shifted(c), shifted(s))):
        assert ct.is_contiguous()
        qo, ko = b200k.rope_qk(_t(q, dt), _t(k, dt), ct, st, interleaved=True)
        torch.cuda.synchronize()
        _close(qo, rq, dt)
        _close(ko, rk, dt)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_devices_in_one_process():
    """Per-device launch set-up (the raised shared-memory limit and the cached
    pipeline shape belong to each device's context): rows of 64 KB, whose
    pipeline needs more than 48 KB of shared memory, on cuda:0 then cuda:1."""
    x = _randn((512, 16384), "f32", 1.0, 5)
    w = _randn((16384,), "f32", 0.1, 6) + 1
    ref = O.rmsnorm(x, w, "f32")
    for d in (0, 1):
        xt = torch.from_numpy(x).to(f"cuda:{d}")
        wt = torch.from_numpy(w).to(f"cuda:{d}")
        y = b200k.rmsnorm(xt, wt)
        torch.cuda.synchronize(d)
        ok, err, bad = allclose_report(y.cpu().numpy(), ref, *tol_for("rmsnorm", "f32"))
        assert ok, f"cuda:{d}: max err {err}, {bad} bad"


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("M", [3, 700, 2000, 8000])
def test_cross_entropy_few_rows_per_block(dt, M):
    """Vocabulary-length rows with few rows per resident block (a shard of
    the logits on one of many GPUs, so the last round of rows leaves most
    blocks idle).  Sampled rows against the oracle, including
    ignored rows, a bad target (NaN) and targets in the first and last chunk
    of a row, plus the mean over all rows."""
    V = 128256
    g = torch.Generator(device="cuda").manual_seed(M)
    x = (torch.randn((M, V), generator=g, device="cuda") * 3).to(TDT[dt])
    t = torch.randint(0, V, (M,), generator=g, device="cuda")
    t[::17] = -100
    t[0] = 0
    if M > 2:
        t[1] = V - 1
        t[2] = V + 5  # outside [0, V): NaN
    out = b200k.cross_entropy(x, t)
    rows = np.unique(np.concatenate([[0, 1, M - 1], np.arange(0, M, max(1, M // 13))]))
    rows = rows[rows != 2] if M > 2 else rows
    xs = x[rows].float().cpu().numpy()
    ts = t[rows].cpu().numpy()
    ref = O.cross_entropy(xs, ts, dt)
    _close(out[rows], ref, dt)
    if M > 2:
        assert torch.isnan(out[2]).item()
        keep = torch.ones(M, dtype=torch.bool, device="cuda")
        keep[2] = False
        x, t = x[keep], t[keep]
    got = float(b200k.cross_entropy_mean(x, t))
    s, c = 0.0, 0
    for r in range(0, x.shape[0], 1024):
        s += float(torch.nn.functional.cross_entropy(x[r:r + 1024].float(), t[r:r + 1024],
                                                     ignore_index=-100, reduction="sum"))
        c += int((t[r:r + 1024] != -100).sum())
    assert abs(got - s / c) <= 1e-3 * abs(s / c), (got, s / c)


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("M,N,pad", [(1500, 1024, 0), (3000, 4096, 0), (5000, 2048, 64),
                                     (1300, 8192, 0), (2400, 1032, 8), (160000, 1024, 0)])
def test_cross_entropy_many_short_rows(dt, M, N, pad):
    """Many rows of 2..16 KB (the warp-per-row ring), strided rows among them,
    and 160000 rows so that each warp walks more than 64 rows (its window of
    read-ahead targets slides).  Ignored rows and out-of-range targets are
    never copied: 0 and NaN.  All rows against the fp32 torch expression,
    sampled rows against the oracle."""
    g = torch.Generator(device="cuda").manual_seed(M + N)
    base = (torch.randn((M, N + pad), generator=g, device="cuda") * 4).to(TDT[dt])
    x = base[:, :N]
    t = torch.randint(0, N, (M,), generator=g, device="cuda")
    t[::13] = -100
    t[0] = 0
    t[1] = N - 1
    t[5::97] = N + 3  # outside [0, N): NaN
    t[7::101] = -7
    out = b200k.cross_entropy(x, t)
    bad = (t != -100) & ((t < 0) | (t >= N))
    assert torch.isnan(out[bad]).all().item()
    ok = ~bad
    xf = x.float()
    ref = torch.logsumexp(xf, dim=1) - xf.gather(1, t.clamp(0, N - 1)[:, None])[:, 0]
    ref = torch.where(t == -100, torch.zeros_like(ref), ref)
    _close(out[ok].float(), ref[ok].to(TDT[dt]).float().cpu().numpy(), dt)
    rows = np.arange(0, M, max(1, M // 29))
    rows = rows[ok.cpu().numpy()[rows]]
    _close(out[rows], O.cross_entropy(x[rows].float().cpu().numpy(), t[rows].cpu().numpy(), dt), dt)


@pytest.mark.parametrize("sdt", DTS)
@pytest.mark.parametrize("M,N", [(3, 48), (1000, 1040), (4096, 4096), (777, 12304), (300000, 16)])
def test_dequant_flat_rows_bit_exact(sdt, M, N):
    """The flat vector kernel finds each vector's row by a multiply-high
    division (1, 3, 65, 256, 769 vectors per row) and builds the int8 values
    as exact floats: the result must equal (q.float() * scale.float()).half()
    bit for bit, for fp16, bf16 and fp32 scales."""
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    q = torch.randint(-128, 128, (M, N), generator=g, device="cuda", dtype=torch.int8)
    sc = (torch.rand((M, 1), generator=g, device="cuda") * 0.05 + 0.001).to(TDT[sdt])
    sc[::5] = -sc[::5]
    got = b200k.dequant_int8(q, sc)
    want = (q.float() * sc.float()).to(torch.float16)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("M,N", [(5, 24), (1000, 1032), (3000, 4096)])
def test_bias_gelu_flat_columns(dt, M, N):
    """bias_gelu's vector kernel takes each vector's column from the
    multiply-high division: against the oracle on every row."""
    x = _randn((M, N), dt, 2.0, M + 1)
    b = _randn((N,), dt, 0.5, N + 2)
    got = b200k.bias_gelu(_t(x, dt), _t(b, dt))
    _close(got, O.bias_gelu(x, b, dt), dt)


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("op", ["softmax", "softcap_softmax", "log_softmax", "softmax_scale"])
@pytest.mark.parametrize("M,N,pad", [(3000, 1032, 0), (5000, 2048, 0), (700, 1040, 16),
                                     (20000, 2048, 0)])
def test_softmax_family_pipelined_narrow_rows(dt, op, M, N, pad):
    """Rows of 129..256 16-byte vectors (fp16/bf16 1032..2048 values, fp32
    1040 and 2048) through the bulk-copy pipeline with 64-thread blocks, many
    rows per block, strided rows among them: sampled rows against the oracle,
    every row against the fp32 torch expression."""
    g = torch.Generator(device="cuda").manual_seed(M + N + pad)
    base = (torch.randn((M, N + pad), generator=g, device="cuda") * 8).to(TDT[dt])
    x = base[:, :N]
    scale = torch.tensor([0.37], device="cuda").to(TDT[dt])
    fn = getattr(b200k, op)
    out = fn(x, scale) if op == "softmax_scale" else fn(x)
    xf = x.float()
    if op == "softcap_softmax":
        xf = 30.0 * torch.tanh(xf / 30.0)
    elif op == "softmax_scale":
        xf = xf * scale.float()[0]
    want = torch.log_softmax(xf, -1) if op == "log_softmax" else torch.softmax(xf, -1)
    _close(out, want.to(TDT[dt]).float().cpu().numpy(), dt)
    rows = np.arange(0, M, max(1, M // 17))
    xs = x[rows].float().cpu().numpy()
    o = getattr(O, op)
    ref = o(xs, scale.float().cpu().numpy(), dt) if op == "softmax_scale" else o(xs, dt)
    _close(out[rows], ref, dt)


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("op", ["entropy", "kl_div", "cumsum"])
@pytest.mark.parametrize("shape,scale", [((3000, 1024), 1.0), ((700, 8192), 8.0),
                                         ((333, 4096), 64.0), ((64, 512), 1.0)])
def test_reductions_pipelined(dt, op, shape, scale):
    """entropy / kl_div / cumsum on aligned rows whose inputs fit one ring
    stage (the bulk-copy pipelined kernels: one merge of (max, sum, weighted
    sum) per row, fp32 run + fp64 thread offsets for the scan), at scales
    1 / 8 / 64 and more rows than resident blocks, against the oracle on
    sampled rows (all rows for the small case)."""
    M, N = shape
    if dt == "f32" and N * 4 * (2 if op == "kl_div" else 1) > (64 << 10):
        pytest.skip("row above one ring stage: the register / streaming kernels")
    kind = regimes.OPS[op].kind
    case = regimes.make_case(kind, 17, M, N, dt, scale)
    ins = to_cuda(case)
    out = b200k.get_op(op)(*ins)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([[0, M - 1], np.arange(0, M, max(1, M // 23))]))
    sub = [(v[rows] if v.ndim == 2 else v, tag) for v, tag in case]
    ref = regimes.reference(op, sub)
    ok, err, bad = allclose_report(out.float().cpu().numpy()[rows], ref, *tol_for(op, dt))
    assert ok, f"{op} {dt} {shape} x{scale}: max err {err}, {bad} bad"
