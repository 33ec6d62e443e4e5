"""Benchmark of the b200k kernels on the op suite's named configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl b200k|reference]

One JSON line on stdout (rank 0).  Metric: achieved HBM GB/s of the op
(algorithmic bytes: compulsory reads + writes, per step) aggregated over all
ranks, with the % of the measured HBM peak in `roofline`.

Workloads (synthetic data of the named shapes):
  chain     (default) residual add -> LayerNorm -> GELU-tanh, bf16,
            x, r [16384, 8192], outputs (h = x + r, y), eps 1e-5
  rmsnorm   x [4096, 4096] fp16, w = 1 + 0.1 N(0,1), eps 1e-6
  swiglu    gate, up [8192, 14336] bf16, N(0,1)*2
  rope      q [8,4096,32,128], k [8,4096,8,128] bf16, tables [4096, 64] (neox)
  rope_interleaved   same shapes, GPT-J pairs
  ce        logits [32768, 128256] bf16, N(0,1)*3, 5% targets = -100,
            mean loss over valid rows (one exchange of [loss sum, valid
            count] between the ranks inside every step)
  ce_fwd_bwd  same logits: mean loss and its gradient in one pass
Every workload is one fixed problem whose rows are split across the ranks
(strong scaling): rank r of N owns the contiguous rows shard_rows(M, r, N)
(the batch for rope, the tokens for ce).

Timing: W warm-up steps, then exactly K steps captured in one CUDA graph and
replayed between CUDA events on the launching stream (the graph removes the
host's launch gaps, which dominate the microsecond shards of the small
configurations; `--graph 0` launches step by step).  Each rank holds enough
input sets, used in rotation, that a step's inputs were last touched at least
3 x L2 of traffic earlier, so every step reads from HBM.  The reported time
is the maximum over ranks; the per-rank spread is printed beside it.  After
the timed region the last timed output is checked against the reference's
PyTorch expression on the same inputs (`parity`), as ouroboros/harness.py
does after its timing loop.

Baselines on the same device and inputs (N = 1): the reference's PyTorch
expressions in eager mode, under torch.compile (default mode, the reference
harness's baseline) and under torch.compile max-autotune-no-cudagraphs (its
strong baseline, ouroboros/harness.py:282-287).

--impl reference times the CPU implementation of the same workload (the
oracle's numpy restatement of ouroboros/specs.py, all host cores) on a bounded
sample of rows per step, on rank 0 only.
"""
from __future__ import annotations

import argparse
import collections
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ouroboros-kernelsmith_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
ROTATE_BYTES = 3 * L2_BYTES  # per-rank traffic between two uses of one input set
FALLBACK_HBM_GBS = 6650.0
# the spec's allclose tolerance per output dtype: the element-wise minimum of
# ouroboros/specs.py:41-45 and fp16 1e-2 / bf16 2e-2 (rtol, atol)
TOL = {torch.float16: (1e-2, 2e-3), torch.bfloat16: (2e-2, 8e-3), torch.float32: (2e-4, 2e-5)}
CE_MEAN_RTOL = 1e-3  # relative tolerance of the reduced cross-entropy scalar


# ---------------------------------------------------------------------------
# peaks / clocks
def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            v = float(json.load(f)["hbm_gbs"])
        return v, "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index, period=0.002):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period = period
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "n_samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "n_samples": len(self.samples)}


# ---------------------------------------------------------------------------
# workloads
def _randn(shape, dtype, device, seed, scale=1.0, shift=0.0):
    """N(0,1)*scale+shift in `dtype`, generated in row blocks of at most 2^30
    elements (keeps the fp32 temporary small for the 8 GB logits)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = torch.empty(shape, dtype=dtype, device=device)
    flat = out.view(shape[0], -1) if len(shape) > 1 else out.view(-1, 1)
    step = max(1, (1 << 30) // max(1, flat.shape[1]))
    for r in range(0, flat.shape[0], step):
        n = min(step, flat.shape[0] - r)
        flat[r:r + n] = (torch.randn((n, flat.shape[1]), generator=g, device=device,
                                     dtype=torch.float32) * scale + shift).to(dtype)
    return out


def _close(got, want, dtype):
    """(ok, max abs error) of |got - want| <= atol + rtol |want|, element-wise,
    at the spec tolerance of `dtype`, computed in fp32 on the device."""
    rtol, atol = TOL[dtype]
    g, w = got.float(), want.float()
    err = (g - w).abs()
    ok = bool((err <= atol + rtol * w.abs()).all()) and bool(torch.isfinite(g).all())
    return ok, float(err.max()) if err.numel() else 0.0


class Workload:
    """One named configuration, row-sharded over the ranks.

    Subclasses define the row count (attribute ROWS_ATTR), `make_set(k)` (the
    k-th input set of this rank's shard), `run(*inputs)` (the b200k call),
    `expr(*inputs)` (the reference's PyTorch expression of the same outputs,
    used for the eager / compile baselines and the parity check) and
    `bytes_per_step()` (algorithmic bytes of this rank's shard)."""
    name = ""
    scaling = "strong"
    dtype = "bf16"
    launches_per_step = 1
    ROWS_ATTR = "M"
    graphable = True  # the step can be captured in a CUDA graph

    def rows_total(self):
        return int(getattr(self, self.ROWS_ATTR))

    def set_rows(self, n):
        setattr(self, self.ROWS_ATTR, int(n))

    def setup(self, device, rank, world):
        import b200k
        from b200k.dist import shard_rows
        self.b2k = b200k
        self.device, self.rank, self.world = device, rank, world
        self.r0, self.r1 = shard_rows(self.rows_total(), rank, world)
        self.rows = self.r1 - self.r0
        self.make_shared()
        per = max(1, self.bytes_per_step())
        self.nsets = int(max(1, min(64, -(-ROTATE_BYTES // per))))
        self.sets = [self.make_set(k) for k in range(self.nsets)]
        self.i = 0
        self.last_set = 0

    def make_shared(self):
        """Operands every rank holds in full (weights, tables)."""

    def seed(self, k, j):
        """Seed of operand j of input set k on this rank."""
        return 100003 * self.rank + 1009 * k + 17 * j + 1

    def next_set(self):
        k = self.i % self.nsets
        self.i += 1
        self.last_set = k
        return self.sets[k]

    def step(self):
        return self.run(*self.next_set())

    def eager_step(self):
        return self.expr(*self.next_set())

    def compile_step(self, mode):
        """The reference expressions under torch.compile (the reference
        harness's own baselines, ouroboros/harness.py:250-290)."""
        fn = torch.compile(self.expr, mode=mode, dynamic=False)
        return lambda: fn(*self.next_set())

    def poke(self):
        """One large in-range value written into the first input of every set
        before timing (ouroboros/harness.py:229-250): a result cached across
        calls would miss it and fail the check after the timed region."""
        for k, s in enumerate(self.sets):
            flat = s[0].view(-1)
            flat[(7919 * (k + 1)) % flat.numel()] = 60.0

    def verify(self, out):
        """Compares the output of the last step with the reference
        expression on that step's inputs."""
        want = self.expr(*self.sets[self.last_set])
        ok, err = _close(out, want, out.dtype)
        return {"parity": ok, "max_abs_err": err, "checked": "all rows vs the fp32 torch expression"}

    def config(self) -> dict: ...
    def bytes_per_step(self) -> int: ...
    def make_set(self, k): ...
    def run(self, *inputs): ...
    def expr(self, *inputs): ...

    def e2e_api(self):
        return ("b200k.host.RowsHostGraph (pinned host buffers; each run replays the "
                "host->device copies, the kernels and the device->host copies of every "
                f"{self.host_graph.chunk_rows}-row chunk, overlapped on three streams)")

    def _host_graph(self, fn, row_inputs, other_inputs, out):
        from b200k.host import RowsHostGraph
        self.host_graph = RowsHostGraph(fn, row_inputs, other_inputs, out=out,
                                        device=self.device)

    def e2e_step(self, timing):
        self.host_graph.run(timing)

    def e2e_verify(self):
        """The host outputs of the last end-to-end run against the device op on
        the same inputs (the device op's launch may differ by chunk size, so
        at the spec tolerance of the output dtype)."""
        want = self.run(*self.sets[0])
        want = tuple(want) if isinstance(want, (tuple, list)) else (want,)
        got = self.host_graph.out
        got = tuple(got) if isinstance(got, (tuple, list)) else (got,)
        return all(_close(g.to(self.device), w, w.dtype)[0] for g, w in zip(got, want))


class Chain(Workload):
    """x + r -> LayerNorm -> GELU-tanh, outputs (h, y): add_layernorm_gelu of
    ouroboros/chains.py:69-87 plus the residual stream h, 16384 x 8192 bf16."""
    name = "chain_add_layernorm_gelu"
    M, N = 16384, 8192

    def make_shared(self):
        self.w = _randn((self.N,), torch.bfloat16, self.device, 3, 0.1, 1.0)
        self.b = _randn((self.N,), torch.bfloat16, self.device, 4, 0.02)

    def make_set(self, k):
        return (_randn((self.rows, self.N), torch.bfloat16, self.device, self.seed(k, 1)),
                _randn((self.rows, self.N), torch.bfloat16, self.device, self.seed(k, 2)))

    def run(self, x, r):
        return self.b2k.fused_add_norm(x, r, self.w, self.b, norm="layer", act="gelu")

    def bytes_per_step(self):
        # read x, r; write h, y (bf16); read gamma, beta
        return 4 * self.rows * self.N * 2 + 2 * self.N * 2

    def config(self):
        return {"workload": "add_layernorm_gelu_tanh_h_y", "M": self.M, "N": self.N,
                "outputs": "h=x+r, y=gelu_tanh(LN(h)*g+b)", "eps": 1e-5}

    def expr(self, x, r):
        # ouroboros/chains.py:69-87 (add_layernorm_gelu) in torch, plus h
        hf = x.float() + r.float()
        mu = hf.mean(-1, keepdim=True)
        hc = hf - mu
        n = hc * torch.rsqrt((hc * hc).mean(-1, keepdim=True) + 1e-5) * self.w.float() \
            + self.b.float()
        y = 0.5 * n * (1.0 + torch.tanh(0.7978845608028654 * (n + 0.044715 * n * n * n)))
        return hf.to(torch.bfloat16), y.to(torch.bfloat16)

    def verify(self, out):
        h, y = out
        h_want, y_want = self.expr(*self.sets[self.last_set])
        ok_y, err = _close(y, y_want, torch.bfloat16)
        ok_h = bool(torch.equal(h, h_want))
        return {"parity": ok_y and ok_h, "max_abs_err": err, "h_bit_exact": ok_h,
                "checked": "all rows: h bit-exact, y vs the fp32 torch expression"}

    def e2e_setup(self):
        x, r = self.sets[0]
        self.hx, self.hr = x.cpu().pin_memory(), r.cpu().pin_memory()
        self.hw, self.hb = self.w.cpu().pin_memory(), self.b.cpu().pin_memory()
        self.hh = torch.empty_like(self.hx).pin_memory()
        self.hy = torch.empty_like(self.hx).pin_memory()
        b2k = self.b2k
        self._host_graph(lambda x, r, w, b: b2k.fused_add_norm(x, r, w, b, norm="layer",
                                                               act="gelu"),
                         [self.hx, self.hr], [self.hw, self.hb], (self.hh, self.hy))
        return (2 * self.rows * self.N * 2 + 2 * self.N * 2, 2 * self.rows * self.N * 2)

    # CPU: oracle restatement of the same chain on float32 values
    def cpu_prepare(self):
        from oracle.numerics import bf16_round
        rows = self.cpu_rows_total = min(self.M, 4096)
        g = np.random.default_rng(0)
        self.cx = bf16_round(g.standard_normal((rows, self.N), dtype=np.float32))
        self.cr = bf16_round(g.standard_normal((rows, self.N), dtype=np.float32))
        self.cw = bf16_round(1 + 0.1 * g.standard_normal(self.N, dtype=np.float32))
        self.cb = bf16_round(0.02 * g.standard_normal(self.N, dtype=np.float32))

    def cpu_run(self, r0, r1):
        from oracle import ops as O
        from oracle.numerics import rnd
        h = rnd(self.cx[r0:r1] + self.cr[r0:r1], "bf16")
        y = O.chain("layer", True, "gelu", [self.cx[r0:r1], self.cr[r0:r1], self.cw, self.cb],
                    "bf16")
        return h, y

    def cpu_bytes_per_row(self):
        return 4 * self.N * 2


class RMSNorm(Workload):
    """rmsnorm x [4096, 4096] fp16, w = 1 + 0.1 N(0,1), eps 1e-6
    (ouroboros/specs.py:75-78)."""
    name = "rmsnorm"
    dtype = "fp16"
    M = N = 4096
    # a 13 us step: time at least 500 of them as another configuration, so
    # the graph launch and the first launch's ramp are < 0.5 % of the region
    min_steps = 500

    def make_shared(self):
        self.w = _randn((self.N,), torch.float16, self.device, 3, 0.1, 1.0)

    def make_set(self, k):
        return (_randn((self.rows, self.N), torch.float16, self.device, self.seed(k, 1)),)

    def run(self, x):
        return self.b2k.rmsnorm(x, self.w)

    def bytes_per_step(self):
        return 2 * self.rows * self.N * 2 + self.N * 2

    def expr(self, x):
        xf = x.float()  # ouroboros/specs.py:75-78
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype) * self.w

    def config(self):
        return {"workload": "rmsnorm", "M": self.M, "N": self.N, "eps": 1e-6}

    def e2e_setup(self):
        self.hx = self.sets[0][0].cpu().pin_memory()
        self.hw = self.w.cpu().pin_memory()
        self.hy = torch.empty_like(self.hx).pin_memory()
        self._host_graph(self.b2k.rmsnorm, [self.hx], [self.hw], self.hy)
        return (self.rows * self.N * 2 + self.N * 2, self.rows * self.N * 2)

    def cpu_prepare(self):
        from oracle.numerics import f16_round
        g = np.random.default_rng(0)
        self.cx = f16_round(g.standard_normal((self.M, self.N), dtype=np.float32))
        self.cw = f16_round(1 + 0.1 * g.standard_normal(self.N, dtype=np.float32))
        self.cpu_rows_total = self.M

    def cpu_run(self, r0, r1):
        from oracle import ops as O
        return O.rmsnorm(self.cx[r0:r1], self.cw, "f16")

    def cpu_bytes_per_row(self):
        return 2 * self.N * 2


class SwiGLU(Workload):
    """silu(gate) * up, gate/up [8192, 14336] bf16, N(0,1)*2
    (ouroboros/specs.py:85-87)."""
    name = "swiglu"
    M, N = 8192, 14336

    def make_set(self, k):
        return (_randn((self.rows, self.N), torch.bfloat16, self.device, self.seed(k, 1), 2.0),
                _randn((self.rows, self.N), torch.bfloat16, self.device, self.seed(k, 2), 2.0))

    def run(self, g, u):
        return self.b2k.swiglu(g, u)

    def bytes_per_step(self):
        return 3 * self.rows * self.N * 2

    def expr(self, g, u):  # ouroboros/specs.py:85-87
        return (torch.nn.functional.silu(g.float()) * u.float()).to(g.dtype)

    def config(self):
        return {"workload": "swiglu", "M": self.M, "N": self.N}

    def e2e_setup(self):
        g, u = self.sets[0]
        self.hg, self.hu = g.cpu().pin_memory(), u.cpu().pin_memory()
        self.hy = torch.empty_like(self.hg).pin_memory()
        self._host_graph(self.b2k.swiglu, [self.hg, self.hu], [], self.hy)
        return (2 * self.rows * self.N * 2, self.rows * self.N * 2)

    def cpu_prepare(self):
        from oracle.numerics import bf16_round
        g = np.random.default_rng(0)
        rows = self.cpu_rows_total = 1024
        self.cg = bf16_round(2 * g.standard_normal((rows, self.N), dtype=np.float32))
        self.cu = bf16_round(2 * g.standard_normal((rows, self.N), dtype=np.float32))

    def cpu_run(self, r0, r1):
        from oracle import ops as O
        return O.swiglu(self.cg[r0:r1], self.cu[r0:r1], "bf16")

    def cpu_bytes_per_row(self):
        return 3 * self.N * 2


class CrossEntropy(Workload):
    """Mean CE over valid tokens, logits [32768, 128256] bf16, N(0,1)*3, 5%
    targets = -100 (ouroboros/specs.py:239-241 reduced over the valid rows);
    the [loss sum, valid count] pair of every rank is exchanged inside every
    step (peer-memory exchange fused into the reducing kernel, or an NCCL
    all-reduce)."""
    name = "cross_entropy_mean"
    launches_per_step = 3  # row losses, shard reduce, mean (2 with the peer exchange)
    T, V = 32768, 128256
    ROWS_ATTR = "T"

    def setup(self, device, rank, world):
        super().setup(device, rank, world)
        self.exchange = "none (1 rank)"
        if world > 1:
            # collective set-up of the peer-memory exchange (every rank, same order)
            from b200k.dist import ce_exchange
            if ce_exchange(None, device) is not None:
                # mean: row losses + fused reduce / exchange / mean; loss +
                # gradient: valid count, count exchange, fused kernel, fused
                # reduce / exchange / mean
                self.launches_per_step = 2 if type(self) is CrossEntropy else 4
                self.exchange = "peer memory (CUDA IPC over NVLink), fused into the reduce kernel"
            else:
                self.exchange = "NCCL all-reduce"
                self.graphable = False

    def make_set(self, k):
        x = _randn((self.rows, self.V), torch.bfloat16, self.device, self.seed(k, 1), 3.0)
        g = torch.Generator(device=self.device).manual_seed(self.seed(k, 2))
        t = torch.randint(0, self.V, (self.rows,), generator=g, device=self.device,
                          dtype=torch.int64)
        drop = torch.rand((self.rows,), generator=g, device=self.device) < 0.05
        return (x, torch.where(drop, torch.full_like(t, -100), t))

    def run(self, x, t):
        return self.b2k.cross_entropy_mean(x, t)

    def bytes_per_step(self):
        return self.rows * self.V * 2 + self.rows * 8

    def bytes_needed(self):
        """Bytes the step has to move: the algorithmic bytes less the logits
        of rows whose target is ignore_index (their loss is 0 without reading
        them)."""
        t = self.sets[0][1]
        ignored = int((t == -100).sum())
        return self.bytes_per_step() - ignored * self.V * 2

    def expr(self, x, t):
        # ouroboros/specs.py:239-241 reduced to the mean over valid rows
        return torch.nn.functional.cross_entropy(x.float(), t, ignore_index=-100)

    def _ref_mean(self, x, t):
        """fp64 sum of the fp32 per-row losses and the valid count of this
        rank's shard (row chunks of F.cross_entropy), summed over the ranks
        with an NCCL all-reduce that is independent of the path under test."""
        s = torch.zeros((2,), dtype=torch.float64, device=self.device)
        step = 2048
        for r in range(0, x.shape[0], step):
            xs, ts = x[r:r + step].float(), t[r:r + step]
            s[0] += torch.nn.functional.cross_entropy(xs, ts, ignore_index=-100,
                                                      reduction="sum").double()
            s[1] += (ts != -100).sum().double()
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(s, op=dist.ReduceOp.SUM)
        return float(s[0] / s[1])

    def verify(self, out):
        want = self._ref_mean(*self.sets[self.last_set])
        got = float(out)
        err = abs(got - want)
        ok = math.isfinite(got) and err <= CE_MEAN_RTOL * abs(want)
        return {"parity": ok, "max_abs_err": err, "mean": got, "reference_mean": want,
                "checked": f"mean over all {self.T} rows of all ranks vs F.cross_entropy in fp32 "
                           f"(row chunks, NCCL-summed), rtol {CE_MEAN_RTOL}"}

    def config(self):
        return {"workload": "cross_entropy_mean", "T": self.T, "V": self.V,
                "ignore_index": -100, "ignore_frac": 0.05,
                "note": "rows whose target is ignore_index are not read (their loss is 0)"}

    def e2e_setup(self):
        # host buffers for a bounded slice (the full 8.4 GB does not need to
        # sit in pinned memory): 4096 rows
        x, t = self.sets[0]
        self.e2e_rows = min(4096, self.rows)
        self.hx = x[:self.e2e_rows].cpu().pin_memory()
        self.ht = t[:self.e2e_rows].cpu().pin_memory()
        return (self.e2e_rows * (self.V * 2 + 8), 4)

    def e2e_bytes(self):
        return self.e2e_rows * (self.V * 2 + 8)

    def e2e_api(self):
        return ("b200k.cross_entropy_mean on a 4096-row slice copied from pinned host memory, "
                "fp32 mean copied back")

    def e2e_step(self, timing):
        cur = torch.cuda.current_stream(self.device)
        timing[0].record(cur)
        x = self.hx.to(self.device, non_blocking=True)
        t = self.ht.to(self.device, non_blocking=True)
        out = self.b2k.cross_entropy_mean(x, t)
        host = torch.empty((), dtype=torch.float32, pin_memory=True)
        host.copy_(out, non_blocking=True)
        timing[1].record(cur)
        cur.synchronize()

    def cpu_prepare(self):
        from oracle.numerics import bf16_round
        g = np.random.default_rng(0)
        rows = self.cpu_rows_total = 256
        self.cx = bf16_round(3 * g.standard_normal((rows, self.V), dtype=np.float32))
        self.ct = g.integers(0, self.V, size=rows).astype(np.int64)

    def cpu_run(self, r0, r1):
        from oracle import ops as O
        return O.cross_entropy_sum_count(self.cx[r0:r1], self.ct[r0:r1])

    def cpu_bytes_per_row(self):
        return self.V * 2 + 8


class CrossEntropyFwdBwd(CrossEntropy):
    """The same logits: mean CE over valid tokens and d loss / d logits (bf16)
    in one pass over the logits."""
    name = "cross_entropy_fwd_bwd"
    launches_per_step = 4  # valid count, fused fwd+bwd, shard reduce, mean

    def run(self, x, t):
        return self.b2k.cross_entropy_fwd_bwd(x, t)

    def bytes_per_step(self):
        return 2 * self.rows * self.V * 2 + self.rows * 8  # logits read once, gradient written once

    def compile_step(self, mode):
        return None  # the step runs autograd's backward: no single compiled graph

    def expr(self, x, t):
        xf = x.float().requires_grad_(True)
        loss = torch.nn.functional.cross_entropy(xf, t, ignore_index=-100)
        loss.backward()
        return loss.detach(), xf.grad.to(torch.bfloat16)

    def verify(self, out):
        loss, dx = out
        x, t = self.sets[self.last_set]
        want = self._ref_mean(x, t)
        got = float(loss)
        ok_l = math.isfinite(got) and abs(got - want) <= CE_MEAN_RTOL * abs(want)
        # gradient of sampled rows against autograd of the same rows' losses,
        # scaled by the global valid count
        n_valid = float((t != -100).sum())
        if self.world > 1:
            import torch.distributed as dist
            c = torch.tensor([n_valid], dtype=torch.float64, device=self.device)
            dist.all_reduce(c, op=dist.ReduceOp.SUM)
            n_valid = float(c)
        rows = torch.arange(0, x.shape[0], max(1, x.shape[0] // 64), device=self.device)
        xf = x[rows].float().requires_grad_(True)
        torch.nn.functional.cross_entropy(xf, t[rows], ignore_index=-100,
                                          reduction="sum").backward()
        # compared at the scale of p - onehot (the gradient times the valid count)
        ok_g, err = _close(dx[rows].float() * n_valid, xf.grad, torch.bfloat16)
        return {"parity": ok_l and ok_g, "max_abs_err": err, "mean": got, "reference_mean": want,
                "checked": "mean over all rows (rtol 1e-3) and the gradient of 64 sampled rows "
                           "vs autograd in fp32"}

    def config(self):
        c = super().config()
        c["workload"] = "cross_entropy_fwd_bwd"
        c["outputs"] = "mean loss (fp32) and d loss / d logits (bf16)"
        return c

    def e2e_api(self):
        return ("b200k.cross_entropy_fwd_bwd on a 4096-row slice copied from pinned host memory, "
                "loss and gradient copied back")

    def e2e_setup(self):
        h2d, _ = super().e2e_setup()
        self.hg = torch.empty((self.e2e_rows, self.V), dtype=torch.bfloat16).pin_memory()
        return h2d, 4 + self.e2e_rows * self.V * 2

    def e2e_bytes(self):
        return self.e2e_rows * (2 * self.V * 2 + 8)

    def e2e_step(self, timing):
        cur = torch.cuda.current_stream(self.device)
        timing[0].record(cur)
        x = self.hx.to(self.device, non_blocking=True)
        t = self.ht.to(self.device, non_blocking=True)
        loss, dx = self.b2k.cross_entropy_fwd_bwd(x, t)
        host = torch.empty((), dtype=torch.float32, pin_memory=True)
        host.copy_(loss, non_blocking=True)
        self.hg.copy_(dx, non_blocking=True)
        timing[1].record(cur)
        cur.synchronize()

    def cpu_run(self, r0, r1):
        from oracle import ops as O
        return (O.cross_entropy_sum_count(self.cx[r0:r1], self.ct[r0:r1]),
                O.cross_entropy_grad(self.cx[r0:r1], self.ct[r0:r1], "bf16"))

    def cpu_bytes_per_row(self):
        return 2 * self.V * 2 + 8


class RoPE(Workload):
    """q [8,4096,32,128], k [8,4096,8,128] bf16, positions 0..S-1, theta 10000,
    tables [S, 64] computed in fp32 and cast to bf16; q and k rotated in one
    launch into fresh outputs.  Ranks split the batch."""
    name = "rope_qk"
    B, S, H, Hk, D = 8, 4096, 32, 8, 128
    interleaved = False
    ROWS_ATTR = "B"

    def make_shared(self):
        inv = 10000.0 ** (-torch.arange(0, self.D, 2, device=self.device, dtype=torch.float32)
                          / self.D)
        ang = torch.arange(self.S, device=self.device, dtype=torch.float32)[:, None] * inv[None, :]
        self.cos = ang.cos().to(torch.bfloat16)
        self.sin = ang.sin().to(torch.bfloat16)

    def make_set(self, k):
        return (_randn((self.rows, self.S, self.H, self.D), torch.bfloat16, self.device,
                       self.seed(k, 1)),
                _randn((self.rows, self.S, self.Hk, self.D), torch.bfloat16, self.device,
                       self.seed(k, 2)))

    def run(self, q, k):
        return self.b2k.rope_qk(q, k, self.cos, self.sin, interleaved=self.interleaved)

    def bytes_per_step(self):
        qk = (self.rows * self.S * (self.H + self.Hk) * self.D) * 2
        return 2 * qk + 2 * self.S * (self.D // 2) * 2

    def expr(self, q, k):
        # ouroboros/specs.py:96-102 / :228-236 with the tables broadcast over heads
        c = self.cos.float()[None, :, None, :]
        s = self.sin.float()[None, :, None, :]
        out = []
        for t in (q, k):
            tf = t.float()
            if self.interleaved:
                o = torch.empty_like(tf)
                o[..., 0::2] = tf[..., 0::2] * c - tf[..., 1::2] * s
                o[..., 1::2] = tf[..., 1::2] * c + tf[..., 0::2] * s
            else:
                h = self.D // 2
                rot = torch.cat([-tf[..., h:], tf[..., :h]], dim=-1)
                o = tf * torch.cat([c, c], -1) + rot * torch.cat([s, s], -1)
            out.append(o.to(t.dtype))
        return tuple(out)

    def verify(self, out):
        want = self.expr(*self.sets[self.last_set])
        res = [_close(o, w, torch.bfloat16) for o, w in zip(out, want)]
        return {"parity": all(r[0] for r in res), "max_abs_err": max(r[1] for r in res),
                "checked": "all of q and k vs the fp32 torch expression"}

    def config(self):
        return {"workload": "rope_qk_interleaved" if self.interleaved else "rope_qk_neox",
                "q": [self.B, self.S, self.H, self.D], "k": [self.B, self.S, self.Hk, self.D],
                "tables": [self.S, self.D // 2], "theta": 10000.0}

    def e2e_setup(self):
        q, k = self.sets[0]
        self.hq, self.hk = q.cpu().pin_memory(), k.cpu().pin_memory()
        self.hc, self.hs = self.cos.cpu().pin_memory(), self.sin.cpu().pin_memory()
        self.hqo = torch.empty_like(self.hq).pin_memory()
        self.hko = torch.empty_like(self.hk).pin_memory()
        b2k, inter = self.b2k, self.interleaved
        self._host_graph(lambda q, k, c, s: b2k.rope_qk(q, k, c, s, interleaved=inter),
                         [self.hq, self.hk], [self.hc, self.hs], (self.hqo, self.hko))
        qk = (self.rows * self.S * (self.H + self.Hk) * self.D) * 2
        return (qk + 2 * self.S * (self.D // 2) * 2, qk)

    def cpu_prepare(self):
        from oracle.numerics import bf16_round
        g = np.random.default_rng(0)
        self.cq = bf16_round(g.standard_normal((1, self.S, self.H, self.D), dtype=np.float32))
        self.ck = bf16_round(g.standard_normal((1, self.S, self.Hk, self.D), dtype=np.float32))
        inv = 10000.0 ** (-np.arange(0, self.D, 2, dtype=np.float32) / self.D)
        ang = np.arange(self.S, dtype=np.float32)[:, None] * inv[None, :]
        self.cc, self.cs = bf16_round(np.cos(ang)), bf16_round(np.sin(ang))
        self.cpu_rows_total = self.S  # a "row" is one position of one sequence

    def cpu_run(self, r0, r1):
        from oracle import ops as O
        return O.rope_qk_tables(self.cq[:, r0:r1], self.ck[:, r0:r1], self.cc[r0:r1],
                                self.cs[r0:r1], "bf16", interleaved=self.interleaved)

    def cpu_bytes_per_row(self):
        return 2 * (self.H + self.Hk) * self.D * 2


class RoPEInterleaved(RoPE):
    name = "rope_qk_interleaved"
    interleaved = True


WORKLOADS = {"chain": Chain, "rmsnorm": RMSNorm, "swiglu": SwiGLU, "ce": CrossEntropy,
             "ce_fwd_bwd": CrossEntropyFwdBwd,
             "rope": RoPE, "rope_interleaved": RoPEInterleaved}


# ---------------------------------------------------------------------------
# E2E MLP block (ouroboros/e2e_block_bench.py:94-148): add_rmsnorm -> gate/up
# GEMMs -> swiglu -> down GEMM, fp16, GEMMs by cuBLAS (torch.matmul) in every
# path; the b200k path replaces the two non-GEMM ops.
def run_mlp_block(args, device):
    import b200k
    R = args.rows or 8192
    H, F = 4096, 11008
    g = torch.Generator(device=device).manual_seed(7)
    rnd = lambda *shape, scale=1.0: (torch.randn(shape, generator=g, device=device) * scale).half()
    x, res, w = rnd(R, H), rnd(R, H), rnd(H)
    Wg, Wu, Wd = rnd(H, F, scale=H ** -0.5), rnd(H, F, scale=H ** -0.5), rnd(F, H, scale=F ** -0.5)

    def block_eager(x, res, w, Wg, Wu, Wd):
        h = x.float() + res.float()
        rms = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6)
        hn = (h * rms).to(x.dtype) * w
        gate, up = hn @ Wg, hn @ Wu
        return (torch.nn.functional.silu(gate) * up) @ Wd

    def block_ours(x, res, w, Wg, Wu, Wd):
        hn = b200k.add_rmsnorm(x, res, w)
        gate, up = hn @ Wg, hn @ Wu
        return b200k.swiglu(gate, up) @ Wd

    def nongemm_eager(x, res, w):
        h = x.float() + res.float()
        rms = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6)
        return (h * rms).to(x.dtype) * w

    inputs = (x, res, w, Wg, Wu, Wd)
    ref = block_eager(*inputs)
    out = block_ours(*inputs)
    err = float((out.float() - ref.float()).abs().max())
    ok = bool(torch.allclose(out.float(), ref.float(), rtol=3e-2, atol=2e-2))
    stream = torch.cuda.current_stream(device)

    def t(fn, *a):
        for _ in range(3):
            fn(*a)
        torch.cuda.synchronize()
        return StepTimer(lambda: fn(*a), max(10, args.steps), stream, graph=False).run()

    te, to = t(block_eager, *inputs), t(block_ours, *inputs)
    tne, tno = t(nongemm_eager, x, res, w), t(b200k.add_rmsnorm, x, res, w)
    line = {"metric": "MLP block tokens/s (add_rmsnorm -> GEMMs -> swiglu -> GEMM)",
            "value": round(R / (to * 1e-3), 1), "unit": "tokens/s", "n_gpus": 1,
            "higher_is_better": True, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": "mlp_block", "rows": R, "hidden": H, "ffn": F},
            "correct_vs_eager": ok, "max_abs_err_vs_eager": err,
            "block_ms": {"eager": round(te, 4), "b200k": round(to, 4)},
            "speedup_vs_eager": round(te / to, 4),
            "nongemm_ms": {"eager": round(tne, 4), "b200k": round(tno, 4)},
            "amdahl_bound_vs_eager": round(1.0 / (1.0 - (tne - tno) / te), 4)}
    emit(line)
    return 0 if ok else 1


# ---------------------------------------------------------------------------
# Shape grid (ouroboros/rebench_shapes.py:37-41): every listed op at every
# (M, N) cell in fp16 and bf16 — b200k GB/s and % of the HBM peak, torch eager
# (and, with --grid-compile, torch.compile) time of the reference expression,
# each timed --repeats times (ouroboros/rebench_stability.py:17-55) with input
# sets rotated so every call reads from HBM, and a parity check of the whole
# output against the reference expression.  One JSON line per op.
MATRIX_GRID = [(1024, 4096), (4096, 4096), (8192, 4096), (4096, 8192), (16384, 2048), (256, 16384)]
ROPE_GRID = [(8192, 128), (32768, 128), (65536, 64), (16384, 256)]


def _eager_table():
    F = torch.nn.functional
    C = 0.7978845608028654

    def gelu(t):
        return 0.5 * t * (1.0 + torch.tanh(C * (t + 0.044715 * t * t * t)))

    def ln(h, w, b):
        mu = h.mean(-1, keepdim=True)
        hc = h - mu
        return hc * torch.rsqrt((hc * hc).mean(-1, keepdim=True) + 1e-5) * w.float() + b.float()

    def rot(xf):
        h = xf.shape[-1] // 2
        return torch.cat([-xf[..., h:], xf[..., :h]], -1)

    def rms(h):
        return h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6)

    def rope_inter(x, c, s):
        xf, cf, sf = x.float(), c.float(), s.float()
        o = torch.empty_like(xf)
        o[..., 0::2] = xf[..., 0::2] * cf - xf[..., 1::2] * sf
        o[..., 1::2] = xf[..., 1::2] * cf + xf[..., 0::2] * sf
        return o.to(x.dtype)

    def qknorm_rope(x, w, c, s):
        n = rms(x.float()) * w.float()
        return (n * c.float() + rot(n) * s.float()).to(x.dtype)

    def entropy(x):
        xf = x.float()
        lse = torch.logsumexp(xf, dim=-1, keepdim=True)
        return (lse.squeeze(-1) - (xf * torch.exp(xf - lse)).sum(-1)).to(x.dtype)

    def kl_div(x, y):
        lx = x.float() - torch.logsumexp(x.float(), dim=-1, keepdim=True)
        ly = y.float() - torch.logsumexp(y.float(), dim=-1, keepdim=True)
        return (torch.exp(lx) * (lx - ly)).sum(-1).to(x.dtype)

    return {  # the expressions of ouroboros/specs.py / chains.py, eager
        "rmsnorm": lambda x, w: rms(x.float()).to(x.dtype) * w,
        "rmsnorm_gemma": lambda x, w: (rms(x.float()) * (1.0 + w.float())).to(x.dtype),
        "softmax": lambda x: torch.softmax(x.float(), -1).to(x.dtype),
        "log_softmax": lambda x: torch.log_softmax(x.float(), -1).to(x.dtype),
        "softcap_softmax": lambda x: torch.softmax(30.0 * torch.tanh(x.float() / 30.0), -1).to(x.dtype),
        "swiglu": lambda g, u: (F.silu(g.float()) * u.float()).to(g.dtype),
        "glu": lambda g, u: (torch.sigmoid(g.float()) * u.float()).to(g.dtype),
        "geglu": lambda g, u: (gelu(g.float()) * u.float()).to(g.dtype),
        "gelu": lambda x: gelu(x.float()).to(x.dtype),
        "silu": lambda x: (x.float() * torch.sigmoid(x.float())).to(x.dtype),
        "add_rmsnorm": lambda x, r, w: rms(x.float() + r.float()).to(x.dtype) * w,
        "layernorm": lambda x, w, b: ln(x.float(), w, b).to(x.dtype),
        "add_layernorm": lambda x, r, w, b: ln(x.float() + r.float(), w, b).to(x.dtype),
        "layernorm_gelu": lambda x, w, b: gelu(ln(x.float(), w, b)).to(x.dtype),
        "add_layernorm_gelu": lambda x, r, w, b: gelu(ln(x.float() + r.float(), w, b)).to(x.dtype),
        "add_rmsnorm_silu": lambda x, r, w: F.silu(rms(x.float() + r.float()) * w.float()).to(x.dtype),
        "cross_entropy": lambda x, t: F.cross_entropy(x.float(), t, reduction="none").to(x.dtype),
        "rope": lambda x, c, s: (x.float() * c.float() + rot(x.float()) * s.float()).to(x.dtype),
        "rope_interleaved": rope_inter,
        "qknorm_rope": qknorm_rope,
        "dequant_int8": lambda q, sc: (q.float() * sc.float()).to(torch.float16),
        "cumsum": lambda x: torch.cumsum(x.float(), dim=-1).to(x.dtype),
        "entropy": entropy,
        "kl_div": kl_div,
    }


# op -> input kind of _grid_inputs
GRID_OPS = {"rmsnorm": "rms", "rmsnorm_gemma": "rms", "softmax": "x", "log_softmax": "x",
            "softcap_softmax": "x", "swiglu": "gate_up", "glu": "gate_up", "geglu": "gate_up",
            "gelu": "x", "silu": "x", "add_rmsnorm": "add_rms", "layernorm": "ln",
            "add_layernorm": "add_ln", "layernorm_gelu": "ln", "add_layernorm_gelu": "add_ln",
            "add_rmsnorm_silu": "add_rms", "cross_entropy": "ce", "rope": "rope",
            "rope_interleaved": "rope_inter", "qknorm_rope": "qkr", "dequant_int8": "dequant",
            "cumsum": "x", "entropy": "x", "kl_div": "gate_up"}


def _grid_inputs(kind, M, N, dt, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    rn = lambda *s: torch.randn(s, generator=g, device=device).to(dt)
    if kind == "x":
        return (rn(M, N),)
    if kind in ("rms",):
        return (rn(M, N), rn(N))
    if kind == "ln":
        return (rn(M, N), rn(N), rn(N))
    if kind == "add_rms":
        return (rn(M, N), rn(M, N), rn(N))
    if kind == "add_ln":
        return (rn(M, N), rn(M, N), rn(N), rn(N))
    if kind == "gate_up":
        return (rn(M, N), rn(M, N))
    if kind == "ce":
        return (rn(M, N), torch.randint(0, N, (M,), generator=g, device=device))
    if kind == "dequant":
        q = torch.randint(-128, 128, (M, N), generator=g, device=device, dtype=torch.int8)
        return (q, (torch.rand((M, 1), generator=g, device=device) * 0.02).to(dt))
    ang = torch.randn((M, N // 2), generator=g, device=device)
    c, s = ang.cos(), ang.sin()
    if kind == "rope_inter":
        return (rn(M, N), c.to(dt), s.to(dt))
    cos, sin = torch.cat([c, c], -1).to(dt), torch.cat([s, s], -1).to(dt)
    if kind == "rope":
        return (rn(M, N), cos, sin)
    if kind == "qkr":
        return (rn(M, N), rn(N), cos, sin)
    raise KeyError(kind)


def _algo_bytes(args, out):
    return sum(t.numel() * t.element_size() for t in args) + out.numel() * out.element_size()


def _cycle(fn, sets):
    state = {"i": 0}

    def f():
        s = sets[state["i"] % len(sets)]
        state["i"] += 1
        return fn(*s)
    return f


def _time_cell(fn, sets, stream, repeats):
    """ms per call (one figure per repeat) of fn over the rotating input sets,
    from a CUDA graph; stream launches where the expression cannot be
    captured."""
    steps = len(sets) * max(1, -(-20 // len(sets)))
    try:
        return StepTimer(_cycle(fn, sets), steps, stream, graph=True, hold=len(sets)).run_many(
            repeats)
    except Exception:
        torch.cuda.synchronize()
        return StepTimer(_cycle(fn, sets), steps, stream, graph=False).run_many(repeats)


def run_grid(args, device):
    import b200k
    eager = _eager_table()
    peak, _ = hbm_peak()
    stream = torch.cuda.current_stream(device)
    ops = list(GRID_OPS) if args.grid in ("1", "all") else args.grid.split(",")
    tdt = {"fp16": torch.float16, "bf16": torch.bfloat16}
    for op in ops:
        kind = GRID_OPS[op]
        cells = ROPE_GRID if kind in ("rope", "rope_inter", "qkr") else MATRIX_GRID
        if args.cells:
            want = {tuple(int(v) for v in c.split("x")) for c in args.cells.split(",")}
            cells = [c for c in cells if c in want] or sorted(want)
        res = []
        for (M, N) in cells:
            for dname in [d for d in ("fp16", "bf16") if d in args.dtypes.split(",")]:
                dt = tdt[dname]
                probe = _grid_inputs(kind, M, N, dt, device, 1000 + M + N)
                run = b200k.get_op(op)
                out = run(*probe)
                e = eager[op]
                ok, err = _close(out, e(*probe), out.dtype)
                nbytes = _algo_bytes(probe, out)
                nsets = int(max(1, min(64, -(-ROTATE_BYTES // nbytes))))
                sets = [probe] + [_grid_inputs(kind, M, N, dt, device, 1000 + M + N + 7 * k)
                                  for k in range(1, nsets)]
                ms = _time_cell(run, sets, stream, args.repeats)
                med = statistics.median(ms)
                cell = {"M": M, "N": N, "dtype": dname, "parity": bool(ok),
                        "max_abs_err": err, "us": round(med * 1e3, 2),
                        "GBs": round(nbytes / (med * 1e-3) / 1e9, 1),
                        "frac": round(nbytes / (med * 1e-3) / 1e9 / peak, 3),
                        "input_sets": nsets}
                if args.repeats > 1:
                    cell["us_repeats"] = [round(v * 1e3, 2) for v in ms]
                    cell["spread"] = round((max(ms) - min(ms)) / med, 4)
                em = statistics.median(_time_cell(e, sets, stream, 1))
                cell["eager_us"] = round(em * 1e3, 2)
                cell["speedup_vs_eager"] = round(em / med, 2)
                for mode in ([m for m in args.grid_compile.split(",") if m]
                             if args.grid_compile else []):
                    key = "compile" if mode == "default" else mode
                    try:
                        # a fresh dynamo cache per cell: the reference expression
                        # is the same function for every cell, and past the
                        # recompile limit dynamo would run it eagerly
                        torch._dynamo.reset()
                        fn = torch.compile(e, mode=mode, dynamic=False)
                        for _ in range(3):
                            fn(*probe)
                        torch.cuda.synchronize()
                        cm = statistics.median(_time_cell(fn, sets, stream, 1))
                        cell[f"{key}_us"] = round(cm * 1e3, 2)
                        cell[f"speedup_vs_{key}"] = round(cm / med, 2)
                    except Exception as ex:  # a compiler failure is reported, not fatal
                        torch.cuda.synchronize()
                        cell[f"{key}_unavailable"] = f"{type(ex).__name__}: {str(ex)[:100]}"
                res.append(cell)
                del probe, out, sets
        sp = [c["speedup_vs_eager"] for c in res]
        geo = float(np.exp(np.mean(np.log(sp)))) if sp else None
        line = {"op": op, "cells": res, "all_parity": all(c["parity"] for c in res),
                "geomean_speedup_vs_eager": round(geo, 3) if geo else None,
                "mean_frac": round(float(np.mean([c["frac"] for c in res])), 3),
                "timing": "CUDA graph of >= 20 calls over rotating input sets (>= 3 x L2 "
                          "between two uses of a set), median of the repeats"}
        for key in ("compile", "max-autotune-no-cudagraphs"):
            sp = [c[f"speedup_vs_{key}"] for c in res if f"speedup_vs_{key}" in c]
            if sp:
                line[f"geomean_speedup_vs_{key}"] = round(float(np.exp(np.mean(np.log(sp)))), 3)
        emit(line)
    return 0


# ---------------------------------------------------------------------------
# device timing
class StepTimer:
    """Times `steps` calls of fn() with CUDA events on `stream`.

    graph=True: the calls are captured into one CUDA graph and the graph is
    replayed (once untimed, then between the events).  During capture the
    outputs of the last `hold` calls are kept alive, so consecutive calls
    write distinct buffers (a buffer is reused only every `hold` calls, the
    same period as the rotating input sets).  `last` is the output of the
    last call, valid after every replay while the timer lives."""

    def __init__(self, fn, steps, stream, graph=True, hold=1):
        self.fn, self.steps, self.stream = fn, int(steps), stream
        self.graph = None
        self.last = None
        if graph:
            side = torch.cuda.Stream()
            side.wait_stream(stream)
            with torch.cuda.stream(side):  # warm-up on a side stream before capture
                fn()
            stream.wait_stream(side)
            torch.cuda.synchronize()
            keep = collections.deque(maxlen=max(1, hold))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(self.steps):
                    keep.append(fn())
            self.last = keep[-1]
            self.graph = g
            g.replay()
            torch.cuda.synchronize()

    def _once(self, pre=None):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if pre is not None:
            pre()
        e0.record(self.stream)
        if self.graph is not None:
            self.graph.replay()
        else:
            for _ in range(self.steps):
                self.last = self.fn()
        e1.record(self.stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / self.steps

    def run(self, pre=None):
        """ms per call over one timed pass; `pre` (untimed) runs right before
        the start event."""
        return self._once(pre)

    def run_many(self, repeats):
        return [self._once() for _ in range(max(1, repeats))]

    def close(self):
        self.last = None
        self.graph = None


# ---------------------------------------------------------------------------
# CPU timing (oracle on the host cores)
def cpu_measure(wl, budget_s=10.0, threads=None, rows_per_task=64):
    """Runs the oracle over row chunks on `threads` host threads for about
    budget_s seconds; returns (GB/s, threads, rows processed, seconds)."""
    from concurrent.futures import ThreadPoolExecutor
    threads = threads or os.cpu_count() or 1
    wl.cpu_prepare()
    total = wl.cpu_rows_total
    rows_per_task = max(1, min(rows_per_task, total))
    done_rows = 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        while True:
            futs = []
            for i in range(threads):
                r0 = (i * rows_per_task) % max(1, total - rows_per_task + 1)
                futs.append(ex.submit(wl.cpu_run, r0, r0 + rows_per_task))
            for f in futs:
                f.result()
            done_rows += threads * rows_per_task
            el = time.perf_counter() - t0
            if el >= budget_s:
                break
    gbs = done_rows * wl.cpu_bytes_per_row() / el / 1e9
    return gbs, threads, done_rows, el


# ---------------------------------------------------------------------------
class Ranks:
    """The process group plumbing of the bench (None when N = 1)."""

    def __init__(self, dist, device):
        self.dist, self.device = dist, device

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def gather(self, v):
        """[v of rank 0, v of rank 1, ...] (floats)."""
        if self.dist is None:
            return [float(v)]
        t = torch.tensor([float(v)], dtype=torch.float64, device=self.device)
        out = [torch.empty_like(t) for _ in range(self.dist.get_world_size())]
        self.dist.all_gather(out, t)
        return [float(o) for o in out]


def measure_device(wl, ranks, stream, local, steps, warmup, graph=True):
    """Times `steps` steps of wl after `warmup` untimed ones and checks the
    last timed output.  Returns a dict: ms (max over ranks), ms_rank (this
    rank's), per_rank [min, median, max], clocks, parity record."""
    for _ in range(warmup):
        wl.step()
    torch.cuda.synchronize()
    timer = StepTimer(wl.step, steps, stream, graph=graph and wl.graphable, hold=wl.nsets)
    captured_last = wl.last_set
    # ranks whose steps wait for one another (the cross-entropy exchange)
    # start the timed region together: one untimed exchanging step first
    pre = wl.step if (wl.world > 1 and getattr(wl, "exchange", "").startswith("peer")) else None
    ranks.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms = timer.run(pre=pre)
    ranks.barrier()
    if timer.graph is not None:
        wl.last_set = captured_last
    parity = wl.verify(timer.last)
    launch = "cuda_graph" if timer.graph is not None else "stream"
    timer.close()
    per = ranks.gather(ms)
    ok_all = ranks.gather(1.0 if parity["parity"] else 0.0)
    parity["parity"] = all(v == 1.0 for v in ok_all)
    return {"ms": max(per), "ms_rank": ms, "per_rank": per, "clocks": clk.summary(),
            "check": parity, "launch": launch, "steps": steps}


def measure_eager(wl, stream, steps=5):
    try:
        for _ in range(2):
            wl.eager_step()
        torch.cuda.synchronize()
        return StepTimer(wl.eager_step, steps, stream, graph=False).run()
    except torch.cuda.OutOfMemoryError:
        torch.cuda.empty_cache()
        return None


def measure_compile(wl, stream, mode, steps=10):
    """ms per step of the reference expressions under torch.compile (timed
    from a CUDA graph like the workload's own kernel, stream launches where
    the compiled code cannot be captured), or a one-line reason when that
    baseline cannot be had."""
    try:
        torch._dynamo.reset()  # a fresh cache: no recompile limit carried over
        st = wl.compile_step(mode)
        if st is None:
            return None, "not compiled: the step runs autograd"
        for _ in range(3):  # compiles on the first call
            st()
        torch.cuda.synchronize()
        steps = max(steps, wl.nsets)
        try:
            return StepTimer(st, steps, stream, graph=True, hold=wl.nsets).run(), None
        except Exception:
            torch.cuda.synchronize()
        return StepTimer(st, steps, stream, graph=False).run(), None
    except torch.cuda.OutOfMemoryError:
        torch.cuda.empty_cache()
        return None, "out of memory"
    except Exception as e:  # a compiler failure is reported, not fatal
        torch.cuda.synchronize()
        return None, f"{type(e).__name__}: {str(e)[:120]}"


_OUT = None


def _json_out():
    """The stream the JSON lines go to: the process's original stdout.  On
    first use file descriptor 1 is pointed at stderr, so that whatever a
    library prints (NCCL's version banner, compiler logs) cannot land beside
    the JSON line."""
    global _OUT
    if _OUT is None:
        sys.stdout.flush()
        fd = os.dup(1)
        os.dup2(2, 1)
        _OUT = os.fdopen(fd, "w")
    return _OUT


def emit(obj):
    print(json.dumps(obj), file=_json_out(), flush=True)


COMPILE_MODES = ("default", "max-autotune-no-cudagraphs")


def _baselines(wl, stream, args, ms_rank, world, entry):
    """Adds the eager and torch.compile baselines of wl to `entry` (the
    compile modes at N = 1 only: compiling per rank adds minutes and no
    information)."""
    if not args.no_eager:
        e = measure_eager(wl, stream, 3 if wl.bytes_per_step() > (1 << 30) else 5)
        if e is not None:
            entry["eager_ms_per_step"] = round(e, 5)
            entry["speedup_vs_eager"] = round(e / ms_rank, 3)
    if args.no_compile or (world > 1 and not args.compile_all_ranks):
        return
    for mode in [m for m in args.compile_modes.split(",") if m]:
        key = "compile" if mode == "default" else "max_autotune"
        c, why = measure_compile(wl, stream, mode)
        if c:
            entry[f"{key}_ms_per_step"] = round(c, 5)
            entry[f"speedup_vs_{key}"] = round(c / ms_rank, 3)
        else:
            entry[f"{key}_unavailable"] = why
        torch._dynamo.reset()


def _ce_parts(wl, stream, steps):
    """Cross-entropy step split into its kernels: the row-loss kernel alone
    (b200k.cross_entropy, per-row losses) against the whole step."""
    x, t = wl.sets[0]
    f = lambda: wl.b2k.cross_entropy(x, t)
    f()
    torch.cuda.synchronize()
    return StepTimer(f, steps, stream, graph=True).run()


def run_config(name, wl, args, ranks, stream, local, steps, warmup, peak, world):
    """Measures one workload; returns its JSON entry (and keeps the figures
    the headline needs in entry['_raw'])."""
    r = measure_device(wl, ranks, stream, local, steps, warmup, graph=bool(args.graph))
    bytes_rank = wl.bytes_per_step()
    total = sum(ranks.gather(bytes_rank))
    per = sorted(r["per_rank"])
    entry = {"value": round(total / (r["ms"] * 1e-3) / 1e9, 2), "unit": "GB/s",
             "ms_per_step": round(r["ms"], 5),
             "frac": round(bytes_rank / (r["ms_rank"] * 1e-3) / 1e9 / peak, 4),
             "per_rank_ms": {"min": round(per[0], 5), "median": round(statistics.median(per), 5),
                             "max": round(per[-1], 5)},
             "parity": r["check"]["parity"], "check": r["check"],
             "scaling": wl.scaling, "config": wl.config(), "rows_per_rank": wl.rows,
             "input_sets": wl.nsets, "launch": r["launch"], "steps": steps,
             "gpu_launches": steps * wl.launches_per_step}
    # what bounds a rank's step when its shard is small: the HBM time of its
    # bytes at the copy peak against the step it took
    floor_us = bytes_rank / (peak * 1e9) * 1e6
    step_us = r["ms_rank"] * 1e3
    entry["shard"] = {"bytes_per_rank": bytes_rank, "hbm_floor_us": round(floor_us, 3),
                      "step_us": round(step_us, 3)}
    if entry["frac"] < 0.9:
        entry["shard"]["limit"] = (
            f"{bytes_rank / 1e6:.1f} MB per rank: {floor_us:.2f} us of HBM time at the copy peak "
            f"inside a {step_us:.2f} us step; the other {step_us - floor_us:.2f} us are the "
            f"launch, the first rows' loads and the last rows' stores, which do not shrink with "
            f"the shard")
    if hasattr(wl, "bytes_needed"):
        need = wl.bytes_needed()
        entry["bytes_needed"] = need
        entry["frac_on_bytes_needed"] = round(need / (r["ms_rank"] * 1e-3) / 1e9 / peak, 4)
    if isinstance(wl, CrossEntropy) and type(wl) is CrossEntropy:
        entry["exchange"] = wl.exchange
        if wl.exchange.startswith("peer"):
            from b200k.dist import exchange_status
            entry["exchange_status"] = exchange_status(None, wl.device)
        rk = _ce_parts(wl, stream, steps)
        entry["row_kernel_ms"] = round(rk, 5)
        entry["reduce_exchange_ms"] = round(max(0.0, r["ms_rank"] - rk), 5)
    entry["_raw"] = r
    entry["_bytes_rank"] = bytes_rank
    return entry


def main():
    _json_out()  # from here on, fd 1 is stderr; the JSON lines keep the real stdout
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="chain", choices=sorted(WORKLOADS) + ["mlp_block"])
    ap.add_argument("--impl", default="b200k", choices=["b200k", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the measurement of the other configurations")
    ap.add_argument("--extra-steps", type=int, default=100,
                    help="timed steps of each other configuration")
    ap.add_argument("--no-eager", action="store_true")
    ap.add_argument("--no-compile", action="store_true",
                    help="skip the torch.compile baselines")
    ap.add_argument("--compile-modes", default=",".join(COMPILE_MODES),
                    help="torch.compile modes timed as baselines (N = 1)")
    ap.add_argument("--compile-all-ranks", action="store_true",
                    help="also time the compile baselines when N > 1")
    ap.add_argument("--graph", type=int, default=1,
                    help="time the steps from a CUDA graph (1) or launch them one by one (0)")
    ap.add_argument("--grid", default="",
                    help="shape-grid mode: comma list of ops (or 'all'); one JSON line per op")
    ap.add_argument("--cells", default="",
                    help="grid mode: only these shapes, comma list of MxN (e.g. 32768x128)")
    ap.add_argument("--dtypes", default="fp16,bf16", help="grid mode: dtypes to run")
    ap.add_argument("--repeats", type=int, default=1, help="grid mode: timings per cell")
    ap.add_argument("--grid-compile", default="",
                    help="grid mode: comma list of torch.compile modes to time per cell")
    ap.add_argument("--rows", type=int, default=0,
                    help="override the row count of the workload (M; batch for rope; "
                         "tokens for ce) — small cases for profiler captures")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.grid:
        torch.cuda.set_device(local)
        sys.exit(run_grid(args, torch.device("cuda", local)))
    if args.workload == "mlp_block":
        torch.cuda.set_device(local)
        sys.exit(run_mlp_block(args, torch.device("cuda", local)))
    wl = WORKLOADS[args.workload]()
    if args.rows > 0:
        wl.set_rows(args.rows)

    if args.impl == "reference":
        return run_reference(args, wl, rank, world)

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
    ranks = Ranks(dist, device)
    stream = torch.cuda.current_stream(device)
    peak, peak_kind = hbm_peak()

    wl.setup(device, rank, world)
    wl.poke()
    head = run_config(wl.name, wl, args, ranks, stream, local, args.steps, args.warmup, peak,
                      world)
    raw = head.pop("_raw")
    bytes_rank = head.pop("_bytes_rank")
    ms_max, ms = raw["ms"], raw["ms_rank"]
    total_bytes = sum(ranks.gather(bytes_rank))
    value = total_bytes / (ms_max * 1e-3) / 1e9
    achieved = bytes_rank / (ms * 1e-3) / 1e9  # this rank's kernel: bytes / launch time
    base = {}
    _baselines(wl, stream, args, ms, world, base)

    # end to end through the host-buffer API (pinned host in, pinned host out)
    e2e = None
    if not args.no_e2e:
        h2d, d2h = wl.e2e_setup()
        times = []
        for i in range(3 + max(3, min(args.steps, 10))):
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ranks.barrier()
            wl.e2e_step(ev)
            if i >= 3:
                times.append(ev[0].elapsed_time(ev[1]))
        e_ms = max(ranks.gather(statistics.median(times)))
        e_bytes = wl.e2e_bytes() if hasattr(wl, "e2e_bytes") else wl.bytes_per_step()
        e_total = sum(ranks.gather(e_bytes))
        e2e = {"value": round(e_total / (e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(e_ms, 4), "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "api": wl.e2e_api()}
        if hasattr(wl, "host_graph"):
            e2e["parity"] = all(ranks.gather(1.0 if wl.e2e_verify() else 0.0))
            del wl.host_graph  # releases the captured pipeline's device buffers

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, threads, rows, el = cpu_measure(wl, args.cpu_budget)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{rows} rows of the same workload in {el:.1f} s (numpy oracle, "
                         f"{threads} threads)"}

    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp) and args.rows == 0 and world == 1:
        try:
            with open(tp) as f:
                traffic = json.load(f).get(wl.name)
        except Exception:
            traffic = None

    wl_cfg, wl_scaling, wl_dtype = wl.config(), wl.scaling, wl.dtype
    launches = args.steps * wl.launches_per_step
    del wl
    torch.cuda.empty_cache()
    extra = {}
    if not args.no_extra:
        for name in ("rmsnorm", "swiglu", "rope", "rope_interleaved", "ce"):
            if name == args.workload:
                continue
            w2 = WORKLOADS[name]()
            w2.setup(device, rank, world)  # full configuration (no --rows)
            w2.poke()
            steps2 = max(args.extra_steps, w2.nsets, getattr(w2, "min_steps", 0))
            entry = run_config(w2.name, w2, args, ranks, stream, local, steps2, 5, peak, world)
            m2 = entry.pop("_raw")["ms_rank"]
            entry.pop("_bytes_rank")
            if name == "rmsnorm" and args.graph:
                # the same steps launched one by one from the host
                r = measure_device(w2, ranks, stream, local, steps2, 3, graph=False)
                entry["stream_launch"] = {
                    "ms_per_step": round(r["ms"], 5),
                    "frac": round(w2.bytes_per_step() / (r["ms_rank"] * 1e-3) / 1e9 / peak, 4),
                    "parity": r["check"]["parity"]}
            _baselines(w2, stream, args, m2, world, entry)
            extra[w2.name] = entry
            del w2
            torch.cuda.empty_cache()

    line = {
        "metric": "achieved HBM GB/s (algorithmic bytes / step time), aggregate over GPUs",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max, 5), "higher_is_better": True,
        "scaling": wl_scaling, "vs_baseline": None, "dtype": wl_dtype, "data": "synthetic",
        "config": dict(wl_cfg, parallelism=f"rows split over {world} GPUs" if world > 1
                       else "1 GPU", launch=head["launch"],
                       l2=f"{head['input_sets']} rotating input set(s) per rank: >= 3 x L2 of "
                          "traffic between two uses of a set"),
        "parity": head["parity"], "check": head["check"],
        "per_rank_ms": head["per_rank_ms"], "rows_per_rank": head["rows_per_rank"],
        "shard": head["shard"],
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_source": peak_kind, "algorithmic_bytes_per_launch": bytes_rank},
        "e2e": e2e,
        "cpu_baseline": cpu,
        "baselines": base or None,
        "gpu_launches": launches,
        "clocks": raw["clocks"],
        "other_configs": extra or None,
    }
    for k in ("bytes_needed", "frac_on_bytes_needed", "exchange", "exchange_status",
              "row_kernel_ms", "reduce_exchange_ms"):
        if k in head:
            line[k] = head[k]
    if rank == 0:
        emit(line)
    if dist is not None:
        torch.cuda.synchronize()
        dist.barrier()
        from b200k.dist import close_exchanges
        close_exchanges()  # peer mappings of the cross-entropy exchange
        dist.destroy_process_group()


def run_reference(args, wl, rank, world):
    """CPU implementation of the same workload (oracle port, all host threads)."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    wl.cpu_prepare()
    from concurrent.futures import ThreadPoolExecutor
    rows_per_task = 32
    per_step_rows = threads * rows_per_task
    total = wl.cpu_rows_total
    times = []
    with ThreadPoolExecutor(threads) as ex:
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            futs = [ex.submit(wl.cpu_run, (k * rows_per_task) % max(1, total - rows_per_task + 1),
                              (k * rows_per_task) % max(1, total - rows_per_task + 1) + rows_per_task)
                    for k in range(threads)]
            for f in futs:
                f.result()
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
    s = statistics.median(times)
    gbs = per_step_rows * wl.cpu_bytes_per_row() / s / 1e9
    line = {
        "impl": "reference",
        "metric": "achieved HBM GB/s (algorithmic bytes / step time), aggregate over GPUs",
        "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(s * 1e3, 3), "higher_is_better": True,
        "scaling": wl.scaling, "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic",
        "config": wl.config(),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{per_step_rows} rows per step (numpy restatement of "
                                   "ouroboros/specs.py, one row chunk per thread)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


if __name__ == "__main__":
    main()
