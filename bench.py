"""Benchmark of the b200k kernels on the op suite's named configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl b200k|reference]

One JSON line on stdout (rank 0).  Metric: achieved HBM GB/s of the op
(algorithmic bytes: compulsory reads + writes, per step) aggregated over all
ranks, with the % of the measured HBM peak in `roofline`.

Workloads (synthetic data of the named shapes, seeded per rank):
  chain     (default) residual add -> LayerNorm -> GELU-tanh, bf16,
            x, r [16384, 8192], outputs (h = x + r, y), eps 1e-5
  rmsnorm   x [4096, 4096] fp16, w = 1 + 0.1 N(0,1), eps 1e-6
  swiglu    gate, up [8192, 14336] bf16, N(0,1)*2
  rope      q [8,4096,32,128], k [8,4096,8,128] bf16, tables [4096, 64] (neox)
  rope_interleaved   same shapes, GPT-J pairs
  ce        logits [32768, 128256] bf16, N(0,1)*3, 5% targets = -100,
            mean loss over valid rows (rows split across ranks, NCCL
            all-reduce of [loss sum, valid count])
  ce_fwd_bwd  same logits: mean loss and its gradient in one pass
Each rank processes a full configuration (weak scaling) except `ce`, whose
32768 rows are split across ranks (strong scaling).

Baselines on the same device and inputs: the reference's PyTorch expressions
in eager mode (`eager`) and under torch.compile (`compile`, the reference
harness's own baseline; `--compile-mode max-autotune-no-cudagraphs` is its
strong one); `--compile` adds the compile baseline to the other configs.

--impl reference times the CPU implementation of the same workload (the
oracle's numpy restatement of ouroboros/specs.py, all host cores) on a bounded
sample of rows per step, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
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
FALLBACK_HBM_GBS = 6650.0


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
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * scale
            + shift).to(dtype)


class Workload:
    name = ""
    scaling = "weak"
    dtype = "bf16"
    launches_per_step = 1
    graph_steps = 0  # > 0: time from a CUDA graph of this many steps (launch-bound sizes)

    def e2e_api(self):
        return "b200k.host.run_rows_host (pinned host buffers, copies overlapped with kernels)"

    ROWS_ATTR = "M"

    def set_rows(self, n):
        setattr(self, self.ROWS_ATTR, int(n))

    def compile_step(self, mode):
        """The eager reference expressions of the step under torch.compile
        (the reference harness's own baseline, ouroboros/harness.py:250-290)."""
        return torch.compile(self.eager_step, mode=mode, dynamic=False)

    def setup(self, device, rank, world): ...
    def step(self): ...
    def bytes_per_step(self) -> int: ...
    def config(self) -> dict: ...
    def e2e_setup(self): ...
    def e2e_step(self, timing): ...
    def cpu_rows(self) -> int: ...
    def cpu_run(self, r0, r1): ...


class Chain(Workload):
    """x + r -> LayerNorm -> GELU-tanh, outputs (h, y); configs[1] shape."""
    name = "chain_add_layernorm_gelu"
    M, N = 16384, 8192

    def setup(self, device, rank, world):
        import b200k
        self.b2k = b200k
        s = 1000 * rank
        self.x = _randn((self.M, self.N), torch.bfloat16, device, s + 1)
        self.r = _randn((self.M, self.N), torch.bfloat16, device, s + 2)
        self.w = _randn((self.N,), torch.bfloat16, device, s + 3, 0.1, 1.0)
        self.b = _randn((self.N,), torch.bfloat16, device, s + 4, 0.02)
        self.device = device

    def step(self):
        return self.b2k.fused_add_norm(self.x, self.r, self.w, self.b, norm="layer", act="gelu")

    def bytes_per_step(self):
        # read x, r; write h, y (bf16); read gamma, beta
        return 4 * self.M * self.N * 2 + 2 * self.N * 2

    def config(self):
        return {"workload": "add_layernorm_gelu_tanh_h_y", "M": self.M, "N": self.N,
                "outputs": "h=x+r, y=gelu_tanh(LN(h)*g+b)", "eps": 1e-5,
                "l2": "inputs exceed L2 (1 GiB working set per step)"}

    def eager_step(self):
        # ouroboros/chains.py:69-87 (add_layernorm_gelu) in torch eager, plus h
        hf = self.x.float() + self.r.float()
        mu = hf.mean(-1, keepdim=True)
        hc = hf - mu
        n = hc * torch.rsqrt((hc * hc).mean(-1, keepdim=True) + 1e-5) * self.w.float() + self.b.float()
        y = (0.5 * n * (1.0 + torch.tanh(0.7978845608028654 * (n + 0.044715 * n * n * n))))
        return hf.to(torch.bfloat16), y.to(torch.bfloat16)

    def e2e_setup(self):
        self.hx = self.x.cpu().pin_memory()
        self.hr = self.r.cpu().pin_memory()
        self.hw = self.w.cpu()
        self.hb = self.b.cpu()
        self.hh = torch.empty_like(self.hx).pin_memory()
        self.hy = torch.empty_like(self.hx).pin_memory()
        return (2 * self.M * self.N * 2 + 2 * self.N * 2, 2 * self.M * self.N * 2)

    def e2e_step(self, timing):
        from b200k.host import run_rows_host
        b2k = self.b2k
        run_rows_host(lambda x, r, w, b: b2k.fused_add_norm(x, r, w, b, norm="layer", act="gelu"),
                      [self.hx, self.hr], [self.hw, self.hb], out=(self.hh, self.hy),
                      device=self.device, timing=timing)

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
    """rmsnorm x [4096, 4096] fp16; buffers rotate over 8 sets."""
    name = "rmsnorm"
    dtype = "fp16"
    M = N = 4096
    SETS = 8
    graph_steps = 8

    def setup(self, device, rank, world):
        import b200k
        self.b2k = b200k
        s = 1000 * rank
        self.xs = [_randn((self.M, self.N), torch.float16, device, s + 10 + i) for i in range(self.SETS)]
        self.w = _randn((self.N,), torch.float16, device, s + 3, 0.1, 1.0)
        self.i = 0
        self.device = device

    def step(self):
        x = self.xs[self.i % self.SETS]
        self.i += 1
        return self.b2k.rmsnorm(x, self.w)

    def bytes_per_step(self):
        return 2 * self.M * self.N * 2 + self.N * 2

    def eager_step(self):
        x = self.xs[self.i % self.SETS]
        self.i += 1
        return self._expr(x, self.w)

    @staticmethod
    def _expr(x, w):
        xf = x.float()  # ouroboros/specs.py:75-78
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype) * w

    def compile_step(self, mode):
        fn = torch.compile(self._expr, mode=mode, dynamic=False)

        def st():
            x = self.xs[self.i % self.SETS]
            self.i += 1
            return fn(x, self.w)
        return st

    def config(self):
        return {"workload": "rmsnorm", "M": self.M, "N": self.N, "eps": 1e-6,
                "l2": f"{self.SETS} rotating input sets ({self.SETS * self.M * self.N * 2 >> 20} MiB) "
                      "so consecutive steps read cold data"}

    def e2e_setup(self):
        self.hx = self.xs[0].cpu().pin_memory()
        self.hw = self.w.cpu()
        self.hy = torch.empty_like(self.hx).pin_memory()
        return (self.M * self.N * 2 + self.N * 2, self.M * self.N * 2)

    def e2e_step(self, timing):
        from b200k.host import run_rows_host
        run_rows_host(self.b2k.rmsnorm, [self.hx], [self.hw], out=self.hy, device=self.device,
                      timing=timing)

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
    """silu(gate) * up, gate/up [8192, 14336] bf16, N(0,1)*2."""
    name = "swiglu"
    M, N = 8192, 14336

    def setup(self, device, rank, world):
        import b200k
        self.b2k = b200k
        s = 1000 * rank
        self.g = _randn((self.M, self.N), torch.bfloat16, device, s + 21, 2.0)
        self.u = _randn((self.M, self.N), torch.bfloat16, device, s + 22, 2.0)
        self.device = device

    def step(self):
        return self.b2k.swiglu(self.g, self.u)

    def bytes_per_step(self):
        return 3 * self.M * self.N * 2

    def eager_step(self):  # ouroboros/specs.py:85-87
        return (torch.nn.functional.silu(self.g.float()) * self.u.float()).to(self.g.dtype)

    def config(self):
        return {"workload": "swiglu", "M": self.M, "N": self.N,
                "l2": "inputs exceed L2 (470 MB read per step)"}

    def e2e_setup(self):
        self.hg = self.g.cpu().pin_memory()
        self.hu = self.u.cpu().pin_memory()
        self.hy = torch.empty_like(self.hg).pin_memory()
        return (2 * self.M * self.N * 2, self.M * self.N * 2)

    def e2e_step(self, timing):
        from b200k.host import run_rows_host
        run_rows_host(self.b2k.swiglu, [self.hg, self.hu], [], out=self.hy, device=self.device,
                      timing=timing)

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
    """mean CE over valid tokens, logits [32768, 128256] bf16,
    N(0,1)*3, 5% targets = -100; rows split across ranks (strong scaling),
    NCCL all-reduce of [loss sum, valid count] inside every step."""
    name = "cross_entropy_mean"
    scaling = "strong"
    launches_per_step = 3  # row losses, shard reduce, mean (2 with the peer exchange)
    T, V = 32768, 128256
    ROWS_ATTR = "T"

    def setup(self, device, rank, world):
        import b200k
        from b200k.dist import shard_rows
        self.b2k = b200k
        self.r0, self.r1 = shard_rows(self.T, rank, world)
        rows = self.r1 - self.r0
        g = torch.Generator(device=device).manual_seed(500 + rank)
        self.x = (torch.randn((rows, self.V), generator=g, device=device, dtype=torch.float32)
                  * 3.0).to(torch.bfloat16) if rows * self.V < (1 << 31) else self._chunked(
                      rows, device, g)
        t = torch.randint(0, self.V, (rows,), generator=g, device=device, dtype=torch.int64)
        drop = torch.rand((rows,), generator=g, device=device) < 0.05
        self.t = torch.where(drop, torch.full_like(t, -100), t)
        self.world = world
        self.device = device
        if world > 1 and type(self) is CrossEntropy:
            # collective set-up of the peer-memory exchange (every rank, same order):
            # row losses + fused reduce / exchange / mean = 2 launches per step
            from b200k.dist import ce_exchange
            if ce_exchange(None, device) is not None:
                self.launches_per_step = 2

    def _chunked(self, rows, device, g):
        out = torch.empty((rows, self.V), dtype=torch.bfloat16, device=device)
        step = 4096
        for r in range(0, rows, step):
            n = min(step, rows - r)
            out[r:r + n] = (torch.randn((n, self.V), generator=g, device=device) * 3.0).to(
                torch.bfloat16)
        return out

    def step(self):
        return self.b2k.cross_entropy_mean(self.x, self.t)

    def bytes_per_step(self):
        rows = self.r1 - self.r0
        return rows * self.V * 2 + rows * 8

    def eager_step(self):
        # ouroboros/specs.py:239-241 reduced to the mean over valid rows
        return torch.nn.functional.cross_entropy(self.x.float(), self.t, ignore_index=-100)

    def config(self):
        return {"workload": "cross_entropy_mean", "T": self.T, "V": self.V,
                "ignore_index": -100, "ignore_frac": 0.05,
                "l2": "inputs exceed L2 (8.4 GB of logits per step)",
                "note": "rows whose target is ignore_index are not read (their loss is 0)"}

    def e2e_setup(self):
        # host buffers for a bounded slice (the full 8.4 GB does not need to
        # sit in pinned memory): 4096 rows
        self.e2e_rows = min(4096, self.r1 - self.r0)
        self.hx = self.x[:self.e2e_rows].cpu().pin_memory()
        self.ht = self.t[:self.e2e_rows].cpu().pin_memory()
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
    """configs[4] with the gradient: mean CE over valid tokens and
    d loss / d logits (bf16) in one pass over the logits."""
    name = "cross_entropy_fwd_bwd"
    launches_per_step = 4  # valid count, fused fwd+bwd, shard reduce, mean

    def step(self):
        return self.b2k.cross_entropy_fwd_bwd(self.x, self.t)

    def bytes_per_step(self):
        rows = self.r1 - self.r0
        return 2 * rows * self.V * 2 + rows * 8  # logits read once, gradient written once

    def compile_step(self, mode):
        return None  # the step runs autograd's backward: no single compiled graph

    def eager_step(self):
        xf = self.x.float().requires_grad_(True)
        loss = torch.nn.functional.cross_entropy(xf, self.t, ignore_index=-100)
        loss.backward()
        return loss.detach(), xf.grad.to(torch.bfloat16)

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
    """q [8,4096,32,128], k [8,4096,8,128] bf16, positions 0..S-1,
    theta 10000, tables [S, 64] computed in fp32 and cast to bf16; q and k
    rotated in one launch into fresh outputs."""
    name = "rope_qk"
    B, S, H, Hk, D = 8, 4096, 32, 8, 128
    interleaved = False
    ROWS_ATTR = "B"

    def setup(self, device, rank, world):
        import b200k
        self.b2k = b200k
        s = 1000 * rank
        self.q = _randn((self.B, self.S, self.H, self.D), torch.bfloat16, device, s + 31)
        self.k = _randn((self.B, self.S, self.Hk, self.D), torch.bfloat16, device, s + 32)
        inv = 10000.0 ** (-torch.arange(0, self.D, 2, device=device, dtype=torch.float32) / self.D)
        ang = torch.arange(self.S, device=device, dtype=torch.float32)[:, None] * inv[None, :]
        self.cos = ang.cos().to(torch.bfloat16)
        self.sin = ang.sin().to(torch.bfloat16)
        self.device = device

    def step(self):
        return self.b2k.rope_qk(self.q, self.k, self.cos, self.sin, interleaved=self.interleaved)

    def bytes_per_step(self):
        qk = (self.B * self.S * (self.H + self.Hk) * self.D) * 2
        return 2 * qk + 2 * self.S * (self.D // 2) * 2

    def eager_step(self):
        # ouroboros/specs.py:96-102 / :228-236 with the tables broadcast over heads
        c = self.cos.float()[None, :, None, :]
        s = self.sin.float()[None, :, None, :]
        out = []
        for t in (self.q, self.k):
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

    def config(self):
        return {"workload": "rope_qk_interleaved" if self.interleaved else "rope_qk_neox",
                "q": [self.B, self.S, self.H, self.D], "k": [self.B, self.S, self.Hk, self.D],
                "tables": [self.S, self.D // 2], "theta": 10000.0,
                "l2": "inputs exceed L2 (336 MB read per step)"}

    def e2e_setup(self):
        self.hq = self.q.cpu().pin_memory()
        self.hk = self.k.cpu().pin_memory()
        self.hc, self.hs = self.cos.cpu(), self.sin.cpu()
        self.hqo = torch.empty_like(self.hq).pin_memory()
        self.hko = torch.empty_like(self.hk).pin_memory()
        qk = (self.B * self.S * (self.H + self.Hk) * self.D) * 2
        return (qk + 2 * self.S * (self.D // 2) * 2, qk)

    def e2e_step(self, timing):
        from b200k.host import run_rows_host
        b2k, inter = self.b2k, self.interleaved
        run_rows_host(lambda q, k, c, s: b2k.rope_qk(q, k, c, s, interleaved=inter),
                      [self.hq, self.hk], [self.hc, self.hs], out=(self.hqo, self.hko),
                      device=self.device, timing=timing)

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
        return time_steps(lambda: fn(*a), max(10, args.steps), stream)[0]

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
# time of the reference expression, and a parity check of sampled rows
# against the CPU oracle.  One JSON line per op.
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

    return {  # the expressions of ouroboros/specs.py / chains.py, eager
        "rmsnorm": lambda x, w: (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype) * w,
        "rmsnorm_gemma": lambda x, w: (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * (1.0 + w.float())).to(x.dtype),
        "softmax": lambda x: torch.softmax(x.float(), -1).to(x.dtype),
        "log_softmax": lambda x: torch.log_softmax(x.float(), -1).to(x.dtype),
        "softcap_softmax": lambda x: torch.softmax(30.0 * torch.tanh(x.float() / 30.0), -1).to(x.dtype),
        "swiglu": lambda g, u: (F.silu(g.float()) * u.float()).to(g.dtype),
        "glu": lambda g, u: (torch.sigmoid(g.float()) * u.float()).to(g.dtype),
        "geglu": lambda g, u: (gelu(g.float()) * u.float()).to(g.dtype),
        "gelu": lambda x: gelu(x.float()).to(x.dtype),
        "silu": lambda x: (x.float() * torch.sigmoid(x.float())).to(x.dtype),
        "add_rmsnorm": lambda x, r, w: ((x.float() + r.float()) * torch.rsqrt((x.float() + r.float()).pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype) * w,
        "layernorm": lambda x, w, b: ln(x.float(), w, b).to(x.dtype),
        "add_layernorm": lambda x, r, w, b: ln(x.float() + r.float(), w, b).to(x.dtype),
        "layernorm_gelu": lambda x, w, b: gelu(ln(x.float(), w, b)).to(x.dtype),
        "add_layernorm_gelu": lambda x, r, w, b: gelu(ln(x.float() + r.float(), w, b)).to(x.dtype),
        "add_rmsnorm_silu": lambda x, r, w: F.silu((x.float() + r.float()) * torch.rsqrt((x.float() + r.float()).pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).to(x.dtype),
        "cross_entropy": lambda x, t: F.cross_entropy(x.float(), t, reduction="none").to(x.dtype),
        "rope": lambda x, c, s: (x.float() * c.float() + rot(x.float()) * s.float()).to(x.dtype),
        "rope_interleaved": None,
        "qknorm_rope": None,
    }


GRID_OPS = ["rmsnorm", "rmsnorm_gemma", "softmax", "log_softmax", "softcap_softmax", "swiglu",
            "glu", "geglu", "gelu", "silu", "add_rmsnorm", "layernorm", "add_layernorm",
            "layernorm_gelu", "add_layernorm_gelu", "add_rmsnorm_silu", "cross_entropy", "rope",
            "rope_interleaved", "qknorm_rope"]


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
    ang = torch.randn((M, N // 2), generator=g, device=device)
    c, s = ang.cos(), ang.sin()
    if kind == "rope_inter":
        return (rn(M, N), c.to(dt), s.to(dt))
    cos, sin = torch.cat([c, c], -1).to(dt), torch.cat([s, s], -1).to(dt)
    if kind == "rope":
        return (rn(M, N), cos, sin)
    if kind == "qkr":
        return (rn(M, N), rn(N), cos, sin)
    if kind == "arr":
        return (rn(M, N), rn(M, N), rn(N), cos, sin)
    raise KeyError(kind)


def _algo_bytes(args, out):
    return sum(t.numel() * t.element_size() for t in args) + out.numel() * out.element_size()


def run_grid(args, device):
    import b200k
    from oracle import regimes
    from oracle.numerics import allclose_report, tol_for
    eager = _eager_table()
    peak, _ = hbm_peak()
    stream = torch.cuda.current_stream(device)
    ops = args.grid.split(",") if args.grid not in ("1", "all") else GRID_OPS
    tdt = {"fp16": torch.float16, "bf16": torch.bfloat16}
    odt = {"fp16": "f16", "bf16": "bf16"}
    for op in ops:
        kind = regimes.OPS[op].kind
        cells = ROPE_GRID if kind in ("rope", "rope_inter", "qkr", "arr") else MATRIX_GRID
        if args.cells:
            want = {tuple(int(v) for v in c.split("x")) for c in args.cells.split(",")}
            cells = [c for c in cells if c in want] or sorted(want)
        res = []
        for (M, N) in cells:
            for dname in [d for d in ("fp16", "bf16") if d in args.dtypes.split(",")]:
                inp = _grid_inputs(kind, M, N, tdt[dname], device, 1000 + M + N)
                run = b200k.get_op(op)
                out = run(*inp)
                # parity: 16 sampled rows against the oracle
                rows = torch.unique(torch.randint(0, M, (16,), generator=torch.Generator().manual_seed(M)))
                sub = []
                for t in inp:
                    v = t.float().cpu().numpy() if t.is_floating_point() else t.cpu().numpy()
                    if (t.dim() >= 2 and t.shape[0] == M) or (t.dim() == 1 and not t.is_floating_point()):
                        v = v[rows.numpy()]
                    tag = odt[dname] if t.is_floating_point() else "i64"
                    sub.append((v, tag))
                ref = regimes.reference(op, sub)
                got = out.float().cpu().numpy()[rows.numpy()]
                ok = allclose_report(got, ref, *tol_for(op, odt[dname]))[0]
                ms, _ = time_steps(lambda: run(*inp), 20, stream, graph_steps=10)
                nbytes = _algo_bytes(inp, out)
                cell = {"M": M, "N": N, "dtype": dname, "parity": bool(ok),
                        "us": round(ms * 1e3, 2), "GBs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                        "frac": round(nbytes / (ms * 1e-3) / 1e9 / peak, 3)}
                e = eager.get(op)
                if e is not None:
                    e(*inp)
                    torch.cuda.synchronize()
                    em, _ = time_steps(lambda: e(*inp), 10, stream, graph_steps=5)
                    cell["eager_us"] = round(em * 1e3, 2)
                    cell["speedup_vs_eager"] = round(em / ms, 2)
                res.append(cell)
                del inp, out
        sp = [c["speedup_vs_eager"] for c in res if "speedup_vs_eager" in c]
        geo = float(np.exp(np.mean(np.log(sp)))) if sp else None
        emit({"op": op, "cells": res, "all_parity": all(c["parity"] for c in res),
              "geomean_speedup_vs_eager": round(geo, 3) if geo else None,
              "mean_frac": round(float(np.mean([c["frac"] for c in res])), 3)})
    return 0


# ---------------------------------------------------------------------------
# device timing
def time_steps(fn, steps, stream, graph_steps=0):
    """ms per step of fn() over `steps` steps, CUDA events on `stream`.  With
    graph_steps > 0 the steps are captured into a CUDA graph of graph_steps
    calls (host launch overhead removed) and the graph is replayed."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph_steps > 0:
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(graph_steps):
                fn()
        stream.wait_stream(side)
        with torch.cuda.graph(g):
            for _ in range(graph_steps):
                fn()
        reps = max(1, (steps + graph_steps - 1) // graph_steps)
        g.replay()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / (reps * graph_steps), reps * graph_steps
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, steps


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
def measure_device(wl, args, stream, barrier, dist, device, local, sample_clocks=True):
    """(ms per step max over ranks, ms this rank, steps timed, clock summary)."""
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms, steps = time_steps(wl.step, args.steps, stream, wl.graph_steps if args.graph else 0)
    barrier()
    ms_max = ms
    if dist is not None:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    return ms_max, ms, steps, clk.summary()


def measure_eager(wl, stream, steps=5):
    if not hasattr(wl, "eager_step"):
        return None
    try:
        for _ in range(2):
            wl.eager_step()
        torch.cuda.synchronize()
        ms, _ = time_steps(wl.eager_step, steps, stream)
        return ms
    except torch.cuda.OutOfMemoryError:
        torch.cuda.empty_cache()
        return None


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


def measure_compile(wl, stream, mode, steps=5, graph_steps=0):
    """ms per step of the reference expressions under torch.compile, or a
    one-line reason when that baseline cannot be had.  graph_steps > 0 times
    it from a CUDA graph, as the workload's own kernel is timed."""
    try:
        st = wl.compile_step(mode)
        if st is None:
            return None, "not compiled: the step runs autograd"
        for _ in range(3):  # compiles on the first call
            st()
        torch.cuda.synchronize()
        if graph_steps > 0:
            try:
                ms, _ = time_steps(st, max(steps, 2 * graph_steps), stream, graph_steps)
                return ms, None
            except Exception:
                torch.cuda.synchronize()
        ms, _ = time_steps(st, steps, stream)
        return ms, None
    except torch.cuda.OutOfMemoryError:
        torch.cuda.empty_cache()
        return None, "out of memory"
    except Exception as e:  # a compiler failure is reported, not fatal
        torch.cuda.synchronize()
        return None, f"{type(e).__name__}: {str(e)[:120]}"


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
                    help="skip the device-only measurement of the other configurations")
    ap.add_argument("--no-eager", action="store_true")
    ap.add_argument("--no-compile", action="store_true",
                    help="skip the torch.compile baseline of the headline workload")
    ap.add_argument("--compile", action="store_true",
                    help="also time the torch.compile baseline of the other configurations")
    ap.add_argument("--compile-mode", default="default",
                    help="torch.compile mode of the baseline (the reference harness's strong "
                         "baseline is max-autotune-no-cudagraphs)")
    ap.add_argument("--graph", type=int, default=1,
                    help="launch small workloads from a CUDA graph (1) or one by one (0)")
    ap.add_argument("--grid", default="",
                    help="shape-grid mode: comma list of ops (or 'all'); one JSON line per op")
    ap.add_argument("--cells", default="",
                    help="grid mode: only these shapes, comma list of MxN (e.g. 32768x128)")
    ap.add_argument("--dtypes", default="fp16,bf16", help="grid mode: dtypes to run")
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
        sys.path.insert(0, ROOT)
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

    def barrier():
        if dist is not None:
            dist.barrier()

    stream = torch.cuda.current_stream(device)
    wl.setup(device, rank, world)
    ms_max, ms, steps_timed, clocks = measure_device(wl, args, stream, barrier, dist, device, local)

    # every rank's bytes_per_step is its own share (a full configuration for
    # the weakly scaled workloads, its row shard for ce), so the job moves
    # world x that per step
    total_bytes = wl.bytes_per_step() * world
    value = total_bytes / (ms_max * 1e-3) / 1e9
    peak, peak_kind = hbm_peak()
    # the dominant kernel is timed with its step (any small companion
    # kernels of the step count against it, which only lowers the figure)
    achieved = wl.bytes_per_step() / (ms * 1e-3) / 1e9

    eager = None
    if not args.no_eager:
        e_ms = measure_eager(wl, stream)
        if e_ms is not None:
            eager = {"ms_per_step": round(e_ms, 4), "speedup": round(e_ms / ms, 2),
                     "what": "the reference's PyTorch expressions (ouroboros/specs.py), eager"}
    compiled = None
    if not args.no_compile:
        c_ms, why = measure_compile(wl, stream, args.compile_mode,
                                    graph_steps=wl.graph_steps if args.graph else 0)
        compiled = ({"ms_per_step": round(c_ms, 4), "speedup": round(c_ms / ms, 2)} if c_ms
                    else {"unavailable": why})
        compiled.update({"mode": args.compile_mode,
                         "what": "the same expressions under torch.compile (the reference "
                                 "harness's baseline)"})

    # end to end through the host-buffer API (pinned host in, pinned host out)
    e2e = None
    if not args.no_e2e:
        h2d, d2h = wl.e2e_setup()
        times = []
        for i in range(3 + max(3, min(args.steps, 10))):
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            barrier()
            wl.e2e_step(ev)
            if i >= 3:
                times.append(ev[0].elapsed_time(ev[1]))
        e_ms = statistics.median(times)
        if dist is not None:
            t = torch.tensor([e_ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        e_bytes = wl.e2e_bytes() if hasattr(wl, "e2e_bytes") else wl.bytes_per_step()
        e_total = e_bytes * world
        e2e = {"value": round(e_total / (e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(e_ms, 4), "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "api": wl.e2e_api()}

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

    # the fields of the line that need the configured workload
    wl_cfg, wl_bytes = wl.config(), wl.bytes_per_step()
    wl_scaling, wl_dtype, wl_graph = wl.scaling, wl.dtype, wl.graph_steps

    # the other named configurations, device time only
    extra = {}
    # kernels of this library launched inside the headline timed region
    launches = steps_timed * wl.launches_per_step
    if not args.no_extra:
        del wl
        torch.cuda.empty_cache()
        for name in ("rmsnorm", "swiglu", "rope", "rope_interleaved", "ce"):
            if name == args.workload:
                continue
            w2 = WORKLOADS[name]()
            w2.setup(device, rank, world)  # full configuration (no --rows)
            a2 = argparse.Namespace(**vars(args))
            a2.steps, a2.warmup = (40 if name != "ce" else 10), 5
            m2, m2_local, st2, ck2 = measure_device(w2, a2, stream, barrier, dist, device, local)
            tb = w2.bytes_per_step() * world
            per_rank = w2.bytes_per_step() / (m2_local * 1e-3) / 1e9
            entry = {"value": round(tb / (m2 * 1e-3) / 1e9, 2), "unit": "GB/s",
                     "ms_per_step": round(m2, 5), "frac": round(per_rank / peak, 4),
                     "scaling": w2.scaling, "config": w2.config(),
                     "launch": "cuda_graph" if (args.graph and w2.graph_steps) else "stream",
                     "gpu_launches": st2 * w2.launches_per_step}
            if not args.no_eager:
                e2 = measure_eager(w2, stream, 3)
                if e2 is not None:
                    entry["eager_ms_per_step"] = round(e2, 4)
                    entry["speedup_vs_eager"] = round(e2 / m2_local, 2)
            if args.compile:
                c2, why = measure_compile(w2, stream, args.compile_mode, 3,
                                          w2.graph_steps if args.graph else 0)
                if c2:
                    entry["compile_ms_per_step"] = round(c2, 4)
                    entry["speedup_vs_compile"] = round(c2 / m2_local, 2)
                else:
                    entry["compile_unavailable"] = why
            extra[w2.name] = entry
            del w2
            torch.cuda.empty_cache()
    else:
        del wl

    line = {
        "metric": "achieved HBM GB/s (algorithmic bytes / step time), aggregate over GPUs",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max, 5), "higher_is_better": True,
        "scaling": wl_scaling, "vs_baseline": None, "dtype": wl_dtype, "data": "synthetic",
        "config": dict(wl_cfg, parallelism=f"rows x{world}" if world > 1 else "1 GPU",
                       launch="cuda_graph" if (args.graph and wl_graph) else "stream"),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": wl_bytes},
        "e2e": e2e,
        "cpu_baseline": cpu,
        "eager": eager,
        "compile": compiled,
        "gpu_launches": launches,
        "clocks": clocks,
        "other_configs": extra or None,
    }
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
