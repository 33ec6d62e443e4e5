"""Helpers of the GPU parity tests: oracle cases -> CUDA tensors, and the
harness discipline of ouroboros/harness.py:171-202 (kernel on clones, input
mutation check, shape and dtype check, allclose against the reference)."""
from __future__ import annotations

import numpy as np
import torch

from oracle.numerics import allclose_report, tol_for

TDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def to_cuda(case, device="cuda"):
    out = []
    for vals, tag in case:
        if tag == "i8":
            out.append(torch.from_numpy(vals.astype(np.int8)).to(device))
        elif tag == "i64":
            out.append(torch.from_numpy(vals.astype(np.int64)).to(device))
        else:
            out.append(torch.from_numpy(np.ascontiguousarray(vals, dtype=np.float32))
                       .to(device).to(TDT[tag]))
    return out


def out_dtype(op, case):
    if op == "dequant_int8":
        return torch.float16
    return TDT[case[0][1]]


def run_checked(op, run, case, ref, rows=None):
    """Runs `run` on CUDA clones of `case`, enforces the harness contract and
    compares with `ref` (float32 values; `rows` selects the compared rows)."""
    inputs = to_cuda(case)
    clones = [t.clone() for t in inputs]
    out = run(*clones)
    torch.cuda.synchronize()
    for a, b in zip(inputs, clones):
        assert torch.equal(a, b), f"{op}: kernel mutated an input"
    assert out.dtype == out_dtype(op, case), f"{op}: dtype {out.dtype}"
    want_shape = tuple(ref.shape) if rows is None else None
    if want_shape is not None:
        assert tuple(out.shape) == want_shape, f"{op}: shape {tuple(out.shape)} != {want_shape}"
    o = out.float().cpu().numpy()
    if rows is not None:
        o = o[rows]
    dt = case[0][1] if case[0][1] in TDT else "f16"
    rtol, atol = tol_for(op, dt)
    ok, err, bad = allclose_report(o, ref, rtol, atol)
    return ok, err, bad
