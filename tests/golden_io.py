"""Loader of the golden vectors in tests/golden/ (made by make_golden.py
from the reference's own SPECS[op].reference on CPU)."""
from __future__ import annotations

import json
import os

import numpy as np

from oracle.numerics import bf16_from_bits

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_ops():
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        return sorted(json.load(f)["ops"])


def load(op: str):
    """[(recipe dict, reference output as float32 values)]"""
    z = np.load(os.path.join(GOLDEN, f"{op}.npz"))
    recs = json.loads(bytes(z["recipes"]).decode())
    out = []
    for i, r in enumerate(recs):
        a = z[f"out{i}"]
        if r["out_tag"] == "bf16":
            v = bf16_from_bits(a)
        else:
            v = a.astype(np.float32)
        out.append((r, v.reshape(r["out_shape"])))
    return out
