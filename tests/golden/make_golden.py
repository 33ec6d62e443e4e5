"""Generate the golden vectors of tests/golden/ from the REFERENCE itself.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py --reference /root/reference

For every op of ouroboros/specs.py (SPECS, specs.py:666-872 plus the chain
ops registered at :1001-1017; the *_short variants share their base op's
reference and are not repeated) it builds seeded cases with
oracle.regimes.make_case, runs `SPECS[op].reference` on CPU tensors, and
stores the reference output (in its storage dtype) together with the case
recipe and a SHA-256 of the inputs.  The tests regenerate the inputs from the
recipe, check the hash, and compare the oracle (CPU) and the CUDA kernels
(GPU) against these outputs.  This script is the only file that imports the
reference; nothing at test or run time reads it.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import regimes  # noqa: E402
from oracle.numerics import bf16_bits  # noqa: E402


def case_recipes(op: str):
    """Small cases per op: odd N, high magnitude, every dtype, few rows."""
    k = regimes.OPS[op].kind
    if k in ("rope", "rope_inter", "qkr", "arr"):
        return [dict(kind=k, seed=700 + D, M=37, N=D, dt=dt, scale=64.0)
                for D, dt in [(128, "f16"), (256, "bf16"), (64, "f16"), (128, "f32")]]
    if k == "rms_wide":
        return [dict(kind=k, seed=90, M=1, N=131072, dt="f16", scale=64.0),
                dict(kind=k, seed=92, M=2, N=65537, dt="bf16", scale=32.0)]
    if k == "int8":
        return [dict(kind=k, seed=71, M=4, N=4097, dt="f16", scale=1.0),
                dict(kind=k, seed=72, M=2, N=8192, dt="f16", scale=1.0)]
    aux = 8.0 if k == "gate_up" else (4.0 if k == "x_bias" else 1.0)
    chain = op not in EXPLICIT
    if chain:
        return [dict(kind=k, seed=91, M=2, N=4097, dt="f16", scale=64.0, aux=aux),
                dict(kind=k, seed=92, M=2, N=1024, dt="bf16", scale=64.0, aux=aux),
                dict(kind=k, seed=93, M=2, N=257, dt="f32", scale=8.0, aux=aux)]
    out = [dict(kind=k, seed=91, M=4, N=4097, dt="f16", scale=64.0, aux=aux),
           dict(kind=k, seed=92, M=4, N=4097, dt="bf16", scale=64.0, aux=aux),
           dict(kind=k, seed=93, M=2, N=8192, dt="f16", scale=32.0, aux=aux),
           dict(kind=k, seed=94, M=3, N=1024, dt="f32", scale=8.0, aux=aux),
           dict(kind=k, seed=95, M=5, N=128, dt="bf16", scale=1.0, aux=aux)]
    if k == "ce":
        out.append(dict(kind=k, seed=96, M=64, N=512, dt="bf16", scale=3.0, ignore=0.25))
    return out


EXPLICIT = {"rmsnorm", "softmax", "swiglu", "add_rmsnorm", "rope", "layernorm", "add_layernorm",
            "geglu", "qknorm_rope", "gelu", "silu", "relu2", "bias_gelu", "reglu", "l2norm",
            "log_softmax", "softmax_scale", "layernorm_gelu", "add_rmsnorm_rope", "dequant_int8",
            "softcap_softmax", "rmsnorm_gemma", "glu", "rope_interleaved", "cross_entropy",
            "cumsum", "entropy", "kl_div", "rmsnorm_wide"}


def build_case(r):
    return regimes.make_case(r["kind"], r["seed"], r["M"], r["N"], r["dt"], r["scale"],
                             r.get("aux", 1.0), r.get("ignore", 0.0))


def input_hash(case) -> str:
    h = hashlib.sha256()
    for vals, tag in case:
        h.update(tag.encode())
        h.update(np.ascontiguousarray(vals).tobytes())
    return h.hexdigest()


def to_torch(case):
    import torch
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
    out = []
    for vals, tag in case:
        if tag == "i8":
            out.append(torch.from_numpy(vals.astype(np.int8)))
        elif tag == "i64":
            out.append(torch.from_numpy(vals.astype(np.int64)))
        else:
            out.append(torch.from_numpy(np.ascontiguousarray(vals, dtype=np.float32)).to(tdt[tag]))
    return out


def encode_out(t):
    """Reference output tensor -> (array in its storage format, dtype tag)."""
    import torch
    if t.dtype == torch.bfloat16:
        return bf16_bits(t.float().numpy()), "bf16"
    if t.dtype == torch.float16:
        return t.numpy().astype(np.float16), "f16"
    return t.float().numpy().astype(np.float32), "f32"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--ops", default="")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "ouroboros"))
    import torch
    import specs  # the reference's op definitions

    torch.set_num_threads(os.cpu_count() or 1)
    ops = [o for o in regimes.OPS if not o.endswith("_short")]
    if args.ops:
        ops = args.ops.split(",")
    manifest = {}
    mpath = os.path.join(HERE, "manifest.json")
    if args.ops and os.path.exists(mpath):  # partial regeneration keeps the rest
        with open(mpath) as f:
            manifest = json.load(f)["ops"]
    for op in ops:
        ref = specs.SPECS[op].reference
        arrays = {}
        recs = []
        for i, r in enumerate(case_recipes(op)):
            case = build_case(r)
            with torch.no_grad():
                out = ref(*to_torch(case))
            enc, tag = encode_out(out)
            arrays[f"out{i}"] = enc
            recs.append(dict(r, sha256=input_hash(case), out_tag=tag, out_shape=list(out.shape)))
        arrays["recipes"] = np.frombuffer(json.dumps(recs).encode(), dtype=np.uint8)
        np.savez_compressed(os.path.join(HERE, f"{op}.npz"), **arrays)
        manifest[op] = len(recs)
        print(f"{op}: {len(recs)} cases")
    # run() argument names per op, from the spec's signature hint (the
    # drop-in contract: same inputs in the same order)
    import re
    sigs = {}
    for name, spec in specs.SPECS.items():
        m = re.search(r"def run\(([^)]*)\)", spec.signature_hint)
        sigs[name] = [a.strip() for a in m.group(1).split(",")] if m else None
    with open(os.path.join(HERE, "signatures.json"), "w") as f:
        json.dump(sigs, f, indent=0, sort_keys=True)
    with open(mpath, "w") as f:
        json.dump({"ops": dict(sorted(manifest.items())), "torch": torch.__version__,
                   "source": "ouroboros/specs.py SPECS[op].reference on CPU"}, f, indent=1)


if __name__ == "__main__":
    main()
