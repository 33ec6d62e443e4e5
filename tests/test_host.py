"""Host-side logic of the drop-in boundary, without a GPU: the op table
mirrors every spec of ouroboros/specs.py with the same run() arity, the
harness candidate sources are valid Python, inputs that are not CUDA
tensors are refused (there is no CPU path), and row sharding partitions."""
import ast
import inspect
import json
import os

import pytest
import torch

import b200k
from b200k import dist, registry
from oracle import regimes

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_registry_covers_every_spec():
    assert set(b200k.OPS) == set(regimes.OPS)
    assert len(b200k.OPS) == 118


def test_run_signatures_match_the_specs():
    sigs = json.load(open(os.path.join(GOLDEN, "signatures.json")))
    assert set(sigs) == set(b200k.OPS)
    for name, args in sigs.items():
        fn = b200k.get_op(name)
        params = [p for p in inspect.signature(fn).parameters.values()
                  if p.default is inspect.Parameter.empty and p.kind == p.POSITIONAL_OR_KEYWORD]
        assert len(params) == len(args), f"{name}: {len(params)} vs spec {args}"


def test_get_op_unknown_name():
    with pytest.raises(KeyError):
        b200k.get_op("no_such_op")


def test_candidate_sources_parse():
    for name in b200k.OPS:
        src = registry.candidate_source(name, "/opt/b200k")
        tree = ast.parse(src)
        assert any(isinstance(n, ast.FunctionDef) and n.name == "run" for n in tree.body)


@pytest.mark.parametrize("name", ["rmsnorm", "softmax", "swiglu", "rope", "cross_entropy",
                                  "add_layernorm_gelu", "dequant_int8"])
def test_cpu_tensors_are_refused(name):
    info = regimes.OPS[name]
    case = regimes.make_case(info.kind, 1, 4, 128 if "rope" not in name else 64, "f32", 1.0)
    tens = []
    for v, tag in case:
        if tag == "i8":
            tens.append(torch.from_numpy(v.astype("int8")))
        elif tag == "i64":
            tens.append(torch.from_numpy(v.astype("int64")))
        else:
            tens.append(torch.from_numpy(v))
    with pytest.raises(ValueError, match="CUDA"):
        b200k.get_op(name)(*tens)


def test_shard_rows_partition():
    for M in (0, 1, 7, 32768, 32769):
        for world in (1, 2, 3, 4, 8):
            spans = [dist.shard_rows(M, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == M
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        dist.shard_rows(10, 2, 2)
