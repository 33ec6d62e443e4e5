"""The allocation-free cross-entropy entry point.

b2k_cross_entropy_mean_noalloc serves callers that cannot allocate device
memory (a host whose device memory is owned by another runtime, or an FFI
binding with device pointers but no allocator): its scratch is a fixed
buffer inside libb200k.so.  This test calls it through the C ABI, twice in a
row on different inputs (so stale scratch from the first call cannot leak
into the second), and compares each result with the allocating path
(b2k_cross_entropy -> b2k_ce_reduce -> b2k_ce_mean with caller scratch) at
the cross-entropy tolerance of the other tests (1e-3 relative).  It also
checks that a row count above the built-in limit is refused before any
launch.  The file sorts last so a stop-at-first-failure run has already run
every other test; it needs nothing from them.
"""
import pytest
import torch

import b200k
from b200k import _lib

pytestmark = pytest.mark.gpu

MAX_ROWS = 262144  # B2K_NOALLOC_MAX_ROWS in include/b200k.h


def _noalloc(x, t, ignore=-100):
    out = torch.empty((), dtype=torch.float32, device=x.device)
    st = _lib.lib.b2k_cross_entropy_mean_noalloc(
        x.data_ptr(), x.stride(0), t.data_ptr(), x.shape[0], x.shape[1], _lib.BF16, ignore,
        out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.OK, _lib.last_error()
    return out


def _inputs(M, V, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn((M, V), generator=g, device="cuda") * 3).to(torch.bfloat16)
    t = torch.randint(0, V, (M,), generator=g, device="cuda")
    t[torch.rand((M,), generator=g, device="cuda") < 0.05] = -100
    return x, t


def test_noalloc_matches_allocating_path_twice():
    for M, V, seed in [(4096, 128256, 1), (777, 32000, 2)]:
        x, t = _inputs(M, V, seed)
        want = float(b200k.cross_entropy_mean(x, t))
        got = float(_noalloc(x, t))
        assert abs(got - want) <= 1e-3 * abs(want), (M, V, got, want)


def test_noalloc_rejects_too_many_rows():
    st = _lib.lib.b2k_cross_entropy_mean_noalloc(None, 0, None, MAX_ROWS + 1, 16, _lib.BF16,
                                                 -100, None, None)
    assert st == _lib.EINVAL
    assert "exceed" in _lib.last_error()
