"""The allocation-free cross-entropy entry point.

b2k_cross_entropy_mean_noalloc serves callers that cannot allocate device
memory (a host whose device memory is owned by another runtime, or an FFI
binding with device pointers but no allocator): its scratch is a fixed
buffer inside libb200k.so.  This test calls it through the C ABI, twice in a
row on different inputs (so stale scratch from the first call cannot leak
into the second), and compares each result with the allocating path
(b2k_cross_entropy -> b2k_ce_reduce -> b2k_ce_mean with caller scratch).
Both run the same kernels in the same order on the same inputs, so the means
must be equal bit for bit: a tolerance could hide stale or aliased scratch.
The row count exactly at the built-in limit is accepted, zero rows give NaN
(no valid row, as the allocating path), and one row above the limit is
refused before any launch.  The file sorts last so a stop-at-first-failure
run has already run every other test; it needs nothing from them.
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


def _bits(t):
    return t.view(torch.int32).item()


def test_noalloc_matches_allocating_path_twice():
    for M, V, seed in [(4096, 128256, 1), (777, 32000, 2)]:
        x, t = _inputs(M, V, seed)
        want = b200k.cross_entropy_mean(x, t)
        got = _noalloc(x, t)
        assert _bits(got) == _bits(want), (M, V, float(got), float(want))


def test_noalloc_at_the_row_limit_and_empty():
    x, t = _inputs(MAX_ROWS, 64, 3)
    want = b200k.cross_entropy_mean(x, t)
    got = _noalloc(x, t)
    assert _bits(got) == _bits(want), (float(got), float(want))
    e = torch.empty((0, 64), dtype=torch.bfloat16, device="cuda")
    te = torch.empty((0,), dtype=torch.int64, device="cuda")
    assert torch.isnan(_noalloc(e, te)).item()
    assert torch.isnan(b200k.cross_entropy_mean(e, te)).item()


def test_noalloc_rejects_too_many_rows():
    st = _lib.lib.b2k_cross_entropy_mean_noalloc(None, 0, None, MAX_ROWS + 1, 16, _lib.BF16,
                                                 -100, None, None)
    assert st == _lib.EINVAL
    assert "exceed" in _lib.last_error()
