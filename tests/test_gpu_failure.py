"""Failure path of the device pipelines, exercised without faulting the GPU:
a bounded wait on a barrier that nothing completes must give up after its
short limit, report the timeout to the host, and leave the context usable
(a normal kernel runs correctly afterwards)."""
import numpy as np
import pytest
import torch

import b200k
from b200k import _lib
from oracle import ops as O
from oracle.numerics import allclose_report, bf16_round

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_survives():
    torch.cuda.synchronize()
    _lib.lib.b2k_pipeline_timeouts(1)  # clear
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = _lib.lib.b2k_selftest_bounded_wait(50_000_000, status.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert st == _lib.OK, _lib.last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    assert _lib.lib.b2k_pipeline_timeouts(1) == 1
    # the context still works: a pipelined kernel gives correct results
    g = np.random.default_rng(3)
    x = bf16_round(g.standard_normal((64, 4096), dtype=np.float32))
    w = bf16_round(g.standard_normal(4096, dtype=np.float32))
    y = b200k.rmsnorm(torch.from_numpy(x).cuda().to(torch.bfloat16),
                      torch.from_numpy(w).cuda().to(torch.bfloat16))
    ok, err, _ = allclose_report(y.float().cpu().numpy(), O.rmsnorm(x, w, "bf16"), 2e-2, 8e-3)
    assert ok, err
    assert _lib.lib.b2k_pipeline_timeouts(1) == 0
