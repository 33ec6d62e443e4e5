"""Fused forward + backward cross-entropy (b2k_cross_entropy_fwd_bwd): the
mean loss and d(mean loss)/d logits against the CPU oracle (softmax minus
one-hot over the valid-row count) on the pipelined path (long rows) and the
row-kernel path (short / odd rows), in place and out of place, plus one
check against torch autograd in fp32.  301 rows give every persistent block
a second row, 3 rows leave most blocks idle, and 40000-wide rows end in a
partial chunk (the first chunk of the back-to-front gradient pass)."""
import numpy as np
import pytest
import torch

import b200k
from gpu_util import to_cuda
from oracle import ops as O
from oracle import regimes
from oracle.numerics import allclose_report, tol_for

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("shape", [(37, 4097), (96, 1000), (24, 128256), (8, 65536),
                                   (301, 40000), (3, 40000)])
@pytest.mark.parametrize("inplace", [False, True])
def test_fwd_bwd_against_oracle(dt, shape, inplace):
    M, V = shape
    case = regimes.make_case("ce", 17, M, V, dt, 3.0, ignore_frac=0.1)
    x, t = to_cuda(case)
    tn = case[1][0].astype(np.int64)
    n_valid = int((tn != -100).sum())
    xin = x.clone() if inplace else x
    loss, dx = b200k.cross_entropy_fwd_bwd(xin, t, grad_scale=float(n_valid), inplace=inplace)
    torch.cuda.synchronize()
    s, c = O.cross_entropy_sum_count(case[0][0], tn)
    assert abs(float(loss) - s / c) <= 1e-3 * abs(s / c)
    # grad_scale = n_valid makes the gradient softmax - onehot, O(1) entries
    ref = O.cross_entropy_grad(case[0][0], tn, dt, grad_scale=float(n_valid))
    ok, err, bad = allclose_report(dx.float().cpu().numpy(), ref, *tol_for("cross_entropy", dt))
    assert ok, f"max err {err}, {bad} bad"
    if inplace:
        assert dx.data_ptr() == xin.data_ptr()
    else:
        assert torch.equal(x, to_cuda(case)[0])  # logits untouched


def test_fwd_bwd_matches_autograd():
    g = torch.Generator(device="cuda").manual_seed(5)
    x = (torch.randn((64, 32000), generator=g, device="cuda") * 3).to(torch.bfloat16)
    t = torch.randint(0, 32000, (64,), generator=g, device="cuda")
    t[::7] = -100
    loss, dx = b200k.cross_entropy_fwd_bwd(x, t)
    xf = x.float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(xf, t, ignore_index=-100)
    ref.backward()
    r = float(ref.detach())
    assert abs(float(loss) - r) <= 1e-3 * abs(r)
    n_valid = int((t != -100).sum())
    got = dx.float() * n_valid
    want = xf.grad * n_valid
    assert torch.allclose(got, want, rtol=2e-2, atol=8e-3), float((got - want).abs().max())


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("grad_scale", [-3.0, 0.0])
def test_fwd_bwd_nonpositive_grad_scale(dt, grad_scale):
    """A positive scale is folded into the exponent of the 16-bit gradient
    pass; zero and negative scales take the plain multiply."""
    M, V = 24, 128256
    case = regimes.make_case("ce", 23, M, V, dt, 3.0, ignore_frac=0.1)
    x, t = to_cuda(case)
    tn = case[1][0].astype(np.int64)
    n_valid = int((tn != -100).sum())
    _, dx = b200k.cross_entropy_fwd_bwd(x, t, grad_scale=grad_scale * n_valid)
    ref = O.cross_entropy_grad(case[0][0], tn, dt, grad_scale=grad_scale * n_valid)
    ok, err, bad = allclose_report(dx.float().cpu().numpy(), ref, *tol_for("cross_entropy", dt))
    assert ok, f"max err {err}, {bad} bad"
