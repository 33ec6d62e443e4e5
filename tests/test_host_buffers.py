"""Host-buffer entry points (b200k.host): pinned host inputs in, pinned host
outputs back, with the copies of one chunk overlapped with the kernels of
another.  Every chunk's result must equal the device op applied to the same
rows on the device (bit for bit: same kernel, same rows)."""
import pytest
import torch

from b200k.host import RowsHostGraph, _chunk_rows, run_rows_host


def test_chunk_rows_checks_the_row_inputs():
    assert _chunk_rows([torch.zeros(10, 4)], None, 64) == (10, 4)
    assert _chunk_rows([torch.zeros(10, 4)], 3, 64) == (10, 3)
    with pytest.raises(ValueError):
        _chunk_rows([torch.zeros(10, 4), torch.zeros(9, 4)], None, 64)
    with pytest.raises(ValueError):
        _chunk_rows([torch.zeros(10, 4)], 0, 64)


def test_zero_rows_need_host_outputs():
    with pytest.raises(ValueError):
        run_rows_host(lambda x: x, [torch.zeros(0, 4)])


def test_captured_pipeline_takes_pinned_buffers_only():
    t = torch.zeros(3, 4)
    with pytest.raises(ValueError):
        RowsHostGraph(lambda x: x, [t], out=t)


def _per_chunk(fn, row_inputs, other_inputs, chunk_rows):
    """Device op on each chunk of the rows, concatenated (host tensors)."""
    rows = row_inputs[0].shape[0]
    others = [t.cuda() for t in other_inputs]
    outs = []
    for r0 in range(0, rows, chunk_rows):
        res = fn(*[t[r0:r0 + chunk_rows].cuda() for t in row_inputs], *others)
        outs.append(tuple(res) if isinstance(res, (tuple, list)) else (res,))
    return tuple(torch.cat([o[i] for o in outs]).cpu() for i in range(len(outs[0])))


def _pinned(*shape, dtype, seed, scale=1.0, offset=0.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale + offset).to(dtype).pin_memory()


@pytest.mark.gpu
@pytest.mark.parametrize("chunk_rows", [None, 700, 1])
def test_run_rows_host_rmsnorm(chunk_rows):
    import b200k
    M, N = 3000 if chunk_rows != 1 else 37, 1024
    x = _pinned(M, N, dtype=torch.float16, seed=1)
    w = _pinned(N, dtype=torch.float16, seed=2)
    got = run_rows_host(b200k.rmsnorm, [x], [w], chunk_rows=chunk_rows)
    assert got.is_pinned() and got.shape == x.shape
    (want,) = _per_chunk(b200k.rmsnorm, [x], [w], chunk_rows or M)
    assert torch.equal(got, want)


@pytest.mark.gpu
def test_run_rows_host_two_outputs_into_given_buffers():
    import b200k
    M, N = 2500, 2048
    fn = lambda x, r, w, b: b200k.fused_add_norm(x, r, w, b, norm="layer", act="gelu")
    x = _pinned(M, N, dtype=torch.bfloat16, seed=3)
    r = _pinned(M, N, dtype=torch.bfloat16, seed=4)
    w = _pinned(N, dtype=torch.bfloat16, seed=5, scale=0.1, offset=1.0)
    b = _pinned(N, dtype=torch.bfloat16, seed=6, scale=0.02)
    h = torch.empty_like(x).pin_memory()
    y = torch.empty_like(x).pin_memory()
    ret = run_rows_host(fn, [x, r], [w, b], out=(h, y), chunk_rows=600)
    assert ret[0] is h and ret[1] is y
    hw, yw = _per_chunk(fn, [x, r], [w, b], 600)
    assert torch.equal(h, hw) and torch.equal(y, yw)


@pytest.mark.gpu
def test_run_rows_host_zero_rows():
    import b200k
    x = torch.empty((0, 1024), dtype=torch.float16).pin_memory()
    w = _pinned(1024, dtype=torch.float16, seed=7)
    y = torch.empty_like(x).pin_memory()
    assert run_rows_host(b200k.rmsnorm, [x], [w], out=y) is y


@pytest.mark.gpu
def test_captured_pipeline_replays_new_host_data():
    """Each run() copies the current contents of the bound host buffers: new
    data written into them between runs reaches the device and comes back."""
    import b200k
    M, N, C = 4100, 2048, 512  # 9 chunks, the last one ragged
    fn = lambda x, r, w, b: b200k.fused_add_norm(x, r, w, b, norm="layer", act="gelu")
    x = _pinned(M, N, dtype=torch.bfloat16, seed=8)
    r = _pinned(M, N, dtype=torch.bfloat16, seed=9)
    w = _pinned(N, dtype=torch.bfloat16, seed=10, scale=0.1, offset=1.0)
    b = _pinned(N, dtype=torch.bfloat16, seed=11, scale=0.02)
    h = torch.empty_like(x).pin_memory()
    y = torch.empty_like(x).pin_memory()
    pipe = RowsHostGraph(fn, [x, r], [w, b], out=(h, y), chunk_rows=C)
    for seed in (12, 13):
        x.copy_(_pinned(M, N, dtype=torch.bfloat16, seed=seed))
        w.copy_(_pinned(N, dtype=torch.bfloat16, seed=seed + 100, scale=0.1, offset=1.0))
        h.zero_()
        y.zero_()
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        out = pipe.run(ev)
        assert out[0] is h and ev[0].elapsed_time(ev[1]) > 0
        hw, yw = _per_chunk(fn, [x, r], [w, b], C)
        assert torch.equal(h, hw) and torch.equal(y, yw)


@pytest.mark.gpu
def test_captured_pipeline_single_output():
    import b200k
    M, N = 1000, 4096
    g = _pinned(M, N, dtype=torch.bfloat16, seed=14)
    u = _pinned(M, N, dtype=torch.bfloat16, seed=15)
    y = torch.empty_like(g).pin_memory()
    pipe = RowsHostGraph(b200k.swiglu, [g, u], [], out=y)
    assert pipe.run() is y
    (want,) = _per_chunk(b200k.swiglu, [g, u], [], pipe.chunk_rows)
    assert torch.equal(y, want)
