"""Cross-entropy mean with the exchange in the reducing kernel
(b2k_ce_reduce_exchange_mean).  One GPU: a single rank gives exactly the
b2k_ce_reduce + b2k_ce_mean result, and a second "rank" whose flag nothing
ever sets makes the bounded wait give up, report the timeout and leave the
context usable (no GPU fault, no hang).  Two GPUs (skipped with fewer): two
ranks whose exchange buffers are mapped into each other with CUDA IPC
reproduce the single-GPU mean over all rows, over several steps (both slot
parities), with the same bits on both ranks."""
import os
import socket

import numpy as np
import pytest
import torch

import b200k
from b200k import _lib

pytestmark = pytest.mark.gpu


def _loss_rows(M=3000, V=4096, seed=3):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn((M, V), generator=g, device="cuda") * 3).to(torch.bfloat16)
    t = torch.randint(0, V, (M,), generator=g, device="cuda")
    t[::9] = -100
    row = torch.empty((M,), dtype=torch.float32, device="cuda")
    st = _lib.lib.b2k_cross_entropy(x.data_ptr(), V, t.data_ptr(), row.data_ptr(), M, V,
                                    _lib.BF16, _lib.F32, -100,
                                    torch.cuda.current_stream().cuda_stream)
    assert st == _lib.OK, _lib.last_error()
    return x, t, row


def _call(row, t, peers, rank, world, limit_ns, status=None):
    sc = torch.empty(2, dtype=torch.float64, device="cuda")
    out = torch.empty((), dtype=torch.float32, device="cuda")
    if status is not None:
        st = _lib.lib.b2k_ce_reduce_exchange_mean(
            row.data_ptr(), t.data_ptr(), row.numel(), -100, peers.data_ptr(), rank, world,
            limit_ns, sc.data_ptr(), out.data_ptr(), status.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
        assert st == _lib.OK, _lib.last_error()
        torch.cuda.synchronize()
        return sc, out, int(status.item())
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    st = _lib.lib.b2k_ce_reduce_exchange_mean(
        row.data_ptr(), t.data_ptr(), row.numel(), -100, peers.data_ptr(), rank, world, limit_ns,
        sc.data_ptr(), out.data_ptr(), status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.OK, _lib.last_error()
    torch.cuda.synchronize()
    return sc, out, int(status.item())


def test_single_rank_matches_reduce_and_mean():
    x, t, row = _loss_rows()
    buf = torch.zeros(int(_lib.lib.b2k_ce_exchange_bytes(1)), dtype=torch.uint8, device="cuda")
    peers = torch.tensor([buf.data_ptr()], dtype=torch.int64, device="cuda")
    ref_sc = torch.empty(2, dtype=torch.float64, device="cuda")
    ref = torch.empty((), dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert _lib.lib.b2k_ce_reduce(row.data_ptr(), t.data_ptr(), row.numel(), -100,
                                  ref_sc.data_ptr(), s) == _lib.OK
    assert _lib.lib.b2k_ce_mean(ref_sc.data_ptr(), ref.data_ptr(), s) == _lib.OK
    for _ in range(3):  # epochs 1..3: both slot parities
        sc, out, status = _call(row, t, peers, 0, 1, 1_000_000_000)
        assert status == 0
        assert torch.equal(sc, ref_sc) and torch.equal(out, ref)
    assert float(out) == pytest.approx(float(b200k.cross_entropy_mean(x, t)), rel=0, abs=0)


def test_missing_rank_times_out_and_context_survives():
    torch.cuda.synchronize()
    _lib.lib.b2k_pipeline_timeouts(1)
    _, t, row = _loss_rows(M=500)
    nb = int(_lib.lib.b2k_ce_exchange_bytes(2))
    mine = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    other = torch.zeros(nb, dtype=torch.uint8, device="cuda")  # "rank 1": nothing publishes
    peers = torch.tensor([mine.data_ptr(), other.data_ptr()], dtype=torch.int64, device="cuda")
    sc, out, status = _call(row, t, peers, 0, 2, 50_000_000)  # 50 ms
    assert status == 1 and np.isnan(float(out))
    assert _lib.lib.b2k_pipeline_timeouts(1) == 1
    # the context still works
    x, t2, _ = _loss_rows(M=64, seed=4)
    assert np.isfinite(float(b200k.cross_entropy_mean(x, t2)))
    assert _lib.lib.b2k_pipeline_timeouts(1) == 0


def test_single_rank_pair_exchange_returns_the_pair():
    """b2k_exchange_pair with one rank: the global pair is the local one, over
    several calls (both slot parities), status 0."""
    buf = torch.zeros(int(_lib.lib.b2k_ce_exchange_bytes(1)), dtype=torch.uint8, device="cuda")
    peers = torch.tensor([buf.data_ptr()], dtype=torch.int64, device="cuda")
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    for k in range(3):
        local = torch.tensor([1234.5 + k, 7.0 * k], dtype=torch.float64, device="cuda")
        glob = torch.empty(2, dtype=torch.float64, device="cuda")
        st = _lib.lib.b2k_exchange_pair(local.data_ptr(), peers.data_ptr(), 0, 1, 1_000_000_000,
                                        glob.data_ptr(), status.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
        assert st == _lib.OK, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.equal(glob, local) and int(status.item()) == 0


def test_failed_exchange_stays_failed_and_writes_nothing():
    """After a wait ran out, the status word is sticky: the next call with it
    returns NaN at once, publishes nothing into any buffer and leaves the
    epoch counter alone."""
    _lib.lib.b2k_pipeline_timeouts(1)
    _, t, row = _loss_rows(M=500)
    nb = int(_lib.lib.b2k_ce_exchange_bytes(2))
    mine = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    other = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    peers = torch.tensor([mine.data_ptr(), other.data_ptr()], dtype=torch.int64, device="cuda")
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    _, out, st = _call(row, t, peers, 0, 2, 50_000_000, status)
    assert st == 1 and np.isnan(float(out))
    snap_mine, snap_other = mine.clone(), other.clone()
    _, out, st = _call(row, t, peers, 0, 2, 50_000_000, status)
    assert st == 1 and np.isnan(float(out))
    assert torch.equal(mine, snap_mine) and torch.equal(other, snap_other)
    assert _lib.lib.b2k_pipeline_timeouts(1) == 1  # only the first call waited


def test_peer_flag_ahead_is_an_error():
    """A peer flag above this rank's epoch (a peer that gave up waiting and
    stepped on) is reported as status 2, not taken as an arrival."""
    _lib.lib.b2k_pipeline_timeouts(1)
    _, t, row = _loss_rows(M=500)
    nb = int(_lib.lib.b2k_ce_exchange_bytes(2))
    mine = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    other = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    # the first call runs epoch 1 (slot parity 1); rank 1's flag of parity 1
    # in this rank's buffer sits after the 2 x 2 pairs of 16 B and the three
    # flags before it: byte 2*2*16 + (1*2 + 1)*8 = 88.  Epoch 3 = two ahead.
    mine[88:96] = torch.tensor([3], dtype=torch.int64).view(torch.uint8).cuda()
    peers = torch.tensor([mine.data_ptr(), other.data_ptr()], dtype=torch.int64, device="cuda")
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    _, out, st = _call(row, t, peers, 0, 2, 2_000_000_000, status)
    assert st == 2 and np.isnan(float(out))
    assert _lib.lib.b2k_pipeline_timeouts(1) == 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from b200k import dist as bd
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        g = torch.Generator(device="cuda").manual_seed(11)
        M, V = 4001, 8192
        x = (torch.randn((M, V), generator=g, device="cuda") * 3).to(torch.bfloat16)
        t = torch.randint(0, V, (M,), generator=g, device="cuda")
        t[::7] = -100
        r0, r1 = bd.shard_rows(M, rank, world)
        outs = [float(b200k.cross_entropy_mean(x[r0:r1], t[r0:r1])) for _ in range(5)]
        used = bd.ce_exchange(None, torch.device("cuda", rank)) is not None
        # the fused loss + gradient: valid count and loss sum over peer memory
        loss, dx = b200k.cross_entropy_fwd_bwd(x[r0:r1], t[r0:r1])
        q.put((rank, outs, used, float(loss), dx.float().cpu()))
        torch.cuda.synchronize()
        dist.barrier()
        bd.close_exchanges()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_ranks_match_one_gpu():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # single-GPU reference over all rows
    g = torch.Generator(device="cuda").manual_seed(11)
    M, V = 4001, 8192
    x = (torch.randn((M, V), generator=g, device="cuda") * 3).to(torch.bfloat16)
    t = torch.randint(0, V, (M,), generator=g, device="cuda")
    t[::7] = -100
    ref = float(b200k.cross_entropy_mean(x, t))
    ref_loss, ref_dx = b200k.cross_entropy_fwd_bwd(x, t)
    ref_dx = ref_dx.float().cpu()
    res.sort(key=lambda r: r[0])
    for rank, outs, used, loss, dx in res:
        assert used, f"rank {rank} did not use the peer-memory exchange"
        assert all(o == outs[0] for o in outs)
        # the row losses are the same; sums of two fp64 halves vs one pass may
        # differ in the last bits of the fp64 sum, not in the fp32 mean
        assert abs(outs[0] - ref) <= 1e-6 * abs(ref), (outs[0], ref)
        assert abs(loss - float(ref_loss)) <= 1e-6 * abs(float(ref_loss)), (loss, float(ref_loss))
        r0, r1 = (0, 2001) if rank == 0 else (2001, 4001)
        # the same global valid count scales every rank's rows: equal bits
        assert torch.equal(dx, ref_dx[r0:r1]), f"rank {rank}: gradient differs"
    assert res[0][1][0] == res[1][1][0]  # every rank gets the same bits
    assert res[0][3] == res[1][3]
