"""Multi-process host logic on CPU (gloo, world size 2): the row-sharded
cross-entropy protocol (per-shard [loss sum, valid count], SUM all-reduce,
division) equals the single-process mean, and a rank that dies before the
collective makes the survivor fail with an error inside the process-group
timeout instead of hanging."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(rank, world, port, timeout_s):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "ouroboros-kernelsmith_b200"))
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _ce_worker(rank, world, port, result_dir):
    dist = _setup(rank, world, port, 30)
    import torch
    from b200k.dist import allreduce_sumcount, mean_from_sumcount, shard_rows
    from oracle import regimes, ops as O
    case = regimes.make_case("ce", 5, 37, 1000, "bf16", 3.0, ignore_frac=0.2)
    x, t = case[0][0], case[1][0].astype(np.int64)
    r0, r1 = shard_rows(x.shape[0], rank, world)
    s, c = O.cross_entropy_sum_count(x[r0:r1], t[r0:r1])
    sc = torch.tensor([s, float(c)], dtype=torch.float64)
    allreduce_sumcount(sc)
    np.save(os.path.join(result_dir, f"mean{rank}.npy"), np.array([mean_from_sumcount(sc)]))
    dist.destroy_process_group()


def test_sharded_ce_mean_matches_single_process(tmp_path):
    port = _free_port()
    mp.start_processes(_ce_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    sys.path.insert(0, ROOT)
    from oracle import regimes, ops as O
    case = regimes.make_case("ce", 5, 37, 1000, "bf16", 3.0, ignore_frac=0.2)
    s, c = O.cross_entropy_sum_count(case[0][0], case[1][0].astype(np.int64))
    want = s / c
    for r in range(2):
        got = float(np.load(tmp_path / f"mean{r}.npy")[0])
        assert abs(got - want) <= 1e-12 * max(1.0, abs(want))


def _death_worker(rank, world, port, result_dir):
    dist = _setup(rank, world, port, 4)
    import time
    import torch
    if rank == 1:
        os._exit(0)  # leaves between steps, before the collective
    t0 = time.time()
    sc = torch.ones(2, dtype=torch.float64)
    try:
        dist.all_reduce(sc)
        status = "no-error"
    except Exception as e:  # noqa: BLE001
        status = "error:" + type(e).__name__
    with open(os.path.join(result_dir, "rank0.txt"), "w") as f:
        f.write(f"{status} {time.time() - t0:.1f}")


def test_dead_rank_is_an_error_not_a_hang(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_death_worker, args=(2, port, str(tmp_path)), nprocs=2,
                             start_method="spawn", join=False)
    deadline = 60
    import time
    t0 = time.time()
    while not ctx.join(timeout=1):
        if time.time() - t0 > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail("survivor rank hung past the deadline")
    txt = (tmp_path / "rank0.txt").read_text()
    status, secs = txt.split()
    assert status.startswith("error"), txt
    assert float(secs) < 30
