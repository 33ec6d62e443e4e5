"""Row sharding across the GPUs of one node (one process per GPU).

Every op of the suite is row-independent, so a batch of M rows is split into
contiguous shards and each rank runs the kernels on its own rows with no
data exchange.  The only exchange is the reduced cross-entropy: each rank
reduces its shard to [sum of valid-row losses, number of valid rows] (two
fp64 values) and the pairs are summed across ranks before the division —
by b2k_ce_reduce_exchange_mean, one kernel that reduces, pushes its pair
into every rank's exchange buffer over NVLink (buffers mapped between the
processes with CUDA IPC) and waits (bounded) for the others' pairs, or,
where that mapping is not available, by one SUM all-reduce over NCCL.
"""
from __future__ import annotations

import os
import threading

import torch

from . import _lib as L


def shard_rows(M: int, rank: int, world: int) -> tuple[int, int]:
    """[r0, r1) of rank `rank`: contiguous, sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"b200k: bad rank {rank} of {world}")
    base, extra = divmod(M, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def allreduce_sumcount(sumcount: torch.Tensor, group=None) -> torch.Tensor:
    """In-place SUM all-reduce of a [loss_sum, valid_count] pair over the
    process group (no-op without an initialised group of size > 1)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(sumcount, op=dist.ReduceOp.SUM, group=group)
    return sumcount


def mean_from_sumcount(sumcount: torch.Tensor) -> float:
    """Host-side form of b2k_ce_mean (for CPU tests of the protocol)."""
    s, c = float(sumcount[0]), float(sumcount[1])
    return s / c if c else float("nan")


# ---------------------------------------------------------------------------
# peer-memory exchange for the reduced cross-entropy

_XCHG: dict = {}
_XCHG_LOCK = threading.Lock()
XCHG_LIMIT_NS = 2_000_000_000  # bounded device wait for the other ranks


def _group_key(group):
    import torch.distributed as dist
    g = group if group is not None else dist.group.WORLD
    return g, getattr(g, "group_name", None) or str(id(g))


def close_exchanges():
    """Release every exchange buffer (call before destroy_process_group)."""
    with _XCHG_LOCK:
        for x in _XCHG.values():
            if x is not None:
                x.close()
        _XCHG.clear()


class CeExchange:
    """One rank's exchange buffer and the device table of every rank's buffer
    as mapped in this process, set up once per (process group, device): each
    rank allocates its buffer (b2k_ce_exchange_alloc), the 64-byte CUDA IPC
    handles are all-gathered over the process group, and every peer buffer is
    opened with b2k_ipc_open (plain peer mapping over NVLink).  Every rank
    takes the same collectives whatever fails locally; `ok` says whether this
    rank's side worked (the caller agrees on it across ranks)."""

    def __init__(self, group, device):
        import ctypes
        import torch.distributed as dist
        g, _ = _group_key(group)
        self.world = dist.get_world_size(g)
        self.rank = dist.get_rank(g)
        self.device = device
        self.buf = None
        self.opened = []
        self.ok = False
        with torch.cuda.device(device):
            h = (ctypes.c_uint8 * 64)()
            local_ok = 1
            try:
                p = ctypes.c_void_p()
                L.check(L.lib.b2k_ce_exchange_alloc(self.world, ctypes.byref(p)),
                        "b2k_ce_exchange_alloc")
                self.buf = p.value
                L.check(L.lib.b2k_ipc_handle(ctypes.c_void_p(self.buf), h), "b2k_ipc_handle")
            except Exception:
                local_ok = 0
            mine = torch.tensor(list(bytes(h)) + [local_ok], dtype=torch.uint8, device=device)
            allh = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(allh, mine, group=g)
            allh = [t.cpu().tolist() for t in allh]
            if not all(t[64] == 1 for t in allh):
                return
            try:
                ptrs = []
                for r, t in enumerate(allh):
                    if r == self.rank:
                        ptrs.append(self.buf)
                        continue
                    q = ctypes.c_void_p()
                    L.check(L.lib.b2k_ipc_open((ctypes.c_uint8 * 64)(*t[:64]), ctypes.byref(q)),
                            "b2k_ipc_open")
                    self.opened.append(q.value)
                    ptrs.append(q.value)
                self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)
                # sticky failure word of the exchange kernel (0 = healthy) and
                # its copy in pinned host memory, read without a host sync
                self.status = torch.zeros(1, dtype=torch.int32, device=device)
                self.status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
                self.status_event = torch.cuda.Event()
                self.failed = 0
                torch.cuda.synchronize(device)
                self.ok = True
            except Exception:
                self.ok = False

    _WHY = {1: "a rank's wait for the others' [loss sum, valid count] ran out",
            2: "a peer ran two steps ahead (it had given up waiting)"}

    def _raise(self, v):
        self.failed = v
        raise L.B200KError(
            f"b200k: the cross-entropy exchange of rank {self.rank}/{self.world} failed "
            f"(status {v}: {self._WHY.get(v, 'unknown')}); its means since then are NaN. "
            "Set up the process group and the exchange again (close_exchanges()).")

    def raise_if_failed(self):
        """Raises if an earlier call on this rank reported a failure.  Reads
        the status copied after the previous call only once that copy has
        completed (no host synchronisation)."""
        if self.failed:
            self._raise(self.failed)
        if torch.cuda.is_current_stream_capturing():
            return  # no event query inside a stream capture
        if self.status_event.query():
            v = int(self.status_host[0])
            if v:
                self._raise(v)

    def after_launch(self):
        """Queues, on the current stream, the copy of the status word to pinned
        host memory (skipped while the stream is being captured into a CUDA
        graph; exchange_status() reads it after a replay)."""
        if torch.cuda.is_current_stream_capturing():
            return
        self.status_host.copy_(self.status, non_blocking=True)
        self.status_event.record(torch.cuda.current_stream(self.device))

    def check_now(self) -> int:
        """Synchronises the device and returns the status word (0 = healthy)."""
        torch.cuda.synchronize(self.device)
        return int(self.status.item())

    def close(self):
        """Unmap the peers' buffers and free this rank's (after the last use)."""
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for q in self.opened:
                L.lib.b2k_ipc_close(q)
            self.opened = []
            if self.buf is not None:
                L.lib.b2k_ce_exchange_free(self.buf)
                self.buf = None


def ce_exchange(group, device):
    """The cached CeExchange of (group, device), or None when the peer-memory
    path is off (B2K_CE_P2P=0), there is one rank, or the peer mapping cannot
    be set up on every rank (the caller then uses the NCCL all-reduce)."""
    import torch.distributed as dist
    if os.environ.get("B2K_CE_P2P", "1") == "0":
        return None
    if not (dist.is_available() and dist.is_initialized()):
        return None
    g, name = _group_key(group)
    if dist.get_world_size(g) < 2:
        return None
    key = (name, device.index)
    with _XCHG_LOCK:
        if key not in _XCHG:
            x = CeExchange(group, device)
            # every rank takes the same path: peer memory only if all ranks have
            # it.  The agreement also orders every rank's mapping before any
            # rank's first write into a peer buffer.
            ok = torch.tensor([1 if x.ok else 0], dtype=torch.int32, device=device)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=g)
            if int(ok.item()) == 1:
                _XCHG[key] = x
            else:
                x.close()
                _XCHG[key] = None
        return _XCHG[key]


def exchange_status(group=None, device=None) -> int | None:
    """The status word of the cached cross-entropy exchange of (group,
    device) after a device synchronisation: 0 healthy, 1 a wait ran out, 2 a
    peer ran ahead; None when no peer-memory exchange is in use."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return None
    device = device or torch.device("cuda", torch.cuda.current_device())
    _, name = _group_key(group)
    x = _XCHG.get((name, device.index))
    return None if x is None else x.check_now()
