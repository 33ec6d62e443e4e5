"""Host-buffer entry points: run a b200k row op on inputs that live in (pinned)
host memory and get the results back in host memory, with the transfers
overlapped with the kernels.

The rows are cut into chunks.  Chunk i is copied host->device on one stream,
computed on a second and copied device->host on a third, so the PCIe
transfers in both directions and the kernel of different chunks run at the
same time (the H2D and D2H copy engines work in parallel on full-duplex
PCIe).  Operands that are not row-shaped (weights, biases) are copied once
per call.

With equal bandwidth B in both directions, S bytes each way and chunks of at
most s bytes, such a two-stage pipeline ends after (S + s) / B: only a
smaller largest chunk shortens it, and every chunk costs host time to
enqueue (copies, events, the op's launch).

* run_rows_host: enqueues the chunks on every call; returns after the last
  device->host copy has completed.
* RowsHostGraph: captures the same work once, for fixed host buffers, into
  a CUDA graph; each run() replays every copy and kernel with no per-chunk
  host work, so its time does not depend on how busy the host's cores are.

Measured on B200 (PCIe Gen5: 55 GB/s one way, 50 GB/s each way when both
directions run) with x + r -> LayerNorm -> GELU over 16384 x 8192 bf16, 537
MB each way: replays take 12.0-12.3 ms with 8 or 16 MB per operand per chunk
(4 MB: 13.0 ms, 1 MB: 20 ms: per-copy overhead on the device), while the
eager path took 12 to 87 ms for the same chunks depending on host load.
"""
from __future__ import annotations

import torch


def _chunk_rows(row_inputs, chunk_rows, chunk_bytes):
    rows = row_inputs[0].shape[0]
    for t in row_inputs:
        if t.shape[0] != rows:
            raise ValueError("b200k.host: row inputs must share their first dimension")
    if chunk_rows is None:
        row_bytes = max(t[0].numel() * t.element_size() for t in row_inputs) if rows else 1
        chunk_rows = max(1, min(rows, chunk_bytes // max(1, row_bytes)))
    if chunk_rows < 1:
        raise ValueError("b200k.host: chunk_rows must be positive")
    return rows, chunk_rows


def _enqueue(fn, row_inputs, other_inputs, out, chunk_rows, device, n_slots, start,
             capturing):
    """Enqueues every chunk's copies and kernel behind `start` (an event on
    the current stream) and joins the streams back into the current stream.
    Returns (host outputs, single, device outputs kept for a capture)."""
    rows = row_inputs[0].shape[0]
    n_chunks = (rows + chunk_rows - 1) // chunk_rows
    cur = torch.cuda.current_stream(device)
    s_in = torch.cuda.Stream(device)
    s_run = torch.cuda.Stream(device)
    s_out = torch.cuda.Stream(device)
    s_in.wait_event(start)
    s_run.wait_event(start)
    s_out.wait_event(start)

    with torch.cuda.stream(s_in):
        others = [t.to(device, non_blocking=True) for t in other_inputs]
    ev_others = torch.cuda.Event()
    ev_others.record(s_in)
    s_run.wait_event(ev_others)

    slots = [[torch.empty((chunk_rows,) + tuple(t.shape[1:]), dtype=t.dtype, device=device)
              for t in row_inputs] for _ in range(min(n_slots, n_chunks))]
    ev_loaded = [torch.cuda.Event() for _ in range(n_chunks)]
    ev_used = [torch.cuda.Event() for _ in range(n_chunks)]
    ev_done = [torch.cuda.Event() for _ in range(n_chunks)]
    host_out = None if out is None else (tuple(out) if isinstance(out, (tuple, list)) else (out,))
    single = False
    keep = []  # device outputs of every chunk, alive until the call returns

    for i in range(n_chunks):
        r0 = i * chunk_rows
        r1 = min(rows, r0 + chunk_rows)
        n = r1 - r0
        slot = slots[i % len(slots)]
        # H2D of chunk i once chunk i - n_slots has been consumed
        with torch.cuda.stream(s_in):
            if i >= len(slots):
                s_in.wait_event(ev_used[i - len(slots)])
            for d, h in zip(slot, row_inputs):
                d[:n].copy_(h[r0:r1], non_blocking=True)
            ev_loaded[i].record(s_in)
        # compute chunk i
        with torch.cuda.stream(s_run):
            s_run.wait_event(ev_loaded[i])
            res = fn(*[d[:n] for d in slot], *others)
            ev_used[i].record(s_run)
            res = tuple(res) if isinstance(res, (tuple, list)) else (res,)
            if capturing:
                keep.append(res)  # graph-pool memory: keep it out of reuse
            else:
                for t in res:
                    t.record_stream(s_out)
            ev_done[i].record(s_run)
        if host_out is None:
            if capturing:
                raise ValueError("b200k.host: a captured pipeline needs its host outputs")
            single = len(res) == 1
            host_out = tuple(torch.empty((rows,) + tuple(t.shape[1:]), dtype=t.dtype,
                                         pin_memory=True) for t in res)
        if len(res) != len(host_out):
            raise ValueError("b200k.host: the op returned %d outputs for %d host buffers"
                             % (len(res), len(host_out)))
        # D2H of chunk i
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[i])
            for h, d in zip(host_out, res):
                h[r0:r1].copy_(d, non_blocking=True)
    cur.wait_stream(s_out)
    return host_out, single, keep


def run_rows_host(fn, row_inputs, other_inputs=(), *, out=None, chunk_rows=None,
                  device=None, n_slots=3, timing=None):
    """fn(*row_chunks, *other_inputs) -> Tensor or tuple of Tensors, applied to
    row chunks of `row_inputs` (host tensors with the same number of rows);
    results are written into `out` (host tensors, allocated pinned if None;
    required when there are no rows).  Returns the tuple of host outputs (or
    the single output).  `timing`, a
    pair of CUDA events, is recorded around all device work of the call."""
    device = torch.device(device or "cuda")
    # ~32 MB per operand per chunk: large enough to amortise the per-chunk
    # host work, small enough that the pipeline fills quickly
    rows, chunk_rows = _chunk_rows(row_inputs, chunk_rows, 32 << 20)
    if rows == 0 and out is None:
        # the outputs' shapes come from the op's first chunk; with no rows
        # there is none
        raise ValueError("b200k.host: zero rows need the host outputs (`out`)")
    cur = torch.cuda.current_stream(device)
    start = timing[0] if timing else torch.cuda.Event()
    start.record(cur)
    host_out, single = out, False
    if rows:
        host_out, single, _ = _enqueue(fn, row_inputs, other_inputs, out, chunk_rows, device,
                                       n_slots, start, capturing=False)
    if timing:
        timing[1].record(cur)
    cur.synchronize()
    if out is not None:
        return out
    return host_out[0] if single else host_out


class RowsHostGraph:
    """The work of run_rows_host, captured once for fixed host buffers.

    `row_inputs`, `other_inputs` and `out` must be pinned host tensors; they
    stay bound to the graph, so a caller refills the same input buffers and
    calls run() again.  Each run() replays the host->device copies of all
    inputs, the op on every chunk and the device->host copies of all outputs,
    and returns `out` once the last copy has completed.  Construction runs
    the pipeline once eagerly (loads the library, checks the call) and then
    captures it; the device buffers of the chunks stay allocated in the
    graph's memory pool while the object lives.
    """

    def __init__(self, fn, row_inputs, other_inputs=(), *, out, chunk_rows=None, device=None,
                 n_slots=3):
        self.device = torch.device(device or "cuda")
        # ~8 MB per operand per chunk: the replay has no per-chunk host work
        rows, chunk_rows = _chunk_rows(row_inputs, chunk_rows, 8 << 20)
        if rows == 0:
            raise ValueError("b200k.host: a captured pipeline needs at least one row")
        outs = tuple(out) if isinstance(out, (tuple, list)) else (out,)
        for t in list(row_inputs) + list(other_inputs) + list(outs):
            if t.device.type != "cpu" or not t.is_pinned():
                raise ValueError("b200k.host: RowsHostGraph takes pinned host tensors")
        self.out = out
        run_rows_host(fn, row_inputs, other_inputs, out=out, chunk_rows=chunk_rows,
                      device=self.device, n_slots=n_slots)
        self.graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.graph(self.graph, stream=side):
            start = torch.cuda.Event()
            start.record(side)
            _, _, self._keep = _enqueue(fn, row_inputs, other_inputs, outs, chunk_rows,
                                        self.device, n_slots, start, capturing=True)
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.chunk_rows = chunk_rows

    def run(self, timing=None):
        cur = torch.cuda.current_stream(self.device)
        if timing:
            timing[0].record(cur)
        self.graph.replay()
        if timing:
            timing[1].record(cur)
        cur.synchronize()
        return self.out
