"""Host-buffer entry point: run a b200k row op on inputs that live in (pinned)
host memory and get the results back in host memory, with the transfers
overlapped with the kernels.

The rows are cut into chunks.  Chunk i is copied host->device on one stream,
computed on a second and copied device->host on a third, so the PCIe
transfers in both directions and the kernel of different chunks run at the
same time (the H2D and D2H copy engines work in parallel on full-duplex
PCIe).  Operands that are not row-shaped (weights, biases) are copied once.
The call returns after the last device->host copy has completed.
"""
from __future__ import annotations

import torch


def run_rows_host(fn, row_inputs, other_inputs=(), *, out=None, chunk_rows=None,
                  device=None, n_slots=3, timing=None):
    """fn(*row_chunks, *other_inputs) -> Tensor or tuple of Tensors, applied to
    row chunks of `row_inputs` (host tensors with the same number of rows);
    results are written into `out` (host tensors, allocated pinned if None).
    Returns the tuple of host outputs (or the single output).  `timing`, a
    pair of CUDA events, is recorded around all device work of the call."""
    device = torch.device(device or "cuda")
    rows = row_inputs[0].shape[0]
    for t in row_inputs:
        if t.shape[0] != rows:
            raise ValueError("b200k.host: row inputs must share their first dimension")
    if chunk_rows is None:
        # ~32 MB per operand per chunk: large enough to amortise launches,
        # small enough that the pipeline fills quickly
        row_bytes = max(t[0].numel() * t.element_size() for t in row_inputs)
        chunk_rows = max(1, min(rows, (32 << 20) // max(1, row_bytes)))
    n_chunks = (rows + chunk_rows - 1) // chunk_rows
    cur = torch.cuda.current_stream(device)
    s_in = torch.cuda.Stream(device)
    s_run = torch.cuda.Stream(device)
    s_out = torch.cuda.Stream(device)
    start = timing[0] if timing else torch.cuda.Event()
    start.record(cur)
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
    ev_sent = [torch.cuda.Event() for _ in range(n_chunks)]
    outs_dev = [None] * n_chunks
    host_out = None if out is None else (out if isinstance(out, (tuple, list)) else (out,))
    single = False

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
            for t in res:
                t.record_stream(s_out)
            outs_dev[i] = res
            ev_done[i].record(s_run)
        if host_out is None:
            single = len(res) == 1
            host_out = tuple(torch.empty((rows,) + tuple(t.shape[1:]), dtype=t.dtype,
                                         pin_memory=True) for t in res)
        # D2H of chunk i
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[i])
            for h, d in zip(host_out, res):
                h[r0:r1].copy_(d, non_blocking=True)
            ev_sent[i].record(s_out)
        outs_dev[i] = None
    cur.wait_stream(s_out)
    if timing:
        timing[1].record(cur)
    cur.synchronize()
    if out is not None and not isinstance(out, (tuple, list)):
        return host_out[0]
    return host_out[0] if single else host_out
