"""Searching a sequence of host query batches with the copies overlapped.

A serving loop takes batch after batch from host memory. Searched one at a
time on one stream, each batch's host→device copy and its results' copy back
add to the search. Here batch i + 1's queries are copied in on a copy stream
while batch i is searched, and batch i's results go back on another copy
stream while batch i + 1 is searched; every batch is still copied in, searched
and copied out. The reference searches arrays that MLX keeps in unified
memory and has no copies to hide (python/metalfaiss/index/ivf_flat_index.py:95-151).
"""
from __future__ import annotations

from typing import Callable, Sequence, Tuple

import torch

from .search_result import SearchResult


def search_host_batches(search: Callable[[torch.Tensor], SearchResult],
                        batches: Sequence[torch.Tensor],
                        outs: Sequence[Tuple[torch.Tensor, torch.Tensor]],
                        device) -> None:
    """Runs search(queries on `device`) over every host batch, the results of
    batch i copied into outs[i] = (distances, labels), host tensors of the
    result's shapes (pinned, for the copies to be asynchronous).

    `search` enqueues its work on the current stream (every index search
    does). The copies are enqueued on two streams of their own, ordered
    against the current stream by events; on return the current stream waits
    for the last copy, so the results are in place once it is synchronized.
    Two device buffers hold the queries: batch i + 1 is copied in while batch
    i is searched, batch i + 2 only after batch i's search is done."""
    dev = torch.device(device)
    n = len(batches)
    if len(outs) != n:
        raise ValueError(f"{n} batches but {len(outs)} result buffers")
    if n == 0:
        return
    cur = torch.cuda.current_stream(dev)
    h2d = torch.cuda.Stream(dev)
    d2h = torch.cuda.Stream(dev)
    # nothing of this call starts before the work already on the current stream
    h2d.wait_stream(cur)
    d2h.wait_stream(cur)
    bufs = [None, None]
    freed = [None, None]

    def copy_in(i):
        slot = i % 2
        hb = batches[i]
        if bufs[slot] is None or bufs[slot].shape != hb.shape or bufs[slot].dtype != hb.dtype:
            # allocated on the current stream, which waits for each copy
            # into it before using it
            bufs[slot] = torch.empty(hb.shape, dtype=hb.dtype, device=dev)
        with torch.cuda.stream(h2d):
            if freed[slot] is not None:
                h2d.wait_event(freed[slot])
            bufs[slot].copy_(hb, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(h2d)
        return ev

    ready = copy_in(0)
    for i in range(n):
        nxt = copy_in(i + 1) if i + 1 < n else None
        cur.wait_event(ready)
        r = search(bufs[i % 2])
        done = torch.cuda.Event()
        done.record(cur)
        freed[i % 2] = done
        D_out, I_out = outs[i]
        with torch.cuda.stream(d2h):
            d2h.wait_event(done)
            D_out.copy_(r.distances, non_blocking=True)
            I_out.copy_(r.labels, non_blocking=True)
        # the results stay allocated until the copy stream has read them
        r.distances.record_stream(d2h)
        r.labels.record_stream(d2h)
        ready = nxt
    cur.wait_stream(d2h)
    cur.wait_stream(h2d)
