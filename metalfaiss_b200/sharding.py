"""Database sharding over the GPUs of one node (one process per GPU).

The reference has no multi-device code (python/metalfaiss/faissmlx/resources.py:24-26);
its tests describe the intent: a sharded flat index equal to the single one
(python/metalfaiss/unittest/test_mlx_multi_gpu.py:49-65) and an IVF index
sharded with a shared quantizer (:86-119), and its facade stubs IndexShards
(python/metalfaiss/faiss_compat.py:326-366).

* IVFFlat: inverted lists are partitioned over the ranks by greedy LPT on list
  size; the coarse quantizer is replicated, and so are the first rows of every
  list (the head bank: the rows the bound pass reads, about 2.1 M rows of the
  20 M-row index). A search has two exchange steps:
  1. each rank runs the coarse step for its share of the queries and, from the
     head bank, those queries' upper bounds on the k-th distance; one
     all-gather gives every rank all (nq, nprobe) probe lists and nq bounds;
  2. each rank scans only the lists it owns, keeping rows within the bound,
     and one all-gather of the (nq, k) partial results (distances and labels
     in one buffer) feeds the on-device merge, which reads them in place.
  Without a head bank the bounds come from the ranks that hold each query's
  nearest list and a MIN all-reduce (a third exchange step).
* Flat: contiguous row shards; labels are global ids; one all-gather + merge.
Collectives go through torch.distributed (NCCL on GPUs, gloo in CPU tests).
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from . import _native as nat
from .search_result import SearchResult


def lpt_partition(sizes, world: int) -> np.ndarray:
    """Owner rank of each list: lists in decreasing size, each to the currently
    least-loaded rank (ties to the lower rank)."""
    sizes = np.asarray(sizes, np.int64)
    owners = np.zeros(len(sizes), np.int32)
    if world <= 1:
        return owners
    load = np.zeros(world, np.int64)
    for l in np.argsort(-sizes, kind="stable"):
        r = int(np.argmin(load))
        owners[l] = r
        load[r] += sizes[l]
    return owners


def row_shard(n: int, rank: int, world: int):
    """Contiguous [begin, end) rows of `rank` (sizes differ by at most one)."""
    base, rem = divmod(n, world)
    begin = rank * base + min(rank, rem)
    return begin, begin + base + (1 if rank < rem else 0)


def gather_partials(D: torch.Tensor, I: torch.Tensor, group=None):
    """All-gather of each rank's (nq, k) results → (nq, world, k) on every rank."""
    world = dist.get_world_size(group)
    nq, k = D.shape
    if dist.get_backend(group) == "nccl":
        gd = torch.empty((world * nq, k), dtype=D.dtype, device=D.device)
        gi = torch.empty((world * nq, k), dtype=I.dtype, device=I.device)
        dist.all_gather_into_tensor(gd, D.contiguous(), group=group)
        dist.all_gather_into_tensor(gi, I.contiguous(), group=group)
        gd = gd.view(world, nq, k)
        gi = gi.view(world, nq, k)
    else:
        ld = [torch.empty_like(D) for _ in range(world)]
        li = [torch.empty_like(I) for _ in range(world)]
        dist.all_gather(ld, D.contiguous(), group=group)
        dist.all_gather(li, I.contiguous(), group=group)
        gd = torch.stack(ld)
        gi = torch.stack(li)
    return gd.permute(1, 0, 2).contiguous(), gi.permute(1, 0, 2).contiguous()


def gather_rows(local: torch.Tensor, n: int, group=None) -> torch.Tensor:
    """All-gather of row shards: rank r holds rows row_shard(n, r, world) of an
    (n, ...) array; every rank gets the whole array, in row order."""
    world = dist.get_world_size(group)
    m = -(-n // world) if n else 0
    buf = torch.zeros((m,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    buf[: local.shape[0]] = local
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * m,) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        dist.all_gather_into_tensor(out, buf.contiguous(), group=group)
        parts = list(out.split(m)) if m else [out] * world
    else:
        parts = [torch.empty_like(buf) for _ in range(world)]
        dist.all_gather(parts, buf.contiguous(), group=group)
    rows = []
    for r in range(world):
        b, e = row_shard(n, r, world)
        rows.append(parts[r][: e - b])
    return torch.cat(rows)


def _half(n: int) -> int:
    return (n + 1) // 2


def probe_buffer(nq: int, nprobe: int, rank: int, world: int, device):
    """This rank's send buffer of exchange_probes and the views the coarse
    step and the bound pass write into: int64 words, first the (m, nprobe)
    probes of its m = row_shard queries, then the m bounds as float32 (the
    layout of every rank is sized for the largest share)."""
    b, e = row_shard(nq, rank, world)
    mmax = -(-nq // world) if nq else 0
    send = torch.empty(mmax * nprobe + _half(mmax), dtype=torch.int64, device=device)
    m = e - b
    probes = send[: m * nprobe].view(m, nprobe)
    bound = send[mmax * nprobe:].view(torch.float32)[:m]
    return send, probes, bound


def exchange_probes(send: torch.Tensor, nq: int, nprobe: int, group=None):
    """One all-gather of every rank's probe_buffer → the (nq, nprobe) probes
    and (nq,) bounds of all queries, in query order, on every rank."""
    world = dist.get_world_size(group)
    if nq == 0:  # every rank has the same batch, so none of them gathers
        return (torch.empty((0, nprobe), dtype=torch.int64, device=send.device),
                torch.empty(0, dtype=torch.float32, device=send.device))
    mmax = -(-nq // world)
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world, send.numel()), dtype=send.dtype, device=send.device)
        dist.all_gather_into_tensor(out, send, group=group)
    else:
        parts = [torch.empty_like(send) for _ in range(world)]
        dist.all_gather(parts, send, group=group)
        out = torch.stack(parts)
    bounds = out[:, mmax * nprobe:].view(torch.float32)
    probes, bound = [], []
    for r in range(world):
        b, e = row_shard(nq, r, world)
        probes.append(out[r, : (e - b) * nprobe].view(e - b, nprobe))
        bound.append(bounds[r, : e - b])
    return torch.cat(probes), torch.cat(bound)


def partial_buffer(nq: int, k: int, device):
    """A send buffer for gather_packed and its (nq, k) float32 distance and
    int64 label views: int64 words, the distances first (padded to a word),
    then the labels."""
    hd = _half(nq * k)
    send = torch.empty(hd + nq * k, dtype=torch.int64, device=device)
    D = send[:hd].view(torch.float32)[: nq * k].view(nq, k)
    I = send[hd:].view(nq, k)
    return send, D, I


def gather_packed(send: torch.Tensor, group=None) -> torch.Tensor:
    """One all-gather of every rank's partial_buffer → (world, words)."""
    world = dist.get_world_size(group)
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world, send.numel()), dtype=send.dtype, device=send.device)
        dist.all_gather_into_tensor(out, send, group=group)
        return out
    parts = [torch.empty_like(send) for _ in range(world)]
    dist.all_gather(parts, send, group=group)
    return torch.stack(parts)


def unpack_partials(buf: torch.Tensor, nq: int, k: int):
    """Views of gather_packed's output: (world, nq, k) distances and labels."""
    world = buf.shape[0]
    hd = _half(nq * k)
    D = buf[:, :hd].view(torch.float32)[:, : nq * k].view(world, nq, k)
    I = buf[:, hd:].view(world, nq, k)
    return D, I


def merge_packed(buf: torch.Tensor, nq: int, k_in: int, k: int) -> SearchResult:
    """The (nq, k) merge of gather_packed's output, read in place by
    mf_topk_merge_strided (part p's slot j of query q: distance word
    p * 2 * words + q * k_in + j of the float32 view, label p * words +
    hd + q * k_in + j)."""
    world, words = buf.shape
    hd = _half(nq * k_in)
    D = torch.empty((nq, k), dtype=torch.float32, device=buf.device)
    I = torch.empty((nq, k), dtype=torch.int64, device=buf.device)
    if nq:
        nat.call("mf_topk_merge_strided", buf.device.index, nat.stream_of(buf.device),
                 nat.ptr(buf), k_in, 2 * words, nat.ptr(buf[:, hd:]), k_in, words, nq, world,
                 k_in, k, nat.ptr(D), nat.ptr(I))
    return SearchResult(D, I)


def head_rows(labels: torch.Tensor, nlist: int, rows: int) -> torch.Tensor:
    """Positions, ascending, of the first `rows` rows (in input order) of each
    list, given every row's list: the rows of a head bank."""
    n = labels.shape[0]
    if n == 0:
        return torch.empty(0, dtype=torch.int64, device=labels.device)
    order = torch.sort(labels, stable=True).indices
    counts = torch.bincount(labels, minlength=nlist)
    starts = torch.cumsum(counts, 0) - counts
    pos = torch.arange(n, device=labels.device) - starts[labels[order]]
    return torch.sort(order[pos < rows]).values


def merge_partials(pd: torch.Tensor, pi: torch.Tensor, k: int) -> SearchResult:
    """(nq, parts, k_in) → (nq, k) with the on-device merge kernel."""
    nq, parts, k_in = pd.shape
    D = torch.empty((nq, k), dtype=torch.float32, device=pd.device)
    I = torch.empty((nq, k), dtype=torch.int64, device=pd.device)
    if nq:
        nat.call("mf_topk_merge", pd.device.index, nat.stream_of(pd.device), nat.ptr(pd),
                 nat.ptr(pi), nq, parts, k_in, k, nat.ptr(D), nat.ptr(I))
    return SearchResult(D, I)


def _empty_like_index(index):
    from .index_ivf_flat import IVFFlatIndex

    out = IVFFlatIndex(index.d, index.nlist, quantizer=index.quantizer,
                       metric_type=index.metric_type, device=index.device,
                       residuals=index._residuals)
    out._is_trained = index.is_trained
    out.nprobe = index.nprobe
    return out


def keep_lists(index, keep_mask: np.ndarray, max_rows: Optional[int] = None):
    """A copy of an IVFFlatIndex holding only the lists where keep_mask is True
    (the other lists stay empty), and of those only the first max_rows rows
    when given; shares the quantizer."""
    out = _empty_like_index(index)
    sizes = index.list_sizes()
    keep = np.asarray(keep_mask, bool)
    new_sizes = np.where(keep, sizes, 0)
    if max_rows is not None:
        new_sizes = np.minimum(new_sizes, max_rows)
    offsets = np.zeros(index.nlist + 1, np.int64)
    np.cumsum(new_sizes, out=offsets[1:])
    dev = index.device
    if index.ntotal:
        list_of_row = torch.repeat_interleave(torch.arange(index.nlist, device=dev),
                                              torch.from_numpy(sizes).to(dev))
        row_mask = torch.from_numpy(keep).to(dev)[list_of_row]
        if max_rows is not None:
            starts = torch.from_numpy(index.list_offsets.cpu().numpy()[:-1]).to(dev)
            pos = torch.arange(index.ntotal, device=dev) - starts[list_of_row]
            row_mask &= pos < max_rows
        out._vecs = index._vecs[: index.ntotal][row_mask].contiguous()
        out._norms = index._norms[: index.ntotal][row_mask].contiguous()
        out._lo = (index._lo[: index.ntotal][row_mask].contiguous()
                   if index._lo is not None else None)
        out._ids = index._ids[: index.ntotal][row_mask].contiguous()
        out._ntotal = int(out._ids.shape[0])
    out._offsets = torch.from_numpy(offsets).to(dev)
    order = np.argsort(-new_sizes, kind="stable").astype(np.int32)
    out._order = torch.from_numpy(order).to(dev)
    return out


def train_kmeans_sharded(x: torch.Tensor, k: int, niter: int, init: torch.Tensor,
                         group=None) -> torch.Tensor:
    """Lloyd's k-means over the union of every rank's points x (this rank's
    share, padded rows as from the index): each iteration assigns the local
    points, all-reduces the per-cluster fp64 sums and sizes, and applies the
    same update on every rank, so the centroids stay identical everywhere.
    `init` (k, padded d) must be the same on all ranks (e.g. broadcast from
    rank 0). The reference trains on one device only
    (python/metalfaiss/clustering/any_clustering.py:62-124)."""
    from .clustering import apply_sums, assign, cluster_sums, compute_norms

    c = init.clone().contiguous()
    cache = nat.Workspace(x.device)
    for _ in range(int(niter)):
        labels, _ = assign(x, c, compute_norms(c), cache)
        sums, counts = cluster_sums(x, labels, k, cache)
        dist.all_reduce(sums, op=dist.ReduceOp.SUM, group=group)
        dist.all_reduce(counts, op=dist.ReduceOp.SUM, group=group)
        apply_sums(sums, counts, c)
    return c


def empty_heads(index):
    """An empty index with index's quantizer, to receive a head bank from
    add_owned_rows."""
    return _empty_like_index(index)


def head_bank(index):
    """The head bank of a whole IVFFlatIndex: a copy holding the first
    mf_ivf_bound_rows() rows of every list (what the bound pass reads)."""
    return keep_lists(index, np.ones(index.nlist, bool), nat.load().mf_ivf_bound_rows())


def add_owned_rows(index, xs, rank: int, world: int, ids=None, heads=None) -> np.ndarray:
    """Sharded IVF build: `index` (trained; the same centroids on every rank)
    receives only the rows of xs whose list this rank owns. Every rank
    assigns all rows once (the same result everywhere), the lists are
    partitioned by greedy LPT on their sizes, and each rank appends its own
    lists' rows with their global ids (row positions in xs, or `ids`), in
    input order. Returns the owner rank of every list. The database held by
    a rank is about 1/world of the whole. `heads` (an empty index with the
    same centroids), when given, receives the head bank: the first
    mf_ivf_bound_rows() rows of every list, the same on every rank."""
    from ._tensors import as_ids, as_matrix

    dev = index.device
    x = as_matrix(xs, index.d, dev)
    n = x.shape[0]
    labels = index._coarse_assign(x)
    sizes = torch.bincount(labels, minlength=index.nlist).cpu().numpy()
    owners = lpt_partition(sizes, world)
    mine = torch.from_numpy(owners == rank).to(dev)[labels]
    gid = (torch.arange(n, dtype=torch.int64, device=dev) if ids is None
           else as_ids(ids, n, dev))
    index._add_assigned(x[mine].contiguous(), gid[mine].contiguous(),
                        labels[mine].contiguous())
    if heads is not None:
        h = head_rows(labels, index.nlist, nat.load().mf_ivf_bound_rows())
        heads._add_assigned(x[h].contiguous(), gid[h].contiguous(), labels[h].contiguous())
    return owners


class ShardedIVF:
    """This rank's share of an IVFFlat index; search() returns the merged global top-k.

    Built from a whole index (this rank keeps a copy of its own lists and
    the head bank) or, with `owners` from add_owned_rows, from an index that
    holds only this rank's lists already (and `heads`, the head bank
    add_owned_rows filled, if any)."""

    def __init__(self, index, rank: int, world: int, group=None, owners=None, heads=None):
        self.rank, self.world, self.group = rank, world, group
        if owners is None:
            owners = lpt_partition(index.list_sizes(), world)
            self.local = keep_lists(index, owners == rank)
            heads = head_bank(index) if heads is None else heads
        else:
            self.local = index
        self.heads = heads
        self.owners = np.asarray(owners)
        # a list here collects (phase, CUDA event) pairs of each search
        self.phase_events = None

    @property
    def nprobe(self):
        return self.local.nprobe

    @nprobe.setter
    def nprobe(self, v):
        self.local.nprobe = v

    def _mark(self, name):
        # phase boundaries on the current stream, when a caller asked for them
        if self.phase_events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.phase_events.append((name, ev))

    def search(self, xq, k: int) -> SearchResult:
        idx = self.local
        xq = idx._prepare_query(xq)
        k = int(k)
        nq = xq.shape[0]
        idx._check_k(k)
        P = min(idx.nprobe, idx.nlist)
        self._mark("start")
        if self.heads is not None:
            return self._search_heads(xq, k, P)
        # 1. coarse step over this rank's share of the queries
        b, e = row_shard(nq, self.rank, self.world)
        if e > b:
            mine = idx.quantizer._search_padded(xq[b:e], P, map_ids=False).labels
        else:
            mine = torch.empty((0, P), dtype=torch.int64, device=idx.device)
        self._mark("coarse")
        probes = gather_rows(mine, nq, self.group).contiguous()
        self._mark("gather probes")
        # 2. bounds from the ranks that hold each query's nearest list
        bound = idx._probe_bound(xq, probes, k)
        self._mark("bound pass")
        dist.all_reduce(bound, op=dist.ReduceOp.MIN, group=self.group)
        self._mark("reduce bounds")
        # 3. this rank's lists, within the bound; then gather and merge
        local = idx._search_bounded(xq, k, probes, bound)
        self._mark("list scan")
        pd, pi = gather_partials(local.distances, local.labels, self.group)
        self._mark("gather partials")
        out = merge_partials(pd, pi, k)
        self._mark("merge")
        return out

    def _search_heads(self, xq, k: int, P: int) -> SearchResult:
        idx = self.local
        nq = xq.shape[0]
        dev = idx.device
        if nq == 0 or k == 0:  # the same on every rank: no exchange
            return SearchResult(torch.empty((nq, k), dtype=torch.float32, device=dev),
                                torch.empty((nq, k), dtype=torch.int64, device=dev))
        # 1. this rank's share of the queries: coarse step and bounds (from
        #    the head bank), written into the send buffer; one all-gather
        b, e = row_shard(nq, self.rank, self.world)
        send, mine, mine_bound = probe_buffer(nq, P, self.rank, self.world, dev)
        if e > b:
            scratch = torch.empty((e - b, P), dtype=torch.float32, device=dev)
            idx.quantizer._search_padded(xq[b:e], P, map_ids=False, out=(scratch, mine))
        self._mark("coarse")
        if e > b:
            self.heads._probe_bound(xq[b:e], mine, k, out=mine_bound)
        self._mark("bound pass")
        probes, bound = exchange_probes(send, nq, P, self.group)
        self._mark("gather probes")
        # 2. this rank's lists, within the bound, into the partials' send
        #    buffer; one all-gather; the merge reads the gathered buffer
        psend, D, I = partial_buffer(nq, k, dev)
        idx._search_bounded(xq, k, probes, bound, out=(D, I))
        self._mark("list scan")
        gathered = gather_packed(psend, self.group)
        self._mark("gather partials")
        out = merge_packed(gathered, nq, k, k)
        self._mark("merge")
        return out


class ShardedFlat:
    """Contiguous row shard of a flat database (global ids); search() merges.

    Built from the whole index (this rank copies rows row_shard(...)), or
    with local=True from an index that already holds only this rank's rows
    under their global ids."""

    def __init__(self, index, rank: int, world: int, group=None, local: bool = False):
        from .index_flat import FlatIndex

        self.rank, self.world, self.group = rank, world, group
        if local:
            self.local = index
            return
        b, e = row_shard(index.ntotal, rank, world)
        self.local = FlatIndex(index.d, index.metric_type, index.device, index._residuals)
        if e > b:
            self.local.add(index.xb[b:e], index.ids[b:e])

    def search(self, xq, k: int) -> SearchResult:
        kk = k if self.local.ntotal >= k else self.local.ntotal
        nq = len(xq)
        if kk > 0:
            local = self.local.search(xq, kk)
            D, I = local.distances, local.labels
        else:
            D = torch.empty((nq, 0), device=self.local.device)
            I = torch.empty((nq, 0), dtype=torch.int64, device=self.local.device)
        if kk < k:  # pad so every rank contributes (nq, k)
            D = torch.cat([D, torch.full((nq, k - kk), float("inf"), device=D.device)], 1)
            I = torch.cat([I, torch.full((nq, k - kk), -1, dtype=torch.int64, device=I.device)], 1)
        pd, pi = gather_partials(D, I, self.group)
        return merge_partials(pd, pi, k)
