"""FAISS-style facade over the B200 search path
(python/metalfaiss/faiss_compat.py of the reference: IndexFlatL2 / IndexFlatIP
:56-115, IndexIVFFlat :115-147, IndexShards / IndexReplicas :326-366,
normalize_L2 / index_factory / write_index / read_index :372-437).

The reference leaves IndexShards and IndexReplicas as stubs that raise; this
module implements what their docstrings describe, in one process over any set
of CUDA devices:
* IndexShards splits add() over its child indexes (contiguous row blocks,
  successive global ids) and merges their top-k on the device
  (mf_topk_merge) after each child searched on its own GPU. With children on
  different GPUs the searches overlap: every child call only enqueues work on
  its device, and the partial results cross to the merge device as peer copies.
* IndexReplicas mirrors add() to every child and splits the queries of a
  search across them, so replicas on different GPUs search in parallel.
The multi-process form (one process per GPU, NCCL) is sharding.ShardedIVF /
ShardedFlat.
"""
from __future__ import annotations

import re
from typing import List, Optional

import numpy as np
import torch

from . import _native as nat
from .errors import InvalidArgumentError
from .index_flat import FlatIndex
from .index_io import read_index as _read_index
from .index_io import write_index as _write_index
from .index_ivf_flat import IVFFlatIndex
from .metric_type import MetricType
from .search_result import SearchResult


def _unwrap(index):
    return getattr(index, "_impl", index)


class _Wrapper:
    """Common forwarding of the reference's wrappers."""

    _impl = None

    @property
    def d(self) -> int:
        return self._impl.d

    @property
    def ntotal(self) -> int:
        return self._impl.ntotal

    @property
    def is_trained(self) -> bool:
        return self._impl.is_trained

    @property
    def metric_type(self) -> MetricType:
        return self._impl.metric_type

    @property
    def device(self):
        return self._impl.device

    def train(self, xs) -> None:
        self._impl.train(xs)

    def add(self, xs, ids=None) -> None:
        self._impl.add(xs, ids)

    def add_with_ids(self, xs, ids) -> None:
        self._impl.add(xs, ids)

    def search(self, xs, k: int) -> SearchResult:
        return self._impl.search(xs, k)

    def range_search(self, xs, radius: float):
        return self._impl.range_search(xs, radius)

    def reconstruct(self, key: int):
        return self._impl.reconstruct(key)

    def reset(self) -> None:
        self._impl.reset()

    def __len__(self) -> int:
        return self._impl.ntotal


class IndexFlatL2(_Wrapper):
    """python/metalfaiss/faiss_compat.py:56-85: a FlatIndex with metric L2."""

    def __init__(self, d: int, device=None):
        self._impl = FlatIndex(d, MetricType.L2, device=device)


class IndexFlatIP(_Wrapper):
    """python/metalfaiss/faiss_compat.py:86-113: a FlatIndex with metric INNER_PRODUCT
    (distances are negated inner products, ascending, as the reference returns them)."""

    def __init__(self, d: int, device=None):
        self._impl = FlatIndex(d, MetricType.INNER_PRODUCT, device=device)


class IndexIVFFlat(_Wrapper):
    """python/metalfaiss/faiss_compat.py:115-147. The quantizer passed in is
    used as the coarse quantizer (the reference builds its own and ignores it);
    metric is "L2", "IP" / "INNER_PRODUCT" or a MetricType."""

    def __init__(self, quantizer, d: int, nlist: int, metric="L2", device=None):
        m = {"IP": MetricType.INNER_PRODUCT}.get(metric, metric) if isinstance(metric, str) \
            else metric
        q = _unwrap(quantizer) if quantizer is not None else None
        if q is not None and not isinstance(q, FlatIndex):
            raise InvalidArgumentError("the quantizer must be a flat index")
        self._impl = IVFFlatIndex(d, nlist, quantizer=q, metric_type=m,
                                  device=device if q is None else q.device)

    @property
    def nlist(self) -> int:
        return self._impl.nlist

    @property
    def nprobe(self) -> int:
        return self._impl.nprobe

    @nprobe.setter
    def nprobe(self, value: int) -> None:
        self._impl.nprobe = value

    @property
    def quantizer(self) -> FlatIndex:
        return self._impl.quantizer


def _merge_on(device, parts, k: int) -> SearchResult:
    """(D, I) results of several children, each (nq, k) on any device, merged
    into the k best per query on `device` (mf_topk_merge)."""
    nq = parts[0][0].shape[0]
    pd = torch.empty((nq, len(parts), k), dtype=torch.float32, device=device)
    pi = torch.empty((nq, len(parts), k), dtype=torch.int64, device=device)
    for j, (D, I) in enumerate(parts):
        pd[:, j].copy_(D, non_blocking=True)
        pi[:, j].copy_(I, non_blocking=True)
    D = torch.empty((nq, k), dtype=torch.float32, device=device)
    I = torch.empty((nq, k), dtype=torch.int64, device=device)
    if nq:
        nat.call("mf_topk_merge", device.index, nat.stream_of(device), nat.ptr(pd), nat.ptr(pi),
                 nq, len(parts), k, k, nat.ptr(D), nat.ptr(I))
    return SearchResult(D, I)


def _padded(res: SearchResult, k: int) -> tuple:
    """A child's result widened to k slots with (+inf, -1) (a child holding
    fewer than k rows returns fewer)."""
    D, I = res.distances, res.labels
    if D.shape[1] < k:
        nq = D.shape[0]
        D = torch.cat([D, torch.full((nq, k - D.shape[1]), float("inf"), device=D.device)], 1)
        I = torch.cat([I, torch.full((nq, k - I.shape[1]), -1, dtype=torch.int64,
                                     device=I.device)], 1)
    return D, I


class IndexShards:
    """python/metalfaiss/faiss_compat.py:326-345 (a stub there): the database
    split over child indexes, searched by all, merged on the first child's
    device. add() gives each child a contiguous block of rows; with
    successive_ids (the default) the rows keep their global positions as ids.
    Children may live on different GPUs; their searches overlap."""

    def __init__(self, d: int, threaded: bool = False, successive_ids: bool = True):
        self.d = int(d)
        self.threaded = threaded  # kept for parity: child calls are asynchronous already
        self.successive_ids = successive_ids
        self.children: List[object] = []
        self._ntotal_added = 0

    def add_shard(self, index) -> None:
        if _unwrap(index).d != self.d:
            raise InvalidArgumentError(f"shard dimension {_unwrap(index).d} != {self.d}")
        self.children.append(index)

    @property
    def ntotal(self) -> int:
        return sum(_unwrap(c).ntotal for c in self.children)

    @property
    def is_trained(self) -> bool:
        return all(_unwrap(c).is_trained for c in self.children)

    def train(self, xs) -> None:
        for c in self.children:
            _unwrap(c).train(xs)

    def add(self, xs, ids=None) -> None:
        if not self.children:
            raise InvalidArgumentError("IndexShards has no shards")
        n = len(xs)
        if ids is None and self.successive_ids:
            ids = np.arange(self._ntotal_added, self._ntotal_added + n, dtype=np.int64)
        ns = len(self.children)
        for j, c in enumerate(self.children):
            b, e = j * n // ns, (j + 1) * n // ns
            if e > b:
                _unwrap(c).add(xs[b:e], None if ids is None else ids[b:e])
        self._ntotal_added += n

    def search(self, xs, k: int) -> SearchResult:
        if not self.children:
            raise InvalidArgumentError("IndexShards has no shards")
        k = int(k)
        kids = [_unwrap(c) for c in self.children]
        dev = kids[0].device
        parts = []
        for c in kids:
            q = xs.to(c.device) if torch.is_tensor(xs) else xs
            kk = min(k, c.ntotal)
            if kk == 0:
                nq = len(xs)
                parts.append((torch.full((nq, k), float("inf"), device=c.device),
                              torch.full((nq, k), -1, dtype=torch.int64, device=c.device)))
                continue
            parts.append(_padded(c.search(q, kk), k))
        return _merge_on(dev, parts, k)


class IndexReplicas:
    """python/metalfaiss/faiss_compat.py:348-366 (a stub there): every child
    holds the whole database; a search splits its queries across the
    children (contiguous blocks, in order) and concatenates the results on the
    first child's device. Children on different GPUs search in parallel."""

    def __init__(self, d: int):
        self.d = int(d)
        self.children: List[object] = []

    def add_replica(self, index) -> None:
        if _unwrap(index).d != self.d:
            raise InvalidArgumentError(f"replica dimension {_unwrap(index).d} != {self.d}")
        self.children.append(index)

    @property
    def ntotal(self) -> int:
        return _unwrap(self.children[0]).ntotal if self.children else 0

    def train(self, xs) -> None:
        for c in self.children:
            _unwrap(c).train(xs)

    def add(self, xs, ids=None) -> None:
        if not self.children:
            raise InvalidArgumentError("IndexReplicas has no replicas")
        for c in self.children:
            _unwrap(c).add(xs, ids)

    def search(self, xs, k: int) -> SearchResult:
        if not self.children:
            raise InvalidArgumentError("IndexReplicas has no replicas")
        kids = [_unwrap(c) for c in self.children]
        dev = kids[0].device
        nq, nr = len(xs), len(kids)
        outs = []
        for j, c in enumerate(kids):
            b, e = j * nq // nr, (j + 1) * nq // nr
            if e > b:
                q = xs[b:e].to(c.device) if torch.is_tensor(xs) else xs[b:e]
                outs.append(c.search(q, k))
        D = torch.cat([r.distances.to(dev, non_blocking=True) for r in outs])
        I = torch.cat([r.labels.to(dev, non_blocking=True) for r in outs])
        return SearchResult(D, I)


def normalize_L2(x):
    """python/metalfaiss/faiss_compat.py:372-379: rows scaled to unit L2 norm in
    place (norms clamped at 1e-20); numpy or torch."""
    if torch.is_tensor(x):
        n = torch.linalg.vector_norm(x, dim=1, keepdim=True).clamp_min_(1e-20)
        x.div_(n)
        return x
    n = np.maximum(np.linalg.norm(x, axis=1, keepdims=True), 1e-20)
    x /= n.astype(x.dtype)
    return x


_IVF_FLAT = re.compile(r"^IVF(\d+),Flat$")


def index_factory(d: int, description: str, metric=MetricType.L2, device=None):
    """python/metalfaiss/faiss_compat.py:382-411 for the descriptions this path
    covers: "Flat", "FlatIP", "IVF{n},Flat" (metric L2 unless given)."""
    s = description.replace(" ", "")
    m = MetricType.coerce(metric)
    if s == "Flat":
        return IndexFlatIP(d, device) if m == MetricType.INNER_PRODUCT else IndexFlatL2(d, device)
    if s == "FlatIP":
        return IndexFlatIP(d, device)
    hit = _IVF_FLAT.match(s)
    if hit:
        q = IndexFlatIP(d, device) if m == MetricType.INNER_PRODUCT else IndexFlatL2(d, device)
        return IndexIVFFlat(q, d, int(hit.group(1)), m)
    raise InvalidArgumentError(f"Unsupported factory string: {description}")


def write_index(index, path: str) -> None:
    """python/metalfaiss/faiss_compat.py:414-421."""
    _write_index(_unwrap(index), path)


def read_index(path: str, device=None):
    """python/metalfaiss/faiss_compat.py:424-427: the index as its core class."""
    return _read_index(path, device)


__all__ = ["IndexFlatL2", "IndexFlatIP", "IndexIVFFlat", "IndexShards", "IndexReplicas",
           "normalize_L2", "index_factory", "write_index", "read_index"]
