"""IVFFlatIndex on the B200 (drop-in for python/metalfaiss/index/ivf_flat_index.py:21-157).

Layout in HBM: the inverted lists are one CSR bank — list_vecs (N, d) fp32
sorted by list (input order inside a list), list_norms (N), list_ids (N) int64
and list_offsets (nlist+1) int64 — plus the centroids held by the coarse
quantizer (a FlatIndex). search() runs entirely on the device: coarse top-nprobe
(fused distance + warp top-k), grouping of the (query, probe) pairs by list, a
list-major scan that streams each probed list once per group of up to 128
queries (the tensor-core tile; lists probed by at most 16 queries go to a
few-query scan), and an on-device merge of the nprobe partial top-k lists per
query. L2 searches with k <= 16 and 64 <= d <= 128 run as an fp16 filter plus
an exact refinement (mf_ivf_search_filtered), with the same results.

The reference class cannot run end to end (its train never clusters, its add
and search raise AttributeError: python/metalfaiss/index/ivf_flat_index.py:71,89-90,138);
this class implements what those methods document.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _native as nat
from ._tensors import as_ids, as_matrix, default_device, padded_dim, stores_residuals
from .clustering import ClusteringParameters, assign, compute_norms, subsample, train_kmeans
from .errors import BadStateError, InvalidArgumentError, NotImplementedFaissError
from .index_flat import FlatIndex
from .metric_type import SUPPORTED_METRICS, MetricType
from .search_result import SearchRangeResult, SearchResult


class IVFFlatIndex:
    """IVFFlatIndex(quantizer, d, nlist) as in the reference
    (python/metalfaiss/index/ivf_flat_index.py:24), or IVFFlatIndex(d, nlist,
    quantizer=None) as its tests construct it
    (python/metalfaiss/unittest/test_mlx_index.py:54,84)."""

    def __init__(self, *args, quantizer: Optional[FlatIndex] = None, d: Optional[int] = None,
                 nlist: Optional[int] = None, metric_type=MetricType.L2, device=None,
                 clustering: Optional[ClusteringParameters] = None, residuals: bool = True):
        if args and isinstance(args[0], FlatIndex):
            quantizer = args[0]
            args = args[1:]
        if len(args) >= 1:
            d = args[0]
        if len(args) >= 2:
            nlist = args[1]
        if len(args) >= 3:
            if quantizer is None and isinstance(args[2], FlatIndex):
                quantizer = args[2]
            else:
                metric_type = args[2]
        if d is None or nlist is None:
            raise InvalidArgumentError("IVFFlatIndex needs d and nlist")
        self.d = int(d)
        self._nlist = int(nlist)
        if self.d <= 0 or self._nlist <= 0:
            raise InvalidArgumentError(f"bad IVFFlatIndex shape d={d} nlist={nlist}")
        self.metric_type = MetricType.coerce(metric_type)
        # residuals=False: no stored tf32 residuals (half the memory; the scan
        # derives them for d <= 128)
        self._residuals = bool(residuals)
        self._cq = None  # (key, IVF over the centroids) for the coarse step's bound
        if self.metric_type not in SUPPORTED_METRICS:
            raise NotImplementedFaissError(f"metric {self.metric_type.name} is not supported")
        self.device = default_device(device if device is not None else
                                     (quantizer.device if quantizer is not None else None))
        if quantizer is None:
            qmetric = MetricType.INNER_PRODUCT if self.metric_type == MetricType.INNER_PRODUCT else MetricType.L2
            quantizer = FlatIndex(self.d, qmetric, self.device)
        if quantizer.d != self.d:
            raise InvalidArgumentError(f"quantizer dimension {quantizer.d} != {self.d}")
        self._quantizer = quantizer
        self._nprobe = 1
        self._dp = padded_dim(self.d)
        self.clustering = clustering or ClusteringParameters()
        self._is_trained = quantizer.ntotal == self._nlist
        self._ws = None
        self._direct_map = None
        self._clear_lists()

    # --------------------------------------------------------------- state
    def _clear_lists(self):
        dev = self.device
        self._offsets = torch.zeros(self._nlist + 1, dtype=torch.int64, device=dev) \
            if torch.cuda.is_available() else None
        self._vecs = None
        self._norms = None
        self._lo = None  # tf32 residuals of _vecs (tensor-core scan operand)
        self._ids = None
        self._order = None
        self._ntotal = 0
        self._direct_map = None
        self._fbank = None  # filter search bank (fp16 residuals, norms, list stats)

    @property
    def nlist(self) -> int:
        return self._nlist

    @property
    def nprobe(self) -> int:
        return self._nprobe

    @nprobe.setter
    def nprobe(self, value: int) -> None:
        """python/metalfaiss/index/ivf_flat_index.py:48-52."""
        if int(value) < 1:
            raise ValueError("nprobe must be positive")
        self._nprobe = int(value)

    @property
    def quantizer(self) -> FlatIndex:
        return self._quantizer

    @property
    def is_trained(self) -> bool:
        return self._is_trained

    @property
    def ntotal(self) -> int:
        return self._ntotal

    def __len__(self) -> int:
        return self._ntotal

    @property
    def centroids(self) -> torch.Tensor:
        return self._quantizer.xb

    @property
    def list_offsets(self) -> torch.Tensor:
        return self._offsets

    def list_sizes(self) -> np.ndarray:
        return np.diff(self._offsets.cpu().numpy())

    def _workspace(self):
        if self._ws is None:
            self._ws = nat.Workspace(self.device)
        return self._ws

    # ---------------------------------------------------------------- train
    def train(self, xs, niter: Optional[int] = None, seed: Optional[int] = None) -> None:
        """Seeded k-means for the coarse centroids (the reference's train only
        calls the quantizer's no-op train, python/metalfaiss/index/ivf_flat_index.py:59-72)."""
        nat.require_cuda(self.device)
        x = as_matrix(xs, self.d, self.device, "training data")
        if x.shape[0] == 0:
            raise InvalidArgumentError("Empty training data")
        if x.shape[0] < self._nlist:
            raise InvalidArgumentError(
                f"need at least nlist={self._nlist} training points, got {x.shape[0]}")
        p = self.clustering
        x = subsample(x, self._nlist, p)
        c = train_kmeans(x, self._nlist, p.niter if niter is None else niter,
                         p.seed if seed is None else seed)
        self.set_centroids(c[:, : self.d])

    def set_centroids(self, centroids) -> None:
        """Installs given centroids in the quantizer (trained state)."""
        c = as_matrix(centroids, self.d, self.device, "centroids")
        if c.shape[0] != self._nlist:
            raise InvalidArgumentError(f"expected {self._nlist} centroids, got {c.shape[0]}")
        self._quantizer.reset()
        self._quantizer.add(c[:, : self.d])
        self._is_trained = True
        self._fbank = None

    # ------------------------------------------------------------------ add
    def _coarse_assign(self, x: torch.Tensor) -> torch.Tensor:
        q = self._quantizer
        if q.metric_type == MetricType.L2:
            labels, _ = assign(x, q._xb.buf[: q.ntotal], q._norms.buf[: q.ntotal])
            return labels
        return q._search_padded(x, 1, map_ids=False).labels.reshape(-1).contiguous()

    def add(self, xs, ids=None) -> None:
        """Assign each row to its nearest centroid and append it to that list
        (python/metalfaiss/index/ivf_flat_index.py:74-93). Default ids continue
        from ntotal (the reference restarts them at 0 on every call, :91)."""
        if not self._is_trained:
            raise BadStateError("Index must be trained before adding vectors")
        nat.require_cuda(self.device)
        x = as_matrix(xs, self.d, self.device)
        n = x.shape[0]
        if n == 0:
            return
        idt = (torch.arange(self._ntotal, self._ntotal + n, dtype=torch.int64, device=self.device)
               if ids is None else as_ids(ids, n, self.device))
        self._add_assigned(x, idt, self._coarse_assign(x))

    def _add_assigned(self, x: torch.Tensor, idt: torch.Tensor, labels: torch.Tensor) -> None:
        """Appends padded rows x with ids idt to the lists `labels` (int64,
        one per row) names: the CSR merge of IVFFlatIndex.add, for callers
        that have assigned the rows already (a sharded build)."""
        n = x.shape[0]
        if n == 0:
            return
        norms = compute_norms(x)
        total = self._ntotal + n
        out_off = torch.empty(self._nlist + 1, dtype=torch.int64, device=self.device)
        out_vecs = torch.empty((total, self._dp), dtype=torch.float32, device=self.device)
        out_norms = torch.empty(total, dtype=torch.float32, device=self.device)
        out_ids = torch.empty(total, dtype=torch.int64, device=self.device)
        nbytes = nat.workspace_size("mf_ivf_add_workspace_size", self._ntotal, n, self._nlist)
        ws = self._workspace().get(nbytes)
        nat.call("mf_ivf_add", self.device.index, nat.stream_of(self.device), self._nlist, self._dp,
                 nat.ptr(self._offsets), nat.ptr(self._vecs), nat.ptr(self._norms),
                 nat.ptr(self._ids), self._ntotal, nat.ptr(x), nat.ptr(norms), nat.ptr(idt),
                 nat.ptr(labels), n, nat.ptr(out_off), nat.ptr(out_vecs), nat.ptr(out_norms),
                 nat.ptr(out_ids), nat.ptr(ws), ws.numel())
        self._offsets, self._vecs, self._norms, self._ids = out_off, out_vecs, out_norms, out_ids
        if stores_residuals(self._dp, self._residuals):
            self._lo = torch.empty_like(out_vecs)
            nat.call("mf_tf32_residual", self.device.index, nat.stream_of(self.device),
                     nat.ptr(out_vecs), total, self._dp, nat.ptr(self._lo))
        else:
            self._lo = None  # the tensor-core scan derives them
        self._ntotal = total
        self._direct_map = None
        self._fbank = None
        sizes = np.diff(out_off.cpu().numpy())
        # Largest lists first: the scan hands out work in this order.
        order = np.argsort(-sizes, kind="stable").astype(np.int32)
        self._order = torch.from_numpy(order).to(self.device)

    def _install_lists(self, offsets: torch.Tensor, vecs: torch.Tensor, ids: torch.Tensor) -> None:
        """Installs a CSR bank as it stands (offsets (nlist + 1) int64; vecs
        (N, d) grouped by list; ids (N) int64): what read_index restores,
        without reassigning any row."""
        n = int(vecs.shape[0])
        self._clear_lists()
        if n == 0:
            return
        x = as_matrix(vecs, self.d, self.device)
        self._offsets = offsets.to(self.device, torch.int64).contiguous()
        self._vecs = x
        self._norms = compute_norms(x)
        self._ids = ids.to(self.device, torch.int64).contiguous()
        if stores_residuals(self._dp, self._residuals):
            self._lo = torch.empty_like(x)
            nat.call("mf_tf32_residual", self.device.index, nat.stream_of(self.device),
                     nat.ptr(x), n, self._dp, nat.ptr(self._lo))
        self._ntotal = n
        sizes = np.diff(self._offsets.cpu().numpy())
        self._order = torch.from_numpy(np.argsort(-sizes, kind="stable").astype(np.int32)).to(
            self.device)

    def add_with_ids(self, xs, ids) -> None:
        self.add(xs, ids)

    def reset(self) -> None:
        """python/metalfaiss/index/ivf_flat_index.py:153-157 (keeps the trained centroids,
        as FAISS does; the reference also resets its quantizer)."""
        self._clear_lists()

    # --------------------------------------------------------------- search
    def _prepare_query(self, xs):
        if not self._is_trained:
            raise BadStateError("Index must be trained before searching")
        nat.require_cuda(self.device)
        return as_matrix(xs, self.d, self.device, "queries")

    def _empty_lists_guard(self):
        if self._vecs is None:
            # An untouched index: give the kernels a valid empty bank.
            self._vecs = torch.zeros((1, self._dp), dtype=torch.float32, device=self.device)
            self._norms = torch.zeros(1, dtype=torch.float32, device=self.device)
            self._lo = (torch.zeros((1, self._dp), dtype=torch.float32, device=self.device)
                        if stores_residuals(self._dp, self._residuals) else None)
            self._ids = torch.full((1,), -1, dtype=torch.int64, device=self.device)

    def search(self, xs, k: int) -> SearchResult:
        """kNN over the nprobe nearest lists; (nq, k) results padded with
        (+inf, -1) when the probed lists hold fewer than k rows."""
        xq = self._prepare_query(xs)
        k = int(k)
        if k < 0:
            raise InvalidArgumentError(f"k must be non-negative, got {k}")
        nq = xq.shape[0]
        D = torch.empty((nq, k), dtype=torch.float32, device=self.device)
        I = torch.empty((nq, k), dtype=torch.int64, device=self.device)
        if nq == 0 or k == 0:
            return SearchResult(D, I)
        self._check_k(k)
        self._empty_lists_guard()
        q = self._quantizer
        coarse = MetricType.INNER_PRODUCT if self.metric_type == MetricType.INNER_PRODUCT else MetricType.L2
        if q.metric_type != coarse:
            probes = q._search_padded(xq, min(self._nprobe, self._nlist), map_ids=False).labels
            return self._search_preassigned_padded(xq, k, probes)
        cq = self._centroid_index()
        if cq is not None:
            return self._search_preassigned_padded(xq, k, self._coarse_probes(xq, cq))
        if self._filter_ok(k):
            return self._search_filtered(xq, k, D, I)
        m = int(self.metric_type)
        nbytes = nat.workspace_size("mf_ivf_search_workspace_size", nq, self._nlist, self._nprobe,
                                    self._dp, m, k)
        ws = self._workspace().get(nbytes)
        nat.call("mf_ivf_search", self.device.index, nat.stream_of(self.device), nat.ptr(xq), nq,
                 nat.ptr(q._xb.buf), nat.ptr(q._norms.buf), self._nlist, self._nprobe,
                 nat.ptr(self._offsets), nat.ptr(self._vecs), nat.ptr(self._norms),
                 nat.ptr(self._lo), nat.ptr(self._ids), self._vecs.shape[0], nat.ptr(self._order),
                 self._dp, m, k, nat.ptr(D), nat.ptr(I), nat.ptr(ws), ws.numel())
        return SearchResult(D, I)

    # ------------------------------------------------------- filter search
    # L2 searches run as an fp16 tensor-core filter over residuals against the
    # list centroids plus an exact fp32 refinement (mf_ivf_search_filtered):
    # the same exact top-k, with a sixth of the tensor-core work of the 3xTF32
    # scan. The bank (scaled fp16 residuals, their squared norms, per-list
    # bounds and scales) is built on the first such search after an add and
    # kept with the lists.
    filter_search = True

    def _filter_ok(self, k: int) -> bool:
        q = self._quantizer
        return (self.filter_search and self.metric_type == MetricType.L2
                and q.metric_type == MetricType.L2 and self._ntotal > 0
                and q.ntotal == self._nlist
                and nat.load().mf_ivf_filter_eligible(self._dp, int(k), self._ntotal) == 1)

    def _filter_bank(self):
        if self._fbank is None:
            dev = self.device
            n = self._vecs.shape[0]
            h = torch.empty((n, self._dp), dtype=torch.float16, device=dev)
            rn = torch.empty(n, dtype=torch.float32, device=dev)
            rn16 = torch.empty((n, 16), dtype=torch.float16, device=dev)
            stats = torch.empty((self._nlist, 4), dtype=torch.float32, device=dev)
            q = self._quantizer
            nat.call("mf_ivf_filter_bank", dev.index, nat.stream_of(dev), self._nlist, self._dp,
                     nat.ptr(self._offsets), nat.ptr(self._vecs), nat.ptr(self._norms),
                     nat.ptr(q._xb.buf), n, nat.ptr(h), nat.ptr(rn), nat.ptr(rn16),
                     nat.ptr(stats))
            self._fbank = (h, rn, rn16, stats)
        return self._fbank

    def _search_filtered(self, xq, k, D, I) -> SearchResult:
        bf, rn, rn16, stats = self._filter_bank()
        q = self._quantizer
        nq = xq.shape[0]
        nbytes = nat.workspace_size("mf_ivf_search_filtered_workspace_size", nq, self._nlist,
                                    self._nprobe, self._dp, k)
        ws = self._workspace().get(nbytes)
        nat.call("mf_ivf_search_filtered", self.device.index, nat.stream_of(self.device),
                 nat.ptr(xq), nq, nat.ptr(q._xb.buf), nat.ptr(q._norms.buf), self._nlist,
                 self._nprobe, nat.ptr(self._offsets), nat.ptr(self._vecs), nat.ptr(self._norms),
                 nat.ptr(self._lo), nat.ptr(self._ids), self._vecs.shape[0], nat.ptr(self._order),
                 nat.ptr(bf), nat.ptr(rn), nat.ptr(rn16), nat.ptr(stats), self._dp, k, nat.ptr(D),
                 nat.ptr(I), nat.ptr(ws), ws.numel())
        return SearchResult(D, I)

    # ----------------------------------------------- coarse step with a bound
    # Opt-in: with coarse_bound set and at least COARSE_BOUND_MIN_NLIST lists,
    # the coarse step's top-nprobe over the centroids starts from a bound taken
    # from an IVF over the centroids themselves. It pays where the centroids
    # cluster well; on centroids of isotropic mixtures the bound stays loose
    # and the extra passes cost more than they save, so it is off by default.
    coarse_bound = False
    COARSE_BOUND_MIN_NLIST = 2048

    def _centroid_index(self):
        """An IVFFlat index over this index's centroids (~128 centroids per
        list), built on first use and rebuilt when the centroids change; None
        where it does not pay (IP, few lists, small nprobe) or cannot run."""
        q = self._quantizer
        P = min(self._nprobe, self._nlist)
        if (not self.coarse_bound or self.metric_type != MetricType.L2
                or q.metric_type != MetricType.L2
                or self._nlist < self.COARSE_BOUND_MIN_NLIST or P < 8
                or P > nat.load().mf_max_k() or self._dp > 128 or q.ntotal != self._nlist):
            return None
        key = (id(q), q._version)
        if self._cq is not None and self._cq[0] == key:
            return self._cq[1]
        from .clustering import ClusteringParameters as CP
        n2 = max(16, self._nlist // 128)
        cents = q._xb.view()[:, : self.d]
        cq = IVFFlatIndex(self.d, n2, device=self.device,
                          clustering=CP(niter=10, seed=97, max_points_per_centroid=0))
        cq.train(cents)
        cq.add(cents)  # ids = centroid index
        self._cq = (key, cq)
        return cq

    def _coarse_probes(self, xq: torch.Tensor, cq) -> torch.Tensor:
        """Exact top-nprobe centroids: the quantizer's flat search, bounded by
        the nprobe-th distance among the first 128 centroids of the query's
        nearest centroid list (plus the engines' rounding margin)."""
        P = min(self._nprobe, self._nlist)
        near = cq.quantizer._search_padded(xq, 1, map_ids=False).labels.contiguous()
        bound = cq._probe_bound(xq, near, P)
        return self._quantizer._search_bounded(xq, P, bound, map_ids=False).labels.contiguous()

    def _check_k(self, k):
        mk = nat.load().mf_max_k()
        if k > mk or min(self._nprobe, self._nlist) > mk:
            raise NotImplementedFaissError(f"k and nprobe are limited to {mk} on this path")

    def search_preassigned(self, xs, k: int, assign_i, assign_d=None) -> SearchResult:
        """Scan the given lists (nq, nprobe) only
        (python/metalfaiss/unittest/test_mlx_index.py:64-69); assign_d is unused."""
        xq = self._prepare_query(xs)
        probes = assign_i.labels if hasattr(assign_i, "labels") else assign_i
        probes = (probes.to(self.device, torch.int64) if torch.is_tensor(probes)
                  else torch.from_numpy(np.asarray(probes, np.int64)).to(self.device))
        if probes.dim() == 1:
            probes = probes.reshape(-1, 1)
        if probes.shape[0] != xq.shape[0]:
            raise InvalidArgumentError("assign_i must have one row per query")
        k = int(k)
        self._check_k(k)
        self._empty_lists_guard()
        return self._search_preassigned_padded(xq, k, probes.contiguous())

    def _search_preassigned_padded(self, xq, k, probes) -> SearchResult:
        nq = xq.shape[0]
        P = probes.shape[1]
        D = torch.empty((nq, k), dtype=torch.float32, device=self.device)
        I = torch.empty((nq, k), dtype=torch.int64, device=self.device)
        if nq == 0 or k == 0 or P == 0:
            D.fill_(float("inf"))
            I.fill_(-1)
            return SearchResult(D, I)
        m = int(self.metric_type)
        nbytes = nat.workspace_size("mf_ivf_search_preassigned_workspace_size", nq, self._nlist, P,
                                    self._dp, m, k)
        ws = self._workspace().get(nbytes)
        nat.call("mf_ivf_search_preassigned", self.device.index, nat.stream_of(self.device),
                 nat.ptr(xq), nq, nat.ptr(probes), P, self._nlist, nat.ptr(self._offsets),
                 nat.ptr(self._vecs), nat.ptr(self._norms), nat.ptr(self._lo), nat.ptr(self._ids),
                 self._vecs.shape[0], nat.ptr(self._order), self._dp, m, k, nat.ptr(D), nat.ptr(I),
                 nat.ptr(ws), ws.numel())
        return SearchResult(D, I)

    # ------------------------------------------- halves for sharded searches
    def _ivf_args(self, xq, probes, k):
        nq, P = xq.shape[0], probes.shape[1]
        m = int(self.metric_type)
        nbytes = nat.workspace_size("mf_ivf_search_preassigned_workspace_size", nq, self._nlist, P,
                                    self._dp, m, k)
        ws = self._workspace().get(nbytes)
        head = (self.device.index, nat.stream_of(self.device), nat.ptr(xq), nq, nat.ptr(probes), P,
                self._nlist, nat.ptr(self._offsets), nat.ptr(self._vecs), nat.ptr(self._norms),
                nat.ptr(self._lo), nat.ptr(self._ids), self._vecs.shape[0], nat.ptr(self._order),
                self._dp, m, k)
        return head, ws

    def _probe_bound(self, xq: torch.Tensor, probes: torch.Tensor, k: int,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Per query, an upper bound on its k-th distance over its probes, from
        the first rows of its first probe; +inf where this index holds no rows
        of that list (mf_ivf_probe_bound). out: a contiguous (nq,) float32
        tensor to write into."""
        bound = (torch.empty((xq.shape[0],), dtype=torch.float32, device=self.device)
                 if out is None else out)
        if xq.shape[0] == 0 or probes.shape[1] == 0:
            bound.fill_(float("inf"))
            return bound
        self._empty_lists_guard()
        head, ws = self._ivf_args(xq, probes, k)
        nat.call("mf_ivf_probe_bound", *head, nat.ptr(bound), nat.ptr(ws), ws.numel())
        return bound

    def _search_bounded(self, xq: torch.Tensor, k: int, probes: torch.Tensor,
                        bound: torch.Tensor, out=None) -> SearchResult:
        """search_preassigned keeping only rows within bound[q]
        (mf_ivf_search_bounded); fewer than k rows come back padded. out:
        contiguous (nq, k) float32 and int64 tensors to write into."""
        nq = xq.shape[0]
        if out is None:
            D = torch.empty((nq, k), dtype=torch.float32, device=self.device)
            I = torch.empty((nq, k), dtype=torch.int64, device=self.device)
        else:
            D, I = out
        if nq == 0 or k == 0 or probes.shape[1] == 0:
            D.fill_(float("inf"))
            I.fill_(-1)
            return SearchResult(D, I)
        self._empty_lists_guard()
        if self._filter_ok(k):
            bf, rn, rn16, stats = self._filter_bank()
            P = probes.shape[1]
            nbytes = nat.workspace_size("mf_ivf_search_bounded_filtered_workspace_size", nq,
                                        self._nlist, P, self._dp, k)
            ws = self._workspace().get(nbytes)
            nat.call("mf_ivf_search_bounded_filtered", self.device.index,
                     nat.stream_of(self.device), nat.ptr(xq), nq, nat.ptr(probes), P, self._nlist,
                     nat.ptr(self._offsets), nat.ptr(self._vecs), nat.ptr(self._norms),
                     nat.ptr(self._ids), self._vecs.shape[0], nat.ptr(self._order), nat.ptr(bf),
                     nat.ptr(rn), nat.ptr(rn16), nat.ptr(stats), nat.ptr(self._quantizer._xb.buf),
                     self._dp, k,
                     nat.ptr(bound), nat.ptr(D), nat.ptr(I), nat.ptr(ws), ws.numel())
            return SearchResult(D, I)
        head, ws = self._ivf_args(xq, probes, k)
        nat.call("mf_ivf_search_bounded", *head, nat.ptr(bound), nat.ptr(D), nat.ptr(I),
                 nat.ptr(ws), ws.numel())
        return SearchResult(D, I)

    def range_search(self, xs, radius: float) -> SearchRangeResult:
        """Exact range search over the nprobe nearest lists (probe order, then
        list order); see FlatIndex.range_search for the reference's capped form."""
        xq = self._prepare_query(xs)
        nq = xq.shape[0]
        lims = torch.zeros(nq + 1, dtype=torch.int64, device=self.device)
        if nq == 0 or self._ntotal == 0:
            e = torch.empty(0, device=self.device)
            return SearchRangeResult(e.float(), e.long(), lims)
        q = self._quantizer
        coarse = MetricType.INNER_PRODUCT if self.metric_type == MetricType.INNER_PRODUCT else MetricType.L2
        if q.metric_type != coarse:
            raise NotImplementedFaissError("range_search needs the default quantizer metric")
        m = int(self.metric_type)
        nbytes = nat.workspace_size("mf_ivf_range_workspace_size", nq, self._nlist, self._nprobe,
                                    self._dp)
        ws = self._workspace().get(nbytes)
        total = nat.I64(0)
        dev, st = self.device.index, nat.stream_of(self.device)
        nat.call("mf_ivf_range_count", dev, st, nat.ptr(xq), nq, nat.ptr(q._xb.buf),
                 nat.ptr(q._norms.buf), self._nlist, self._nprobe, nat.ptr(self._offsets),
                 nat.ptr(self._vecs), nat.ptr(self._norms), self._dp, m, float(radius),
                 nat.ptr(lims), nat.ctypes.byref(total), nat.ptr(ws), ws.numel())
        n = int(total.value)
        D = torch.empty(max(n, 1), dtype=torch.float32, device=self.device)
        L = torch.empty(max(n, 1), dtype=torch.int64, device=self.device)
        if n:
            nat.call("mf_ivf_range_fill", dev, st, nat.ptr(xq), nq, nat.ptr(q._xb.buf),
                     nat.ptr(q._norms.buf), self._nlist, self._nprobe, nat.ptr(self._offsets),
                     nat.ptr(self._vecs), nat.ptr(self._norms), nat.ptr(self._ids), self._dp, m,
                     float(radius), nat.ptr(lims), nat.ptr(D), nat.ptr(L), nat.ptr(ws), ws.numel())
        return SearchRangeResult(D[:n], L[:n], lims)

    # ----------------------------------------------------------- reconstruct
    def reconstruct(self, key: int) -> torch.Tensor:
        """Vector stored under id `key` (a direct map id → CSR row, built on
        first use; the reference has no IVF reconstruct)."""
        if self._direct_map is None:
            ids = self._ids[: self._ntotal].cpu().numpy() if self._ntotal else np.zeros(0, np.int64)
            order = np.argsort(ids, kind="stable")
            self._direct_map = (ids[order], order)
        sid, order = self._direct_map
        key = int(key)
        pos = np.searchsorted(sid, key)
        if pos >= len(sid) or sid[pos] != key:
            raise InvalidArgumentError(f"id {key} is not in the index")
        return self._vecs[int(order[pos]), : self.d].clone()

    def __repr__(self) -> str:
        return (f"IVFFlatIndex(d={self.d}, nlist={self._nlist}, nprobe={self._nprobe}, "
                f"metric={self.metric_type.name}, ntotal={self._ntotal})")
