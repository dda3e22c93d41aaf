"""IVFPQIndex and ProductQuantizer on the B200 (drop-in for
python/metalfaiss/index/ivf_pq_index.py:25-192 and
python/metalfaiss/index/product_quantizer.py of the reference).

* ProductQuantizer(d, M, nbits): M sub-quantizers of ksub = 2^nbits (<= 256)
  centroids over d / M coordinates each, trained by seeded k-means (25
  iterations, as the reference runs them) on the GPU; compute_codes gives one
  byte per sub-quantizer (mf_pq_encode); decode rebuilds vectors.
* IVFPQIndex(d, nlist, M, nbits=8): coarse centroids by seeded k-means, PQ
  trained on the training rows' residuals against their centroid, lists of
  residual codes as one CSR bank (codes, ids, offsets; rows grouped by list in
  insertion order), searched by the ADC scan mf_ivfpq_search_preassigned over
  the nprobe nearest lists. L2 only, as in the reference.

The reference trains with MLX's random permutations (not reproducible here)
and keeps its lists as Python lists of (id, code) pairs; this class seeds
numpy permutations and keeps one device bank. Empty results are (+inf, -1)
(the reference pads with label 0, :170-174).
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _native as nat
from ._tensors import as_ids, as_matrix, default_device, padded_dim
from .clustering import assign, compute_norms, train_kmeans
from .errors import BadStateError, InvalidArgumentError, NotImplementedFaissError
from .index_flat import FlatIndex
from .metric_type import MetricType
from .search_result import SearchResult

PQ_ITERS = 25  # the reference's k-means iterations (ivf_pq_index.py:59, product_quantizer.py)


class ProductQuantizer:
    """python/metalfaiss/index/product_quantizer.py (FAISS ProductQuantizer)."""

    def __init__(self, d: int, M: int, nbits: int = 8, device=None):
        if M <= 0 or d % M != 0:
            raise InvalidArgumentError(f"Dimension {d} not divisible by number of subquantizers {M}")
        if not 1 <= nbits <= 8:
            raise InvalidArgumentError(f"nbits={nbits}: codes are one byte (1 <= nbits <= 8)")
        if d // M > 32 or M > 64:
            raise InvalidArgumentError(f"M={M}, d={d}: at most 64 sub-quantizers of at most 32 "
                                       "coordinates")
        self.d, self.M, self.nbits = int(d), int(M), int(nbits)
        self.dsub = self.d // self.M
        self.ksub = 1 << self.nbits
        self.code_size = self.M
        # bytes between rows in the device bank: M rounded up to 16, so that a
        # row is whole 16-byte words (the CSR build moves rows as such)
        self.code_pitch = (self.M + 15) // 16 * 16
        self.device = default_device(device)
        self.centroids: Optional[torch.Tensor] = None  # (M, ksub, dsub)

    @property
    def is_trained(self) -> bool:
        return self.centroids is not None

    def train(self, xs, seed: int = 1234, niter: int = PQ_ITERS) -> None:
        """One seeded k-means per sub-space (k = ksub, `niter` Lloyd steps, an
        empty cluster keeps its centroid), on the device."""
        x = as_matrix(xs, self.d, self.device, "training data")
        n = x.shape[0]
        if n < self.ksub:
            raise InvalidArgumentError(f"need at least ksub={self.ksub} training points, got {n}")
        cents = torch.empty((self.M, self.ksub, self.dsub), dtype=torch.float32, device=self.device)
        for m in range(self.M):
            sub = as_matrix(x[:, m * self.dsub:(m + 1) * self.dsub], self.dsub, self.device)
            c = train_kmeans(sub, self.ksub, niter, seed + m)
            cents[m] = c[:, : self.dsub]
        self.centroids = cents.contiguous()

    def _encode(self, x: torch.Tensor, centroids=None, labels=None) -> torch.Tensor:
        if self.centroids is None:
            raise BadStateError("ProductQuantizer must be trained first")
        n, dp = x.shape
        codes = torch.empty((n, self.code_pitch), dtype=torch.uint8, device=self.device)
        if n:
            nat.call("mf_pq_encode", self.device.index, nat.stream_of(self.device), nat.ptr(x), n,
                     dp, self.d, self.M, self.ksub, nat.ptr(self.centroids), nat.ptr(centroids),
                     nat.ptr(labels), nat.ptr(codes), self.code_pitch)
        return codes

    def compute_codes(self, xs) -> torch.Tensor:
        """(n, M) uint8 codes (argmin per sub-space, ties to the lowest code)."""
        x = as_matrix(xs, self.d, self.device)
        return self._encode(x)[:, : self.M]

    def decode(self, codes) -> torch.Tensor:
        """(n, d) reconstructions: the chosen centroid of every sub-space."""
        if self.centroids is None:
            raise BadStateError("ProductQuantizer must be trained first")
        c = torch.as_tensor(codes, device=self.device).long()[:, : self.M]
        parts = [self.centroids[m][c[:, m]] for m in range(self.M)]
        return torch.cat(parts, dim=1)


class IVFPQIndex:
    """python/metalfaiss/index/ivf_pq_index.py:25-192."""

    def __init__(self, d: int, nlist: int, M: int, nbits: int = 8,
                 metric_type=MetricType.L2, device=None, seed: int = 1234):
        if MetricType.coerce(metric_type) != MetricType.L2:
            raise NotImplementedFaissError("IVFPQIndex currently supports L2 metric only")
        if int(nlist) <= 0:
            raise InvalidArgumentError(f"nlist must be positive, got {nlist}")
        self.d = int(d)
        self.metric_type = MetricType.L2
        self._nlist = int(nlist)
        self._nprobe = 1
        self.seed = int(seed)
        self.device = default_device(device)
        self._dp = padded_dim(self.d)
        self._pq = ProductQuantizer(self.d, M, nbits, self.device)
        self._quantizer = FlatIndex(self.d, MetricType.L2, self.device)
        self._is_trained = False
        self._ws = None
        self._clear()

    def _clear(self):
        self._offsets = None
        self._codes = None
        self._ids = None
        self._ntotal = 0

    @property
    def nlist(self) -> int:
        return self._nlist

    @property
    def nprobe(self) -> int:
        return self._nprobe

    @nprobe.setter
    def nprobe(self, value: int) -> None:
        if int(value) < 1:
            raise ValueError("nprobe must be >= 1")
        self._nprobe = int(value)

    @property
    def pq(self) -> ProductQuantizer:
        return self._pq

    @property
    def quantizer(self) -> FlatIndex:
        return self._quantizer

    @property
    def centroids(self) -> torch.Tensor:
        return self._quantizer.xb

    @property
    def is_trained(self) -> bool:
        return self._is_trained

    @property
    def ntotal(self) -> int:
        return self._ntotal

    def __len__(self) -> int:
        return self._ntotal

    def list_sizes(self) -> np.ndarray:
        if self._offsets is None:
            return np.zeros(self._nlist, np.int64)
        return np.diff(self._offsets.cpu().numpy())

    def _workspace(self, nbytes):
        if self._ws is None:
            self._ws = nat.Workspace(self.device)
        return self._ws.get(nbytes)

    def train(self, xs, niter: int = PQ_ITERS) -> None:
        """Coarse k-means over all training rows, then the PQ on their
        residuals against the nearest centroid (:85-102)."""
        nat.require_cuda(self.device)
        x = as_matrix(xs, self.d, self.device, "training data")
        if x.shape[0] == 0:
            raise InvalidArgumentError("Empty training data")
        if x.shape[0] < self._nlist:
            raise InvalidArgumentError(
                f"need at least nlist={self._nlist} training points, got {x.shape[0]}")
        c = train_kmeans(x, self._nlist, niter, self.seed)
        self._quantizer.reset()
        self._quantizer.add(c[:, : self.d])
        labels, _ = assign(x, self._quantizer._xb.buf[: self._nlist],
                           self._quantizer._norms.buf[: self._nlist])
        res = x - self._quantizer._xb.buf[: self._nlist].index_select(0, labels)
        self._pq.train(res[:, : self.d], seed=self.seed + 1, niter=niter)
        self._is_trained = True
        self._clear()

    def add(self, xs, ids=None) -> None:
        """Assign to the nearest centroid, encode the residual, append the code
        to that list (:104-124). Default ids continue from ntotal."""
        if not self._is_trained:
            raise BadStateError("Train index before adding vectors")
        x = as_matrix(xs, self.d, self.device)
        n = x.shape[0]
        if n == 0:
            return
        idt = (torch.arange(self._ntotal, self._ntotal + n, dtype=torch.int64, device=self.device)
               if ids is None else as_ids(ids, n, self.device))
        cents = self._quantizer._xb.buf[: self._nlist]
        labels, _ = assign(x, cents, self._quantizer._norms.buf[: self._nlist])
        codes = self._pq._encode(x, cents, labels)
        # CSR merge of the old bank and the new rows (stable by list): the
        # rows' code bytes travel as opaque 4-byte words through mf_ivf_add
        cw = self._pq.code_pitch // 4
        total = self._ntotal + n
        out_off = torch.empty(self._nlist + 1, dtype=torch.int64, device=self.device)
        out_codes = torch.empty((total, self._pq.code_pitch), dtype=torch.uint8, device=self.device)
        out_nrm = torch.empty(total, dtype=torch.float32, device=self.device)
        out_ids = torch.empty(total, dtype=torch.int64, device=self.device)
        zeros = torch.zeros(n, dtype=torch.float32, device=self.device)
        old_off = (self._offsets if self._offsets is not None else
                   torch.zeros(self._nlist + 1, dtype=torch.int64, device=self.device))
        old_nrm = (torch.zeros(self._ntotal, dtype=torch.float32, device=self.device)
                   if self._ntotal else None)
        nbytes = nat.workspace_size("mf_ivf_add_workspace_size", self._ntotal, n, self._nlist)
        ws = self._workspace(nbytes)
        nat.call("mf_ivf_add", self.device.index, nat.stream_of(self.device), self._nlist, cw,
                 nat.ptr(old_off), nat.ptr(self._codes), nat.ptr(old_nrm), nat.ptr(self._ids),
                 self._ntotal, nat.ptr(codes), nat.ptr(zeros), nat.ptr(idt), nat.ptr(labels), n,
                 nat.ptr(out_off), nat.ptr(out_codes), nat.ptr(out_nrm), nat.ptr(out_ids),
                 nat.ptr(ws), ws.numel())
        self._offsets, self._codes, self._ids = out_off, out_codes, out_ids
        self._ntotal = total

    def add_with_ids(self, xs, ids) -> None:
        self.add(xs, ids)

    def search(self, xs, k: int) -> SearchResult:
        """ADC over the nprobe nearest lists (:127-186)."""
        if not self._is_trained:
            raise BadStateError("Train index before search")
        xq = as_matrix(xs, self.d, self.device, "queries")
        k = int(k)
        if k <= 0:
            raise InvalidArgumentError(f"k must be positive, got {k}")
        nq = xq.shape[0]
        D = torch.full((nq, k), float("inf"), dtype=torch.float32, device=self.device)
        I = torch.full((nq, k), -1, dtype=torch.int64, device=self.device)
        if nq == 0 or self._ntotal == 0:
            return SearchResult(D, I)
        P = min(self._nprobe, self._nlist)
        if P > nat.load().mf_max_k() or k > nat.load().mf_max_k():
            raise NotImplementedFaissError(f"k and nprobe are limited to {nat.load().mf_max_k()}")
        probes = self._quantizer._search_padded(xq, P, map_ids=False).labels.contiguous()
        return self._search_probes(xq, k, probes, D, I)

    def search_preassigned(self, xs, k: int, assign_i) -> SearchResult:
        xq = as_matrix(xs, self.d, self.device, "queries")
        probes = assign_i.labels if hasattr(assign_i, "labels") else assign_i
        probes = torch.as_tensor(np.asarray(probes) if not torch.is_tensor(probes) else probes,
                                 dtype=torch.int64).to(self.device).reshape(xq.shape[0], -1)
        k = int(k)
        D = torch.full((xq.shape[0], k), float("inf"), dtype=torch.float32, device=self.device)
        I = torch.full((xq.shape[0], k), -1, dtype=torch.int64, device=self.device)
        if self._ntotal == 0 or xq.shape[0] == 0:
            return SearchResult(D, I)
        return self._search_probes(xq, k, probes.contiguous(), D, I)

    def _search_probes(self, xq, k, probes, D, I) -> SearchResult:
        nq, P = probes.shape
        nbytes = nat.workspace_size("mf_ivfpq_search_workspace_size", nq, P, k)
        ws = self._workspace(nbytes)
        pq = self._pq
        nat.call("mf_ivfpq_search_preassigned", self.device.index, nat.stream_of(self.device),
                 nat.ptr(xq), nq, self._dp, self.d, nat.ptr(probes), P, self._nlist,
                 nat.ptr(self._quantizer._xb.buf), nat.ptr(pq.centroids), pq.M, pq.ksub,
                 nat.ptr(self._offsets), nat.ptr(self._codes), pq.code_pitch, nat.ptr(self._ids), k,
                 nat.ptr(D), nat.ptr(I), nat.ptr(ws), ws.numel())
        return SearchResult(D, I)

    def list_codes(self):
        """(offsets (nlist + 1), codes (ntotal, M) uint8, ids (ntotal)) of the bank."""
        if self._ntotal == 0:
            return (torch.zeros(self._nlist + 1, dtype=torch.int64),
                    torch.zeros((0, self._pq.M), dtype=torch.uint8), torch.zeros(0, dtype=torch.int64))
        return self._offsets, self._codes[:, : self._pq.M], self._ids

    def reset(self) -> None:
        """Removes the rows; the trained quantizers stay (FAISS semantics; the
        reference also drops its centroids, :188-192)."""
        self._clear()

    def __repr__(self) -> str:
        return (f"IVFPQIndex(d={self.d}, nlist={self._nlist}, M={self._pq.M}, "
                f"nbits={self._pq.nbits}, nprobe={self._nprobe}, ntotal={self._ntotal})")
