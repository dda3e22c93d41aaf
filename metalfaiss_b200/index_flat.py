"""FlatIndex: exact kNN on the B200 (drop-in for python/metalfaiss/indexflat.py:16-151).

Storage: the bank lives in HBM as fp32 rows (padded to a multiple of 4) with
their squared norms (computed once at add time) and int64 ids. search() is one
fused kernel pass per (query tile, row split): distances are formed in
registers and fed straight into a per-query warp top-k, so the (nq, ntotal)
distance matrix of the reference (python/metalfaiss/distances.py:140-173 plus a
full-row argsort, python/metalfaiss/utils/sorting.py:71) never exists.
"""
from __future__ import annotations

import copy
from typing import Optional

import numpy as np
import torch

from . import _native as nat
from ._tensors import GrowBuffer, as_ids, as_matrix, default_device, padded_dim, stores_residuals
from .errors import InvalidArgumentError, NotImplementedFaissError
from .metric_type import SUPPORTED_METRICS, MetricType
from .search_result import SearchRangeResult, SearchResult


class FlatIndex:
    def __init__(self, d: int, metric_type=MetricType.L2, device=None,
                 residuals: bool = True) -> None:
        """residuals=False stores no tf32 residuals (half the memory); for
        d <= 128 the tensor-core scan then derives them itself, a little slower."""
        if int(d) <= 0:
            raise InvalidArgumentError(f"dimension must be positive, got {d}")
        self.d = int(d)
        self.metric_type = MetricType.coerce(metric_type)
        if self.metric_type not in SUPPORTED_METRICS:
            raise NotImplementedFaissError(
                f"metric {self.metric_type.name} is outside the B200 search path "
                "(supported: L2, INNER_PRODUCT, L1, LINF)")
        self.device = default_device(device)
        self._dp = padded_dim(self.d)
        self._xb = GrowBuffer((self._dp,), torch.float32, self.device)
        self._norms = GrowBuffer((), torch.float32, self.device)
        # tf32 residuals, stored only where the tensor-core scan cannot derive them
        self._residuals = bool(residuals)
        self._lo = (GrowBuffer((self._dp,), torch.float32, self.device)
                    if stores_residuals(self._dp, self._residuals) else None)
        self._ids = GrowBuffer((), torch.int64, self.device)
        self._ws = None
        self._version = 0  # bumped by every change of the stored rows
        self.verbose = False

    # ------------------------------------------------------------- state
    @property
    def ntotal(self) -> int:
        return self._xb.n

    @property
    def is_trained(self) -> bool:
        return True

    @property
    def xb(self) -> torch.Tensor:
        """Stored vectors (ntotal, d), python/metalfaiss/indexflat.py:26."""
        return self._xb.view()[:, : self.d]

    @property
    def ids(self) -> torch.Tensor:
        return self._ids.view()

    @property
    def norms(self) -> torch.Tensor:
        return self._norms.view()

    def __len__(self) -> int:
        return self.ntotal

    def _workspace(self):
        if self._ws is None:
            self._ws = nat.Workspace(self.device)
        return self._ws

    # ------------------------------------------------------------ mutation
    def train(self, xs=None) -> None:
        """No-op, python/metalfaiss/indexflat.py:30-34."""

    def add(self, xs, ids: Optional[object] = None) -> None:
        """Append vectors; ids default to ntotal + arange (python/metalfaiss/indexflat.py:36-68)."""
        nat.require_cuda(self.device)
        x = as_matrix(xs, self.d, self.device)
        n = x.shape[0]
        if n == 0:
            return
        if ids is None:
            idt = torch.arange(self.ntotal, self.ntotal + n, dtype=torch.int64, device=self.device)
        else:
            idt = as_ids(ids, n, self.device)
        norms = torch.empty(n, dtype=torch.float32, device=self.device)
        st = nat.stream_of(self.device)
        nat.call("mf_vector_norms", self.device.index, st, nat.ptr(x), n, self._dp, nat.ptr(norms))
        if self._lo is not None:
            lo = torch.empty_like(x)
            nat.call("mf_tf32_residual", self.device.index, st, nat.ptr(x), n, self._dp, nat.ptr(lo))
            self._lo.append(lo)
        self._xb.append(x)
        self._norms.append(norms)
        self._ids.append(idt)
        self._version += 1

    def add_with_ids(self, xs, ids) -> None:
        """64-bit ids (python/metalfaiss/unittest/test_mlx_index.py:231-240)."""
        self.add(xs, ids)

    def reset(self) -> None:
        """python/metalfaiss/indexflat.py:127-133."""
        self._version += 1
        self._xb.reset()
        self._norms.reset()
        if self._lo is not None:
            self._lo.reset()
        self._ids.reset()

    def clone(self) -> "FlatIndex":
        """Deep copy, python/metalfaiss/indexflat.py:142-151."""
        out = FlatIndex(self.d, self.metric_type, self.device, self._residuals)
        if self.ntotal:
            out._xb.append(self._xb.view())
            out._norms.append(self._norms.view())
            if self._lo is not None:
                out._lo.append(self._lo.view())
            out._ids.append(self._ids.view())
        return out

    # --------------------------------------------------------------- search
    def search(self, xs, k: int) -> SearchResult:
        """kNN: distances (nq, min(k, ntotal)) ascending and int64 labels
        (python/metalfaiss/indexflat.py:70-110)."""
        nat.require_cuda(self.device)
        if self.ntotal == 0:
            raise InvalidArgumentError("Index is empty; add vectors before searching.")
        k = int(k)
        if k < 0:
            raise InvalidArgumentError(f"k must be non-negative, got {k}")
        xq = as_matrix(xs, self.d, self.device, "queries")
        return self._search_padded(xq, min(k, self.ntotal))

    def _search_padded(self, xq: torch.Tensor, k: int, map_ids: bool = True,
                       out=None) -> SearchResult:
        """out: contiguous (nq, k) float32 and int64 tensors to write into."""
        nq = xq.shape[0]
        if out is None:
            D = torch.empty((nq, k), dtype=torch.float32, device=self.device)
            I = torch.empty((nq, k), dtype=torch.int64, device=self.device)
        else:
            D, I = out
        if nq == 0 or k == 0:
            return SearchResult(D, I)
        if k > nat.load().mf_max_k():
            raise NotImplementedFaissError(
                f"k={k} exceeds the fused top-k limit {nat.load().mf_max_k()}")
        m = int(self.metric_type)
        ws_bytes = nat.workspace_size("mf_flat_search_workspace_size", nq, self.ntotal, self._dp,
                                      m, k)
        ws = self._workspace().get(ws_bytes)
        nat.call("mf_flat_search", self.device.index, nat.stream_of(self.device), nat.ptr(xq), nq,
                 nat.ptr(self._xb.buf), nat.ptr(self._norms.buf), nat.ptr(self._lo.buf if self._lo is not None else None),
                 self.ntotal, self._dp, m, k,
                 nat.ptr(self._ids.buf) if map_ids else nat.ptr(None), nat.ptr(D), nat.ptr(I),
                 nat.ptr(ws), ws.numel())
        return SearchResult(D, I)

    def _search_bounded(self, xq: torch.Tensor, k: int, bound: torch.Tensor,
                        map_ids: bool = True) -> SearchResult:
        """_search_padded given bound[q], an upper bound on each query's k-th
        distance (mf_flat_search_bounded): the same results, fewer candidates."""
        nq = xq.shape[0]
        D = torch.empty((nq, k), dtype=torch.float32, device=self.device)
        I = torch.empty((nq, k), dtype=torch.int64, device=self.device)
        if nq == 0 or k == 0:
            return SearchResult(D, I)
        m = int(self.metric_type)
        ws_bytes = nat.workspace_size("mf_flat_search_workspace_size", nq, self.ntotal, self._dp,
                                      m, k)
        ws = self._workspace().get(ws_bytes)
        nat.call("mf_flat_search_bounded", self.device.index, nat.stream_of(self.device),
                 nat.ptr(xq), nq, nat.ptr(self._xb.buf), nat.ptr(self._norms.buf),
                 nat.ptr(self._lo.buf if self._lo is not None else None), self.ntotal, self._dp,
                 m, k, nat.ptr(self._ids.buf) if map_ids else nat.ptr(None), nat.ptr(bound),
                 nat.ptr(D), nat.ptr(I), nat.ptr(ws), ws.numel())
        return SearchResult(D, I)

    def assign(self, xs, k: int = 1) -> torch.Tensor:
        """Labels of the k nearest stored vectors (python/metalfaiss/index.py:132-143)."""
        return self.search(xs, k).labels

    def range_search(self, xs, radius: float) -> SearchRangeResult:
        """Every stored vector with distance <= radius (squared for L2, -IP for
        INNER_PRODUCT), in storage order per query. The reference filters a
        kNN capped at k=min(100, ntotal) (python/metalfaiss/index.py:90-130); this
        search is exact and uncapped."""
        nat.require_cuda(self.device)
        xq = as_matrix(xs, self.d, self.device, "queries")
        nq = xq.shape[0]
        lims = torch.zeros(nq + 1, dtype=torch.int64, device=self.device)
        if nq == 0 or self.ntotal == 0:
            e = torch.empty(0, device=self.device)
            return SearchRangeResult(e.float(), e.long(), lims)
        m = int(self.metric_type)
        ws_bytes = nat.workspace_size("mf_flat_range_workspace_size", nq, self.ntotal, self._dp)
        ws = self._workspace().get(ws_bytes)
        total = nat.I64(0)
        dev, st = self.device.index, nat.stream_of(self.device)
        args = (nat.ptr(xq), nq, nat.ptr(self._xb.buf), nat.ptr(self._norms.buf), self.ntotal,
                self._dp, m, float(radius))
        nat.call("mf_flat_range_count", dev, st, *args, nat.ptr(lims), nat.ctypes.byref(total),
                 nat.ptr(ws), ws.numel())
        n = int(total.value)
        D = torch.empty(max(n, 1), dtype=torch.float32, device=self.device)
        L = torch.empty(max(n, 1), dtype=torch.int64, device=self.device)
        if n:
            nat.call("mf_flat_range_fill", dev, st, *args, nat.ptr(self._ids.buf), nat.ptr(lims),
                     nat.ptr(D), nat.ptr(L), nat.ptr(ws), ws.numel())
        return SearchRangeResult(D[:n], L[:n], lims)

    # ---------------------------------------------------------- reconstruct
    def reconstruct(self, key: int) -> torch.Tensor:
        """Row `key` (positional), python/metalfaiss/indexflat.py:112-125."""
        key = int(key)
        if self.ntotal == 0 or key < 0 or key >= self.ntotal:
            raise InvalidArgumentError("Invalid key for reconstruction.")
        return self._xb.view()[key, : self.d].clone()

    def reconstruct_n(self, i0: int, n: int) -> torch.Tensor:
        """Rows [i0, i0+n), python/metalfaiss/index.py:168-178."""
        i0, n = int(i0), int(n)
        if i0 < 0 or n < 0 or i0 + n > self.ntotal:
            raise InvalidArgumentError("Invalid range for reconstruction.")
        return self._xb.view()[i0:i0 + n, : self.d].clone()

    def __deepcopy__(self, memo):
        return self.clone()

    def __repr__(self) -> str:
        return f"FlatIndex(d={self.d}, metric={self.metric_type.name}, ntotal={self.ntotal}, device={self.device})"
