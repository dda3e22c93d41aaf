"""BinaryFlatIndex on the B200 (drop-in for python/metalfaiss/index/binary_flat_index.py:12-165).

Vectors are d binary coordinates (d a multiple of 8, up to 1024), given as
(n, d) arrays of 0/1 values as the reference takes them. They are stored
packed, 32 coordinates per uint32 word (mf_binary_pack), and searched by
Hamming distance (the number of differing coordinates) with the popcount scan
and warp top-k of mf_binary_flat_search: no (nq, ntotal) distance matrix and
no full argsort as in the reference (:79-92).

Results: distances int32, labels int64, ascending, ties to the lower row.
k is clipped to ntotal as the reference clips it (:88-90); an empty index
returns distance INT32_MAX with label -1 (the reference returns zeros, :72-76;
-1 marks "no result" as everywhere else in this package).
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _native as nat
from ._tensors import GrowBuffer, as_ids, default_device
from .errors import InvalidArgumentError
from .search_result import SearchRangeResult, SearchResult

INT32_MAX = 2 ** 31 - 1


class BinaryFlatIndex:
    metric = "hamming"

    def __init__(self, d: int, device=None):
        d = int(d)
        if d <= 0 or d % 8 != 0 or d > 1024:
            raise InvalidArgumentError(f"binary dimension must be a multiple of 8 in [8, 1024], "
                                       f"got {d}")
        self.d = d
        self._W = (d + 31) // 32
        self.device = default_device(device)
        self._codes = GrowBuffer((self._W,), torch.int32, self.device)
        self._ids = GrowBuffer((), torch.int64, self.device)
        self._ws = None

    @property
    def ntotal(self) -> int:
        return self._codes.n

    @property
    def is_trained(self) -> bool:
        return True

    def __len__(self) -> int:
        return self.ntotal

    @property
    def codes(self) -> torch.Tensor:
        """Packed rows (ntotal, ceil(d / 32)) as int32 words."""
        return self._codes.view()

    def train(self, xs=None) -> None:
        """No-op, as for the reference's flat binary index."""

    def _pack(self, xs, name="vectors") -> torch.Tensor:
        nat.require_cuda(self.device)
        if torch.is_tensor(xs):
            x = xs.to(self.device, torch.uint8)
        else:
            x = torch.from_numpy(np.ascontiguousarray(np.asarray(xs), dtype=np.uint8)).to(
                self.device)
        if x.dim() == 1:
            x = x.reshape(1, -1)
        if x.dim() != 2 or x.shape[1] != self.d:
            raise InvalidArgumentError(
                f"{name} have dimension {tuple(x.shape)[1:]} != index dimension {self.d}")
        x = x.contiguous()
        if x.numel() and bool((x > 1).any()):
            raise InvalidArgumentError(f"binary {name} must hold 0 / 1 values")
        n = x.shape[0]
        codes = torch.empty((n, self._W), dtype=torch.int32, device=self.device)
        if n:
            nat.call("mf_binary_pack", self.device.index, nat.stream_of(self.device), nat.ptr(x), n,
                     self.d, nat.ptr(codes))
        return codes

    def add(self, xs, ids=None) -> None:
        """python/metalfaiss/index/binary_flat_index.py:27-48 (ids default to
        ntotal + arange, as the float indexes number them)."""
        codes = self._pack(xs)
        n = codes.shape[0]
        if n == 0:
            return
        idt = (torch.arange(self.ntotal, self.ntotal + n, dtype=torch.int64, device=self.device)
               if ids is None else as_ids(ids, n, self.device))
        self._codes.append(codes)
        self._ids.append(idt)

    def reset(self) -> None:
        self._codes.reset()
        self._ids.reset()

    def _workspace(self, nbytes):
        if self._ws is None:
            self._ws = nat.Workspace(self.device)
        return self._ws.get(nbytes)

    def search(self, xs, k: int) -> SearchResult:
        """python/metalfaiss/index/binary_flat_index.py:50-92."""
        q = self._pack(xs, "queries")
        nq = q.shape[0]
        k = int(k)
        if k <= 0:
            raise InvalidArgumentError(f"k must be positive, got {k}")
        if self.ntotal == 0:
            return SearchResult(torch.full((nq, k), INT32_MAX, dtype=torch.int32, device=self.device),
                                torch.full((nq, k), -1, dtype=torch.int64, device=self.device))
        kk = min(k, self.ntotal)
        D = torch.empty((nq, kk), dtype=torch.float32, device=self.device)
        I = torch.empty((nq, kk), dtype=torch.int64, device=self.device)
        if nq:
            nbytes = nat.workspace_size("mf_binary_flat_search_workspace_size", nq, self.ntotal,
                                        self.d, kk)
            ws = self._workspace(nbytes)
            nat.call("mf_binary_flat_search", self.device.index, nat.stream_of(self.device),
                     nat.ptr(q), nq, nat.ptr(self._codes.buf), self.ntotal, self.d, kk,
                     nat.ptr(self._ids.buf), nat.ptr(D), nat.ptr(I), nat.ptr(ws), ws.numel())
        return SearchResult(D.to(torch.int32), I)

    def range_search(self, xs, radius) -> SearchRangeResult:
        """Every row within Hamming distance <= radius, per query in row order
        (python/metalfaiss/index/binary_flat_index.py:94-150)."""
        q = self._pack(xs, "queries")
        nq = q.shape[0]
        lims = torch.zeros(nq + 1, dtype=torch.int64, device=self.device)
        if nq == 0 or self.ntotal == 0:
            e = torch.empty(0, device=self.device)
            return SearchRangeResult(e.to(torch.int32), e.long(), lims)
        r = int(np.floor(float(radius)))
        nbytes = nat.workspace_size("mf_binary_range_workspace_size", nq, self.ntotal, self.d)
        ws = self._workspace(nbytes)
        total = nat.I64(0)
        dev, st = self.device.index, nat.stream_of(self.device)
        nat.call("mf_binary_range_count", dev, st, nat.ptr(q), nq, nat.ptr(self._codes.buf),
                 self.ntotal, self.d, r, nat.ptr(lims), nat.ctypes.byref(total), nat.ptr(ws),
                 ws.numel())
        n = int(total.value)
        D = torch.empty(max(n, 1), dtype=torch.float32, device=self.device)
        L = torch.empty(max(n, 1), dtype=torch.int64, device=self.device)
        if n:
            nat.call("mf_binary_range_fill", dev, st, nat.ptr(q), nq, nat.ptr(self._codes.buf),
                     self.ntotal, self.d, r, nat.ptr(lims), nat.ptr(self._ids.buf), nat.ptr(D),
                     nat.ptr(L), nat.ptr(ws), ws.numel())
        return SearchRangeResult(D[:n].to(torch.int32), L[:n], lims)

    def reconstruct(self, key):
        """Rows by position as 0/1 uint8 (python/metalfaiss/index/binary_flat_index.py:152-170):
        an int gives (1, d) like the reference, an array of positions (m, d);
        ValueError when a position is outside [0, ntotal)."""
        single = isinstance(key, (int, np.integer))
        pos = np.atleast_1d(np.asarray(key, np.int64))
        if pos.size and (pos.min() < 0 or pos.max() >= self.ntotal):
            raise InvalidArgumentError(f"Indices out of bounds [0, {self.ntotal})")
        rows = self._codes.view()[torch.from_numpy(pos).to(self.device)].contiguous()
        out = torch.empty((len(pos), self.d), dtype=torch.uint8, device=self.device)
        if len(pos):
            nat.call("mf_binary_unpack", self.device.index, nat.stream_of(self.device),
                     nat.ptr(rows), len(pos), self.d, nat.ptr(out))
        return out[:1] if single else out

    def __repr__(self) -> str:
        return f"BinaryFlatIndex(d={self.d}, ntotal={self.ntotal})"
