"""BinaryFlatIndex and BinaryIVFIndex on the B200 (drop-ins for
python/metalfaiss/index/binary_flat_index.py:12-165 and
python/metalfaiss/index/binary_ivf_index.py:19-206).

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
from .errors import BadStateError, InvalidArgumentError, NotImplementedFaissError
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

    def _search_codes(self, q: torch.Tensor, k: int):
        """Hamming kNN of packed queries (nq, W) int32: (distances fp32, labels)."""
        nq = q.shape[0]
        D = torch.empty((nq, k), dtype=torch.float32, device=self.device)
        I = torch.empty((nq, k), dtype=torch.int64, device=self.device)
        if nq:
            nbytes = nat.workspace_size("mf_binary_flat_search_workspace_size", nq, self.ntotal,
                                        self.d, k)
            ws = self._workspace(nbytes)
            nat.call("mf_binary_flat_search", self.device.index, nat.stream_of(self.device),
                     nat.ptr(q), nq, nat.ptr(self._codes.buf), self.ntotal, self.d, k,
                     nat.ptr(self._ids.buf), nat.ptr(D), nat.ptr(I), nat.ptr(ws), ws.numel())
        return D, I

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


class BinaryIVFIndex:
    """BinaryIVFIndex(quantizer, d, nlist), python/metalfaiss/index/binary_ivf_index.py:19-200.

    The coarse quantizer is a BinaryFlatIndex holding the nlist binary
    centroids (as the reference's quantizer does); train() fills it when it is
    not full yet: seeded k-means on the 0/1 coordinates as floats, centroids
    rounded to 0/1 (the binary k-means of FAISS's IndexBinaryIVF). The lists are
    one CSR bank of packed codes, rows padded to whole 16-byte words, built by
    mf_ivf_add; search probes the nprobe nearest centroids (Hamming) and scans
    their lists with mf_binary_ivf_search, ranking ties by probe then by row as
    the reference's candidate order does."""

    metric = "hamming"

    def __init__(self, quantizer: Optional[BinaryFlatIndex] = None, d: Optional[int] = None,
                 nlist: Optional[int] = None, device=None, seed: int = 1234):
        if isinstance(quantizer, (int, np.integer)) and d is not None and nlist is None:
            quantizer, d, nlist = None, quantizer, d  # BinaryIVFIndex(d, nlist)
        if d is None or nlist is None:
            raise InvalidArgumentError("BinaryIVFIndex needs d and nlist")
        if quantizer is None:
            quantizer = BinaryFlatIndex(d, device=device)
        if quantizer.d != int(d):
            raise InvalidArgumentError(
                f"Quantizer dimension {quantizer.d} does not match index dimension {d}")
        if int(nlist) <= 0:
            raise InvalidArgumentError("Number of lists must be positive")
        self.d = int(d)
        self._nlist = int(nlist)
        self._nprobe = 1
        self._quantizer = quantizer
        self.device = quantizer.device
        self.seed = int(seed)
        self._W = (self.d + 31) // 32
        self._pitch = (self._W + 3) // 4 * 4  # words per stored row
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
            raise ValueError("nprobe must be positive")
        self._nprobe = int(value)

    @property
    def quantizer(self) -> BinaryFlatIndex:
        return self._quantizer

    @property
    def is_trained(self) -> bool:
        return self._quantizer.ntotal == self._nlist

    @property
    def ntotal(self) -> int:
        return self._ntotal

    def __len__(self) -> int:
        return self._ntotal

    def _workspace(self, nbytes):
        if self._ws is None:
            self._ws = nat.Workspace(self.device)
        return self._ws.get(nbytes)

    def train(self, xs, niter: int = 10) -> None:
        """Fills the quantizer with nlist binary centroids unless it holds them already."""
        if self.is_trained:
            return
        if self._quantizer.ntotal:
            raise InvalidArgumentError("the quantizer must be empty or hold exactly nlist centroids")
        from .clustering import train_kmeans

        self._quantizer._pack(xs)  # validates shape and 0/1 values
        x = (torch.as_tensor(np.asarray(xs) if not torch.is_tensor(xs) else xs)
             .to(self.device, torch.float32))
        if x.shape[0] < self._nlist:
            raise InvalidArgumentError(f"need at least nlist={self._nlist} training vectors")
        dp = (self.d + 3) // 4 * 4
        xp = torch.zeros((x.shape[0], dp), dtype=torch.float32, device=self.device)
        xp[:, : self.d] = x
        c = train_kmeans(xp, self._nlist, niter, self.seed)[:, : self.d]
        self._quantizer.add((c > 0.5).to(torch.uint8))

    def add(self, xs, ids=None) -> None:
        """python/metalfaiss/index/binary_ivf_index.py:91-112 (ids default to ntotal + i)."""
        if not self.is_trained:
            raise BadStateError("Index must be trained before adding vectors")
        codes = self._quantizer._pack(xs)
        n = codes.shape[0]
        if n == 0:
            return
        idt = (torch.arange(self._ntotal, self._ntotal + n, dtype=torch.int64, device=self.device)
               if ids is None else as_ids(ids, n, self.device))
        labels = self._quantizer._search_codes(codes, 1)[1].reshape(-1).contiguous()
        rows = torch.zeros((n, self._pitch), dtype=torch.int32, device=self.device)
        rows[:, : self._W] = codes
        total = self._ntotal + n
        out_off = torch.empty(self._nlist + 1, dtype=torch.int64, device=self.device)
        out_codes = torch.empty((total, self._pitch), dtype=torch.int32, device=self.device)
        out_nrm = torch.empty(total, dtype=torch.float32, device=self.device)
        out_ids = torch.empty(total, dtype=torch.int64, device=self.device)
        zeros = torch.zeros(n, dtype=torch.float32, device=self.device)
        old_off = (self._offsets if self._offsets is not None else
                   torch.zeros(self._nlist + 1, dtype=torch.int64, device=self.device))
        old_nrm = (torch.zeros(self._ntotal, dtype=torch.float32, device=self.device)
                   if self._ntotal else None)
        nbytes = nat.workspace_size("mf_ivf_add_workspace_size", self._ntotal, n, self._nlist)
        ws = self._workspace(nbytes)
        nat.call("mf_ivf_add", self.device.index, nat.stream_of(self.device), self._nlist,
                 self._pitch, nat.ptr(old_off), nat.ptr(self._codes), nat.ptr(old_nrm),
                 nat.ptr(self._ids), self._ntotal, nat.ptr(rows), nat.ptr(zeros), nat.ptr(idt),
                 nat.ptr(labels), n, nat.ptr(out_off), nat.ptr(out_codes), nat.ptr(out_nrm),
                 nat.ptr(out_ids), nat.ptr(ws), ws.numel())
        self._offsets, self._codes, self._ids = out_off, out_codes, out_ids
        self._ntotal = total

    def search(self, xs, k: int) -> SearchResult:
        """python/metalfaiss/index/binary_ivf_index.py:113-185. Raises on an
        empty index, as the reference does."""
        if self._ntotal == 0:
            raise BadStateError("Index is empty")
        q = self._quantizer._pack(xs, "queries")
        nq = q.shape[0]
        k = int(k)
        if k <= 0 or k > nat.load().mf_max_k():
            raise InvalidArgumentError(f"k={k} outside [1, {nat.load().mf_max_k()}]")
        P = min(self._nprobe, self._nlist)
        if P > 64:
            raise NotImplementedFaissError("nprobe is limited to 64 on the binary IVF path")
        probes = self._quantizer._search_codes(q, P)[1].contiguous()
        D = torch.empty((nq, k), dtype=torch.float32, device=self.device)
        I = torch.empty((nq, k), dtype=torch.int64, device=self.device)
        if nq:
            nbytes = nat.workspace_size("mf_binary_ivf_search_workspace_size", nq, P, k)
            ws = self._workspace(nbytes)
            nat.call("mf_binary_ivf_search", self.device.index, nat.stream_of(self.device),
                     nat.ptr(q), nq, nat.ptr(probes), P, self._nlist, nat.ptr(self._offsets),
                     nat.ptr(self._codes), self._pitch, nat.ptr(self._ids), self.d, k, nat.ptr(D),
                     nat.ptr(I), nat.ptr(ws), ws.numel())
        empty = torch.isinf(D)
        Di = torch.nan_to_num(D, posinf=0.0).to(torch.int32)
        Di = torch.where(empty, torch.full_like(Di, INT32_MAX), Di)
        return SearchResult(Di, I)

    def reconstruct(self, key: int):
        """The 0/1 vector stored under id `key` (python/metalfaiss/index/binary_ivf_index.py:187-200)."""
        if self._ntotal == 0:
            raise BadStateError("Index is empty")
        hit = torch.nonzero(self._ids == int(key))
        if hit.numel() == 0:
            raise InvalidArgumentError(f"Invalid key {key}")
        row = self._codes[int(hit[0, 0])][: self._W].contiguous().reshape(1, -1)
        out = torch.empty((1, self.d), dtype=torch.uint8, device=self.device)
        nat.call("mf_binary_unpack", self.device.index, nat.stream_of(self.device), nat.ptr(row), 1,
                 self.d, nat.ptr(out))
        return out[0]

    def reset(self) -> None:
        """Removes the rows and the quantizer's centroids (as the reference does, :202-206)."""
        self._clear()
        self._quantizer.reset()

    def __repr__(self) -> str:
        return f"BinaryIVFIndex(d={self.d}, nlist={self._nlist}, nprobe={self._nprobe}, ntotal={self._ntotal})"
