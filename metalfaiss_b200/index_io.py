"""Index persistence: write_index / read_index for FlatIndex and IVFFlatIndex
(python/metalfaiss/index/index_io.py:31-115 of the reference).

File layout (little-endian). The reference's framing is kept: a u64 header
length L, then L bytes of UTF-8 JSON, then the index's data. The JSON carries
what the reference writes (type, d, ntotal, is_trained, metric) plus:
  * "format": "metalfaiss_b200/1";
  * the index's own fields (IVFFlatIndex: nlist, nprobe);
  * "arrays": one descriptor per array - name, dtype, shape, and the byte
    offset from the start of the data section, which begins at 8 + L rounded
    up to 64 bytes; every array starts on a 64-byte boundary.
Arrays (rows unpadded, d columns):
  * FlatIndex: xb (ntotal, d) float32, ids (ntotal,) int64;
  * IVFFlatIndex: centroids (nlist, d) float32, list_offsets (nlist + 1,)
    int64, list_vecs (ntotal, d) float32 grouped by list (input order inside a
    list), list_ids (ntotal,) int64.
The inverted lists are stored as the CSR bank the search reads and installed
as written on read (no reassignment), so a read index answers exactly like
the written one. Large arrays stream between the device and the file in
chunks, so the host holds one chunk at a time.

The reference's read_index cannot load an IVFFlat index (it constructs
IVFFlatIndex(d, metric=...), which the class does not accept, :94-95, and the
class has no write/read); this module implements what those lines intend.
"""
from __future__ import annotations

import json
import os
import struct
from typing import Optional

import numpy as np
import torch

from .errors import FormatError, InvalidArgumentError, IOFaissError

FORMAT = "metalfaiss_b200/1"
ALIGN = 64
CHUNK_BYTES = 256 << 20
_DTYPES = {"float32": np.float32, "int64": np.int64}


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def _np_dtype(t) -> str:
    if torch.is_tensor(t):
        name = {torch.float32: "float32", torch.int64: "int64"}.get(t.dtype)
    else:
        name = {np.dtype(np.float32): "float32", np.dtype(np.int64): "int64"}.get(t.dtype)
    if name is None:
        raise InvalidArgumentError(f"unsupported array dtype {t.dtype}")
    return name


def write_file(fname: str, header: dict, arrays) -> None:
    """Writes header + named arrays (torch tensors on any device, or numpy).
    arrays: list of (name, array). 2-D arrays must be row-contiguous."""
    descs, off = [], 0
    for name, a in arrays:
        nbytes = int(a.numel() * a.element_size()) if torch.is_tensor(a) else int(a.nbytes)
        descs.append({"name": name, "dtype": _np_dtype(a), "shape": list(a.shape),
                      "offset": off, "nbytes": nbytes})
        off = _align(off + nbytes)
    head = dict(header, format=FORMAT, arrays=descs)
    hb = json.dumps(head).encode("utf-8")
    data_start = _align(8 + len(hb))
    try:
        with open(fname, "wb") as f:
            f.write(struct.pack("<Q", len(hb)))
            f.write(hb)
            for desc, (_, a) in zip(descs, arrays):
                f.write(b"\0" * (data_start + desc["offset"] - f.tell()))
                _write_array(f, a)
            f.truncate(data_start + off)
    except OSError as e:
        raise IOFaissError(f"cannot write {fname}: {e}") from e


def _write_array(f, a) -> None:
    if not torch.is_tensor(a):
        np.ascontiguousarray(a).tofile(f)
        return
    a = a.contiguous()
    if a.numel() == 0:
        return
    rows = a.shape[0] if a.dim() else 1
    row_bytes = max(1, a[0].numel() * a.element_size()) if a.dim() else a.element_size()
    step = max(1, CHUNK_BYTES // row_bytes)
    for s in range(0, rows, step):
        a[s:s + step].cpu().numpy().tofile(f)


def read_header(fname: str):
    """(header dict, data section start). Raises FormatError on a file that is
    not one of these indexes, IOFaissError when it cannot be read."""
    try:
        size = os.path.getsize(fname)
        with open(fname, "rb") as f:
            raw = f.read(8)
            if len(raw) != 8:
                raise FormatError(f"{fname}: shorter than its header length")
            (hl,) = struct.unpack("<Q", raw)
            if hl == 0 or 8 + hl > size:
                raise FormatError(f"{fname}: header length {hl} outside the file")
            hb = f.read(hl)
    except OSError as e:
        raise IOFaissError(f"cannot read {fname}: {e}") from e
    try:
        head = json.loads(hb.decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise FormatError(f"{fname}: header is not JSON ({e})") from e
    if not isinstance(head, dict) or head.get("format") != FORMAT:
        raise FormatError(f"{fname}: not a {FORMAT} index file")
    data_start = _align(8 + hl)
    for desc in head.get("arrays", []):
        dt = _DTYPES.get(desc.get("dtype"))
        if dt is None:
            raise FormatError(f"{fname}: array {desc.get('name')} has dtype {desc.get('dtype')}")
        want = int(np.prod(desc["shape"], dtype=np.int64)) * np.dtype(dt).itemsize
        if want != desc["nbytes"] or data_start + desc["offset"] + want > size:
            raise FormatError(f"{fname}: array {desc['name']} lies outside the file")
    return head, data_start


def read_array(fname: str, head: dict, data_start: int, name: str) -> np.ndarray:
    """A read-only memory map of one array."""
    for desc in head["arrays"]:
        if desc["name"] == name:
            shape = tuple(desc["shape"])
            if int(np.prod(shape)) == 0:
                return np.zeros(shape, _DTYPES[desc["dtype"]])
            return np.memmap(fname, dtype=_DTYPES[desc["dtype"]], mode="r",
                             offset=data_start + desc["offset"], shape=shape)
    raise FormatError(f"{fname}: no array {name!r}")


def _to_device(a: np.ndarray, device, dtype=None) -> torch.Tensor:
    """Host array (possibly a memory map) to the device, chunk by chunk."""
    out = torch.empty(a.shape, dtype=dtype or torch.from_numpy(np.zeros(0, a.dtype)).dtype,
                      device=device)
    if a.size == 0:
        return out
    row_bytes = max(1, a[0].nbytes if a.ndim > 1 else a.itemsize)
    step = max(1, CHUNK_BYTES // row_bytes)
    for s in range(0, a.shape[0], step):
        out[s:s + step].copy_(torch.from_numpy(np.array(a[s:s + step], copy=True)))
    return out


def write_index(index, fname: str) -> None:
    """Writes a FlatIndex or IVFFlatIndex (python/metalfaiss/index/index_io.py:31-60)."""
    from .index_flat import FlatIndex
    from .index_ivf_flat import IVFFlatIndex

    head = {"type": type(index).__name__, "d": index.d, "ntotal": index.ntotal,
            "is_trained": bool(index.is_trained), "metric": int(index.metric_type)}
    if isinstance(index, IVFFlatIndex):
        n = index.ntotal
        head.update(nlist=index.nlist, nprobe=index.nprobe)
        cents = (index.centroids if index.is_trained
                 else torch.zeros((0, index.d), dtype=torch.float32))
        vecs = index._vecs[:n, : index.d] if n else torch.zeros((0, index.d))
        ids = index._ids[:n] if n else torch.zeros(0, dtype=torch.int64)
        arrays = [("centroids", cents.contiguous()), ("list_offsets", index.list_offsets),
                  ("list_vecs", vecs.contiguous()), ("list_ids", ids)]
    elif isinstance(index, FlatIndex):
        arrays = [("xb", index.xb.contiguous()), ("ids", index.ids)]
    else:
        raise InvalidArgumentError(f"write_index does not take {type(index).__name__}")
    write_file(fname, head, arrays)


def read_index(fname: str, device=None):
    """Reads a file written by write_index onto `device` (default: the current
    CUDA device) (python/metalfaiss/index/index_io.py:62-113)."""
    from .index_flat import FlatIndex
    from .index_ivf_flat import IVFFlatIndex
    from .metric_type import MetricType

    head, start = read_header(fname)
    kind = head.get("type")
    try:
        d = int(head["d"])
        metric = MetricType(int(head["metric"]))
        ntotal = int(head["ntotal"])
    except (KeyError, ValueError, TypeError) as e:
        raise FormatError(f"{fname}: bad header field ({e})") from e
    if kind == "FlatIndex":
        index = FlatIndex(d, metric, device=device)
        xb = read_array(fname, head, start, "xb")
        ids = read_array(fname, head, start, "ids")
        if xb.shape != (ntotal, d) or ids.shape != (ntotal,):
            raise FormatError(f"{fname}: array shapes disagree with ntotal={ntotal}, d={d}")
        if ntotal:
            index.add(_to_device(xb, index.device), _to_device(ids, index.device))
    elif kind == "IVFFlatIndex":
        nlist = int(head["nlist"])
        index = IVFFlatIndex(d, nlist, metric_type=metric, device=device)
        index.nprobe = int(head.get("nprobe", 1))
        cents = read_array(fname, head, start, "centroids")
        offs = np.asarray(read_array(fname, head, start, "list_offsets"), np.int64)
        vecs = read_array(fname, head, start, "list_vecs")
        ids = read_array(fname, head, start, "list_ids")
        if (offs.shape != (nlist + 1,) or vecs.shape != (ntotal, d) or ids.shape != (ntotal,)
                or offs[0] != 0 or offs[-1] != ntotal or np.any(np.diff(offs) < 0)):
            raise FormatError(f"{fname}: inverted lists disagree with nlist={nlist}, "
                              f"ntotal={ntotal}")
        if head.get("is_trained"):
            if cents.shape != (nlist, d):
                raise FormatError(f"{fname}: centroids are {cents.shape}, not ({nlist}, {d})")
            index.set_centroids(_to_device(cents, index.device))
            index._install_lists(_to_device(offs, index.device),
                                 _to_device(vecs, index.device), _to_device(ids, index.device))
        elif ntotal:
            raise FormatError(f"{fname}: an untrained index with {ntotal} rows")
    else:
        raise FormatError(f"{fname}: unknown index type {kind!r}")
    if index.ntotal != ntotal or index.is_trained != bool(head["is_trained"]):
        raise FormatError(f"{fname}: the index read back disagrees with its header")
    return index


__all__ = ["write_index", "read_index", "write_file", "read_header", "read_array", "FORMAT"]
