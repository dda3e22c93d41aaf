"""The index file format (metalfaiss_b200/index_io.py) on the CPU: the
reference's framing (u64 header length + JSON header, as
python/metalfaiss/index/index_io.py:31-60 writes it) followed by 64-byte
aligned arrays; round trips of every array kind, and the errors a damaged or
foreign file raises (FormatError, python/metalfaiss/errors.py:124-128)."""
import json
import struct

import numpy as np
import pytest
import torch

from metalfaiss_b200 import index_io
from metalfaiss_b200.errors import FormatError, IOFaissError


def _arrays():
    rng = np.random.Generator(np.random.PCG64(1))
    return [("centroids", rng.standard_normal((7, 5), dtype=np.float32)),
            ("list_offsets", np.array([0, 2, 2, 9, 10, 10, 13, 13], np.int64)),
            ("list_vecs", torch.from_numpy(rng.standard_normal((13, 5), dtype=np.float32))),
            ("list_ids", torch.arange(13, dtype=torch.int64) * 3),
            ("empty", np.zeros((0, 5), np.float32))]


def test_round_trip_and_layout(tmp_path):
    f = tmp_path / "x.idx"
    arrays = _arrays()
    index_io.write_file(str(f), {"type": "IVFFlatIndex", "d": 5, "ntotal": 13,
                                 "is_trained": True, "metric": 1, "nlist": 7}, arrays)
    raw = f.read_bytes()
    (hl,) = struct.unpack("<Q", raw[:8])
    head = json.loads(raw[8:8 + hl])
    assert head["format"] == index_io.FORMAT and head["type"] == "IVFFlatIndex"
    head2, start = index_io.read_header(str(f))
    assert head2 == head and start % 64 == 0 and start >= 8 + hl
    for desc, (name, a) in zip(head["arrays"], arrays):
        assert desc["name"] == name and desc["offset"] % 64 == 0
        got = index_io.read_array(str(f), head, start, name)
        want = a.numpy() if torch.is_tensor(a) else a
        assert got.dtype == want.dtype and got.shape == want.shape
        np.testing.assert_array_equal(got, want)


def test_chunked_device_writes_match(tmp_path, monkeypatch):
    """Arrays larger than the streaming chunk are written in pieces."""
    monkeypatch.setattr(index_io, "CHUNK_BYTES", 100)
    a = torch.arange(1000 * 3, dtype=torch.float32).reshape(1000, 3)
    f = tmp_path / "c.idx"
    index_io.write_file(str(f), {"type": "FlatIndex"}, [("xb", a)])
    head, start = index_io.read_header(str(f))
    np.testing.assert_array_equal(index_io.read_array(str(f), head, start, "xb"), a.numpy())
    back = index_io._to_device(index_io.read_array(str(f), head, start, "xb"), "cpu")
    assert torch.equal(back, a)


def test_foreign_and_damaged_files(tmp_path):
    f = tmp_path / "bad.idx"
    f.write_bytes(b"\x01\x02")
    with pytest.raises(FormatError):
        index_io.read_header(str(f))
    f.write_bytes(struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(FormatError):
        index_io.read_header(str(f))
    hb = json.dumps({"type": "FlatIndex", "format": "other"}).encode()
    f.write_bytes(struct.pack("<Q", len(hb)) + hb)
    with pytest.raises(FormatError):
        index_io.read_header(str(f))
    # a truncated data section
    good = tmp_path / "good.idx"
    index_io.write_file(str(good), {"type": "FlatIndex"}, _arrays()[:2])
    raw = good.read_bytes()
    f.write_bytes(raw[:-8])
    with pytest.raises(FormatError):
        index_io.read_header(str(f))
    with pytest.raises(IOFaissError):
        index_io.read_header(str(tmp_path / "missing.idx"))
    with pytest.raises(FormatError):
        index_io.read_index(str(good))  # a FlatIndex header without d / metric
