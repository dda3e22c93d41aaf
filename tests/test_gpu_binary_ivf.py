"""BinaryIVFIndex (Hamming coarse quantizer + packed inverted lists) on the
device against the oracle's restatement of the reference's search
(python/metalfaiss/index/binary_ivf_index.py:113-185): integer work, so
distances and labels must be identical, ties going to the earlier probe and
then to the earlier row of the list on both sides."""
import numpy as np
import pytest

from metalfaiss_b200 import BinaryFlatIndex, BinaryIVFIndex
from metalfaiss_b200.errors import BadStateError, InvalidArgumentError, NotImplementedFaissError
from oracle import oracle

pytestmark = pytest.mark.gpu

INT32_MAX = 2 ** 31 - 1
G = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "reference_golden.npz")


def _bits(n, d, seed, p=0.5):
    return (np.random.Generator(np.random.PCG64(seed)).random((n, d)) < p).astype(np.uint8)


def _lists(xb, ids, cents):
    """Each row in its nearest centroid's list (ties to the lower centroid), in add order."""
    _, a = oracle.hamming_search(xb, cents, 1)
    a = a[:, 0]
    rows = [xb[a == l] for l in range(len(cents))]
    lid = [ids[a == l] for l in range(len(cents))]
    return rows, lid


def _check(idx, xq, cents, rows, lid, nprobe, k):
    idx.nprobe = nprobe
    D, I = idx.search(xq, k).numpy()
    D_ref, I_ref, _ = oracle.hamming_ivf_search(xq, cents, rows, lid, nprobe, k)
    empty = np.isinf(D_ref)
    D_ref = np.nan_to_num(D_ref, posinf=0).astype(np.int64)
    D_ref[empty] = INT32_MAX
    assert D.dtype == np.int32
    np.testing.assert_array_equal(D.astype(np.int64), D_ref)
    np.testing.assert_array_equal(I, I_ref)


def _index_with(cents):
    q = BinaryFlatIndex(cents.shape[1])
    q.add(cents)
    return BinaryIVFIndex(q, cents.shape[1], len(cents))


@pytest.mark.parametrize("tag", [str(t) for t in G["binivf_cases"]])
def test_binary_ivf_golden(cuda_device, tag):
    """Against BinaryIVFIndex.search run from the reference's own module;
    missing slots are (INT32_MAX, -1) here and (inf, 0) there."""
    xb, xq, cents, ids = (G[tag + s] for s in ("_xb", "_xq", "_cents", "_ids"))
    idx = _index_with(cents)
    idx.add(xb, ids)
    idx.nprobe = int(G[tag + "_nprobe"])
    D, I = idx.search(xq, G[tag + "_D"].shape[1]).numpy()
    pad = np.isinf(G[tag + "_D"])
    np.testing.assert_array_equal(D[~pad].astype(np.int64), G[tag + "_D"][~pad].astype(np.int64))
    np.testing.assert_array_equal(I[~pad], G[tag + "_I"][~pad])
    assert (D[pad] == INT32_MAX).all() and (I[pad] == -1).all()


@pytest.mark.parametrize("d", [64, 72, 128, 256])
def test_binary_ivf_equals_oracle(cuda_device, d):
    # clustered rows: 32 seeds, each row flips a few bits of its seed
    rng = np.random.Generator(np.random.PCG64(d))
    seeds = _bits(32, d, seed=d + 1)
    n = 6000
    xb = seeds[rng.integers(0, 32, n)] ^ (rng.random((n, d)) < 0.1).astype(np.uint8)
    xq = seeds[rng.integers(0, 32, 50)] ^ (rng.random((50, d)) < 0.1).astype(np.uint8)
    xq[:2] = xb[[3, 4000]]
    cents = xb[rng.choice(n, 32, replace=False)]
    idx = _index_with(cents)
    assert idx.is_trained
    ids = np.arange(n, dtype=np.int64)
    idx.add(xb)
    rows, lid = _lists(xb, ids, cents)
    for nprobe in (1, 4, 32):
        for k in (1, 10, 100):
            _check(idx, xq, cents, rows, lid, nprobe, k)


def test_binary_ivf_batches_ids_and_padding(cuda_device):
    """Two add batches with explicit ids (each list keeps add order), k above
    the candidate count (inf / -1 padding), nprobe above nlist (clipped)."""
    d = 128
    xb = _bits(3000, d, seed=11, p=0.3)
    xq = _bits(40, d, seed=12, p=0.3)
    cents = xb[:16].copy()
    ids = np.arange(3000, dtype=np.int64) * 7 + 5
    idx = _index_with(cents)
    idx.add(xb[:1700], ids[:1700])
    idx.add(xb[1700:], ids[1700:])
    assert idx.ntotal == 3000 and len(idx) == 3000
    rows, lid = _lists(xb, ids, cents)
    _check(idx, xq, cents, rows, lid, 2, 256)   # lists hold ~190 rows each: padding
    _check(idx, xq, cents, rows, lid, 100, 50)  # nprobe clipped to nlist
    # reconstruct by id, then reset
    np.testing.assert_array_equal(idx.reconstruct(int(ids[2500])).cpu().numpy(), xb[2500])
    with pytest.raises(InvalidArgumentError):
        idx.reconstruct(6)
    idx.reset()
    assert idx.ntotal == 0 and not idx.is_trained


def test_binary_ivf_train_and_errors(cuda_device):
    d = 64
    xb = _bits(4000, d, seed=21)
    idx = BinaryIVFIndex(d, 20)  # BinaryIVFIndex(d, nlist) builds its own quantizer
    assert not idx.is_trained
    with pytest.raises(BadStateError):
        idx.add(xb)
    idx.train(xb)
    assert idx.is_trained and idx.quantizer.ntotal == 20
    with pytest.raises(BadStateError):
        idx.search(xb[:3], 5)  # empty index raises, as the reference does
    idx.add(xb)
    cents = np.stack([idx.quantizer.reconstruct(i).cpu().numpy().reshape(-1) for i in range(20)])
    rows, lid = _lists(xb, np.arange(4000, dtype=np.int64), cents)
    _check(idx, _bits(30, d, seed=22), cents, rows, lid, 3, 10)
    wide = BinaryIVFIndex(d, 70)
    wide.train(xb)
    wide.add(xb[:100])
    wide.nprobe = 65
    with pytest.raises(NotImplementedFaissError):
        wide.search(xb[:3], 5)
    with pytest.raises(ValueError):
        idx.nprobe = 0
    with pytest.raises(InvalidArgumentError):
        BinaryIVFIndex(BinaryFlatIndex(32), 64, 4)
    with pytest.raises(InvalidArgumentError):
        BinaryIVFIndex(BinaryFlatIndex(64), 64, 0)
