"""BinaryFlatIndex (Hamming distance over packed codes) on the device against
the oracle and the reference's own outputs: integer work, so distances and
labels must be identical (ties go to the lower row on both sides)."""
import numpy as np
import pytest
import torch

from metalfaiss_b200 import BinaryFlatIndex
from metalfaiss_b200.errors import InvalidArgumentError
from oracle import oracle

pytestmark = pytest.mark.gpu

G = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "reference_golden.npz")


def _bits(n, d, seed, p=0.5):
    return (np.random.Generator(np.random.PCG64(seed)).random((n, d)) < p).astype(np.uint8)


@pytest.mark.parametrize("tag", [str(t) for t in G["binary_cases"]])
def test_binary_golden(cuda_device, tag):
    xb, xq = G[tag + "_xb"], G[tag + "_xq"]
    idx = BinaryFlatIndex(xb.shape[1])
    idx.add(xb)
    k = G[tag + "_D"].shape[1]
    D, I = idx.search(xq, k).numpy()
    assert D.dtype == np.int32
    np.testing.assert_array_equal(D, G[tag + "_D"])
    np.testing.assert_array_equal(I, G[tag + "_I"])
    np.testing.assert_array_equal(idx.reconstruct(5).cpu().numpy(), G[tag + "_rec"])


@pytest.mark.parametrize("d", [8, 64, 72, 256, 1024])
@pytest.mark.parametrize("k", [1, 10, 100, 256])
def test_binary_knn_equals_oracle(cuda_device, d, k):
    xb = _bits(5000, d, seed=d + k)
    xq = _bits(77, d, seed=d + k + 1)
    xq[:3] = xb[[0, 17, 4999]]
    idx = BinaryFlatIndex(d)
    idx.add(xb)
    D, I = idx.search(xq, k).numpy()
    D_ref, I_ref = oracle.hamming_search(xq, xb, k)
    np.testing.assert_array_equal(D, D_ref)
    np.testing.assert_array_equal(I, I_ref)
    # self-queries find distance 0 (their own row, or a lower duplicate of it
    # when d is small enough for duplicates)
    assert (D[:3, 0] == 0).all()
    if d >= 64:
        assert list(I[:3, 0]) == [0, 17, 4999]


def test_binary_many_rows_merged_splits_and_ids(cuda_device):
    """Enough rows for many splits merged on the device; ids mapped after the merge."""
    d = 128
    xb = _bits(150_000, d, seed=5, p=0.3)
    xq = _bits(40, d, seed=6, p=0.3)
    ids = np.arange(150_000, dtype=np.int64) * 3 + 11
    idx = BinaryFlatIndex(d)
    idx.add(xb[:70_000], ids[:70_000])
    idx.add(xb[70_000:], ids[70_000:])
    D, I = idx.search(xq, 50).numpy()
    D_ref, I_ref = oracle.hamming_search(xq, xb, 50, ids)
    np.testing.assert_array_equal(D, D_ref)
    np.testing.assert_array_equal(I, I_ref)


@pytest.mark.parametrize("d,radius", [(64, 20), (256, 110), (72, 0), (128, -1)])
def test_binary_range_equals_oracle(cuda_device, d, radius):
    xb = _bits(20_000, d, seed=d)
    xq = _bits(45, d, seed=d + 1)
    xq[0] = xb[123]
    idx = BinaryFlatIndex(d)
    idx.add(xb)
    res = idx.range_search(xq, radius)
    lims_ref, D_ref, L_ref = oracle.hamming_range(xq, xb, radius)
    np.testing.assert_array_equal(res.lims.cpu().numpy(), lims_ref)
    np.testing.assert_array_equal(res.distances.cpu().numpy(), D_ref)
    np.testing.assert_array_equal(res.labels.cpu().numpy(), L_ref)


def test_binary_reconstruct_empty_and_errors(cuda_device):
    xb = _bits(100, 64, seed=9)
    idx = BinaryFlatIndex(64)
    D, I = idx.search(xb[:4], 3).numpy()
    assert (I == -1).all() and (D == 2 ** 31 - 1).all()
    res = idx.range_search(xb[:4], 10)
    assert res.lims.cpu().numpy().tolist() == [0] * 5
    idx.add(xb)
    np.testing.assert_array_equal(idx.reconstruct(np.array([0, 2, 4])).cpu().numpy(),
                                  xb[[0, 2, 4]])
    np.testing.assert_array_equal(idx.reconstruct(7).cpu().numpy(), xb[7:8])
    with pytest.raises(ValueError):
        idx.reconstruct(100)
    with pytest.raises(ValueError):
        idx.reconstruct(np.array([0, 100]))
    with pytest.raises(ValueError):
        BinaryFlatIndex(63)
    with pytest.raises(InvalidArgumentError):
        idx.add(np.full((2, 64), 2, np.uint8))
    with pytest.raises(InvalidArgumentError):
        idx.search(xb[:2, :32], 3)
    D, I = idx.search(xb[:2], 500).numpy()  # k clipped to ntotal
    assert D.shape == (2, 100)
