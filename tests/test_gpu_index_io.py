"""write_index / read_index round trips on the device
(python/metalfaiss/unittest/test_index_io.py:54-77): the index read back has
the same shape, metric, nprobe and rows, and answers every search exactly as
the written one (distances and labels identical)."""
import numpy as np
import pytest
import torch

from metalfaiss_b200 import FlatIndex, IVFFlatIndex, MetricType, read_index, write_index
from metalfaiss_b200 import synthetic as syn
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("metric", [MetricType.L2, MetricType.INNER_PRODUCT, MetricType.L1])
def test_flat_round_trip(cuda_device, tmp_path, metric):
    x = syn.gaussian(5000, 36, seed=1)
    idx = FlatIndex(36, metric)
    idx.add(x, np.arange(5000, dtype=np.int64) * 11 + 5)
    f = str(tmp_path / "flat.idx")
    write_index(idx, f)
    back = read_index(f)
    assert isinstance(back, FlatIndex) and back.d == 36 and back.ntotal == 5000
    assert back.metric_type == metric
    assert torch.equal(back.ids, idx.ids) and torch.equal(back.xb, idx.xb)
    q = syn.gaussian(50, 36, seed=2)
    D1, I1 = idx.search(q, 7).numpy()
    D2, I2 = back.search(q, 7).numpy()
    np.testing.assert_array_equal(D1, D2)
    np.testing.assert_array_equal(I1, I2)


@pytest.mark.parametrize("d,k", [(64, 10), (36, 20)])
def test_ivf_round_trip(cuda_device, tmp_path, d, k):
    """d=64, k=10 runs the filter search on both sides; d=36, k=20 the exact scan."""
    x, cen, _ = syn.mixture(30000, d, 50, seed=3)
    idx = IVFFlatIndex(d, 50)
    idx.set_centroids(oracle.kmeans_train(x, 50, 2, 3))
    idx.add(x[:20000])
    idx.add(x[20000:], np.arange(10000, dtype=np.int64) + 10 ** 9)
    idx.nprobe = 6
    f = str(tmp_path / "ivf.idx")
    write_index(idx, f)
    back = read_index(f)
    assert isinstance(back, IVFFlatIndex)
    assert (back.d, back.nlist, back.nprobe, back.ntotal) == (d, 50, 6, 30000)
    assert back.is_trained and back.metric_type == MetricType.L2
    assert torch.equal(back.list_offsets, idx.list_offsets)
    assert torch.equal(back.centroids, idx.centroids)
    q, _, _ = syn.mixture(300, d, 50, seed=4, centres=cen)
    D1, I1 = idx.search(q, k).numpy()
    D2, I2 = back.search(q, k).numpy()
    np.testing.assert_array_equal(D1, D2)
    np.testing.assert_array_equal(I1, I2)
    np.testing.assert_array_equal(back.reconstruct(10 ** 9 + 7).cpu().numpy(), x[20007])


def test_untrained_and_empty_ivf_round_trip(cuda_device, tmp_path):
    idx = IVFFlatIndex(16, 8)
    f = str(tmp_path / "u.idx")
    write_index(idx, f)
    back = read_index(f)
    assert not back.is_trained and back.ntotal == 0 and back.nlist == 8
    x = syn.gaussian(100, 16, seed=5)
    idx.set_centroids(x[:8])
    write_index(idx, f)
    back = read_index(f)
    assert back.is_trained and back.ntotal == 0
    torch.testing.assert_close(back.centroids, idx.centroids, rtol=0, atol=0)
