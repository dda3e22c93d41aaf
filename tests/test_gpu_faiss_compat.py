"""The FAISS-style facade (metalfaiss_b200/faiss_compat.py) on the device:
IndexShards equals one index holding every row (the reference's intent,
python/metalfaiss/unittest/test_mlx_multi_gpu.py:49-65 for flat shards,
:86-119 for IVF shards with a shared quantizer), IndexReplicas equals one
index, index_factory builds searchable indexes, and the IO delegates round
trip. Children on a second GPU when the box has one."""
import numpy as np
import pytest
import torch

from metalfaiss_b200 import FlatIndex, IVFFlatIndex, MetricType
from metalfaiss_b200 import faiss_compat as fc
from metalfaiss_b200 import synthetic as syn
from oracle import compare, oracle

pytestmark = pytest.mark.gpu


def _devices(n):
    cnt = torch.cuda.device_count()
    return [torch.device("cuda", i % cnt) for i in range(n)]


@pytest.mark.parametrize("metric", [MetricType.L2, MetricType.INNER_PRODUCT])
def test_flat_shards_equal_single(cuda_device, metric):
    xb = syn.gaussian(30000, 64, seed=1)
    xq = syn.gaussian(200, 64, seed=2)
    single = FlatIndex(64, metric)
    single.add(xb)
    sh = fc.IndexShards(64)
    for dev in _devices(3):
        sh.add_shard(FlatIndex(64, metric, device=dev))
    sh.add(xb)
    assert sh.ntotal == 30000
    D1, I1 = single.search(xq, 20).numpy()
    D2, I2 = sh.search(xq, 20).numpy()
    np.testing.assert_array_equal(I2, I1)
    np.testing.assert_array_equal(D2, D1)


def test_ivf_shards_shared_quantizer_equal_single(cuda_device):
    d, nlist = 64, 64
    x, cen, _ = syn.mixture(40000, d, nlist, seed=3)
    cents = oracle.kmeans_train(x, nlist, 2, 3)
    single = IVFFlatIndex(d, nlist)
    single.set_centroids(cents)
    single.add(x)
    single.nprobe = 8
    sh = fc.IndexShards(d)
    for dev in _devices(2):
        c = IVFFlatIndex(d, nlist, device=dev)
        c.set_centroids(cents)
        c.nprobe = 8
        sh.add_shard(c)
    sh.add(x)
    xq, _, _ = syn.mixture(500, d, nlist, seed=4, centres=cen)
    D1, I1 = single.search(xq, 10).numpy()
    D2, I2 = sh.search(xq, 10).numpy()
    errs = compare.check_knn(D2, I2, D1, I1, compare.exact_lookup(xq, x, oracle.L2),
                             atol=compare.l2_atol(xq, x))
    assert not errs, errs[:5]


def test_replicas_equal_single(cuda_device):
    xb = syn.gaussian(20000, 48, seed=5)
    xq = syn.gaussian(301, 48, seed=6)
    single = FlatIndex(48)
    single.add(xb)
    rep = fc.IndexReplicas(48)
    for dev in _devices(3):
        rep.add_replica(fc.IndexFlatL2(48, device=dev))
    rep.add(xb)
    assert rep.ntotal == 20000
    D1, I1 = single.search(xq, 10).numpy()
    D2, I2 = rep.search(xq, 10).numpy()
    np.testing.assert_array_equal(I2, I1)
    np.testing.assert_array_equal(D2, D1)


def test_factory_ivf_flat_and_io(cuda_device, tmp_path):
    d = 32
    x, cen, _ = syn.mixture(20000, d, 40, seed=7)
    idx = fc.index_factory(d, "IVF40,Flat")
    assert isinstance(idx, fc.IndexIVFFlat) and idx.nlist == 40
    idx.train(x)
    idx.add(x)
    idx.nprobe = 5
    xq, _, _ = syn.mixture(100, d, 40, seed=8, centres=cen)
    D, I = idx.search(xq, 10).numpy()
    impl = idx._impl
    D_ref, I_ref = oracle.ivf_search(xq, impl.centroids.cpu().numpy(),
                                     impl.list_offsets.cpu().numpy(),
                                     impl._vecs[:, :d].cpu().numpy(),
                                     impl._ids[: impl.ntotal].cpu().numpy(), 5, 10)
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq, x, oracle.L2),
                             atol=compare.l2_atol(xq, x))
    assert not errs, errs[:5]
    f = str(tmp_path / "f.idx")
    fc.write_index(idx, f)
    back = fc.read_index(f)
    D2, I2 = back.search(xq, 10).numpy()
    np.testing.assert_array_equal(I2, I)
    flat = fc.index_factory(d, "FlatIP")
    flat.add(x)
    Df, If = flat.search(xq, 5).numpy()
    Dr, Ir = oracle.flat_search(xq, x, 5, oracle.INNER_PRODUCT)
    errs = compare.check_knn(Df, If, Dr, Ir, compare.exact_lookup(xq, x, oracle.INNER_PRODUCT),
                             atol=1e-4)
    assert not errs, errs[:5]


def test_shards_with_fewer_rows_than_k(cuda_device):
    xb = syn.gaussian(10, 16, seed=9)
    sh = fc.IndexShards(16)
    for _ in range(4):
        sh.add_shard(FlatIndex(16))
    sh.add(xb)
    D, I = sh.search(syn.gaussian(3, 16, seed=10), 8).numpy()
    D_ref, I_ref = oracle.flat_search(syn.gaussian(3, 16, seed=10), xb, 8)
    np.testing.assert_array_equal(I, I_ref)
