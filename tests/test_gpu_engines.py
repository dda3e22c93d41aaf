"""The tensor-core (tcgen05, 3xTF32) and SIMT scan engines against each other
and against the oracle, on flat and IVF searches. Engine 2 (like the default)
uses the tensor cores where the shape allows (L2 / inner product, d >= 32,
k <= 32; or k <= 128 with d <= 128, in 64-row tiles with 128-key lists) and
the SIMT scan otherwise. For d <= 128 it keeps the query tile in
tensor memory and derives the rows' tf32 residuals in the kernel; above that
it streams both operands with stored residuals. Engine 3 takes the streamed
form at every d (where residuals are stored: d > 128; the SIMT scan
otherwise); engine 1 forces the SIMT scan."""
import numpy as np
import pytest

from metalfaiss_b200 import FlatIndex, IVFFlatIndex, MetricType
from metalfaiss_b200 import _native as nat
from metalfaiss_b200 import synthetic as syn
from oracle import compare, oracle

pytestmark = pytest.mark.gpu


@pytest.fixture
def engine():
    yield nat.set_scan_engine
    nat.set_scan_engine(0)
    assert nat.device_error(0) == 0, "a bounded device wait timed out"


def _flat(metric, d, n, nq, k, seed, engine_id, data="gauss"):
    nat.set_scan_engine(engine_id)
    if data == "gauss":
        xb, xq = syn.gaussian(n, d, seed), syn.gaussian(nq, d, seed + 1)
    else:
        xb, cen, _ = syn.mixture(n, d, 64, seed)
        xq, _, _ = syn.mixture(nq, d, 64, seed + 1, centres=cen)
    idx = FlatIndex(d, metric)
    idx.add(xb)
    D, I = idx.search(xq, k).numpy()
    return xb, xq, D, I


@pytest.mark.parametrize("eng", [2, 3])
@pytest.mark.parametrize("metric", [MetricType.L2, MetricType.INNER_PRODUCT])
@pytest.mark.parametrize("d,k", [(32, 10), (64, 1), (128, 32), (96, 100), (256, 256), (48, 7),
                                 (160, 10), (192, 32)])
def test_tc_flat_matches_oracle(cuda_device, engine, eng, metric, d, k):
    xb, xq, D, I = _flat(metric, d, 5000, 77, k, seed=d + k, engine_id=eng)
    D_ref, I_ref = oracle.flat_search(xq, xb, k, int(metric))
    atol = compare.l2_atol(xq, xb) if metric == MetricType.L2 else 1e-5 * (1 + np.abs(D_ref).max())
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq, xb, int(metric)), atol=atol)
    assert not errs, errs[:5]


def test_tc_precision_on_mixture(cuda_device, engine):
    """Distances of the 3xTF32 path against fp64 on clustered data (norms ~ 5x the distances)."""
    xb, xq, D, I = _flat(MetricType.L2, 128, 20000, 200, 10, seed=3, engine_id=2, data="mix")
    exact = oracle.pairwise_exact(xq, xb, oracle.L2)
    got = D.astype(np.float64)
    ref = np.take_along_axis(exact, I, 1)
    rel = np.abs(got - ref) / np.maximum(ref, 1e-6)
    print(f"3xTF32 L2 max relative distance error {rel.max():.3e} (median {np.median(rel):.3e})")
    assert rel.max() < 1e-4
    D_ref, I_ref = oracle.flat_search(xq, xb, 10, oracle.L2)
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq, xb, oracle.L2),
                             atol=compare.l2_atol(xq, xb))
    assert not errs, errs[:5]


@pytest.mark.parametrize("d", [64, 160])
@pytest.mark.parametrize("eng", [2, 3])
@pytest.mark.parametrize("nprobe,k", [(1, 10), (8, 32), (16, 100)])
def test_tc_ivf_equals_simt(cuda_device, engine, d, eng, nprobe, k):
    x, cen, _ = syn.mixture(40000, d, 96, seed=7)
    idx = IVFFlatIndex(d, 96)
    idx.set_centroids(oracle.kmeans_train(x, 96, 2, 7))
    idx.add(x)
    idx.nprobe = nprobe
    xq, _, _ = syn.mixture(300, d, 96, seed=8, centres=cen)
    nat.set_scan_engine(1)
    D1, I1 = idx.search(xq, k).numpy()
    nat.set_scan_engine(eng)
    D2, I2 = idx.search(xq, k).numpy()
    look = compare.exact_lookup(xq, x, oracle.L2)
    atol = compare.l2_atol(xq, x)
    errs = compare.check_knn(D2, I2, D1, I1, look, atol=atol)
    assert not errs, errs[:5]
    # and both against the oracle over the index's own lists
    offs = idx.list_offsets.cpu().numpy()
    vecs = idx._vecs[:, :d].cpu().numpy()
    ids = idx._ids[: idx.ntotal].cpu().numpy()
    cents = idx.centroids.cpu().numpy()
    D_ref, I_ref = oracle.ivf_search(xq, cents, offs, vecs, ids, nprobe, k)
    for D, I in ((D1, I1), (D2, I2)):
        errs = compare.check_knn(D, I, D_ref, I_ref, look, atol=atol)
        assert not errs, errs[:5]


@pytest.mark.parametrize("eng", [2, 3])
def test_tc_many_items_persistent(cuda_device, engine, eng):
    """More work items than CTAs, lists of every size, groups of 1..128 queries."""
    x, cen, _ = syn.mixture(60000, 128, 300, seed=9)
    idx = IVFFlatIndex(128, 300)
    idx.set_centroids(x[:300])
    idx.add(x)
    idx.nprobe = 20
    xq, _, _ = syn.mixture(2000, 128, 300, seed=10, centres=cen)
    nat.set_scan_engine(eng)
    D, I = idx.search(xq, 10).numpy()
    offs = idx.list_offsets.cpu().numpy()
    vecs = idx._vecs[:, :128].cpu().numpy()
    ids = idx._ids[: idx.ntotal].cpu().numpy()
    D_ref, I_ref = oracle.ivf_search(xq, x[:300], offs, vecs, ids, 20, 10)
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq, x, oracle.L2),
                             atol=compare.l2_atol(xq, x))
    assert not errs, errs[:5]


@pytest.mark.parametrize("metric", [MetricType.L2, MetricType.INNER_PRODUCT])
def test_tc_without_stored_residuals(cuda_device, engine, metric):
    """residuals=False: the tensor-core scan derives the rows' tf32 residuals in
    shared memory (d <= 128); flat and IVF results match the oracle."""
    nat.set_scan_engine(2)
    x, cen, _ = syn.mixture(30000, 96, 64, seed=17)
    xq, _, _ = syn.mixture(300, 96, 64, seed=18, centres=cen)
    flat = FlatIndex(96, metric, residuals=False)
    flat.add(x)
    assert flat._lo is None
    D, I = flat.search(xq, 10).numpy()
    D_ref, I_ref = oracle.flat_search(xq, x, 10, int(metric))
    atol = compare.l2_atol(xq, x) if metric == MetricType.L2 else 1e-5 * (1 + np.abs(D_ref).max())
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq, x, int(metric)), atol=atol)
    assert not errs, errs[:5]
    ivf = IVFFlatIndex(96, 64, metric_type=metric, residuals=False)
    ivf.set_centroids(oracle.kmeans_train(x, 64, 2, 17))
    ivf.add(x)
    ivf.nprobe = 8
    assert ivf._lo is None
    D2, I2 = ivf.search(xq, 10).numpy()
    nat.set_scan_engine(1)
    D1, I1 = ivf.search(xq, 10).numpy()
    errs = compare.check_knn(D2, I2, D1, I1, compare.exact_lookup(xq, x, int(metric)), atol=atol)
    assert not errs, errs[:5]


@pytest.mark.parametrize("metric", [MetricType.L2, MetricType.INNER_PRODUCT])
@pytest.mark.parametrize("d,k", [(64, 33), (128, 64), (128, 100), (96, 128), (32, 100)])
def test_tc_long_lists_flat(cuda_device, engine, metric, d, k):
    """32 < k <= 128 on the tensor cores (the rank merge into 128-key lists):
    the engine query says so, and the results equal the oracle."""
    nat.set_scan_engine(0)
    assert nat.load().mf_flat_engine(int(metric), d, k, 20000, 1) == 1
    xb, xq, D, I = _flat(metric, d, 20000, 300, k, seed=d * 7 + k, engine_id=0)
    D_ref, I_ref = oracle.flat_search(xq, xb, k, int(metric))
    atol = compare.l2_atol(xq, xb) if metric == MetricType.L2 else 1e-5 * (1 + np.abs(D_ref).max())
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq, xb, int(metric)), atol=atol)
    assert not errs, errs[:5]


def test_tc_unit_rows_ip_k100(cuda_device, engine):
    """The flat inner-product k=100 configuration in miniature: 200k unit rows
    x d=128, 513 unit queries (a partial last query tile), k=100, tensor cores."""
    nat.set_scan_engine(0)
    xb = syn.unit_rows(200_000, 128, seed=51)
    xq = syn.unit_rows(513, 128, seed=52)
    assert nat.load().mf_flat_engine(0, 128, 100, len(xb), 1) == 1
    idx = FlatIndex(128, MetricType.INNER_PRODUCT)
    idx.add(xb)
    D, I = idx.search(xq, 100).numpy()
    D_ref, I_ref = oracle.flat_search(xq, xb, 100, oracle.INNER_PRODUCT)
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq, xb, oracle.INNER_PRODUCT),
                             atol=1e-5)
    assert not errs, errs[:5]


@pytest.mark.parametrize("k", [50, 128])
def test_tc_long_lists_ivf(cuda_device, engine, k):
    """IVF lists with 32 < k <= 128 (exact scan: the filter search takes k <= 16)
    on the tensor cores, against the oracle."""
    nat.set_scan_engine(0)
    d = 128
    x, cen, _ = syn.mixture(40000, d, 64, seed=61)
    idx = IVFFlatIndex(d, 64)
    idx.set_centroids(oracle.kmeans_train(x, 64, 2, 61))
    idx.add(x)
    idx.nprobe = 6
    xq, _, _ = syn.mixture(700, d, 64, seed=62, centres=cen)
    D, I = idx.search(xq, k).numpy()
    offs = idx.list_offsets.cpu().numpy()
    vecs = idx._vecs[:, :d].cpu().numpy()
    ids = idx._ids[: idx.ntotal].cpu().numpy()
    D_ref, I_ref = oracle.ivf_search(xq, idx.centroids.cpu().numpy(), offs, vecs, ids, 6, k)
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq, x, oracle.L2),
                             atol=compare.l2_atol(xq, x))
    assert not errs, errs[:5]
