"""IVFFlatIndex, k-means and the merge kernel on the GPU against the CPU oracle."""
import numpy as np
import pytest
import torch

from metalfaiss_b200 import FlatIndex, IVFFlatIndex, MetricType, clustering
from metalfaiss_b200 import _native as nat
from metalfaiss_b200 import synthetic as syn
from oracle import compare, oracle

pytestmark = pytest.mark.gpu


def _ivf_pair(d, n, nlist, seed, metric=MetricType.L2):
    x, cen, _ = syn.mixture(n, d, nlist, seed)
    init = oracle.kmeans_init(x, nlist, seed)
    cents = oracle.kmeans_train(x, nlist, 3, seed, init=init)
    idx = IVFFlatIndex(d, nlist, metric_type=metric)
    idx.set_centroids(cents)
    idx.add(x)
    return idx, x, cents, gpu_lists(idx), cen


def gpu_lists(idx):
    """The index's own CSR lists, so the oracle checks the search on the same
    lists (the list build is checked separately against oracle.ivf_build)."""
    return (idx._offsets.cpu().numpy(), idx._vecs[:, : idx.d].cpu().numpy(),
            idx._ids[: idx.ntotal].cpu().numpy())


def _check_ivf(idx, xq, x, cents, lists, nprobe, k, metric):
    idx.nprobe = nprobe
    D, I = idx.search(xq, k).numpy()
    offsets, vecs, ids = lists
    # Probes from the GPU's own coarse step would differ only at coarse near-ties;
    # the oracle recomputes them in fp32 the reference's way.
    D_ref, I_ref = oracle.ivf_search(xq, cents, offsets, vecs, ids, nprobe, k, int(metric))
    atol = compare.l2_atol(xq, x) if metric == MetricType.L2 else 1e-4 * (1 + np.abs(D_ref[np.isfinite(D_ref)]).max())
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq, x, int(metric)), atol=atol)
    assert not errs, errs[:5]
    return D, I


@pytest.mark.parametrize("nprobe,k", [(1, 10), (8, 10), (1, 32), (8, 32)])
def test_ivf_config_c2_sweep(cuda_device, nprobe, k):
    """IVFFlat L2, d=64, N=32768 mixture of 128 clusters, nlist=128, Q=16."""
    idx, x, cents, lists, cen = _ivf_pair(64, 32768, 128, seed=3)
    xq, _, _ = syn.mixture(16, 64, 128, seed=4, centres=cen)
    _check_ivf(idx, xq, x, cents, lists, nprobe, k, MetricType.L2)


@pytest.mark.parametrize("metric", [MetricType.L2, MetricType.INNER_PRODUCT, MetricType.L1, MetricType.LINF])
def test_ivf_metrics(cuda_device, metric):
    idx, x, cents, lists, cen = _ivf_pair(32, 6000, 40, seed=5, metric=metric)
    xq, _, _ = syn.mixture(50, 32, 40, seed=6, centres=cen)
    if metric == MetricType.INNER_PRODUCT:
        # IP lists are built with an IP quantizer: the build matches the oracle's.
        lab = oracle.flat_search(x, cents, 1, oracle.INNER_PRODUCT)[1][:, 0]
        ref = oracle.ivf_build(x, lab, 40)
        assert np.array_equal(ref[0], lists[0]) and np.array_equal(ref[2], lists[2])
    _check_ivf(idx, xq, x, cents, lists, 5, 10, metric)


def test_ivf_many_queries_and_big_lists(cuda_device):
    idx, x, cents, lists, cen = _ivf_pair(64, 60000, 64, seed=7)
    xq, _, _ = syn.mixture(700, 64, 64, seed=8, centres=cen)
    _check_ivf(idx, xq, x, cents, lists, 6, 20, MetricType.L2)


@pytest.mark.parametrize("filter_search", [True, False])
def test_ivf_long_list_table(cuda_device, filter_search):
    """3,000 lists (past two blocks of the grouping plan: its multi-block
    form), many of them empty, against the oracle on the index's own lists."""
    x, cen, _ = syn.mixture(60_000, 64, 3000, seed=71)
    cents = np.concatenate([x[:: 60_000 // 2000][:2000], cen[:1000] + 50.0])  # 1,000 far, empty
    idx = IVFFlatIndex(64, 3000)
    idx.set_centroids(cents)
    idx.add(x)
    idx.filter_search = filter_search
    xq, _, _ = syn.mixture(900, 64, 3000, seed=72, centres=cen)
    sizes = np.diff(idx._offsets.cpu().numpy())
    assert (sizes == 0).sum() >= 1000
    _check_ivf(idx, xq, x, cents, gpu_lists(idx), 12, 10, MetricType.L2)


def test_ivf_nprobe_all_equals_flat(cuda_device):
    idx, x, cents, lists, cen = _ivf_pair(16, 3000, 12, seed=9)
    xq = syn.gaussian(30, 16, seed=10)
    idx.nprobe = 50  # > nlist: clipped like the reference's quantizer k (flat_index.py:87)
    D, I = idx.search(xq, 15).numpy()
    flat = FlatIndex(16)
    flat.add(x)
    Df, If = flat.search(xq, 15).numpy()
    errs = compare.check_knn(D, I, Df, If, compare.exact_lookup(xq, x, oracle.L2),
                             atol=compare.l2_atol(xq, x))
    assert not errs, errs[:5]


def test_ivf_preassigned_matches_search(cuda_device):
    """python/metalfaiss/unittest/test_mlx_index.py:50-69."""
    idx, x, cents, lists, cen = _ivf_pair(64, 10000, 100, seed=11)
    idx.nprobe = 4
    xq = syn.gaussian(100, 64, seed=12)
    q = FlatIndex(64)
    q.add(idx.centroids)
    assign_d, assign_i = q.search(xq, idx.nprobe)
    d1, i1 = idx.search_preassigned(xq, 10, assign_i, assign_d)
    d2, i2 = idx.search(xq, 10)
    assert torch.equal(i1, i2)
    assert torch.allclose(d1, d2)


def test_ivf_ids_64bit_self_query(cuda_device):
    """python/metalfaiss/unittest/test_mlx_index.py:242-256."""
    x = syn.gaussian(1000, 64, seed=13)
    ids = np.arange(1000, dtype=np.int64) + (1 << 32)
    idx = IVFFlatIndex(64, 10)
    idx.train(x)
    idx.add_with_ids(x, ids)
    D, I = idx.search(x[:10], 1).numpy()
    assert np.array_equal(I[:, 0], ids[:10])
    assert np.array_equal(idx.reconstruct(int(ids[7])).cpu().numpy(), x[7])


def test_ivf_incremental_add_keeps_order(cuda_device):
    idx, x, cents, lists, cen = _ivf_pair(24, 5000, 30, seed=14)
    idx2 = IVFFlatIndex(24, 30)
    idx2.set_centroids(cents)
    for s in range(0, 5000, 1300):
        idx2.add(x[s:s + 1300])
    assert idx2.ntotal == 5000
    assert torch.equal(idx2._offsets, idx._offsets)
    assert torch.equal(idx2._ids, idx._ids)
    assert torch.equal(idx2._vecs, idx._vecs)
    labels, _ = oracle.kmeans_assign(x, cents)
    offsets, vecs, ids = oracle.ivf_build(x, labels, 30)
    assert np.array_equal(idx._offsets.cpu().numpy(), offsets)
    assert np.array_equal(idx._ids.cpu().numpy(), ids)
    assert np.array_equal(idx._vecs[:, :24].cpu().numpy(), vecs)


def test_ivf_empty_lists_and_padding(cuda_device):
    x = syn.gaussian(40, 8, seed=15)
    cents = np.concatenate([x[:3], syn.gaussian(5, 8, seed=16) + 100.0])  # 5 lists stay empty
    idx = IVFFlatIndex(8, 8)
    idx.set_centroids(cents)
    idx.add(x)
    idx.nprobe = 8
    D, I = idx.search(x[:4], 60).numpy()  # k > ntotal: padded with (+inf, -1)
    assert np.all(I[:, 40:] == -1) and np.all(np.isinf(D[:, 40:]))
    assert np.all(I[:, :40] >= 0)
    empty = IVFFlatIndex(8, 8)
    empty.set_centroids(cents)
    D, I = empty.search(x[:2], 5).numpy()
    assert np.all(I == -1)


def test_ivf_range_search(cuda_device):
    idx, x, cents, lists, cen = _ivf_pair(32, 8000, 50, seed=17)
    idx.nprobe = 6
    xq, _, _ = syn.mixture(40, 32, 50, seed=18, centres=cen)
    D10, _ = idx.search(xq, 10).numpy()
    radius = float(np.median(D10[:, -1]))  # the median 10th-NN distance
    lims, D, L = idx.range_search(xq, radius).numpy()
    offsets, vecs, ids = lists
    lims_ref, D_ref, L_ref = oracle.ivf_range_search(xq, cents, offsets, vecs, ids, 6, radius)
    errs = compare.check_range(lims, D, L, lims_ref, D_ref, L_ref,
                               compare.exact_lookup(xq, x, oracle.L2), radius,
                               atol=compare.l2_atol(xq, x))
    assert not errs, errs[:5]


def test_kmeans_assign_update_step(cuda_device):
    x = syn.gaussian(20000, 32, seed=19)
    c = x[:200].copy()
    dev = cuda_device
    xt = torch.from_numpy(x).to(dev)
    ct = torch.from_numpy(c).to(dev)
    lab, dist = clustering.assign(xt, ct)
    lab_ref, dist_ref = oracle.kmeans_assign(x, c)
    lab = lab.cpu().numpy()
    mism = np.nonzero(lab != lab_ref)[0]
    if len(mism):
        ex = oracle.pairwise_exact(x[mism], c, oracle.L2)
        a = ex[np.arange(len(mism)), lab[mism]]
        b = ex[np.arange(len(mism)), lab_ref[mism]]
        assert np.all(np.abs(a - b) <= 1e-5 * np.abs(b) + compare.l2_atol(x, c))
    assert np.allclose(dist.cpu().numpy(), dist_ref, rtol=1e-4, atol=compare.l2_atol(x, c))
    lab_t = torch.from_numpy(lab_ref).to(dev)
    counts = clustering.update(xt, lab_t, ct)
    c_ref, counts_ref = oracle.kmeans_update(x, lab_ref, c)
    assert np.array_equal(counts.cpu().numpy(), counts_ref)
    assert np.allclose(ct.cpu().numpy(), c_ref, rtol=1e-5, atol=1e-6)


def test_kmeans_empty_cluster_keeps_centroid(cuda_device):
    x = syn.gaussian(500, 8, seed=20)
    c = np.concatenate([x[:4], np.full((2, 8), 1e3, np.float32)])
    xt = torch.from_numpy(x).to(cuda_device)
    ct = torch.from_numpy(c).to(cuda_device)
    lab, _ = clustering.assign(xt, ct)
    counts = clustering.update(xt, lab, ct)
    assert counts.cpu().numpy()[4:].sum() == 0
    assert np.array_equal(ct.cpu().numpy()[4:], c[4:])


def test_kmeans_train_matches_oracle_on_separated_data(cuda_device):
    x, cen, _ = syn.mixture(12000, 16, 24, seed=21)
    got = clustering.kmeans_clustering(x, 16, 24, clustering.ClusteringParameters(niter=10, seed=5, max_points_per_centroid=0)).cpu().numpy()
    ref = oracle.kmeans_train(x, 24, 10, 5)
    assert np.allclose(got, ref, rtol=1e-4, atol=1e-4)


def test_topk_merge_capi(cuda_device):
    rng = np.random.default_rng(22)
    nq, parts, kin, k = 37, 5, 12, 20
    pd = np.sort(rng.standard_normal((nq, parts, kin)).astype(np.float32), axis=2)
    pl = rng.integers(0, 1 << 40, size=(nq, parts, kin)).astype(np.int64)
    pl[:, 4, 6:] = -1
    pd[:, 4, 6:] = np.inf
    dev = cuda_device
    tpd, tpl = torch.from_numpy(pd).to(dev), torch.from_numpy(pl).to(dev)
    D = torch.empty((nq, k), dtype=torch.float32, device=dev)
    I = torch.empty((nq, k), dtype=torch.int64, device=dev)
    nat.call("mf_topk_merge", 0, nat.stream_of(dev), nat.ptr(tpd), nat.ptr(tpl), nq, parts, kin, k,
             nat.ptr(D), nat.ptr(I))
    flatd = pd.reshape(nq, -1)
    flatl = pl.reshape(nq, -1)
    order = np.argsort(np.where(flatl >= 0, flatd, np.inf), axis=1, kind="stable")[:, :k]
    assert np.array_equal(D.cpu().numpy(), np.take_along_axis(flatd, order, 1))
    assert np.array_equal(I.cpu().numpy(), np.take_along_axis(flatl, order, 1))


def test_ivf_coarse_bound_path_equals_plain(cuda_device):
    """With coarse_bound on and nlist >= 2048 the coarse step starts from a
    bound taken from an IVF over the centroids; its probes and the search
    results must equal those of the unbounded coarse step (mf_ivf_search)."""
    x, cen, _ = syn.mixture(200_000, 64, 2048, seed=61)
    idx = IVFFlatIndex(64, 2048)
    idx.set_centroids(x[:: 200_000 // 2048][:2048])
    idx.add(x)
    idx.nprobe = 24
    idx.coarse_bound = True
    idx.filter_search = False  # both sides on the exact 3xTF32 scan
    xq, _, _ = syn.mixture(3000, 64, 2048, seed=62, centres=cen)
    xt = idx._prepare_query(xq)
    cq = idx._centroid_index()
    assert cq is not None
    probes_b = idx._coarse_probes(xt, cq).cpu().numpy()
    probes_p = idx.quantizer._search_padded(xt, 24, map_ids=False).labels.cpu().numpy()
    assert np.array_equal(probes_b, probes_p)
    D1, I1 = idx.search(xq, 10).numpy()          # bounded coarse step
    old = IVFFlatIndex.COARSE_BOUND_MIN_NLIST
    try:
        IVFFlatIndex.COARSE_BOUND_MIN_NLIST = 1 << 30
        D2, I2 = idx.search(xq, 10).numpy()      # mf_ivf_search
    finally:
        IVFFlatIndex.COARSE_BOUND_MIN_NLIST = old
    np.testing.assert_array_equal(I1, I2)
    np.testing.assert_array_equal(D1, D2)
