"""The multi-GPU IVF search's device steps, with its ranks emulated in one
process on one GPU: the lists split over W ranks by LPT (keep_lists), each
rank's bound from mf_ivf_probe_bound, their minimum (what the MIN all-reduce
gives every rank), each rank's mf_ivf_search_bounded over its own lists, and
the on-device merge. The merged result must equal the unsharded search.
The collectives themselves are covered on CPU ranks (test_sharding_gloo)."""
import numpy as np
import pytest
import torch

from metalfaiss_b200 import IVFFlatIndex, MetricType
from metalfaiss_b200 import _native as nat
from metalfaiss_b200 import synthetic as syn
from metalfaiss_b200.sharding import keep_lists, lpt_partition, merge_partials
from oracle import compare, oracle

pytestmark = pytest.mark.gpu


@pytest.fixture
def engine():
    yield nat.set_scan_engine
    nat.set_scan_engine(0)
    assert nat.device_error(0) == 0, "a bounded device wait timed out"


def _index(metric, d=64, n=40000, nlist=96, seed=21):
    x, cen, _ = syn.mixture(n, d, nlist, seed)
    if metric == MetricType.INNER_PRODUCT:
        x = x / np.linalg.norm(x, axis=1, keepdims=True)
    idx = IVFFlatIndex(d, nlist, metric_type=metric)
    idx.set_centroids(oracle.kmeans_train(x, nlist, 2, seed))
    idx.add(x)
    xq, _, _ = syn.mixture(500, d, nlist, seed + 1, centres=cen)
    if metric == MetricType.INNER_PRODUCT:
        xq = xq / np.linalg.norm(xq, axis=1, keepdims=True)
    return idx, x, xq


@pytest.mark.parametrize("eng", [0, 1])
@pytest.mark.parametrize("metric", [MetricType.L2, MetricType.INNER_PRODUCT])
@pytest.mark.parametrize("world", [2, 3])
def test_emulated_ranks_equal_single(cuda_device, engine, eng, metric, world):
    nat.set_scan_engine(eng)
    idx, x, xq_np = _index(metric)
    idx.nprobe = 8
    k = 10
    ref = idx.search(xq_np, k)
    xq = idx._prepare_query(xq_np)
    probes = idx.quantizer._search_padded(xq, idx.nprobe, map_ids=False).labels.contiguous()
    owners = lpt_partition(idx.list_sizes(), world)
    shards = [keep_lists(idx, owners == r) for r in range(world)]
    bounds = [s._probe_bound(xq, probes, k) for s in shards]
    bound = torch.stack(bounds).min(0).values
    # every query's bound comes from the one rank holding its nearest list
    finite = torch.stack([torch.isfinite(b) for b in bounds]).sum(0)
    assert int(finite.max()) <= 1
    parts = [s._search_bounded(xq, k, probes, bound) for s in shards]
    pd = torch.stack([p.distances for p in parts], 1).contiguous()
    pi = torch.stack([p.labels for p in parts], 1).contiguous()
    got = merge_partials(pd, pi, k)
    D, I = got.numpy()
    D_ref, I_ref = ref.numpy()
    m = oracle.L2 if metric == MetricType.L2 else oracle.INNER_PRODUCT
    atol = compare.l2_atol(xq_np, x) if metric == MetricType.L2 else 1e-5 * (1 + np.abs(D_ref).max())
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq_np, x, m), atol=atol)
    assert not errs, errs[:5]


def test_kmeans_sums_over_shards_equal_update(cuda_device):
    """mf_kmeans_sums on shards + a summed (all-reduced) total + mf_kmeans_apply
    equals mf_kmeans_update on all points; an empty cluster keeps its centroid."""
    from metalfaiss_b200 import clustering
    from metalfaiss_b200.sharding import row_shard

    x, _, _ = syn.mixture(30000, 64, 50, seed=31)
    xt = torch.from_numpy(x).cuda()
    c = torch.from_numpy(np.concatenate([x[:49], np.full((1, 64), 1e3, np.float32)])).cuda()
    labels, _ = clustering.assign(xt, c, clustering.compute_norms(c))
    ref = c.clone()
    counts_ref = clustering.update(xt, labels, ref)
    assert int(counts_ref[-1]) == 0
    tot_s = tot_n = None
    for r in range(3):
        b, e = row_shard(len(x), r, 3)
        s, n = clustering.cluster_sums(xt[b:e].contiguous(), labels[b:e].contiguous(), 50)
        tot_s = s if tot_s is None else tot_s + s
        tot_n = n if tot_n is None else tot_n + n
    got = c.clone()
    clustering.apply_sums(tot_s, tot_n, got)
    assert torch.equal(tot_n, counts_ref)
    assert torch.equal(got[-1], c[-1])
    torch.testing.assert_close(got, ref, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_build_holds_each_rank_its_own_lists(cuda_device, world):
    """add_owned_rows: each emulated rank adds only the rows of the lists it
    owns (LPT over the sizes every rank computes alike), under global ids and
    in input order. The ranks' banks partition the whole one exactly, and the
    bounded filter searches over them merge to the unsharded search."""
    from metalfaiss_b200.sharding import add_owned_rows

    d, nlist, k = 64, 96, 10
    x, cen, _ = syn.mixture(40000, d, nlist, seed=41)
    cents = oracle.kmeans_train(x, nlist, 2, 41)
    full = IVFFlatIndex(d, nlist)
    full.set_centroids(cents)
    full.add(x)
    shards, owners = [], None
    for r in range(world):
        s = IVFFlatIndex(d, nlist)
        s.set_centroids(cents)
        o = add_owned_rows(s, x, r, world)
        assert owners is None or np.array_equal(o, owners)
        owners = o
        shards.append(s)
    assert np.array_equal(owners, lpt_partition(full.list_sizes(), world))
    assert sum(s.ntotal for s in shards) == full.ntotal
    offs = full.list_offsets.cpu().numpy()
    for r, s in enumerate(shards):
        so = s.list_offsets.cpu().numpy()
        for l in range(nlist):
            n_l = so[l + 1] - so[l]
            if owners[l] != r:
                assert n_l == 0
                continue
            assert n_l == offs[l + 1] - offs[l]
            torch.testing.assert_close(s._ids[so[l]:so[l + 1]], full._ids[offs[l]:offs[l + 1]],
                                       rtol=0, atol=0)
            torch.testing.assert_close(s._vecs[so[l]:so[l + 1]],
                                       full._vecs[offs[l]:offs[l + 1]], rtol=0, atol=0)
    xq_np, _, _ = syn.mixture(500, d, nlist, seed=42, centres=cen)
    full.nprobe = 8
    ref = full.search(xq_np, k)
    xq = full._prepare_query(xq_np)
    probes = full.quantizer._search_padded(xq, 8, map_ids=False).labels.contiguous()
    bound = torch.stack([s._probe_bound(xq, probes, k) for s in shards]).min(0).values
    parts = [s._search_bounded(xq, k, probes, bound) for s in shards]
    pd = torch.stack([p.distances for p in parts], 1).contiguous()
    pi = torch.stack([p.labels for p in parts], 1).contiguous()
    D, I = merge_partials(pd, pi, k).numpy()
    D_ref, I_ref = ref.numpy()
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq_np, x, oracle.L2),
                             atol=compare.l2_atol(xq_np, x))
    assert not errs, errs[:5]
