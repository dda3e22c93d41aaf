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


@pytest.mark.parametrize("metric", [MetricType.L2, MetricType.INNER_PRODUCT])
@pytest.mark.parametrize("world", [2, 3])
def test_head_bank_search_equals_single(cuda_device, engine, metric, world):
    """The head-bank form of the multi-GPU search, ranks emulated in one
    process: each rank's coarse step and bounds (from the head bank, the first
    mf_ivf_bound_rows() rows of every list) for its share of the queries,
    written into its probe_buffer; the buffers concatenated as the all-gather
    leaves them; bounded scans into partial_buffers; merge_packed over the
    stacked buffers. Equal to merge_partials over the same partials, and to
    the unsharded search."""
    from metalfaiss_b200.sharding import (head_bank, merge_packed, partial_buffer,
                                          probe_buffer, row_shard, unpack_partials)

    idx, x, xq_np = _index(metric)
    idx.nprobe = P = 8
    k = 10
    ref = idx.search(xq_np, k)
    xq = idx._prepare_query(xq_np)
    nq = xq.shape[0]
    heads = head_bank(idx)
    R = nat.load().mf_ivf_bound_rows()
    sizes, hsizes = idx.list_sizes(), heads.list_sizes()
    assert np.array_equal(hsizes, np.minimum(sizes, R))
    owners = lpt_partition(sizes, world)
    shards = [keep_lists(idx, owners == r) for r in range(world)]
    sends = []
    for r in range(world):
        b, e = row_shard(nq, r, world)
        send, mine, mine_bound = probe_buffer(nq, P, r, world, xq.device)
        scratch = torch.empty((e - b, P), dtype=torch.float32, device=xq.device)
        idx.quantizer._search_padded(xq[b:e], P, map_ids=False, out=(scratch, mine))
        heads._probe_bound(xq[b:e], mine, k, out=mine_bound)
        sends.append(send)
    # what exchange_probes unpacks from the all-gather's (world, words) output
    gathered = torch.stack(sends)
    bounds = gathered[:, -(-nq // world) * P:].view(torch.float32)
    shares = [row_shard(nq, r, world) for r in range(world)]
    probes = torch.cat([gathered[r, : (e - b) * P].view(e - b, P)
                        for r, (b, e) in enumerate(shares)])
    bound = torch.cat([bounds[r, : e - b] for r, (b, e) in enumerate(shares)])
    full_probes = idx.quantizer._search_padded(xq, P, map_ids=False).labels
    assert torch.equal(probes, full_probes)
    # the head bank's bound is a bound: at least the exact k-th distance
    D_ref, I_ref = ref.numpy()
    assert bool((bound.cpu().numpy() >= D_ref[:, k - 1]).all())
    psends = []
    for s in shards:
        psend, Dv, Iv = partial_buffer(nq, k, xq.device)
        s._search_bounded(xq, k, probes, bound, out=(Dv, Iv))
        psends.append(psend)
    buf = torch.stack(psends)
    D, I = merge_packed(buf, nq, k, k).numpy()
    pd, pi = unpack_partials(buf, nq, k)
    D2, I2 = merge_partials(pd.permute(1, 0, 2).contiguous(), pi.permute(1, 0, 2).contiguous(),
                            k).numpy()
    assert np.array_equal(I, I2) and np.array_equal(D, D2)
    m = oracle.L2 if metric == MetricType.L2 else oracle.INNER_PRODUCT
    atol = compare.l2_atol(xq_np, x) if metric == MetricType.L2 else 1e-5 * (1 + np.abs(D_ref).max())
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq_np, x, m), atol=atol)
    assert not errs, errs[:5]


def test_strided_merge_matches_contiguous(cuda_device):
    """mf_topk_merge_strided over a part-major layout with padded rows equals
    mf_topk_merge over the (nq, parts, k_in) copy, ties and empty slots
    included."""
    g = torch.Generator().manual_seed(3)
    nq, parts, k_in, k = 37, 5, 12, 9
    d = torch.randint(0, 6, (nq, parts, k_in), generator=g).float()  # many ties
    d = d.sort(-1).values
    l = torch.randint(0, 1000, (nq, parts, k_in), generator=g)
    l[torch.rand((nq, parts, k_in), generator=g) < 0.2] = -1
    d[l < 0] = float("inf")
    dev = torch.device("cuda", 0)
    ref = merge_partials(d.to(dev), l.to(dev), k)
    # part-major, each part's block padded by 3 elements
    pad = 3
    bd = torch.full((parts, nq * k_in + pad), 7.0)
    bl = torch.full((parts, nq * k_in + pad), 5, dtype=torch.int64)
    bd[:, : nq * k_in] = d.permute(1, 0, 2).reshape(parts, -1)
    bl[:, : nq * k_in] = l.permute(1, 0, 2).reshape(parts, -1)
    bd, bl = bd.to(dev), bl.to(dev)
    D = torch.empty((nq, k), device=dev)
    I = torch.empty((nq, k), dtype=torch.int64, device=dev)
    nat.call("mf_topk_merge_strided", 0, nat.stream_of(dev), nat.ptr(bd), k_in, nq * k_in + pad,
             nat.ptr(bl), k_in, nq * k_in + pad, nq, parts, k_in, k, nat.ptr(D), nat.ptr(I))
    assert torch.equal(D, ref.distances) and torch.equal(I, ref.labels)
