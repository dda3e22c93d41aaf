"""The search path at the full sizes of its benchmark configurations, checked
through properties that do not need a CPU run over the whole data, plus the
oracle on a few sampled queries or points:

* flat INNER_PRODUCT, 10M unit rows x d=128, Q=10000, k=100: ascending rows,
  self-queries return themselves first, sampled queries equal the oracle;
* IVFFlat L2, 20M rows from a 16384-cluster mixture, nlist=16384, nprobe=32
  (the benchmarked index, built once for the module): the k=10 search, by the
  default filter search and by the exact scan, on 64 sampled queries against
  the oracle (its own coarse step, then the probed lists); range search at
  radius = median 10th-NN distance: every reported distance within the
  radius, every kNN result within the radius reported, sampled queries equal
  the oracle over their probed lists;
* k-means, 5M points x d=256, K=4096: sampled assignments equal the oracle's
  argmin, sampled cluster means equal the oracle's, sizes sum to N.

Inputs are generated on the device from fixed seeds (the mixtures of the
benchmark), so each test holds 5-25 GB of HBM and runs for seconds."""
import gc

import numpy as np
import pytest
import torch

from metalfaiss_b200 import FlatIndex, IVFFlatIndex, MetricType, clustering
from metalfaiss_b200 import _native as nat
from metalfaiss_b200 import synthetic as syn
from metalfaiss_b200.clustering import ClusteringParameters
from oracle import compare, oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _release():
    yield
    gc.collect()
    torch.cuda.empty_cache()


def test_flat_ip_10m_k100(cuda_device):
    dev = torch.device("cuda", 0)
    n, d, nq, k = 10_000_000, 128, 10_000, 100
    xb = syn.torch_unit_rows(n, d, 41, dev)
    xq = syn.torch_unit_rows(nq, d, 42, dev)
    self_rows = torch.arange(0, n, n // 64, device=dev)[:64]
    xq[:64] = xb[self_rows]
    idx = FlatIndex(d, MetricType.INNER_PRODUCT)
    idx.add(xb)
    D, I = idx.search(xq, k)
    assert D.shape == (nq, k) and I.shape == (nq, k)
    assert bool((D[:, 1:] >= D[:, :-1]).all()), "rows must be ascending"
    assert bool((I >= 0).all())
    assert torch.equal(I[:64, 0], self_rows)
    # sampled queries against the oracle (exact fp64 inner products, on the host)
    sample = [0, 77, 5003, nq - 1]
    xb_h = xb.cpu().numpy()
    for q in sample:
        qv = xq[q:q + 1].cpu().numpy()
        ip = np.concatenate([(xb_h[s:s + 1_000_000].astype(np.float64) @ qv[0].astype(np.float64))
                             for s in range(0, n, 1_000_000)])
        ref_i = np.argsort(-ip, kind="stable")[:k]
        got_d = D[q].cpu().numpy()
        got_i = I[q].cpu().numpy()
        np.testing.assert_allclose(got_d, -ip[ref_i], rtol=1e-4, atol=1e-5)
        # labels equal except where the exact values are near-ties
        diff = np.nonzero(got_i != ref_i)[0]
        for j in diff:
            assert abs(ip[got_i[j]] - ip[ref_i[j]]) <= 1e-5 * (1 + abs(ip[ref_i[j]]))


IVF20M = dict(n=20_000_000, d=128, nlist=16384, nq=10_000, nprobe=32, k=10, seed=1234)


@pytest.fixture(scope="module")
def ivf20m():
    """The benchmarked IVFFlat index: 20M rows from the 16384-cluster mixture,
    nlist=16384 trained by seeded k-means (10 iterations on a 256-per-list
    subsample), 10000 queries from the same mixture, nprobe=32 (the same seeds
    and training as the benchmark's index)."""
    c = IVF20M
    dev = torch.device("cuda", 0)
    x, cen = syn.torch_mixture(c["n"], c["d"], c["nlist"], c["seed"], dev)
    params = ClusteringParameters(niter=10, seed=c["seed"], max_points_per_centroid=256)
    idx = IVFFlatIndex(c["d"], c["nlist"], device=dev, clustering=params)
    idx.train(x)
    idx.add(x)
    del x
    torch.cuda.empty_cache()
    xq, _ = syn.torch_mixture(c["nq"], c["d"], c["nlist"], c["seed"] + 1, dev, centres=cen)
    idx.nprobe = c["nprobe"]
    yield idx, xq
    del idx, xq
    gc.collect()
    torch.cuda.empty_cache()


def _probed_rows(idx, lists):
    """Rows of the given lists, in list order, with a CSR over them."""
    offs = idx.list_offsets.cpu().numpy()
    sizes = np.array([offs[l + 1] - offs[l] for l in lists], np.int64)
    sub = np.zeros(len(lists) + 1, np.int64)
    np.cumsum(sizes, out=sub[1:])
    rows = np.concatenate([np.arange(offs[l], offs[l + 1]) for l in lists])
    return rows, sub


@pytest.mark.parametrize("filtered", [True, False], ids=["filter", "exact"])
def test_ivf_20m_knn_sampled_oracle(cuda_device, ivf20m, filtered):
    """The benchmarked search (k=10) on 64 sampled queries against the oracle:
    the oracle's own coarse step over all 16384 centroids, then the exact
    top-k over the rows of the probed lists. The default L2 path is the fp16
    filter search with its exact refinement; it must rescan no list here and
    no bounded device wait may time out."""
    idx, xq = ivf20m
    c = IVF20M
    d, k, P = c["d"], c["k"], c["nprobe"]
    dev = xq.device
    nat.filter_rescans(0, reset=True)
    idx.filter_search = filtered
    try:
        assert idx._filter_ok(k) == filtered
        D, I = idx.search(xq, k)
    finally:
        idx.filter_search = True
    torch.cuda.synchronize()
    assert nat.device_error(0) == 0, "a bounded device wait timed out"
    if filtered:
        assert nat.filter_rescans(0, reset=True) == 0
    rng = np.random.Generator(np.random.PCG64(20))
    sample = np.unique(np.concatenate([np.linspace(0, c["nq"] - 1, 32).astype(np.int64),
                                       rng.choice(c["nq"], 32, replace=False)]))
    assert len(sample) >= 60
    cents = idx.centroids[:, :d].cpu().numpy()
    qs = xq[torch.from_numpy(sample).to(dev)].cpu().numpy()
    probes_ref = oracle.coarse_probes(qs, cents, P)
    probes_gpu = idx.quantizer._search_padded(idx._prepare_query(xq), P,
                                              map_ids=False).labels.cpu().numpy()[sample]
    Dg, Ig = D.cpu().numpy()[sample], I.cpu().numpy()[sample]
    for t in range(len(sample)):
        pr = probes_ref[t]
        if set(pr.tolist()) != set(probes_gpu[t].tolist()):
            # only a near-tie at the last probe may differ
            exact = oracle.pairwise_exact(qs[t:t + 1], cents, oracle.L2)[0]
            a = np.sort(exact[pr])
            b = np.sort(exact[probes_gpu[t]])
            assert np.allclose(a, b, rtol=1e-5, atol=0), (sample[t], a[-3:], b[-3:])
            pr = probes_gpu[t]
        rows, sub = _probed_rows(idx, pr)
        rt = torch.from_numpy(rows).to(dev)
        vecs = idx._vecs[rt][:, :d].cpu().numpy()
        ids = idx._ids[rt].cpu().numpy()
        qv = qs[t:t + 1]
        D_ref, I_ref = oracle.ivf_search(qv, cents, sub, vecs, ids, P, k,
                                         probes=np.arange(len(pr))[None, :])
        errs = compare.check_knn(Dg[t:t + 1], Ig[t:t + 1], D_ref, I_ref,
                                 compare.exact_lookup(qv, vecs, oracle.L2, ids),
                                 atol=compare.l2_atol(qv, vecs))
        assert not errs, (int(sample[t]), errs[:3])


def test_ivf_20m_range_search(cuda_device, ivf20m):
    idx, xq = ivf20m
    dev = xq.device
    nq, d, nprobe, k = IVF20M["nq"], IVF20M["d"], IVF20M["nprobe"], IVF20M["k"]
    D, I = idx.search(xq, k)
    radius = float(D[:, k - 1].median())
    res = idx.range_search(xq, radius)
    lims = res.lims.cpu().numpy()
    rd = res.distances.cpu().numpy()
    rl = res.labels.cpu().numpy()
    assert lims[0] == 0 and np.all(np.diff(lims) >= 0) and lims[-1] == len(rd)
    assert np.all(rd <= radius)
    # every kNN result inside the ball is in the range result
    Dh, Ih = D.cpu().numpy(), I.cpu().numpy()
    for q in range(0, nq, 97):
        inside = set(Ih[q][Dh[q] <= radius].tolist())
        assert inside <= set(rl[lims[q]:lims[q + 1]].tolist()), q
    # sampled queries against the oracle over their probed lists
    probes = idx.quantizer._search_padded(idx._prepare_query(xq), nprobe,
                                          map_ids=False).labels.cpu().numpy()
    for q in (3, 4242, nq - 2):
        rows, _ = _probed_rows(idx, probes[q])
        rt = torch.from_numpy(rows).to(dev)
        vecs = idx._vecs[rt][:, :d].cpu().numpy()
        ids = idx._ids[rt].cpu().numpy()
        qv = xq[q:q + 1].cpu().numpy()
        dist = oracle.pairwise_exact(qv, vecs, oracle.L2)[0]
        atol = compare.l2_atol(qv, vecs)
        want = set(ids[dist <= radius - atol].tolist())      # surely inside
        maybe = set(ids[dist <= radius + atol].tolist())     # inside or a near-tie
        got = set(rl[lims[q]:lims[q + 1]].tolist())
        assert want <= got <= maybe, q


def test_kmeans_5m_d256_k4096(cuda_device):
    dev = torch.device("cuda", 0)
    n, d, K = 5_000_000, 256, 4096
    x, _ = syn.torch_mixture(n, d, K, 77, dev)
    c = clustering.init_centroids(x, K, 77)
    for _ in range(2):
        c_prev = c.clone()
        labels, mind = clustering.assign(x, c, clustering.compute_norms(c))
        counts = clustering.update(x, labels, c)
    assert int(counts.sum()) == n
    # sampled assignments: argmin over all centroids (ties within tolerance)
    rng = np.random.Generator(np.random.PCG64(5))
    pts = np.sort(rng.choice(n, 1000, replace=False))
    xs = x[torch.from_numpy(pts).to(dev)].cpu().numpy()
    cp = c_prev.cpu().numpy()
    lab = labels.cpu().numpy()[pts]
    exact = oracle.pairwise_exact(xs, cp, oracle.L2)
    best = exact.min(1)
    chosen = exact[np.arange(len(pts)), lab]
    assert np.all(chosen <= best + 1e-5 * (1 + best) + compare.l2_atol(xs, cp))
    # sampled cluster means: the update of the last iteration
    lab_all = labels.cpu().numpy()
    for j in (0, 1, 2047, K - 1):
        members = np.nonzero(lab_all == j)[0]
        if len(members) == 0:
            np.testing.assert_array_equal(c[j].cpu().numpy(), cp[j])
            continue
        xm = x[torch.from_numpy(members).to(dev)].cpu().numpy().astype(np.float64)
        np.testing.assert_allclose(c[j].cpu().numpy(), xm.mean(0), rtol=1e-5, atol=1e-5)
