"""Pins the CPU oracle to the reference's own outputs (tests/golden/)."""
from pathlib import Path

import numpy as np
import pytest

from oracle import compare, cport, oracle

G = np.load(Path(__file__).parent / "golden" / "reference_golden.npz")
METRIC = {"L2": oracle.L2, "INNER_PRODUCT": oracle.INNER_PRODUCT, "L1": oracle.L1, "LINF": oracle.LINF}


@pytest.mark.parametrize("tag", ["a", "b"])
def test_pairwise(tag):
    xq, xb = G[f"pairwise_{tag}_xq"], G[f"pairwise_{tag}_xb"]
    np.testing.assert_allclose(oracle.pairwise_f32(xq, xb, oracle.L2), G[f"pairwise_{tag}_l2"], rtol=1e-6, atol=1e-5)
    np.testing.assert_allclose(oracle.pairwise_f32(xq, xb, oracle.L1), G[f"pairwise_{tag}_l1"], rtol=1e-6)
    np.testing.assert_allclose(oracle.pairwise_f32(xq, xb, oracle.LINF), G[f"pairwise_{tag}_linf"], rtol=1e-6)
    # the property the reference's own test checks (test_distances.py:19-35)
    exact = oracle.pairwise_exact(xq, xb, oracle.L2)
    np.testing.assert_allclose(G[f"pairwise_{tag}_l2"], exact, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("tag", list(G["flat_cases"]))
def test_flat_search(tag):
    xb, xq, ids = G[tag + "_xb"], G[tag + "_xq"], G[tag + "_ids"]
    metric, k = (int(v) for v in G[tag + "_meta"])
    D, I = oracle.flat_search(xq, xb, k, metric, ids)
    assert D.shape == G[tag + "_D"].shape  # k clipped to ntotal like the reference
    atol = compare.l2_atol(xq, xb) if metric == oracle.L2 else 1e-5
    errs = compare.check_knn(D, I, G[tag + "_D"], G[tag + "_I"], compare.exact_lookup(xq, xb, metric, ids),
                             atol=atol)
    assert not errs, errs[:3]


@pytest.mark.parametrize("tag", list(G["ivf_cases"]))
def test_ivf_search(tag):
    x, cents, labels, xq = G[tag + "_x"], G[tag + "_cents"], G[tag + "_labels"], G[tag + "_xq"]
    nlist, nprobe, k = (int(v) for v in G[tag + "_meta"])
    # the list build: the oracle's assignment equals the reference quantizer's
    lab = oracle.flat_search(x, cents, 1)[1][:, 0]
    assert np.array_equal(lab, labels)
    offsets, vecs, ids = oracle.ivf_build(x, labels, nlist)
    kk = G[tag + "_D"].shape[1]  # the reference kernel returns min(k, 32) columns
    D, I = oracle.ivf_search(xq, cents, offsets, vecs, ids, nprobe, k)
    errs = compare.check_knn(D[:, :kk], I[:, :kk], G[tag + "_D"], G[tag + "_I"],
                             compare.exact_lookup(xq, x, oracle.L2), atol=compare.l2_atol(xq, x))
    assert not errs, errs[:3]
    # the C port follows the same algorithm
    Dc, Ic = cport.ivf_search(xq, cents, offsets, vecs, ids, nprobe, k, threads=2)
    errs = compare.check_knn(Dc[:, :kk], Ic[:, :kk], G[tag + "_D"], G[tag + "_I"],
                             compare.exact_lookup(xq, x, oracle.L2), atol=compare.l2_atol(xq, x))
    assert not errs, errs[:3]


@pytest.mark.parametrize("k", [1, 10, 32])
def test_list_scan_kernel(k):
    X, ids, Q = G["kernel_X"], G["kernel_ids"].astype(np.int64), G["kernel_Q"]
    offsets = np.array([0, len(X)], np.int64)
    D, I = oracle.ivf_search(Q[None], np.zeros((1, len(Q)), np.float32), offsets, X, ids, 1, k)
    for pre in ("kernel", "kernel_chunked"):
        errs = compare.check_knn(D, I, G[f"{pre}_k{k}_D"][None], G[f"{pre}_k{k}_I"][None],
                                 compare.exact_lookup(Q[None], X, oracle.L2, ids), atol=1e-5)
        assert not errs, (pre, errs[:3])


def test_range_search_matches_reference_below_cap():
    xb, xq, r = G["range_small_xb"], G["range_small_xq"], float(G["range_small_radius"])
    lims, D, I = oracle.range_search_capped(xq, xb, r)
    assert np.array_equal(lims, G["range_small_lims"])
    assert np.array_equal(I, G["range_small_I"])
    np.testing.assert_allclose(D, G["range_small_D"], rtol=1e-6, atol=1e-5)
    # below the cap the exact search returns the same sets
    le, De, Ie = oracle.range_search(xq, xb, r)
    assert np.array_equal(le, lims)
    for q in range(len(xq)):
        assert set(Ie[le[q]:le[q + 1]].tolist()) == set(I[lims[q]:lims[q + 1]].tolist())


def test_range_search_reference_cap():
    """The reference truncates at 100 results per query (python/metalfaiss/index.py:104)."""
    xb, xq, r = G["range_capped_xb"], G["range_capped_xq"], float(G["range_capped_radius"])
    lims, D, I = oracle.range_search_capped(xq, xb, r)
    assert np.array_equal(lims, G["range_capped_lims"]) and np.array_equal(I, G["range_capped_I"])
    le, _, _ = oracle.range_search(xq, xb, r)
    assert np.all(np.diff(le) > 100)  # the exact search finds what the cap drops


def test_kmeans():
    x, perm, iters = G["kmeans_x"], G["kmeans_perm"], int(G["kmeans_iters"])
    k = len(perm)
    c = oracle.kmeans_train(x, k, iters, seed=0, init=x[perm])
    np.testing.assert_allclose(c, G["kmeans_centroids"], rtol=1e-4, atol=1e-4)


def test_hamming_oracle_matches_reference_binary_flat():
    """oracle.hamming_search against BinaryFlatIndex.search run from the
    reference's own module (tests/golden/make_golden.py gen_binary)."""
    g = G
    for tag in g["binary_cases"]:
        tag = str(tag)
        xb, xq = g[tag + "_xb"], g[tag + "_xq"]
        k = g[tag + "_D"].shape[1]
        D, I = oracle.hamming_search(xq, xb, k)
        np.testing.assert_array_equal(D, g[tag + "_D"])
        np.testing.assert_array_equal(I, g[tag + "_I"])
        np.testing.assert_array_equal(xb[5:6], g[tag + "_rec"])


def _binivf_lists(xb, ids, cents):
    """Rows into their nearest centroid's list (ties to the lower centroid), in add order."""
    _, a = oracle.hamming_search(xb, cents, 1)
    a = a[:, 0]
    return [xb[a == l] for l in range(len(cents))], [ids[a == l] for l in range(len(cents))]


def test_hamming_ivf_oracle_matches_reference_binary_ivf():
    """oracle.hamming_ivf_search against BinaryIVFIndex.search run from the
    reference's own module (tests/golden/make_golden.py gen_binary_ivf).
    Missing slots: the reference pads label 0, the oracle -1; both distance inf."""
    for tag in G["binivf_cases"]:
        tag = str(tag)
        xb, xq, cents, ids = (G[tag + s] for s in ("_xb", "_xq", "_cents", "_ids"))
        k = G[tag + "_D"].shape[1]
        rows, lid = _binivf_lists(xb, ids, cents)
        D, I, _ = oracle.hamming_ivf_search(xq, cents, rows, lid, int(G[tag + "_nprobe"]), k)
        np.testing.assert_array_equal(D, G[tag + "_D"])
        pad = np.isinf(D)
        np.testing.assert_array_equal(I[~pad], G[tag + "_I"][~pad])
        assert (I[pad] == -1).all() and (G[tag + "_I"][pad] == 0).all()
    assert any(np.isinf(G[str(t) + "_D"]).any() for t in G["binivf_cases"])  # padding covered


def test_hamming_search_packed_equals_unpacked():
    """The packed host form the benchmark's CPU baseline uses gives
    hamming_search's results, ties (to the lower row) included."""
    rng = np.random.Generator(np.random.PCG64(17))
    for d in (8, 64, 100, 256):
        xb = (rng.random((3000, d)) < 0.5).astype(np.uint8)
        xb[1500:1600] = xb[:100]  # equal rows: equal distances
        xq = (rng.random((9, d)) < 0.5).astype(np.uint8)
        for k in (1, 10, 150):
            D0, I0 = oracle.hamming_search(xq, xb, k)
            D1, I1 = oracle.hamming_search_packed(oracle.pack01_words(xq),
                                                  oracle.pack01_words(xb), k)
            assert np.array_equal(D0, D1) and np.array_equal(I0, I1), (d, k)


def test_ivfpq_oracle_matches_reference_golden():
    """oracle.pq_encode and oracle.ivfpq_search against the reference
    IVFPQIndex's own add and search on installed centroids and codebooks
    (tests/golden/make_golden.py gen_ivfpq): the lists the reference filed
    the rows into, their codes (equal but for fp32 / fp64 near-ties of two
    codewords), and the ADC search's distances and labels over the
    reference's lists and probes."""
    cases = [str(t) for t in G["ivfpq_cases"]]
    assert len(cases) == 3
    for t in cases:
        xb, xq, cents, pqc = G[t + "_xb"], G[t + "_xq"], G[t + "_cents"], G[t + "_pqc"]
        ids, codes, labels = G[t + "_ids"], G[t + "_codes"], G[t + "_labels"]
        nprobe, probes = int(G[t + "_nprobe"]), G[t + "_probes"]
        D, I = G[t + "_D"], G[t + "_I"]
        nlist, k = len(cents), D.shape[1]
        # the reference's assignment: direct-difference fp32 distances, argmin
        lab = np.argmin(np.sum(np.square(xb[:, None, :] - cents[None, :, :]), axis=2), axis=1)
        assert np.array_equal(lab, labels), t
        res = (xb - cents[labels]).astype(np.float64)
        enc = oracle.pq_encode(res, pqc)
        dsub = xb.shape[1] // pqc.shape[0]
        for r, m in np.argwhere(enc != codes):
            sub = res[r, m * dsub:(m + 1) * dsub]
            d_ours = np.sum((pqc[m, enc[r, m]].astype(np.float64) - sub) ** 2)
            d_ref = np.sum((pqc[m, codes[r, m]].astype(np.float64) - sub) ** 2)
            assert abs(d_ours - d_ref) <= 1e-5 * max(d_ref, 1e-30), (t, r, m)
        order = np.argsort(labels, kind="stable")
        offsets = np.zeros(nlist + 1, np.int64)
        np.cumsum(np.bincount(labels, minlength=nlist), out=offsets[1:])
        Do, Io = oracle.ivfpq_search(xq, cents, pqc, offsets, codes[order], ids[order], nprobe, k,
                                     probes=probes)
        assert np.array_equal(Io, I), t
        assert np.array_equal(Do, D), t
