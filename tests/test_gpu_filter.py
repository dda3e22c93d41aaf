"""The IVF filter search (an fp16 tensor-core pass over scaled residuals
against the list centroids, then an exact fp32 refinement;
mf_ivf_search_filtered) against
the CPU oracle and against the exact 3xTF32 scan of the same index:

* mixtures at d = 64, 96, 128 with k from 1 to 16 and nprobe from 1 to 32;
* batches small enough that every list is probed by at most 16 queries (the
  fp16 few-query pass alone), at d = 72 and 80 (not multiples of 32: lanes
  past d carry zeros) and 128;
* duplicated rows, so that more rows tie inside a pair's error window than its
  slots hold: the refinement must rescan those lists and stay exact;
* lists holding fewer than k rows (padded results), data scaled by 1e3 and
  1e-3, an add after a search (the bank is rebuilt), and queries far from
  every centroid."""
import numpy as np
import pytest
import torch

from metalfaiss_b200 import IVFFlatIndex
from metalfaiss_b200 import _native as nat
from metalfaiss_b200 import synthetic as syn
from oracle import compare, oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert nat.device_error(0) == 0, "a bounded device wait timed out"


def _build(x, nlist, seed):
    idx = IVFFlatIndex(x.shape[1], nlist)
    idx.set_centroids(oracle.kmeans_train(x, nlist, 2, seed))
    idx.add(x)
    return idx


def _check(idx, x, xq, nprobe, k):
    """Filter search == oracle over the index's own lists, and == the exact scan."""
    assert nat.load().mf_ivf_filter_eligible(idx._dp, k, idx.ntotal) == 1
    idx.nprobe = nprobe
    D, I = idx.search(xq, k).numpy()
    offsets = idx._offsets.cpu().numpy()
    vecs = idx._vecs[:, : idx.d].cpu().numpy()
    ids = idx._ids[: idx.ntotal].cpu().numpy()
    cents = idx.centroids[: idx.nlist, : idx.d].cpu().numpy()
    D_ref, I_ref = oracle.ivf_search(xq, cents, offsets, vecs, ids, nprobe, k, oracle.L2)
    look = compare.exact_lookup(xq, x, oracle.L2)
    atol = compare.l2_atol(xq, x)
    errs = compare.check_knn(D, I, D_ref, I_ref, look, atol=atol)
    assert not errs, errs[:5]
    idx.filter_search = False
    try:
        De, Ie = idx.search(xq, k).numpy()
    finally:
        idx.filter_search = True
    errs = compare.check_knn(D, I, De, Ie, look, atol=atol)
    assert not errs, errs[:5]
    return D, I


@pytest.mark.parametrize("d,k,nprobe", [(64, 10, 8), (128, 1, 4), (128, 16, 16), (96, 5, 32),
                                        (128, 10, 32)])
def test_filter_equals_oracle_and_exact(cuda_device, d, k, nprobe):
    x, cen, _ = syn.mixture(40000, d, 128, seed=d + k)
    idx = _build(x, 128, seed=d)
    xq, _, _ = syn.mixture(700, d, 128, seed=d + k + 1, centres=cen)
    nat.filter_rescans(0, reset=True)
    _check(idx, x, xq, nprobe, k)


@pytest.mark.parametrize("d,k,nprobe", [(72, 7, 16), (80, 10, 8), (128, 16, 32)])
def test_filter_few_query_lists(cuda_device, d, k, nprobe):
    """16 queries: no list is probed by more than 16, so the few-query pass
    scans every probed list."""
    x, cen, _ = syn.mixture(30000, d, 256, seed=d + 5)
    idx = _build(x, 256, seed=d + 5)
    xq, _, _ = syn.mixture(16, d, 256, seed=d + 6, centres=cen)
    _check(idx, x, xq, nprobe, k)


def test_filter_rescans_tied_rows(cuda_device):
    """Each of 40 points is stored 64 times: a query at one of them sees 64
    rows at the same distance, more than a pair's slots (at most 32) hold, so
    the refinement rescans those lists."""
    d = 64
    x, cen, _ = syn.mixture(20000, d, 64, seed=71)
    base = x[:40].copy()
    x[: 40 * 64] = np.repeat(base, 64, axis=0)
    idx = _build(x, 64, seed=71)
    rng = np.random.Generator(np.random.PCG64(72))
    xq = (base + 1e-3 * rng.standard_normal(base.shape)).astype(np.float32)
    nat.filter_rescans(0, reset=True)
    _check(idx, x, xq, 4, 10)
    assert nat.filter_rescans(0) > 0


def test_filter_short_lists_pad(cuda_device):
    """nlist = 256 over 600 rows: many lists hold fewer than k rows."""
    d = 64
    x, cen, _ = syn.mixture(600, d, 256, seed=81)
    idx = _build(x, 256, seed=81)
    xq, _, _ = syn.mixture(300, d, 256, seed=82, centres=cen)
    D, I = _check(idx, x, xq, 1, 16)
    assert (I == -1).any() and np.isinf(D[I == -1]).all()


@pytest.mark.parametrize("scale", [1e3, 1e-3])
def test_filter_scaled_data(cuda_device, scale):
    d = 128
    x, cen, _ = syn.mixture(30000, d, 100, seed=91)
    x = (x * scale).astype(np.float32)
    idx = _build(x, 100, seed=91)
    xq, _, _ = syn.mixture(400, d, 100, seed=92, centres=cen)
    _check(idx, x, (xq * scale).astype(np.float32), 8, 10)


def test_filter_bank_rebuilt_after_add(cuda_device):
    d = 64
    x, cen, _ = syn.mixture(30000, d, 80, seed=101)
    idx = _build(x[:20000], 80, seed=101)
    xq, _, _ = syn.mixture(300, d, 80, seed=102, centres=cen)
    _check(idx, x[:20000], xq, 6, 10)
    idx.add(x[20000:])
    _check(idx, x, xq, 6, 10)


def test_filter_far_queries(cuda_device):
    """Queries far outside the data: every list is far, the error bounds are
    large against the distances' spread."""
    d = 128
    x, cen, _ = syn.mixture(30000, d, 64, seed=111)
    idx = _build(x, 64, seed=111)
    xq = (syn.gaussian(200, d, seed=112) * 40.0).astype(np.float32)
    _check(idx, x, xq, 8, 10)


@pytest.mark.parametrize("d", [56, 136, 256])
def test_dims_outside_the_filter_take_the_exact_scan(cuda_device, d):
    """L2 indexes whose d the filter search does not take (below 64, above
    128) run the exact scan: same results as the oracle, and the filter bank
    itself refuses those shapes instead of failing inside the refinement."""
    x, cen, _ = syn.mixture(20000, d, 64, seed=121)
    idx = _build(x, 64, seed=121)
    assert nat.load().mf_ivf_filter_eligible(idx._dp, 10, idx.ntotal) == 0
    assert not idx._filter_ok(10)
    xq, _, _ = syn.mixture(300, d, 64, seed=122, centres=cen)
    idx.nprobe = 8
    D, I = idx.search(xq, 10).numpy()
    offsets = idx._offsets.cpu().numpy()
    vecs = idx._vecs[:, : idx.d].cpu().numpy()
    ids = idx._ids[: idx.ntotal].cpu().numpy()
    cents = idx.centroids[: idx.nlist, : idx.d].cpu().numpy()
    D_ref, I_ref = oracle.ivf_search(xq, cents, offsets, vecs, ids, 8, 10, oracle.L2)
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq, x, oracle.L2),
                             atol=compare.l2_atol(xq, x))
    assert not errs, errs[:5]
    dev = idx.device
    n = idx._vecs.shape[0]
    h = torch.empty((n, idx._dp), dtype=torch.float16, device=dev)
    rn = torch.empty(n, dtype=torch.float32, device=dev)
    stats = torch.empty((idx.nlist, 4), dtype=torch.float32, device=dev)
    rn16 = torch.empty((n, 16), dtype=torch.float16, device=dev)
    lib = nat.load()
    status = lib.mf_ivf_filter_bank(dev.index, nat.stream_of(dev), idx.nlist, idx._dp,
                                    nat.ptr(idx._offsets), nat.ptr(idx._vecs),
                                    nat.ptr(idx._norms), nat.ptr(idx.quantizer._xb.buf), n,
                                    nat.ptr(h), nat.ptr(rn), nat.ptr(rn16), nat.ptr(stats))
    assert status == 6, lib.mf_last_error()


@pytest.mark.parametrize("d,nq", [(128, 3000), (64, 2500), (96, 700)])
def test_filter_one_and_two_epilogue_groups_agree(cuda_device, d, nq):
    """The filter pass with one epilogue warpgroup and with two (each taking
    half of every tile's columns, sharing the rows' thresholds and merging at
    the end of an item) gives the same results, and both equal the oracle.
    Batches large enough that most lists are probed by more than 16 queries."""
    x, cen, _ = syn.mixture(60000, d, 48, seed=131 + d)
    idx = _build(x, 48, seed=131 + d)
    xq, _, _ = syn.mixture(nq, d, 48, seed=132 + d, centres=cen)
    lib = nat.load()
    try:
        lib.mf_set_filter_groups(1)
        idx.nprobe = 6
        D1, I1 = idx.search(xq, 10).numpy()
        lib.mf_set_filter_groups(2)
        D2, I2 = _check(idx, x, xq, 6, 10)
    finally:
        lib.mf_set_filter_groups(2)
    np.testing.assert_array_equal(I1, I2)
    np.testing.assert_array_equal(D1, D2)
