"""FlatIndex on the GPU against the CPU oracle (parity rule in oracle/compare.py:
labels exact except near-ties <= 1e-5 relative, distances <= 1e-4 relative)."""
import numpy as np
import pytest
import torch

from metalfaiss_b200 import FlatIndex, MetricType
from metalfaiss_b200 import _native as nat
from metalfaiss_b200 import synthetic as syn
from oracle import compare, oracle

pytestmark = pytest.mark.gpu

METRICS = [MetricType.L2, MetricType.INNER_PRODUCT, MetricType.L1, MetricType.LINF]


def _check(index, xq, xb, k, metric, ids=None):
    res = index.search(xq, k)
    D, I = res.numpy()
    D_ref, I_ref = oracle.flat_search(xq, xb, k, int(metric), ids)
    atol = compare.l2_atol(xq, xb) if metric == MetricType.L2 else 1e-5 * (1 + np.abs(D_ref).max())
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(xq, xb, int(metric), ids),
                             atol=atol)
    assert not errs, errs[:5]
    return D, I


@pytest.mark.parametrize("metric", METRICS)
@pytest.mark.parametrize("d", [4, 8, 64, 128])
def test_flat_metrics(cuda_device, metric, d):
    xb = syn.gaussian(3000, d, seed=10 + d)
    xq = syn.gaussian(70, d, seed=20 + d)
    idx = FlatIndex(d, metric)
    idx.add(xb)
    _check(idx, xq, xb, 10, metric)


@pytest.mark.parametrize("k", [1, 7, 32, 33, 100, 128, 200, 256])
def test_flat_k_sweep(cuda_device, k):
    xb = syn.gaussian(5000, 32, seed=1)
    xq = syn.gaussian(40, 32, seed=2)
    idx = FlatIndex(32)
    idx.add(xb)
    _check(idx, xq, xb, k, MetricType.L2)


@pytest.mark.parametrize("d", [1, 3, 5, 65, 130, 256])
def test_flat_odd_dims(cuda_device, d):
    xb = syn.gaussian(1500, d, seed=3)
    xq = syn.gaussian(33, d, seed=4)
    for metric in METRICS:
        idx = FlatIndex(d, metric)
        idx.add(xb)
        _check(idx, xq, xb, 5, metric)


def test_flat_small_database_clips_k(cuda_device):
    xb = syn.gaussian(7, 16, seed=5)
    xq = syn.gaussian(3, 16, seed=6)
    idx = FlatIndex(16)
    idx.add(xb)
    D, I = _check(idx, xq, xb, 10, MetricType.L2)
    assert D.shape == (3, 7)  # k clipped to ntotal, python/metalfaiss/utils/sorting.py:66-67


def test_flat_config_c1(cuda_device):
    """FlatIndex L2: N=32768 x d=64 N(0,1), Q=16 N(0,1), k=10."""
    xb = syn.gaussian(32768, 64, seed=1)
    xq = syn.gaussian(16, 64, seed=2)
    idx = FlatIndex(64)
    idx.add(xb)
    _check(idx, xq, xb, 10, MetricType.L2)


def test_flat_many_queries_multi_split(cuda_device):
    xb = syn.gaussian(20000, 48, seed=8)
    xq = syn.gaussian(1000, 48, seed=9)
    idx = FlatIndex(48, MetricType.INNER_PRODUCT)
    idx.add(xb)
    _check(idx, xq, xb, 16, MetricType.INNER_PRODUCT)


@pytest.mark.parametrize("metric,k", [(MetricType.INNER_PRODUCT, 100), (MetricType.L2, 10)])
def test_flat_split_major_database(cuda_device, metric, k):
    """A database past 64 MB of fp32 rows and residuals with several query
    tiles: the tensor-core scan takes (row split, query tile) items split-major
    and merges one partial list per split; ids mapped after the merge."""
    xb = syn.unit_rows(80_000, 128, seed=31)
    xq = syn.unit_rows(300, 128, seed=32)
    xq[:2] = xb[[7, 79_999]]
    ids = np.arange(80_000, dtype=np.int64) * 5 + 3
    idx = FlatIndex(128, metric)
    idx.add(xb, ids)
    D, I = _check(idx, xq, xb, k, metric, ids)
    assert list(I[:2, 0]) == [ids[7], ids[79_999]]


@pytest.mark.parametrize("metric,k,nq", [(MetricType.L2, 8, 700), (MetricType.INNER_PRODUCT, 32, 700),
                                         (MetricType.L2, 32, 4500), (MetricType.INNER_PRODUCT, 8, 4500)])
def test_flat_distance_matrix_path_matches_fused(cuda_device, metric, k, nq):
    """k in [8, 32] over 2 to 64 query tiles takes the distance-matrix path
    (every distance written, then one warp per query selects) when the
    workspace holds the matrix; one byte less keeps the fused top-k. The two
    give identical distances and labels, and both match the oracle."""
    from metalfaiss_b200 import _native as nat
    from metalfaiss_b200._tensors import as_matrix

    xb = syn.gaussian(9000, 64, seed=41)
    xq = syn.gaussian(nq, 64, seed=42)
    ids = np.arange(9000, dtype=np.int64) * 3 + 1
    idx = FlatIndex(64, metric)
    idx.add(xb, ids)
    D, I = _check(idx, xq, xb, k, metric, ids)  # full workspace: the matrix path
    q = as_matrix(xq, 64, idx.device, "queries")
    need = nat.workspace_size("mf_flat_search_workspace_size", len(xq), idx.ntotal, idx._dp,
                              int(metric), k)
    ws = torch.empty(need, dtype=torch.uint8, device=idx.device)
    D2 = torch.empty((len(xq), k), dtype=torch.float32, device=idx.device)
    I2 = torch.empty((len(xq), k), dtype=torch.int64, device=idx.device)
    nat.call("mf_flat_search", idx.device.index, nat.stream_of(idx.device), nat.ptr(q), len(xq),
             nat.ptr(idx._xb.buf), nat.ptr(idx._norms.buf),
             nat.ptr(idx._lo.buf if idx._lo is not None else None), idx.ntotal, idx._dp,
             int(metric), k, nat.ptr(idx._ids.buf), nat.ptr(D2), nat.ptr(I2), nat.ptr(ws),
             need - 1)  # one byte short of the matrix: the fused top-k
    np.testing.assert_array_equal(D2.cpu().numpy(), D)
    np.testing.assert_array_equal(I2.cpu().numpy(), I)


def test_flat_ids_64bit_self_query(cuda_device):
    """python/metalfaiss/unittest/test_mlx_index.py:231-240: self-query returns the own 64-bit id."""
    xb = syn.gaussian(1000, 64, seed=11)
    ids = np.arange(1000, dtype=np.int64) + (1 << 32)
    idx = FlatIndex(64)
    idx.add_with_ids(xb, ids)
    D, I = idx.search(xb[:10], 1).numpy()
    assert np.array_equal(I[:, 0], ids[:10])
    assert np.all(D[:, 0] <= compare.l2_atol(xb[:10], xb))


def test_flat_incremental_add_and_reconstruct(cuda_device):
    xb = syn.gaussian(2500, 24, seed=12)
    idx = FlatIndex(24)
    for s in range(0, 2500, 700):
        idx.add(xb[s:s + 700])
    assert idx.ntotal == 2500
    xq = syn.gaussian(20, 24, seed=13)
    _check(idx, xq, xb, 10, MetricType.L2)
    assert np.array_equal(idx.reconstruct(1234).cpu().numpy(), xb[1234])
    assert np.array_equal(idx.reconstruct_n(10, 5).cpu().numpy(), xb[10:15])
    with pytest.raises(ValueError):
        idx.reconstruct(2500)


def test_flat_ties_resolve_to_lower_position(cuda_device):
    xb = np.repeat(syn.gaussian(50, 16, seed=14), 4, axis=0)  # every row 4 times
    xq = syn.gaussian(9, 16, seed=15)
    idx = FlatIndex(16, MetricType.L1)
    idx.add(xb)
    D, I = idx.search(xq, 8).numpy()
    D_ref, I_ref = oracle.flat_search(xq, xb, 8, oracle.L1)
    assert np.array_equal(I, I_ref)


def test_flat_torch_inputs_and_clone(cuda_device):
    xb = torch.from_numpy(syn.gaussian(900, 32, seed=16)).to(cuda_device)
    idx = FlatIndex(32)
    idx.add(xb)
    c = idx.clone()
    idx.reset()
    assert idx.ntotal == 0 and c.ntotal == 900
    xq = syn.gaussian(5, 32, seed=17)
    _check(c, xq, xb.cpu().numpy(), 4, MetricType.L2)


@pytest.mark.parametrize("metric", METRICS)
def test_flat_range_search(cuda_device, metric):
    xb = syn.gaussian(4000, 16, seed=18)
    xq = syn.gaussian(25, 16, seed=19)
    D0, _ = oracle.flat_search(xq, xb, 30, int(metric))
    radius = float(np.median(D0[:, -1]))
    idx = FlatIndex(16, metric)
    idx.add(xb)
    r = idx.range_search(xq, radius)
    lims, D, L = r.numpy()
    lims_ref, D_ref, L_ref = oracle.range_search(xq, xb, radius, int(metric))
    atol = compare.l2_atol(xq, xb) if metric == MetricType.L2 else 1e-4
    errs = compare.check_range(lims, D, L, lims_ref, D_ref, L_ref,
                               compare.exact_lookup(xq, xb, int(metric)), radius, atol=atol)
    assert not errs, errs[:5]
    # row order inside each query
    for q in range(len(xq)):
        seg = L[lims[q]:lims[q + 1]]
        assert np.all(np.diff(seg) > 0)


def test_flat_empty_and_errors(cuda_device):
    idx = FlatIndex(8)
    with pytest.raises(ValueError):
        idx.search(np.zeros((1, 8), np.float32), 1)
    idx.add(syn.gaussian(10, 8, seed=20))
    with pytest.raises(ValueError):
        idx.search(np.zeros((1, 7), np.float32), 1)
    r = idx.search(np.zeros((0, 8), np.float32), 3)
    assert tuple(r.distances.shape) == (0, 3)


@pytest.mark.parametrize("k", [1, 10, 32])
@pytest.mark.parametrize("layout", ["mixture", "near_first", "duplicates"])
def test_flat_many_queries_l2(cuda_device, k, layout):
    """L2 tensor-core flat search of many queries against the oracle: rows
    from a mixture (mixture), the first rows each query's nearest (near_first),
    and the first 2048 rows repeated at 2048..4095 (duplicates: equal
    distances, which the lower row must win). Also equal to
    mf_flat_search_bounded with an infinite bound."""
    d, nb, nq = 64, 20000, 1500
    xb, cen, _ = syn.mixture(nb, d, 32, seed=61)
    xq, _, _ = syn.mixture(nq, d, 32, seed=62, centres=cen)
    if layout == "near_first":
        xb[:nq] = xq + 1e-3 * syn.gaussian(nq, d, seed=63)
    elif layout == "duplicates":
        xb[2048:4096] = xb[:2048]
    idx = FlatIndex(d, MetricType.L2)
    idx.add(xb)
    assert nat.load().mf_flat_engine(int(MetricType.L2), d, k, nb, 1) == 1
    D, I = _check(idx, xq, xb, k, MetricType.L2)
    xqt = torch.from_numpy(xq).cuda()
    inf = torch.full((nq,), float("inf"), device="cuda")
    open_ = idx._search_bounded(xqt, k, inf)
    assert np.array_equal(open_.labels.cpu().numpy(), I)
    assert np.array_equal(open_.distances.cpu().numpy(), D)
    if layout == "duplicates":
        # of two equal rows the lower one comes back first
        for q in range(nq):
            got = set(I[q].tolist())
            assert all(l - 2048 in got for l in I[q] if 2048 <= l < 4096), q
