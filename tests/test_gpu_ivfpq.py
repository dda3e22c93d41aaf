"""IVFPQ on the device (python/metalfaiss/index/ivf_pq_index.py): codes against
the oracle's argmin per sub-space, the ADC search against the oracle's
restatement of IVFPQIndex.search on the index's own centroids, codebooks and
lists, incremental adds, ids, and recall against exact search."""
import numpy as np
import pytest
import torch

from metalfaiss_b200 import _native as nat
from metalfaiss_b200 import synthetic as syn
from metalfaiss_b200.index_ivfpq import IVFPQIndex, ProductQuantizer
from oracle import compare, oracle

pytestmark = pytest.mark.gpu


def _adc_lookup(xq, cents, pq, offsets, codes, ids):
    """exact_of for check_knn: the fp64 ADC distance of (query, label)."""
    pos = {int(v): i for i, v in enumerate(np.asarray(ids).tolist())}
    row_list = np.searchsorted(offsets, np.arange(len(ids)), side="right") - 1
    pq64 = np.asarray(pq, np.float64)
    M, ksub, dsub = pq64.shape

    def exact_of(q, labels):
        out = np.full(len(labels), np.inf)
        for t, lab in enumerate(np.asarray(labels).tolist()):
            if lab < 0:
                continue
            r = pos[lab]
            rec = cents[row_list[r]].astype(np.float64) + np.concatenate(
                [pq64[m][codes[r, m]] for m in range(M)])
            out[t] = float(((xq[q].astype(np.float64) - rec) ** 2).sum())
        return out
    return exact_of


def _bank(idx):
    off, codes, ids = idx.list_codes()
    return off.cpu().numpy(), codes.cpu().numpy(), ids.cpu().numpy()


@pytest.mark.parametrize("d,M,nbits", [(64, 16, 8), (32, 8, 8), (96, 12, 6), (128, 64, 8)])
def test_ivfpq_search_equals_oracle(cuda_device, d, M, nbits):
    nlist = 32
    x, cen, _ = syn.mixture(20000, d, nlist, seed=d + M)
    idx = IVFPQIndex(d, nlist, M, nbits)
    idx.train(x[:8000], niter=8)
    idx.add(x[:12000])
    idx.add(x[12000:], np.arange(8000, dtype=np.int64) + 10 ** 6)
    assert idx.ntotal == 20000
    xq, _, _ = syn.mixture(150, d, nlist, seed=d + M + 1, centres=cen)
    idx.nprobe = 4
    D, I = idx.search(xq, 10).numpy()
    cents = idx.centroids.cpu().numpy()
    pq = idx.pq.centroids.cpu().numpy()
    offs, codes, ids = _bank(idx)
    D_ref, I_ref = oracle.ivfpq_search(xq, cents, pq, offs, codes, ids, 4, 10)
    errs = compare.check_knn(D, I, D_ref, I_ref, _adc_lookup(xq, cents, pq, offs, codes, ids),
                             atol=1e-5 * float(np.abs(D_ref[np.isfinite(D_ref)]).max()))
    assert not errs, errs[:5]
    assert nat.device_error(0) == 0


def test_pq_codes_equal_oracle_argmin(cuda_device):
    d, M = 64, 8
    x = syn.gaussian(5000, d, seed=3)
    pq = ProductQuantizer(d, M, 8)
    pq.train(x, niter=6)
    codes = pq.compute_codes(x).cpu().numpy()
    ref = oracle.pq_encode(x, pq.centroids.cpu().numpy())
    cents = pq.centroids.cpu().numpy().astype(np.float64)
    diff = np.nonzero(codes != ref)
    # a differing code must be a near-tie of the two centroid distances
    for r, m in zip(*diff):
        sub = x[r, m * 8:(m + 1) * 8].astype(np.float64)
        a = ((cents[m][codes[r, m]] - sub) ** 2).sum()
        b = ((cents[m][ref[r, m]] - sub) ** 2).sum()
        assert abs(a - b) <= 1e-5 * max(a, b) + 1e-7, (r, m, a, b)
    assert len(diff[0]) <= 5
    rec = pq.decode(torch.from_numpy(codes)).cpu().numpy()
    np.testing.assert_allclose(rec[:, :8], cents[0][codes[:, 0]], rtol=0, atol=0)


def test_ivfpq_recall_and_empty(cuda_device):
    """Recall@10 of the ADC top-10 against exact L2 at nprobe = nlist, and an
    index with no rows gives (+inf, -1)."""
    d, nlist = 64, 16
    x, cen, _ = syn.mixture(30000, d, nlist, seed=5)
    idx = IVFPQIndex(d, nlist, 32, 8)
    idx.train(x[:10000], niter=8)
    xq, _, _ = syn.mixture(100, d, nlist, seed=6, centres=cen)
    D, I = idx.search(xq, 5).numpy()
    assert (I == -1).all() and np.isinf(D).all()
    idx.add(x)
    idx.nprobe = nlist
    _, I = idx.search(xq, 10).numpy()
    _, I_ex = oracle.flat_search(xq, x, 10)
    recall = np.mean([len(set(a) & set(b)) / 10 for a, b in zip(I, I_ex)])
    print(f"IVFPQ recall@10 (M=32, nbits=8, nprobe=nlist) = {recall:.3f}")
    assert recall > 0.5
