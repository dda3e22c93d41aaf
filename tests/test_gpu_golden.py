"""The CUDA path against the reference's own outputs (tests/golden/), same inputs."""
from pathlib import Path

import numpy as np
import pytest

from metalfaiss_b200 import FlatIndex, IVFFlatIndex, MetricType
from oracle import compare, oracle

pytestmark = pytest.mark.gpu
G = np.load(Path(__file__).parent / "golden" / "reference_golden.npz")


@pytest.mark.parametrize("tag", list(G["flat_cases"]))
def test_flat_vs_reference(cuda_device, tag):
    xb, xq, ids = G[tag + "_xb"], G[tag + "_xq"], G[tag + "_ids"]
    metric, k = (int(v) for v in G[tag + "_meta"])
    idx = FlatIndex(xb.shape[1], MetricType(metric))
    idx.add(xb, ids)
    D, I = idx.search(xq, k).numpy()
    atol = compare.l2_atol(xq, xb) if metric == oracle.L2 else 1e-5
    errs = compare.check_knn(D, I, G[tag + "_D"], G[tag + "_I"], compare.exact_lookup(xq, xb, metric, ids),
                             atol=atol)
    assert not errs, errs[:3]


@pytest.mark.parametrize("tag", list(G["ivf_cases"]))
def test_ivf_vs_reference(cuda_device, tag):
    x, cents, labels, xq = G[tag + "_x"], G[tag + "_cents"], G[tag + "_labels"], G[tag + "_xq"]
    nlist, nprobe, k = (int(v) for v in G[tag + "_meta"])
    idx = IVFFlatIndex(x.shape[1], nlist)
    idx.set_centroids(cents)
    idx.add(x)
    # same lists as the reference's quantizer built
    assert np.array_equal(np.diff(idx.list_offsets.cpu().numpy()), np.bincount(labels, minlength=nlist))
    idx.nprobe = nprobe
    D, I = idx.search(xq, k).numpy()
    kk = G[tag + "_D"].shape[1]
    errs = compare.check_knn(D[:, :kk], I[:, :kk], G[tag + "_D"], G[tag + "_I"],
                             compare.exact_lookup(xq, x, oracle.L2), atol=compare.l2_atol(xq, x))
    assert not errs, errs[:3]


def test_range_vs_reference(cuda_device):
    xb, xq, r = G["range_small_xb"], G["range_small_xq"], float(G["range_small_radius"])
    idx = FlatIndex(xb.shape[1])
    idx.add(xb)
    lims, D, I = idx.range_search(xq, r).numpy()
    errs = compare.check_range(lims, D, I, G["range_small_lims"], G["range_small_D"], G["range_small_I"],
                               compare.exact_lookup(xq, xb, oracle.L2), r, atol=compare.l2_atol(xq, xb))
    assert not errs, errs[:3]
