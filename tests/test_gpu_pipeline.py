"""search_host_batches: host query batches searched with the copies
overlapped give, batch for batch, what the device search gives; batches of
different sizes (the device buffers replaced mid-run) included."""
import numpy as np
import pytest
import torch

from metalfaiss_b200 import FlatIndex, IVFFlatIndex, MetricType
from metalfaiss_b200 import synthetic as syn
from metalfaiss_b200.pipeline import search_host_batches
from oracle import oracle


def test_empty_and_mismatched_inputs():
    search_host_batches(lambda q: None, [], [], "cpu")  # nothing to do, no device touched
    with pytest.raises(ValueError):
        search_host_batches(lambda q: None, [torch.zeros(2, 4)], [], "cpu")


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["ivf", "flat"])
def test_pipelined_batches_equal_device_search(cuda_device, kind):
    d, nlist, k = 64, 64, 10
    x, cen, _ = syn.mixture(30000, d, nlist, seed=51)
    if kind == "ivf":
        idx = IVFFlatIndex(d, nlist)
        idx.set_centroids(oracle.kmeans_train(x, nlist, 2, 51))
        idx.nprobe = 8
    else:
        idx = FlatIndex(d, MetricType.L2)
    idx.add(x)
    sizes = [700, 700, 333, 700, 1, 512]
    xq, _, _ = syn.mixture(sum(sizes), d, nlist, seed=52, centres=cen)
    offs = np.cumsum([0] + sizes)
    batches = [torch.from_numpy(xq[a:b]).pin_memory() for a, b in zip(offs[:-1], offs[1:])]
    outs = [(torch.full((n, k), -1.0).pin_memory(),
             torch.full((n, k), -2, dtype=torch.int64).pin_memory()) for n in sizes]
    dev = torch.device("cuda", 0)
    search_host_batches(lambda q: idx.search(q, k), batches, outs, dev)
    torch.cuda.synchronize(dev)
    for hb, (D_h, I_h) in zip(batches, outs):
        ref = idx.search(hb.to(dev), k)
        assert torch.equal(I_h, ref.labels.cpu())
        assert torch.equal(D_h, ref.distances.cpu())
