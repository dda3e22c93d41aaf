"""mf_flat_search_noalloc (the flat search that uses a fixed device scratch
array instead of a caller workspace) against mf_flat_search, through the C-ABI.

Two searches of different shapes, metrics and engines run back to back on the
one shared scratch array; each must match mf_flat_search on the same inputs
within the tolerances the other parity tests use, and the first also the CPU
oracle directly. Repeating both searches must leave the device's free memory
unchanged: the entry point is for callers that cannot allocate, so a search
that allocated (or cached an allocation) would fail them. Collected last so
that it also runs after every other test has used the library in this
process."""
import ctypes

import numpy as np
import pytest
import torch

from metalfaiss_b200 import _native as nat
from metalfaiss_b200 import synthetic as syn
from metalfaiss_b200.errors import ErrorCode
from oracle import compare, oracle

pytestmark = pytest.mark.gpu

L2, IP = 1, 0


def _bank(n, d, seed, dev):
    xb = torch.from_numpy(syn.gaussian(n, d, seed)).to(dev)
    norms = torch.empty(n, dtype=torch.float32, device=dev)
    lo = torch.empty_like(xb)
    st = nat.stream_of(dev)
    nat.call("mf_vector_norms", dev.index, st, nat.ptr(xb), n, d, nat.ptr(norms))
    nat.call("mf_tf32_residual", dev.index, st, nat.ptr(xb), n, d, nat.ptr(lo))
    ids = torch.arange(n, dtype=torch.int64, device=dev) * 7 + 1000
    return xb, norms, lo, ids


def _with_workspace(dev, xq, xb, norms, lo, ids, metric, k):
    nq, d = xq.shape
    nb = xb.shape[0]
    D = torch.empty((nq, k), dtype=torch.float32, device=dev)
    I = torch.empty((nq, k), dtype=torch.int64, device=dev)
    ws = torch.empty(nat.workspace_size("mf_flat_search_workspace_size", nq, nb, d, metric, k),
                     dtype=torch.uint8, device=dev)
    nat.call("mf_flat_search", dev.index, nat.stream_of(dev), nat.ptr(xq), nq, nat.ptr(xb),
             nat.ptr(norms), nat.ptr(lo), nb, d, metric, k, nat.ptr(ids), nat.ptr(D), nat.ptr(I),
             nat.ptr(ws), ws.numel())
    return D, I


def _noalloc(dev, xq, xb, norms, lo, ids, metric, k):
    nq, d = xq.shape
    nb = xb.shape[0]
    D = torch.full((nq, k), float("nan"), dtype=torch.float32, device=dev)
    I = torch.full((nq, k), -7, dtype=torch.int64, device=dev)
    nat.call("mf_flat_search_noalloc", dev.index, nat.stream_of(dev), nat.ptr(xq), nq,
             nat.ptr(xb), nat.ptr(norms), nat.ptr(lo), nb, d, metric, k, nat.ptr(ids),
             nat.ptr(D), nat.ptr(I))
    return D, I


def _check(xq, xb, ids, metric, got, ref):
    D, I = (t.cpu().numpy() for t in got)
    D_ref, I_ref = (t.cpu().numpy() for t in ref)
    q, b, idn = xq.cpu().numpy(), xb.cpu().numpy(), ids.cpu().numpy()
    if metric == L2:
        atol = compare.l2_atol(q, b)
    else:
        atol = 1e-5 * (1 + np.abs(D_ref).max())
    errs = compare.check_knn(D, I, D_ref, I_ref, compare.exact_lookup(q, b, metric, idn),
                             atol=atol)
    assert not errs, errs[:5]


def test_noalloc_matches_workspace_search_twice(cuda_device):
    dev = torch.device("cuda", 0)
    # call 1: L2 with tf32 residuals (tensor-core engine), k = 10
    xb1, n1, lo1, ids1 = _bank(40000, 64, seed=11, dev=dev)
    xq1 = torch.from_numpy(syn.gaussian(300, 64, 12)).to(dev)
    # call 2: inner product without stored residuals, other shapes, k = 17
    xb2, n2, _, ids2 = _bank(23456, 96, seed=13, dev=dev)
    xq2 = torch.from_numpy(syn.gaussian(129, 96, 14)).to(dev)

    ref1 = _with_workspace(dev, xq1, xb1, n1, lo1, ids1, L2, 10)
    ref2 = _with_workspace(dev, xq2, xb2, n2, None, ids2, IP, 17)
    got1 = _noalloc(dev, xq1, xb1, n1, lo1, ids1, L2, 10)
    got2 = _noalloc(dev, xq2, xb2, n2, None, ids2, IP, 17)
    torch.cuda.synchronize()
    _check(xq1, xb1, ids1, L2, got1, ref1)
    _check(xq2, xb2, ids2, IP, got2, ref2)
    # the first search also against the CPU oracle itself
    q1, b1 = xq1.cpu().numpy(), xb1.cpu().numpy()
    D_or, I_or = oracle.flat_search(q1, b1, 10, oracle.L2, ids1.cpu().numpy())
    errs = compare.check_knn(got1[0].cpu().numpy(), got1[1].cpu().numpy(), D_or, I_or,
                             compare.exact_lookup(q1, b1, oracle.L2, ids1.cpu().numpy()),
                             atol=compare.l2_atol(q1, b1))
    assert not errs, errs[:5]
    assert nat.device_error(0) == 0

    # The same two searches again into buffers allocated up front: the
    # device's free memory must not move (nothing allocated, nothing cached).
    outs = [(torch.empty((xq1.shape[0], 10), dtype=torch.float32, device=dev),
             torch.empty((xq1.shape[0], 10), dtype=torch.int64, device=dev)),
            (torch.empty((xq2.shape[0], 17), dtype=torch.float32, device=dev),
             torch.empty((xq2.shape[0], 17), dtype=torch.int64, device=dev))]
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(dev)
    for (xq, xb, nrm, lo, ids, metric, k), (D, I) in zip(
            [(xq1, xb1, n1, lo1, ids1, L2, 10), (xq2, xb2, n2, None, ids2, IP, 17)], outs):
        nat.call("mf_flat_search_noalloc", dev.index, nat.stream_of(dev), nat.ptr(xq),
                 xq.shape[0], nat.ptr(xb), nat.ptr(nrm), nat.ptr(lo), xb.shape[0], xq.shape[1],
                 metric, k, nat.ptr(ids), nat.ptr(D), nat.ptr(I))
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0, f"device free memory moved by {free0 - free1} bytes"
    assert torch.equal(outs[0][1], got1[1]) and torch.equal(outs[1][1], got2[1])
    assert torch.equal(outs[0][0], got1[0]) and torch.equal(outs[1][0], got2[0])


def test_noalloc_rejects_searches_beyond_the_scratch(cuda_device):
    dev = torch.device("cuda", 0)
    lib = nat.load()
    nq, nb, d, k = 4096, 100000, 128, 256
    need = nat.workspace_size("mf_flat_search_workspace_size", nq, nb, d, L2, k)
    assert need > (16 << 20)
    # sizes are checked before any pointer is used or any kernel launched
    buf = torch.empty(16, dtype=torch.float32, device=dev)
    lab = torch.empty(16, dtype=torch.int64, device=dev)
    status = lib.mf_flat_search_noalloc(0, None, nat.ptr(buf), nq, nat.ptr(buf), nat.ptr(buf),
                                        None, nb, d, L2, k, None, nat.ptr(buf), nat.ptr(lab))
    assert status == ErrorCode.INVALID_ARGS
    msg = lib.mf_last_error().decode()
    assert "static scratch" in msg and str(need) in msg, msg
