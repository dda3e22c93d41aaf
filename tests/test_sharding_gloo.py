"""Host logic of the multi-GPU search on CPU ranks (torch.distributed gloo,
world size 2): list and row partitioning, the all-gather layout of the partial
results, sharded == single search (the intent of the reference's multi-GPU
tests, python/metalfaiss/unittest/test_mlx_multi_gpu.py:49-65,86-119), and a
rank that leaves before the exchange step.

Each rank's local search is the oracle on its shard (the GPU kernels are not
available on CPU); what is under test is the partitioning, the exchange and
the merge order."""
import multiprocessing as mp
import os
import socket
import tempfile
from datetime import timedelta

import numpy as np
import pytest
import torch

from metalfaiss_b200.sharding import (exchange_probes, gather_packed, gather_partials,
                                      gather_rows, head_rows, lpt_partition, partial_buffer,
                                      probe_buffer, row_shard, unpack_partials)
from oracle import oracle

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, port, timeout_s=20):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=WORLD, timeout=timedelta(seconds=timeout_s))
    return dist


def _merge(pd, pi, k):
    """(nq, parts, k) -> (nq, k) ascending by (distance, label); empty slots last."""
    nq = pd.shape[0]
    d = pd.reshape(nq, -1)
    l = pi.reshape(nq, -1)
    D = np.empty((nq, k), np.float32)
    I = np.empty((nq, k), np.int64)
    for q in range(nq):
        lab = np.where(l[q] < 0, np.iinfo(np.int64).max, l[q])
        o = np.lexsort((lab, d[q]))[:k]
        D[q], I[q] = d[q][o], l[q][o]
    return D, I


def _flat_data():
    rng = np.random.Generator(np.random.PCG64(7))
    xb = rng.standard_normal((3001, 16)).astype(np.float32)
    xq = rng.standard_normal((23, 16)).astype(np.float32)
    return xb, xq


def _flat_worker(rank, port, out_dir):
    dist = _init(rank, port)
    try:
        xb, xq = _flat_data()
        k = 9
        b, e = row_shard(len(xb), rank, WORLD)
        D, pos = oracle.flat_search(xq, xb[b:e], k)
        I = pos + b  # global ids of a contiguous row shard
        pd, pi = gather_partials(torch.from_numpy(D), torch.from_numpy(I))
        assert tuple(pd.shape) == (len(xq), WORLD, k)
        # slot r of the gathered layout is rank r's own contribution
        assert np.array_equal(pi[:, rank].numpy(), I)
        Dm, Im = _merge(pd.numpy(), pi.numpy(), k)
        np.savez(os.path.join(out_dir, f"flat{rank}.npz"), D=Dm, I=Im)
    finally:
        dist.destroy_process_group()


def _ivf_data():
    rng = np.random.Generator(np.random.PCG64(11))
    nlist, d = 24, 8
    cents = (2.0 * rng.standard_normal((nlist, d))).astype(np.float32)
    lab = rng.integers(0, nlist, 4000) ** 2 % nlist  # skewed list sizes
    x = (cents[lab] + rng.standard_normal((4000, d))).astype(np.float32)
    xq = (cents[rng.integers(0, nlist, 31)] + rng.standard_normal((31, d))).astype(np.float32)
    offsets, vecs, ids = oracle.ivf_build(x, lab, nlist)
    return cents, offsets, vecs, ids, xq


def _ivf_worker(rank, port, out_dir):
    dist = _init(rank, port)
    try:
        cents, offsets, vecs, ids, xq = _ivf_data()
        nprobe, k = 5, 7
        owners = lpt_partition(np.diff(offsets), WORLD)
        probes = oracle.coarse_probes(xq, cents, nprobe)  # replicated quantizer
        local = np.where(owners[probes] == rank, probes, -1)  # scan only owned lists
        D, I = oracle.ivf_search(xq, cents, offsets, vecs, ids, nprobe, k, probes=local)
        pd, pi = gather_partials(torch.from_numpy(D), torch.from_numpy(I))
        Dm, Im = _merge(pd.numpy(), pi.numpy(), k)
        np.savez(os.path.join(out_dir, f"ivf{rank}.npz"), D=Dm, I=Im)
    finally:
        dist.destroy_process_group()


def _bound_of(xq, offsets, vecs, probes, k, owned, rows=128):
    """The bound a rank contributes: the k-th distance over the first `rows`
    rows of each query's first probe where this rank holds that list, else inf."""
    out = np.full(len(xq), np.inf, np.float32)
    for q in range(len(xq)):
        l = probes[q, 0]
        if l < 0 or not owned[l]:
            continue
        a, b = offsets[l], min(offsets[l + 1], offsets[l] + rows)
        if b - a < k:
            continue
        d = oracle.pairwise_f32(xq[q:q + 1], vecs[a:b], oracle.L2)[0]
        out[q] = np.sort(d)[k - 1]
    return out


def _ivf_bound_worker(rank, port, out_dir):
    """The multi-GPU IVF search's exchange steps: coarse probes computed for
    a row shard of the queries and all-gathered, bounds MIN-reduced, bounded
    local scans, merge."""
    dist = _init(rank, port)
    try:
        cents, offsets, vecs, ids, xq = _ivf_data()
        nprobe, k = 5, 7
        owners = lpt_partition(np.diff(offsets), WORLD)
        b, e = row_shard(len(xq), rank, WORLD)
        mine = torch.from_numpy(oracle.coarse_probes(xq[b:e], cents, nprobe).astype(np.int64))
        probes = gather_rows(mine, len(xq)).numpy()
        assert np.array_equal(probes, oracle.coarse_probes(xq, cents, nprobe))
        bound = torch.from_numpy(_bound_of(xq, offsets, vecs, probes, k, owners == rank))
        dist.all_reduce(bound, op=dist.ReduceOp.MIN)
        local = np.where(owners[probes] == rank, probes, -1)
        D, I = oracle.ivf_search(xq, cents, offsets, vecs, ids, nprobe, k, probes=local)
        keep = D <= bound.numpy()[:, None]
        D = np.where(keep, D, np.inf).astype(np.float32)
        I = np.where(keep, I, -1)
        pd, pi = gather_partials(torch.from_numpy(D), torch.from_numpy(I))
        Dm, Im = _merge(pd.numpy(), pi.numpy(), k)
        np.savez(os.path.join(out_dir, f"ivfb{rank}.npz"), D=Dm, I=Im)
    finally:
        dist.destroy_process_group()


def _ivf_heads_worker(rank, port, out_dir):
    """The head-bank form of the multi-GPU IVF search: each rank computes the
    probes and bounds of its share of the queries (the bounds from a copy of
    every list's first rows), one all-gather shares both, bounded local scans,
    one all-gather of the packed partials, merge."""
    dist = _init(rank, port)
    try:
        cents, offsets, vecs, ids, xq = _ivf_data()
        nprobe, k, nq = 5, 7, len(xq)
        owners = lpt_partition(np.diff(offsets), WORLD)
        b, e = row_shard(nq, rank, WORLD)
        send, mine, mine_bound = probe_buffer(nq, nprobe, rank, WORLD, "cpu")
        mine.copy_(torch.from_numpy(oracle.coarse_probes(xq[b:e], cents, nprobe).astype(np.int64)))
        every = np.ones(len(offsets) - 1, bool)  # the head bank holds every list
        mine_bound.copy_(torch.from_numpy(
            _bound_of(xq[b:e], offsets, vecs, mine.numpy(), k, every)))
        probes_t, bound_t = exchange_probes(send, nq, nprobe)
        probes, bound = probes_t.numpy(), bound_t.numpy()
        assert np.array_equal(probes, oracle.coarse_probes(xq, cents, nprobe))
        assert np.array_equal(bound, _bound_of(xq, offsets, vecs, probes, k, every))
        local = np.where(owners[probes] == rank, probes, -1)
        D, I = oracle.ivf_search(xq, cents, offsets, vecs, ids, nprobe, k, probes=local)
        keep = D <= bound[:, None]
        psend, Dv, Iv = partial_buffer(nq, k, "cpu")
        Dv.copy_(torch.from_numpy(np.where(keep, D, np.inf).astype(np.float32)))
        Iv.copy_(torch.from_numpy(np.where(keep, I, -1)))
        pd, pi = unpack_partials(gather_packed(psend), nq, k)
        assert tuple(pd.shape) == (WORLD, nq, k)
        # part r of the gathered buffer is rank r's own contribution
        assert torch.equal(pi[rank], Iv) and torch.equal(pd[rank], Dv)
        Dm, Im = _merge(pd.permute(1, 0, 2).numpy(), pi.permute(1, 0, 2).numpy(), k)
        np.savez(os.path.join(out_dir, f"ivfh{rank}.npz"), D=Dm, I=Im)
    finally:
        dist.destroy_process_group()


def _exchange_shapes_worker(rank, port, out_dir):
    """exchange_probes for batches with fewer queries than ranks (rank 1's
    share empty) and an empty batch."""
    dist = _init(rank, port)
    try:
        nprobe = 3
        for nq in (0, 1, 2, 3, 7):
            probes = torch.arange(nq * nprobe, dtype=torch.int64).reshape(nq, nprobe)
            bound = torch.arange(nq, dtype=torch.float32) / 4
            b, e = row_shard(nq, rank, WORLD)
            send, mine, mine_bound = probe_buffer(nq, nprobe, rank, WORLD, "cpu")
            assert tuple(mine.shape) == (e - b, nprobe) and mine_bound.numel() == e - b
            mine.copy_(probes[b:e])
            mine_bound.copy_(bound[b:e])
            got_p, got_b = exchange_probes(send, nq, nprobe)
            assert torch.equal(got_p, probes) and torch.equal(got_b, bound), nq
        with open(os.path.join(out_dir, f"shapes{rank}.txt"), "w") as f:
            f.write("ok")
    finally:
        dist.destroy_process_group()


def _gather_rows_worker(rank, port, out_dir):
    dist = _init(rank, port)
    try:
        for n in (0, 1, 5, 8):
            full = torch.arange(n * 3, dtype=torch.int64).reshape(n, 3)
            b, e = row_shard(n, rank, WORLD)
            got = gather_rows(full[b:e], n)
            assert torch.equal(got, full), (n, got, full)
        with open(os.path.join(out_dir, f"rows{rank}.txt"), "w") as f:
            f.write("ok")
    finally:
        dist.destroy_process_group()


def _leaving_worker(rank, port, out_dir):
    """Rank 1 leaves between steps (after set-up, before the exchange); rank 0
    must get an error from its next collective instead of waiting forever."""
    dist = _init(rank, port, timeout_s=5)
    if rank == 1:
        os._exit(3)
    msg = "no error"
    try:
        gather_partials(torch.zeros(4, 3), torch.zeros(4, 3, dtype=torch.int64))
    except Exception as e:  # the failure surfaces on the host as an exception
        msg = f"raised {type(e).__name__}"
    with open(os.path.join(out_dir, "leave0.txt"), "w") as f:
        f.write(msg)
    os._exit(0)


def _run(target, out_dir, limit_s=120):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, port, out_dir)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(limit_s)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return [p.exitcode for p in procs]


def test_lpt_partition_covers_and_balances():
    rng = np.random.Generator(np.random.PCG64(3))
    sizes = (rng.pareto(1.2, 5000) * 100).astype(np.int64)
    for world in (1, 2, 4, 8):
        owners = lpt_partition(sizes, world)
        assert owners.shape == sizes.shape and owners.min() >= 0 and owners.max() < world
        load = np.bincount(owners, weights=sizes, minlength=world)
        # greedy LPT: the heaviest rank exceeds the lightest by at most one list
        assert load.max() - load.min() <= sizes.max()


def test_row_shard_is_a_partition():
    for n in (0, 1, 7, 1000, 1001):
        for world in (1, 2, 3, 8):
            spans = [row_shard(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[r][1] == spans[r + 1][0] for r in range(world - 1))
            sizes = [e - b for b, e in spans]
            assert max(sizes) - min(sizes) <= 1


def test_sharded_flat_equals_single_gloo():
    with tempfile.TemporaryDirectory() as tmp:
        assert _run(_flat_worker, tmp) == [0, 0]
        xb, xq = _flat_data()
        D_ref, I_ref = oracle.flat_search(xq, xb, 9)
        for r in range(WORLD):
            z = np.load(os.path.join(tmp, f"flat{r}.npz"))
            assert np.array_equal(z["I"], I_ref)
            assert np.array_equal(z["D"], D_ref)


def test_sharded_ivf_equals_single_gloo():
    with tempfile.TemporaryDirectory() as tmp:
        assert _run(_ivf_worker, tmp) == [0, 0]
        cents, offsets, vecs, ids, xq = _ivf_data()
        D_ref, I_ref = oracle.ivf_search(xq, cents, offsets, vecs, ids, 5, 7)
        for r in range(WORLD):
            z = np.load(os.path.join(tmp, f"ivf{r}.npz"))
            assert np.array_equal(z["I"], I_ref)
            assert np.allclose(z["D"], D_ref, rtol=0, atol=0)


def test_rank_leaving_before_exchange_is_reported_gloo():
    with tempfile.TemporaryDirectory() as tmp:
        codes = _run(_leaving_worker, tmp, limit_s=90)
        assert codes == [0, 3]
        with open(os.path.join(tmp, "leave0.txt")) as f:
            assert f.read().startswith("raised"), "rank 0 did not see the failure"


def test_gather_rows_gloo():
    with tempfile.TemporaryDirectory() as tmp:
        assert _run(_gather_rows_worker, tmp) == [0, 0]


def test_sharded_ivf_bound_exchange_equals_single_gloo():
    with tempfile.TemporaryDirectory() as tmp:
        assert _run(_ivf_bound_worker, tmp) == [0, 0]
        cents, offsets, vecs, ids, xq = _ivf_data()
        D_ref, I_ref = oracle.ivf_search(xq, cents, offsets, vecs, ids, 5, 7)
        for r in range(WORLD):
            z = np.load(os.path.join(tmp, f"ivfb{r}.npz"))
            assert np.array_equal(z["I"], I_ref)
            assert np.array_equal(z["D"], D_ref)


def _kmeans_data():
    rng = np.random.Generator(np.random.PCG64(5))
    cen = 3.0 * rng.standard_normal((12, 6))
    x = (cen[rng.integers(0, 12, 901)] + rng.standard_normal((901, 6))).astype(np.float32)
    return x, x[rng.permutation(901)[:12]].copy()


def _kmeans_worker(rank, port, out_dir):
    """Sharded Lloyd iterations: local assignment, SUM all-reduce of the fp64
    per-cluster sums and sizes, the same update on every rank."""
    dist = _init(rank, port)
    try:
        x, c = _kmeans_data()
        b, e = row_shard(len(x), rank, WORLD)
        xs = x[b:e]
        for _ in range(4):
            lab, _ = oracle.kmeans_assign(xs, c)
            sums = np.zeros(c.shape, np.float64)
            np.add.at(sums, lab, xs.astype(np.float64))
            cnt = np.bincount(lab, minlength=len(c)).astype(np.int64)
            ts, tc = torch.from_numpy(sums), torch.from_numpy(cnt)
            dist.all_reduce(ts, op=dist.ReduceOp.SUM)
            dist.all_reduce(tc, op=dist.ReduceOp.SUM)
            s, n = ts.numpy(), tc.numpy()
            c = np.where(n[:, None] > 0, s / np.maximum(n, 1)[:, None], c).astype(np.float32)
        np.save(os.path.join(out_dir, f"km{rank}.npy"), c)
    finally:
        dist.destroy_process_group()


def test_sharded_kmeans_equals_single_gloo():
    with tempfile.TemporaryDirectory() as tmp:
        assert _run(_kmeans_worker, tmp) == [0, 0]
        x, c0 = _kmeans_data()
        ref = oracle.kmeans_train(x, len(c0), 4, 0, init=c0)
        c_r = [np.load(os.path.join(tmp, f"km{r}.npy")) for r in range(WORLD)]
        assert np.array_equal(c_r[0], c_r[1])  # identical on every rank
        np.testing.assert_allclose(c_r[0], ref, rtol=1e-6, atol=1e-6)


def test_sharded_ivf_head_bank_exchange_equals_single_gloo():
    with tempfile.TemporaryDirectory() as tmp:
        assert _run(_ivf_heads_worker, tmp) == [0, 0]
        cents, offsets, vecs, ids, xq = _ivf_data()
        D_ref, I_ref = oracle.ivf_search(xq, cents, offsets, vecs, ids, 5, 7)
        for r in range(WORLD):
            z = np.load(os.path.join(tmp, f"ivfh{r}.npz"))
            assert np.array_equal(z["I"], I_ref)
            assert np.array_equal(z["D"], D_ref)


def test_head_rows_are_each_lists_first_rows():
    rng = np.random.Generator(np.random.PCG64(5))
    nlist = 7
    labels = rng.integers(0, nlist, 500) ** 2 % nlist  # skewed, some lists empty
    for rows in (1, 3, 40, 1000):
        got = head_rows(torch.from_numpy(labels), nlist, rows).numpy()
        want = np.sort(np.concatenate([np.flatnonzero(labels == l)[:rows]
                                       for l in range(nlist)]))
        assert np.array_equal(got, want)
    assert head_rows(torch.empty(0, dtype=torch.int64), nlist, 4).numel() == 0


def test_exchange_probes_uneven_and_empty_gloo():
    with tempfile.TemporaryDirectory() as tmp:
        assert _run(_exchange_shapes_worker, tmp) == [0, 0]
