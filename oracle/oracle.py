"""numpy restatement of the reference search path (test infrastructure only).

Conventions follow the reference:
  * L2 distances are squared and clamped at 0 (python/metalfaiss/distances.py:170-173).
  * INNER_PRODUCT distances are negated IP, ranked ascending (python/metalfaiss/indexflat.py:93).
  * top-k is an ascending sort; k is clipped to the number of candidates
    (python/metalfaiss/utils/sorting.py:66-67). Ties go to the lower position
    (a stable sort; MLX's argsort does not promise an order for ties).
"""
from __future__ import annotations

import numpy as np

INNER_PRODUCT, L2, L1, LINF = 0, 1, 2, 3


# ------------------------------------------------------------------ distances
def pairwise_l2sqr_f32(xq: np.ndarray, xb: np.ndarray) -> np.ndarray:
    """fp32 replica of pairwise_L2sqr, python/metalfaiss/distances.py:140-173:
    (||q||^2 + ||x||^2) - (q.x + q.x), clamped at 0."""
    xq = np.ascontiguousarray(xq, np.float32)
    xb = np.ascontiguousarray(xb, np.float32)
    nq = np.sum(np.square(xq), axis=1, keepdims=True, dtype=np.float32)
    nb = np.sum(np.square(xb), axis=1, keepdims=True, dtype=np.float32)
    dot = xq @ xb.T
    d = (nq + nb.T) - (dot + dot)
    return np.maximum(d, np.float32(0.0))


def pairwise_f32(xq: np.ndarray, xb: np.ndarray, metric: int) -> np.ndarray:
    """fp32 distances as the reference's FlatIndex.search computes them
    (python/metalfaiss/indexflat.py:88-99)."""
    xq = np.ascontiguousarray(xq, np.float32)
    xb = np.ascontiguousarray(xb, np.float32)
    if metric == L2:
        return pairwise_l2sqr_f32(xq, xb)
    if metric == INNER_PRODUCT:
        return -(xq @ xb.T)
    return _pairwise_direct(xq, xb, metric, np.float32)


def pairwise_exact(xq: np.ndarray, xb: np.ndarray, metric: int) -> np.ndarray:
    """fp64 distances (the yardstick for tolerances and near-ties)."""
    xq = np.asarray(xq, np.float64)
    xb = np.asarray(xb, np.float64)
    if metric == INNER_PRODUCT:
        return -(xq @ xb.T)
    if metric == L2:
        out = np.empty((xq.shape[0], xb.shape[0]), np.float64)
        for s in range(0, xq.shape[0], 64):
            diff = xq[s:s + 64, None, :] - xb[None, :, :]
            out[s:s + 64] = np.einsum("qnd,qnd->qn", diff, diff)
        return out
    return _pairwise_direct(xq, xb, metric, np.float64)


def _pairwise_direct(xq, xb, metric, dtype):
    """L1 / Linf by broadcast, python/metalfaiss/indexflat.py:96,99 and
    python/metalfaiss/distances.py:305-316."""
    out = np.empty((xq.shape[0], xb.shape[0]), dtype)
    step = max(1, int(2**24 // max(1, xb.shape[0] * xb.shape[1])))
    for s in range(0, xq.shape[0], step):
        a = np.abs(xq[s:s + step, None, :].astype(dtype) - xb[None, :, :].astype(dtype))
        out[s:s + step] = a.sum(axis=2, dtype=dtype) if metric == L1 else a.max(axis=2)
    return out


# --------------------------------------------------------------------- top-k
def topk_ascending(d: np.ndarray, k: int):
    """mlx_topk(largest=False), python/metalfaiss/utils/sorting.py:39-87, with a
    stable order for ties. Returns (values, positions) with k clipped."""
    kk = min(k, d.shape[1])
    order = np.argsort(d, axis=1, kind="stable")[:, :kk]
    return np.take_along_axis(d, order, axis=1), order


def flat_search(xq, xb, k, metric=L2, ids=None):
    """FlatIndex.search, python/metalfaiss/indexflat.py:70-110 (fp32 distances,
    ascending top-k, id map :109)."""
    d = pairwise_f32(xq, xb, metric)
    vals, pos = topk_ascending(d, k)
    labels = pos.astype(np.int64) if ids is None else np.asarray(ids, np.int64)[pos]
    return vals.astype(np.float32), labels


# ----------------------------------------------------------------------- IVF
def coarse_probes(xq, centroids, nprobe, metric=L2):
    """Coarse step of IVFFlatIndex.search: quantizer.search(xs, nprobe),
    python/metalfaiss/index/ivf_flat_index.py:113 → python/metalfaiss/index/flat_index.py:87-93
    (k clipped to ntotal, pairwise_L2sqr, ascending)."""
    _, pos = flat_search(xq, centroids, min(nprobe, len(centroids)), metric)
    return pos


def ivf_build(x, labels, nlist, ids=None):
    """Inverted lists as CSR: rows grouped by list, input order kept inside a
    list. Restates the append loop of IVFFlatIndex.add,
    python/metalfaiss/index/ivf_flat_index.py:89-91 (ids default to the running
    row count, not the batch index: the reference's :91 restarts at 0 per batch)."""
    x = np.asarray(x, np.float32)
    labels = np.asarray(labels, np.int64)
    ids = np.arange(len(x), dtype=np.int64) if ids is None else np.asarray(ids, np.int64)
    order = np.argsort(labels, kind="stable")
    counts = np.bincount(labels, minlength=nlist)
    offsets = np.zeros(nlist + 1, np.int64)
    np.cumsum(counts, out=offsets[1:])
    return offsets, x[order], ids[order]


def ivf_search(xq, centroids, offsets, vecs, ids, nprobe, k, metric=L2, probes=None):
    """IVFFlatIndex.search with the reference's intended semantics,
    python/metalfaiss/index/ivf_flat_index.py:95-151: coarse top-nprobe (:113),
    gather the probed lists in probe order (:118-126), exact top-k over the
    union (ivf_list_topk_l2, python/metalfaiss/faissmlx/kernels/ivf_kernels.py:43-111:
    direct sum of squared differences, ascending), ids through the id table
    (:107-110). Slots beyond the candidates are (+inf, -1); the reference pads
    (+inf, 0) (:128-132) and caps k at 32 (:265)."""
    xq = np.asarray(xq, np.float32)
    if probes is None:
        probes = coarse_probes(xq, centroids, nprobe,
                               INNER_PRODUCT if metric == INNER_PRODUCT else L2)
    nq = xq.shape[0]
    D = np.full((nq, k), np.inf, np.float32)
    I = np.full((nq, k), -1, np.int64)
    for q in range(nq):
        rows = [np.arange(offsets[l], offsets[l + 1]) for l in probes[q] if l >= 0]
        if not rows:
            continue
        rows = np.concatenate(rows)
        if rows.size == 0:
            continue
        X = vecs[rows]
        if metric == L2:
            diff = X - xq[q][None, :]
            dist = np.einsum("nd,nd->n", diff, diff, dtype=np.float32)
        else:
            dist = pairwise_f32(xq[q:q + 1], X, metric)[0]
        kk = min(k, rows.size)
        order = np.argsort(dist, kind="stable")[:kk]
        D[q, :kk] = dist[order]
        I[q, :kk] = ids[rows[order]]
    return D, I


# ------------------------------------------------------------------- k-means
def kmeans_assign(x, centroids):
    """argmin_j ||x - c_j||^2, python/metalfaiss/clustering/any_clustering.py:105-106
    (fp64 here; ties to the lowest j like mx.argmin)."""
    d = pairwise_exact(x, centroids, L2)
    lab = np.argmin(d, axis=1)
    return lab.astype(np.int64), d[np.arange(len(x)), lab]


def kmeans_update(x, labels, centroids):
    """Masked mean per cluster; an empty cluster keeps its old centroid,
    python/metalfaiss/clustering/any_clustering.py:109-120 (fp64 sums)."""
    x = np.asarray(x, np.float64)
    k = centroids.shape[0]
    sums = np.zeros((k, x.shape[1]), np.float64)
    np.add.at(sums, labels, x)
    counts = np.bincount(labels, minlength=k)
    out = np.array(centroids, np.float32, copy=True)
    nz = counts > 0
    out[nz] = (sums[nz] / counts[nz, None]).astype(np.float32)
    return out, counts.astype(np.int64)


def kmeans_init(x, k, seed):
    """Initial centroids: k distinct rows from a seeded permutation,
    python/metalfaiss/index/ivf_pq_index.py:63 (numpy PCG64 replaces MLX's PRNG)."""
    perm = np.random.Generator(np.random.PCG64(seed)).permutation(len(x))[:k]
    return np.asarray(x, np.float32)[perm]


def kmeans_train(x, k, niter, seed, init=None):
    """Lloyd iterations with a fixed count and no early stop,
    python/metalfaiss/index/ivf_pq_index.py:59-78 and
    python/metalfaiss/clustering/any_clustering.py:100-122."""
    c = kmeans_init(x, k, seed) if init is None else np.array(init, np.float32)
    for _ in range(niter):
        lab, _ = kmeans_assign(x, c)
        c, _ = kmeans_update(x, lab, c)
    return c


# -------------------------------------------------------------- range search
def range_search(xq, xb, radius, metric=L2, ids=None):
    """Exact range search: every row with distance <= radius, in row order,
    with lims of length nq+1. The reference (python/metalfaiss/index.py:90-130)
    filters a kNN with k = min(100, ntotal) (:104), so it misses rows past the
    100th; this restatement does not cap."""
    d = pairwise_f32(xq, xb, metric)
    mask = d <= np.float32(radius)
    lims = np.zeros(len(xq) + 1, np.int64)
    np.cumsum(mask.sum(axis=1), out=lims[1:])
    qi, ri = np.nonzero(mask)
    labels = ri.astype(np.int64) if ids is None else np.asarray(ids, np.int64)[ri]
    return lims, d[qi, ri].astype(np.float32), labels


def range_search_capped(xq, xb, radius, metric=L2, ids=None):
    """The reference's own range_search: kNN with k=min(100, ntotal), keep
    distance <= radius, python/metalfaiss/index.py:100-130."""
    k = min(100, len(xb))
    D, I = flat_search(xq, xb, k, metric, ids)
    lims = [0]
    ds, ls = [], []
    for q in range(len(xq)):
        m = D[q] <= np.float32(radius)
        ds.append(D[q][m])
        ls.append(I[q][m])
        lims.append(lims[-1] + int(m.sum()))
    return (np.array(lims, np.int64), np.concatenate(ds) if ds else np.zeros(0, np.float32),
            np.concatenate(ls) if ls else np.zeros(0, np.int64))


def ivf_range_search(xq, centroids, offsets, vecs, ids, nprobe, radius, metric=L2):
    """Range search restricted to the probed lists, in probe order then row order."""
    xq = np.asarray(xq, np.float32)
    probes = coarse_probes(xq, centroids, nprobe,
                           INNER_PRODUCT if metric == INNER_PRODUCT else L2)
    lims = [0]
    ds, ls = [], []
    for q in range(len(xq)):
        for l in probes[q]:
            rows = np.arange(offsets[l], offsets[l + 1])
            if rows.size == 0:
                continue
            dist = pairwise_f32(xq[q:q + 1], vecs[rows], metric)[0]
            m = dist <= np.float32(radius)
            ds.append(dist[m])
            ls.append(ids[rows[m]])
        lims.append(sum(len(a) for a in ds))
    return (np.array(lims, np.int64), np.concatenate(ds).astype(np.float32) if ds else np.zeros(0, np.float32),
            np.concatenate(ls).astype(np.int64) if ls else np.zeros(0, np.int64))


# ------------------------------------------------------------ binary (Hamming)
def hamming_distances(xq01, xb01) -> np.ndarray:
    """Number of coordinates where a query and a row differ, the distance
    BinaryFlatIndex.search accumulates (python/metalfaiss/index/binary_flat_index.py:79-86)."""
    xq01 = np.asarray(xq01, np.uint8)
    xb01 = np.asarray(xb01, np.uint8)
    out = np.empty((xq01.shape[0], xb01.shape[0]), np.int32)
    for s in range(0, xq01.shape[0], 16):
        out[s:s + 16] = (xq01[s:s + 16, None, :] != xb01[None, :, :]).sum(axis=2)
    return out


def hamming_search(xq01, xb01, k, ids=None):
    """BinaryFlatIndex.search: ascending distances, k clipped to ntotal (:88-92),
    ties to the lower row (a stable sort)."""
    d = hamming_distances(xq01, xb01)
    kk = min(k, d.shape[1])
    order = np.argsort(d, axis=1, kind="stable")[:, :kk]
    labels = order.astype(np.int64) if ids is None else np.asarray(ids, np.int64)[order]
    return np.take_along_axis(d, order, axis=1), labels


def pack01_words(x01) -> np.ndarray:
    """(n, d) 0/1 rows → (n, ceil(d / 64)) uint64 words, zero padding bits.
    The bit order within a word is fixed, so Hamming distances between rows
    packed alike are those of the 0/1 rows."""
    b = np.packbits(np.asarray(x01, np.uint8), axis=1, bitorder="little")
    pad = (-b.shape[1]) % 8
    if pad:
        b = np.concatenate([b, np.zeros((b.shape[0], pad), np.uint8)], axis=1)
    return np.ascontiguousarray(b).view(np.uint64)


def hamming_search_packed(xq_words, xb_words, k):
    """hamming_search over pack01_words rows: per query the popcount of
    q XOR x summed over the words, then the k smallest with ties to the lower
    row (the stable order of hamming_search), without its (n, d) temporaries."""
    xq_words = np.asarray(xq_words, np.uint64)
    xb_words = np.asarray(xb_words, np.uint64)
    n = len(xb_words)
    kk = min(k, n)
    D = np.empty((len(xq_words), kk), np.int32)
    I = np.empty((len(xq_words), kk), np.int64)
    for i, q in enumerate(xq_words):
        d = np.bitwise_count(xb_words ^ q).sum(axis=1, dtype=np.int32)
        kth = np.partition(d, kk - 1)[kk - 1] if kk < n else d.max()
        cand = np.flatnonzero(d <= kth)  # ascending rows
        order = cand[np.argsort(d[cand], kind="stable")[:kk]]
        D[i], I[i] = d[order], order
    return D, I


def hamming_range(xq01, xb01, radius, ids=None):
    """Rows within Hamming distance <= radius, in row order, with lims
    (python/metalfaiss/index/binary_flat_index.py:94-150)."""
    d = hamming_distances(xq01, xb01)
    mask = d <= radius
    lims = np.zeros(len(d) + 1, np.int64)
    np.cumsum(mask.sum(axis=1), out=lims[1:])
    qi, ri = np.nonzero(mask)
    labels = ri.astype(np.int64) if ids is None else np.asarray(ids, np.int64)[ri]
    return lims, d[qi, ri], labels


def hamming_ivf_search(xq01, centroids01, list_rows01, list_ids, nprobe, k):
    """BinaryIVFIndex.search, python/metalfaiss/index/binary_ivf_index.py:113-185:
    the nprobe Hamming-nearest centroids (hamming_search over them), then the
    probed lists' rows concatenated in probe order (each list in insertion
    order) and ranked by Hamming distance, ties to the earlier candidate (a
    stable sort). Missing slots: distance inf, label -1 (the reference pads
    with label 0, :163-171). list_rows01[l] is list l's (n_l, d) 0/1 array."""
    xq01 = np.asarray(xq01, np.uint8)
    P = min(int(nprobe), len(centroids01))
    _, probes = hamming_search(xq01, centroids01, P)
    D = np.full((len(xq01), k), np.inf, np.float32)
    I = np.full((len(xq01), k), -1, np.int64)
    for i in range(len(xq01)):
        rows = [list_rows01[l] for l in probes[i] if len(list_rows01[l])]
        if not rows:
            continue
        cand = np.concatenate(rows)
        cid = np.concatenate([np.asarray(list_ids[l], np.int64) for l in probes[i]
                              if len(list_rows01[l])])
        dist = hamming_distances(xq01[i:i + 1], cand)[0]
        order = np.argsort(dist, kind="stable")[:k]
        D[i, :len(order)] = dist[order]
        I[i, :len(order)] = cid[order]
    return D, I, probes


# ------------------------------------------------------------------ IVFPQ
def pq_encode(x, pq_centroids):
    """ProductQuantizer.compute_codes (python/metalfaiss/index/product_quantizer.py):
    per sub-space the nearest centroid (fp64 distances; ties to the lowest code)."""
    x = np.asarray(x, np.float64)
    pq = np.asarray(pq_centroids, np.float64)
    M, ksub, dsub = pq.shape
    codes = np.empty((len(x), M), np.uint8)
    for m in range(M):
        sub = x[:, m * dsub:(m + 1) * dsub]
        d = ((sub[:, None, :] - pq[m][None, :, :]) ** 2).sum(axis=2)
        codes[:, m] = np.argmin(d, axis=1)
    return codes


def pq_adc_table(qres, pq_centroids):
    """IVFPQIndex._adc_lut, python/metalfaiss/index/ivf_pq_index.py:115-125:
    LUT[m][j] = |pq[m][j] - qres_m|^2, fp32."""
    pq = np.asarray(pq_centroids, np.float32)
    M, ksub, dsub = pq.shape
    q = np.asarray(qres, np.float32).reshape(M, 1, dsub)
    return np.sum(np.square(pq - q), axis=2, dtype=np.float32)


def ivfpq_search(xq, centroids, pq_centroids, offsets, codes, ids, nprobe, k, probes=None):
    """IVFPQIndex.search, python/metalfaiss/index/ivf_pq_index.py:127-186: coarse
    top-nprobe, per probed list the ADC scores sum_m LUT[m][code_m] (fp32, in m
    order), candidates in probe order, stable ascending top-k. Missing slots
    are (+inf, -1) (the reference pads label 0)."""
    xq = np.asarray(xq, np.float32)
    centroids = np.asarray(centroids, np.float32)
    if probes is None:
        probes = coarse_probes(xq, centroids, nprobe)
    codes = np.asarray(codes)
    M = codes.shape[1]
    D = np.full((len(xq), k), np.inf, np.float32)
    I = np.full((len(xq), k), -1, np.int64)
    for q in range(len(xq)):
        vals, labs = [], []
        for l in probes[q]:
            if l < 0:
                continue
            rows = np.arange(offsets[l], offsets[l + 1])
            if rows.size == 0:
                continue
            lut = pq_adc_table(xq[q] - centroids[l], pq_centroids)
            s = np.zeros(rows.size, np.float32)
            for m in range(M):
                s = s + lut[m][codes[rows, m]]
            vals.append(s)
            labs.append(np.asarray(ids)[rows])
        if not vals:
            continue
        v = np.concatenate(vals)
        lb = np.concatenate(labs)
        kk = min(k, v.size)
        order = np.argsort(v, kind="stable")[:kk]
        D[q, :kk] = v[order]
        I[q, :kk] = lb[order]
    return D, I
