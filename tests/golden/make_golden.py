"""Generates the golden vectors in tests/golden/*.npz by running the
reference's own code (MetalFaiss, read from the reference tree) in this
container.

MLX cannot be installed here, so mlx_numpy_shim.py stands in for `mlx.core`
(numpy arithmetic, stable argsort, numpy PCG64 random numbers) and the Metal
kernel strings run through their C++ build (oracle/ref_msl). Reference modules
are loaded one by one, without executing the package __init__ (which imports
subsystems outside the search path).

Workarounds applied to reference objects, each needed to reach the code under
test and none altering its arithmetic:
  * IVFFlatIndex: `metric_type` is set on the instance (its search reads a
    missing attribute, python/metalfaiss/index/ivf_flat_index.py:138), `is_trained`
    is set (train never sets the attribute that search checks, :72,105), and the
    inverted lists are filled directly with (id, vector) tuples (its add fails,
    :89-90); the lists hold the same rows its add would append.
  * Index.range_search runs on a minimal concrete subclass of the abstract
    Index (python/metalfaiss/index.py:22) whose search is the exported FlatIndex.

Run:  python tests/golden/make_golden.py   (needs the reference tree)
"""
from __future__ import annotations

import importlib
import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
# The reference checkout: METALFAISS_REFERENCE, else its default location.
REF = Path(os.environ.get("METALFAISS_REFERENCE", "/root/reference")) / "python/metalfaiss"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

import mlx_numpy_shim as mxs  # noqa: E402

mxs.install()
os.environ["METALFAISS_ALLOW_CPU"] = "1"


def load_reference():
    """Registers empty package shells so submodules import without their __init__."""
    for pkg, sub in [("metalfaiss", ""), ("metalfaiss.utils", "utils"),
                     ("metalfaiss.types", "types"), ("metalfaiss.index", "index"),
                     ("metalfaiss.faissmlx", "faissmlx"),
                     ("metalfaiss.faissmlx.kernels", "faissmlx/kernels")]:
        m = types.ModuleType(pkg)
        m.__path__ = [str(REF / sub)] if sub else [str(REF)]
        sys.modules[pkg] = m
    mods = {}
    for name in ["metalfaiss.metric_type", "metalfaiss.types.metric_type",
                 "metalfaiss.utils.search_result", "metalfaiss.utils.sorting",
                 "metalfaiss.distances", "metalfaiss.indexflat",
                 "metalfaiss.index.base_index", "metalfaiss.index.flat_index",
                 "metalfaiss.faissmlx.kernels.ivf_kernels", "metalfaiss.index.ivf_flat_index"]:
        try:
            mods[name] = importlib.import_module(name)
        except Exception as e:  # pragma: no cover - reported, the case is skipped
            print(f"[golden] cannot import {name}: {type(e).__name__}: {e}")
    # python/metalfaiss/index.py is shadowed by the python/metalfaiss/index/ package;
    # load the file itself (it holds the only range_search, :90-130).
    spec = importlib.util.spec_from_file_location("metalfaiss._index_py", REF / "index.py")
    mod = importlib.util.module_from_spec(spec)
    mod.__package__ = "metalfaiss"
    sys.modules["metalfaiss._index_py"] = mod
    spec.loader.exec_module(mod)
    mods["metalfaiss._index_py"] = mod
    return mods


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def np_(a):
    return np.asarray(a)


def gen_pairwise(m, out):
    dist = m["metalfaiss.distances"]
    for tag, (nq, nb, d, seed) in {"a": (10, 20, 5, 1), "b": (16, 300, 64, 2)}.items():
        xq = rng(seed).standard_normal((nq, d), dtype=np.float32)
        xb = rng(seed + 100).standard_normal((nb, d), dtype=np.float32)
        out[f"pairwise_{tag}_xq"] = xq
        out[f"pairwise_{tag}_xb"] = xb
        out[f"pairwise_{tag}_l2"] = np_(dist.pairwise_L2sqr(mxs.array(xq), mxs.array(xb)))
        out[f"pairwise_{tag}_l1"] = np_(dist.pairwise_L1(mxs.array(xq), mxs.array(xb)))
        out[f"pairwise_{tag}_linf"] = np_(dist.pairwise_Linf(mxs.array(xq), mxs.array(xb)))


def gen_flat(m, out):
    flat = m["metalfaiss.indexflat"]
    MT = m["metalfaiss.metric_type"].MetricType
    cases = []
    for mi, metric in enumerate([MT.L2, MT.INNER_PRODUCT, MT.L1, MT.LINF]):
        for (n, d, nq, k, seed) in [(500, 16, 8, 10, 3), (1024, 32, 12, 32, 4), (60, 8, 5, 100, 5)]:
            xb = rng(seed + 10 * mi).standard_normal((n, d), dtype=np.float32)
            xq = rng(seed + 10 * mi + 1).standard_normal((nq, d), dtype=np.float32)
            idx = flat.FlatIndex(d, metric)
            ids = None
            if seed == 4:
                ids = (np.arange(n, dtype=np.int64) * 7 + (1 << 33)).tolist()
            idx.add(xb, ids)
            res = idx.search(xq, k)
            tag = f"flat_{metric.name}_{n}_{d}_{k}"
            out[tag + "_xb"] = xb
            out[tag + "_xq"] = xq
            out[tag + "_ids"] = np.asarray(ids if ids is not None else np.arange(n), np.int64)
            out[tag + "_D"] = np_(res.distances).astype(np.float32)
            out[tag + "_I"] = np_(res.indices).astype(np.int64)
            out[tag + "_meta"] = np.array([int(metric.value), k], np.int64)
            cases.append(tag)
    out["flat_cases"] = np.array(cases)


def mixture(n, d, nc, seed, centres=None):
    g = rng(seed)
    if centres is None:
        centres = (rng(seed + 7919).standard_normal((nc, d), dtype=np.float32) * 2.0)
    comp = g.integers(0, nc, size=n)
    return (centres[comp] + g.standard_normal((n, d), dtype=np.float32)).astype(np.float32), centres


def gen_ivf(m, out):
    ivfk = m["metalfaiss.faissmlx.kernels.ivf_kernels"]
    ivfm = m["metalfaiss.index.ivf_flat_index"]
    fi = m["metalfaiss.index.flat_index"]
    TMT = m["metalfaiss.types.metric_type"].MetricType
    cases = []
    for (n, d, nlist, nq, nprobe, k, seed) in [(2500, 32, 32, 10, 4, 10, 6), (2000, 48, 24, 8, 1, 32, 7),
                                               (2500, 16, 40, 12, 8, 5, 8)]:
        x, centres = mixture(n, d, nlist, seed)
        cents = x[rng(seed + 1).permutation(n)[:nlist]].copy()
        # list assignment with the reference quantizer (FlatIndex.search k=1)
        q = fi.FlatIndex(d)
        q.add(cents)
        _, lab = q.search(x, 1)
        lab = np_(lab)[:, 0].astype(np.int64)
        index = ivfm.IVFFlatIndex(q, d, nlist)
        index.metric_type = TMT.L2
        index.is_trained = True
        for i in range(n):
            index._invlists[int(lab[i])].append((i, mxs.array(x[i])))
        index.nprobe = nprobe
        xq, _ = mixture(nq, d, nlist, seed + 2, centres)
        res = index.search(xq, k)
        tag = f"ivf_{n}_{d}_{nlist}_{nprobe}_{k}"
        out[tag + "_x"] = x
        out[tag + "_cents"] = cents
        out[tag + "_labels"] = lab
        out[tag + "_xq"] = xq
        out[tag + "_D"] = np_(res.distances).astype(np.float32)
        out[tag + "_I"] = np_(res.indices).astype(np.int64)
        out[tag + "_meta"] = np.array([nlist, nprobe, k], np.int64)
        cases.append(tag)
    out["ivf_cases"] = np.array(cases)
    # the kernel and its chunked device merge on one gathered candidate set
    X = rng(9).standard_normal((700, 32), dtype=np.float32)
    ids = (np.arange(700) * 3 + 11).astype(np.int32)
    Q = rng(10).standard_normal(32, dtype=np.float32)
    for k in (1, 10, 32):
        v, i = ivfk.ivf_list_topk_l2(mxs.array(Q), mxs.array(X), mxs.array(ids), k)
        out[f"kernel_k{k}_D"] = np_(v)
        out[f"kernel_k{k}_I"] = np_(i).astype(np.int64)
        v, i = ivfk.ivf_list_topk_l2_chunked_device_merge(mxs.array(Q), mxs.array(X), mxs.array(ids), k,
                                                           rows_per_chunk=128)
        out[f"kernel_chunked_k{k}_D"] = np_(v)
        out[f"kernel_chunked_k{k}_I"] = np_(i).astype(np.int64)
    out["kernel_X"], out["kernel_ids"], out["kernel_Q"] = X, ids, Q


def gen_range(m, out):
    Index = m["metalfaiss._index_py"].Index
    flat = m["metalfaiss.indexflat"]
    MT = m["metalfaiss.metric_type"].MetricType

    class FlatRange(Index):
        def __init__(self, d):
            self._f = flat.FlatIndex(d, MT.L2)
            self.d = d

        @property
        def ntotal(self):
            return self._f.ntotal

        def add(self, xs):
            self._f.add(xs)

        def search(self, xs, k):
            return self._f.search(xs, k)

        def reset(self):
            self._f.reset()

    for tag, (n, d, nq, seed) in {"small": (80, 8, 6, 12), "capped": (1500, 4, 5, 13)}.items():
        xb = rng(seed).standard_normal((n, d), dtype=np.float32)
        xq = rng(seed + 1).standard_normal((nq, d), dtype=np.float32)
        r = FlatRange(d)
        r.add(xb)
        dsort = np.sort(((xq[:, None] - xb[None]) ** 2).sum(-1), 1)
        # The reference's SearchRangeResult rejects a query with no hit (its lims
        # length check, python/metalfaiss/utils/search_result.py:61-62, counts only
        # non-empty per-query arrays), so every query gets at least one.
        radius = float(max(np.median(dsort[:, 9]), dsort[:, 0].max() * 1.01))
        if tag == "capped":
            radius *= 6.0  # more than 100 hits per query: the reference's cap shows
        res = r.range_search(xq, radius)
        lims = np_(res.lims).astype(np.int64)
        D = np.concatenate([np_(a) for a in res.distances]) if res.distances else np.zeros(0, np.float32)
        I = np.concatenate([np_(a) for a in res.indices]) if res.indices else np.zeros(0, np.int64)
        out[f"range_{tag}_xb"], out[f"range_{tag}_xq"] = xb, xq
        out[f"range_{tag}_radius"] = np.float32(radius)
        out[f"range_{tag}_lims"], out[f"range_{tag}_D"], out[f"range_{tag}_I"] = lims, D, I.astype(np.int64)


def gen_kmeans(m, out):
    # IVFPQIndex._kmeans, python/metalfaiss/index/ivf_pq_index.py:59-78, needs the
    # product-quantizer modules to import; the k-means step itself is restated
    # there with the same ops as AnyClustering (any_clustering.py:105-120), so the
    # golden k-means runs those ops through the shim here verbatim-by-behaviour:
    import mlx.core as mx  # the shim

    x, _ = mixture(3000, 16, 12, 14)
    k, iters = 12, 6
    mx.random.seed(1234)
    try:
        ivfpq = importlib.import_module("metalfaiss.index.ivf_pq_index")
        mx.random.log.clear()
        cent = ivfpq.IVFPQIndex._kmeans(None, mx.array(x), k, iters)
        perm = mx.random.log[0][1][:k]
        out["kmeans_source"] = np.array("IVFPQIndex._kmeans")
    except Exception as e:  # pragma: no cover
        print(f"[golden] IVFPQIndex._kmeans unavailable ({type(e).__name__}: {e})")
        return
    out["kmeans_x"] = x
    out["kmeans_perm"] = np.asarray(perm, np.int64)
    out["kmeans_iters"] = np.int64(iters)
    out["kmeans_centroids"] = np_(cent).astype(np.float32)


def gen_binary(m, out):
    """BinaryFlatIndex search / reconstruct, python/metalfaiss/index/binary_flat_index.py:27-165.
    The class declares no _add/_train/_search/_reconstruct, which its abstract
    base requires, and assigns the base's read-only ntotal, so it cannot be
    instantiated as written; a subclass supplies those members and leaves the
    class's own add, search and reconstruct in charge. (Its range_search builds
    a SearchRangeResult its own validation rejects; range search is restated
    in the oracle.)"""
    import importlib

    b = importlib.import_module("metalfaiss.index.binary_flat_index")
    noop = lambda self, *a, **k: None  # noqa: E731
    Concrete = type("BinaryFlatConcrete", (b.BinaryFlatIndex,), {
        "_add": noop, "_train": noop, "_search": noop, "_reconstruct": noop,
        "ntotal": property(lambda s: s._ntotal, lambda s, v: setattr(s, "_ntotal", v))})
    cases = []
    for (n, d, nq, k, seed) in [(300, 64, 12, 10, 40), (1000, 256, 9, 32, 41), (50, 8, 5, 60, 42)]:
        x = rng(seed).integers(0, 2, size=(n, d)).astype(np.uint8)
        q = rng(seed + 1).integers(0, 2, size=(nq, d)).astype(np.uint8)
        q[:2] = x[[3, n - 1]]  # two self-queries
        idx = Concrete(d)
        idx.add(mxs.array(x))
        D, I = idx.search(mxs.array(q), k)
        tag = f"binary_{n}_{d}_{k}"
        out[tag + "_xb"] = x
        out[tag + "_xq"] = q
        out[tag + "_D"] = np_(D).astype(np.int32)
        out[tag + "_I"] = np_(I).astype(np.int64)
        out[tag + "_rec"] = np_(idx.reconstruct(5)).astype(np.uint8)
        cases.append(tag)
    out["binary_cases"] = np.array(cases)


def gen_binary_ivf(m, out):
    """BinaryIVFIndex train / add / search, python/metalfaiss/index/binary_ivf_index.py:84-185,
    over a quantizer (the BinaryFlatIndex subclass of gen_binary) that holds
    the centroids: the reference's train() trains the quantizer, which stores
    nothing, so the centroids are added to it first. Ids are passed as a list
    (its `ids[i] if ids else i` tests the container's truth), and vectors as
    nested lists (its _validate_binary tests their truth, binary_index.py:221);
    the quantizer's search turns those lists into arrays, which the IVF's
    _add and _search hand it as they are (binary_flat_index.py:67 reads .shape),
    and wraps its (distances, indices) tuple in the SearchResult whose .labels
    they read (binary_ivf_index.py:115,138)."""
    import importlib

    b = importlib.import_module("metalfaiss.index.binary_flat_index")
    ivf = importlib.import_module("metalfaiss.index.binary_ivf_index")
    sr = importlib.import_module("metalfaiss.utils.search_result")
    noop = lambda self, *a, **k: None  # noqa: E731
    as_arr = lambda xs: mxs.array(np.asarray(xs, np.uint8)) if isinstance(xs, list) else xs  # noqa: E731
    Concrete = type("BinaryFlatConcrete", (b.BinaryFlatIndex,), {
        "_add": noop, "_train": noop, "_search": noop, "_reconstruct": noop,
        "ntotal": property(lambda s: s._ntotal, lambda s, v: setattr(s, "_ntotal", v)),
        "search": lambda s, xs, k: sr.SearchResult(*b.BinaryFlatIndex.search(s, as_arr(xs), k))})
    cases = []
    for (n, d, nlist, nq, k, nprobe, seed) in [(400, 64, 8, 10, 10, 2, 50),
                                               (600, 128, 12, 8, 40, 3, 51),
                                               (200, 72, 6, 6, 90, 1, 52)]:
        x = rng(seed).integers(0, 2, size=(n, d)).astype(np.uint8)
        q = rng(seed + 1).integers(0, 2, size=(nq, d)).astype(np.uint8)
        q[:2] = x[[3, n - 1]]
        cents = x[rng(seed + 2).choice(n, nlist, replace=False)]
        quant = Concrete(d)
        quant.add(mxs.array(cents))
        idx = ivf.BinaryIVFIndex(quant, d, nlist)
        idx.train(x.tolist())
        ids = [int(7 * i + 5) for i in range(n)]
        idx.add(x.tolist(), ids)
        idx.nprobe = nprobe
        res = idx.search(q.tolist(), k)
        D, I = res.distances, res.indices
        tag = f"binivf_{n}_{d}_{nlist}_{k}"
        out[tag + "_xb"] = x
        out[tag + "_xq"] = q
        out[tag + "_cents"] = cents
        out[tag + "_ids"] = np.asarray(ids, np.int64)
        out[tag + "_nprobe"] = np.int64(nprobe)
        out[tag + "_D"] = np_(D).astype(np.float32)
        out[tag + "_I"] = np_(I).astype(np.int64)
        cases.append(tag)
    out["binivf_cases"] = np.array(cases)


def gen_ivfpq(m, out):
    """IVFPQIndex add / search, python/metalfaiss/index/ivf_pq_index.py:101-186,
    on installed coarse centroids and PQ codebooks. Its train draws MLX random
    permutations (:62, product_quantizer.py:57), which the shim does not
    reproduce, so the centroids are seeded rows of the data and each subspace's
    256 codewords seeded rows of the residuals, installed where train leaves
    them (_centroids, pq.centroids, is_trained). add then assigns, encodes and
    files the rows as written, and search probes and scores them through its
    ADC tables. Every query's probed lists hold at least k rows (its search
    stacks one row of k per query). Saved beside D and I: each row's list and
    codes as add filed them, and the probes its search takes (the same shim
    operations, :149-150)."""
    import mlx.core as mx  # the shim

    try:
        ivfpq = importlib.import_module("metalfaiss.index.ivf_pq_index")
    except Exception as e:  # pragma: no cover
        print(f"[golden] IVFPQIndex unavailable ({type(e).__name__}: {e})")
        return
    cases = []
    for (n, d, nlist, M, nq, k, nprobe, seed) in [(2000, 32, 8, 4, 9, 10, 2, 60),
                                                  (3000, 64, 16, 8, 7, 20, 3, 61),
                                                  (1500, 16, 6, 16, 5, 5, 1, 62)]:
        x, cen = mixture(n, d, nlist, seed)
        q, _ = mixture(nq, d, nlist, seed + 1, centres=cen)
        g = rng(seed + 2)
        cents = x[g.choice(n, nlist, replace=False)].copy()
        lab0 = np.argmin(((x[:, None, :] - cents[None, :, :]) ** 2).sum(2), axis=1)
        res0 = x - cents[lab0]
        dsub = d // M
        pick = g.choice(n, 256, replace=False)
        pqc = np.stack([res0[pick, j * dsub:(j + 1) * dsub] for j in range(M)]).astype(np.float32)
        idx = ivfpq.IVFPQIndex(d, nlist, M)
        idx._centroids = mx.array(cents)
        idx._pq.centroids = mx.array(pqc)
        idx.is_trained = True
        ids = [int(3 * i + 1) for i in range(n)]
        idx.add(x.tolist(), ids)
        idx.nprobe = nprobe
        try:
            r = idx.search(q.tolist(), k)
        except Exception as e:  # pragma: no cover
            print(f"[golden] IVFPQ case {n}/{d}: search failed ({type(e).__name__}: {e})")
            continue
        codes = np.zeros((n, M), np.uint8)
        labels = np.zeros(n, np.int64)
        for lid, lst in enumerate(idx._codes):
            for vid, c in lst:
                row = (vid - 1) // 3
                codes[row] = np_(c).astype(np.uint8)
                labels[row] = lid
        cm = mx.array(cents)
        probes = np.stack([np_(mx.argsort(mx.sum(mx.square(mx.subtract(cm, mx.array(qq)[None, :])),
                                                 axis=1))[:nprobe]) for qq in q]).astype(np.int64)
        tag = f"ivfpq_{n}_{d}_{M}_{k}"
        out[tag + "_xb"] = x
        out[tag + "_xq"] = q
        out[tag + "_cents"] = cents
        out[tag + "_pqc"] = pqc
        out[tag + "_ids"] = np.asarray(ids, np.int64)
        out[tag + "_nprobe"] = np.int64(nprobe)
        out[tag + "_probes"] = probes
        out[tag + "_codes"] = codes
        out[tag + "_labels"] = labels
        out[tag + "_D"] = np_(r.distances).astype(np.float32)
        out[tag + "_I"] = np_(r.indices).astype(np.int64)
        cases.append(tag)
    out["ivfpq_cases"] = np.array(cases)


def main():
    mods = load_reference()
    out = {}
    gen_pairwise(mods, out)
    gen_flat(mods, out)
    gen_ivf(mods, out)
    gen_range(mods, out)
    gen_kmeans(mods, out)
    gen_binary(mods, out)
    gen_binary_ivf(mods, out)
    gen_ivfpq(mods, out)
    path = HERE / "reference_golden.npz"
    np.savez_compressed(path, **out)
    print(f"[golden] wrote {path} ({path.stat().st_size // 1024} KiB, {len(out)} arrays)")


if __name__ == "__main__":
    main()
