#!/usr/bin/env python
"""Search-path throughput on B200, with the dominant kernel's roofline and a
CPU baseline. One JSON line per run.

Workloads (--config; the default is the headline):
* ivf20m (headline): IVFFlat L2, d=128, N=20M rows from a Gaussian mixture of
  16384 clusters (centres ~ N(0, 4 I), sigma = 1), nlist=16384 trained by
  seeded k-means on a 256*nlist subsample, Q=10000 queries from the same
  mixture, nprobe=32, k=10. One step = one search of the Q-query batch. The
  database (10.2 GB) is far larger than L2 (126 MB), so no flush is needed
  between steps. ivf32k is the small IVF configuration (d=64, N=32768,
  nlist=128, Q=16; --nprobe / --k give its nprobe x k sweep); ivf2m and ivf4m
  are development sizes.
* flat10m: FlatIndex INNER_PRODUCT, 10M unit rows x d=128, Q=10000 unit
  queries, k=100. flat32k: FlatIndex L2, N=32768 x d=64 N(0,1), Q=16, k=10.
  One step = one search of the batch.
* kmeans5m: k-means on 5M points x d=256 from a 4096-cluster mixture, K=4096;
  one step = one Lloyd iteration (assignment + centroid update); the
  configuration runs 20.
* ivfpq10m: IVFPQ L2, d=128, N=10M mixture rows, nlist=4096, M=16 one-byte
  codes, Q=10000, nprobe=32, k=10. binary10m: BinaryFlatIndex, 256-bit
  uniform random rows, N=10M, Q=1000, k=10. ivfpq32k and binary32k are their
  small cases. One step = one search of the batch.

N>1 GPUs (one process per GPU, NCCL; ivf configurations): the inverted lists
are partitioned over the ranks by greedy LPT on list size and each rank adds
only the rows of its own lists, plus a copy of every list's first 128 rows
(the head bank); each rank runs the coarse step and the bound pass (on the
head bank) for its share of the queries, one all-gather shares the probes and
bounds, every rank scans its own lists, and the (Q, k) partial results are
merged after a second all-gather. The database is fixed as N grows (strong
scaling).

--impl reference times the reference algorithm on the host cores and never
loads this library: for ivf configurations the index is built with plain
torch operations (the same data, training sample, initial centroids and Lloyd
iterations as the library's build) and searched by the oracle's C port of the
reference's IVF search (python/metalfaiss/index/ivf_flat_index.py:95-151 with
the list scan of python/metalfaiss/faissmlx/kernels/ivf_kernels.py:21-122)
over a bounded sample of queries; flat and k-means configurations run the
numpy restatement of the reference (python/metalfaiss/indexflat.py:70-110,
python/metalfaiss/clustering/any_clustering.py:62-124) on a sample.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # The headline workload: IVFFlat L2 at d=128, N=20M, nlist=16384, Q=10000, nprobe=32, k=10.
    "ivf20m": dict(kind="ivf", d=128, n=20_000_000, nlist=16384, nq=10_000, nprobe=32, k=10,
                   niter=10),
    # The small IVF configuration (d=64, N=32768, nlist=128, Q=16).
    "ivf32k": dict(kind="ivf", d=64, n=32768, nlist=128, nq=16, nprobe=8, k=10, niter=10),
    # Mid-size for development runs.
    "ivf2m": dict(kind="ivf", d=128, n=2_000_000, nlist=2048, nq=10_000, nprobe=32, k=10,
                  niter=5),
    # The headline's list count at a fifth of its rows (4 GB on the device with
    # residuals): lists probed by few queries dominate, as at full size; small
    # enough for multi-pass profiler captures.
    "ivf4m": dict(kind="ivf", d=128, n=4_000_000, nlist=16384, nq=10_000, nprobe=32, k=10,
                  niter=5),
    # Flat inner product over 10M unit rows, k=100.
    "flat10m": dict(kind="flat", metric=0, d=128, n=10_000_000, nq=10_000, k=100, data="unit"),
    # The small flat L2 configuration (N(0,1) rows).
    "flat32k": dict(kind="flat", metric=1, d=64, n=32768, nq=16, k=10, data="gaussian"),
    # k-means assignment + update, 5M x d=256, K=4096 (20 iterations).
    "kmeans5m": dict(kind="kmeans", d=256, n=5_000_000, K=4096, niter=20),
    # Small cases of the two GEMM-shaped configurations, for multi-pass
    # profiler captures (a few GB on the device, inputs still past L2).
    "flat1m": dict(kind="flat", metric=0, d=128, n=1_000_000, nq=10_000, k=100, data="unit"),
    "kmeans500k": dict(kind="kmeans", d=256, n=500_000, K=4096, niter=20),
    # IVFPQ L2 (the ADC scan over residual codes): d=128, N=10M rows from a
    # 4096-cluster mixture, nlist=4096, M=16 one-byte codes (16 B per row),
    # Q=10000, nprobe=32, k=10; ivfpq32k is its small case (ivf32k's shapes).
    "ivfpq10m": dict(kind="ivfpq", d=128, n=10_000_000, nlist=4096, M=16, nq=10_000, nprobe=32,
                     k=10, niter=10),
    "ivfpq32k": dict(kind="ivfpq", d=64, n=32768, nlist=128, M=8, nq=16, nprobe=8, k=10,
                     niter=10),
    # BinaryFlatIndex (Hamming): 256-bit rows, N=10M, Q=1000, k=10;
    # binary32k is its small case.
    "binary10m": dict(kind="binary", d=256, n=10_000_000, nq=1000, k=10),
    "binary32k": dict(kind="binary", d=256, n=32768, nq=16, k=10),
}
METRIC_NAMES = {0: "INNER_PRODUCT", 1: "L2"}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def measured_peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, kind) from MEASURED_PEAKS.json, else the fallback."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def gemm_peak(device, tf32: bool, n=8192, reps=10):
    """Dense fp32 GEMM throughput of cuBLAS on this GPU (TFLOP/s, best of
    `reps` n^3 GEMMs, CUDA events): with tf32 the tensor-core TF32 rate (the
    denominator of the 3xTF32 scans), without it the SIMT fp32 rate (the
    denominator of the fp32 FMA scans)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = tf32
    try:
        a = torch.randn(n, n, device=device)
        b = torch.randn(n, n, device=device)
        c = torch.empty(n, n, device=device)
        for _ in range(3):
            torch.matmul(a, b, out=c)
        best = float("inf")
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            torch.cuda.synchronize(device)
            best = min(best, e0.elapsed_time(e1))
        del a, b, c
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled through NVML every
    few milliseconds during the timed region (reads only)."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))

    def __init__(self, cuda_index: int, period_s: float = 0.005):
        self.cuda_index = int(cuda_index)
        self.period = period_s
        self.samples = []
        self.err = None
        self.handle = None
        self.stop_flag = threading.Event()

    def _handle(self, nv):
        # the NVML device with this CUDA device's PCI address (indices may differ)
        try:
            pr = torch.cuda.get_device_properties(self.cuda_index)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def start(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.handle = self._handle(nv)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.handle, nv.NVML_CLOCK_SM)
            self._sample()
        except Exception as e:  # no NVML: report it, do not fail the run
            self.err = f"NVML unavailable ({type(e).__name__})"
            return
        self.samples = []
        self.t = threading.Thread(target=self._loop, daemon=True)
        self.t.start()

    def _sample(self):
        nv = self.nv
        mhz = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
        try:
            mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        except AttributeError:
            mask = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
        self.samples.append((mhz, mask))

    def _loop(self):
        while not self.stop_flag.is_set():
            try:
                self._sample()
            except Exception:
                pass
            time.sleep(self.period)

    def stop(self):
        if self.err is not None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err], "samples": 0}
        self.stop_flag.set()
        self.t.join(timeout=2)
        if not self.samples:  # a region shorter than one period: the clocks right after it
            self._sample()
        sm = [m for m, _ in self.samples]
        reasons = sorted({nm for _, mask in self.samples for nm, bit in self.REASONS if mask & bit})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sm), "source": f"NVML every {int(self.period * 1000)} ms"}


# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the dominant
# kernel (profiles/). Exact search, the all-probes 3xTF32 launch: ivf2m
# measured (2,228,082,688 + 53,105,408 B); ivf20m not captured at full size:
# the ivf2m bytes per probed row (1,142 B: vector, residual and norm once
# each, plus the query tiles) times the 13,287,418 rows probed per batch.
# Filter search, the fp16 tensor-core launch: ivf4m measured (272,680,960 +
# 4,955,904 B over its 918,849 rows); ivf20m: those 302.2 B per row times its
# 4,620,425 rows.
TRAFFIC = {
    "ivf2m": {"bytes": 2281188096, "source": "ncu, measured"},
    "ivf20m": {"bytes": 15177587741, "source": "ncu ivf2m bytes per probed row x probed rows"},
    "ivf4m/filter": {"bytes": 277636864, "source": "ncu, measured"},
    "ivf20m/filter": {"bytes": 1396094796,
                      "source": "ncu ivf4m bytes per row of the filter pass x its rows"},
}


def _synthetic():
    """metalfaiss_b200/synthetic.py on its own (numpy + torch only): the
    reference arm draws the same data without importing this library."""
    spec = importlib.util.spec_from_file_location(
        "_mf_bench_synthetic", os.path.join(ROOT, "metalfaiss_b200", "synthetic.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def workload_config(name, cfg):
    """The `config` object of the JSON line: the workload alone, the same in
    both arms."""
    if cfg["kind"] == "ivf":
        big = cfg["n"] * cfg["d"] * 4 > 126e6
        return {
            "workload": f"{name}: IVFFlat L2 d={cfg['d']} N={cfg['n']} nlist={cfg['nlist']} "
                        f"Q={cfg['nq']} nprobe={cfg['nprobe']} k={cfg['k']}",
            "d": cfg["d"], "N": cfg["n"], "nlist": cfg["nlist"], "Q": cfg["nq"],
            "nprobe": cfg["nprobe"], "k": cfg["k"],
            "l2": ("database larger than L2 (126 MB); no flush" if big else
                   "database fits in L2 (the configuration's own size); no flush"),
        }
    if cfg["kind"] == "flat":
        big = cfg["n"] * cfg["d"] * 4 > 126e6
        return {
            "workload": f"{name}: FlatIndex {METRIC_NAMES[cfg['metric']]} d={cfg['d']} "
                        f"N={cfg['n']} Q={cfg['nq']} k={cfg['k']}",
            "d": cfg["d"], "N": cfg["n"], "Q": cfg["nq"], "k": cfg["k"],
            "metric_type": METRIC_NAMES[cfg["metric"]],
            "l2": ("database larger than L2 (126 MB); no flush" if big else
                   "database fits in L2 (the configuration's own size); no flush"),
        }
    if cfg["kind"] == "ivfpq":
        code_bytes = cfg["n"] * ((cfg["M"] + 15) // 16 * 16)
        return {
            "workload": f"{name}: IVFPQ L2 d={cfg['d']} N={cfg['n']} nlist={cfg['nlist']} "
                        f"M={cfg['M']} (8-bit codes) Q={cfg['nq']} nprobe={cfg['nprobe']} "
                        f"k={cfg['k']}",
            "d": cfg["d"], "N": cfg["n"], "nlist": cfg["nlist"], "M": cfg["M"], "Q": cfg["nq"],
            "nprobe": cfg["nprobe"], "k": cfg["k"],
            "l2": ("codes larger than L2 (126 MB); no flush" if code_bytes > 126e6 else
                   "codes fit in L2 (the configuration's own size); no flush"),
        }
    if cfg["kind"] == "binary":
        return {
            "workload": f"{name}: BinaryFlatIndex Hamming d={cfg['d']} bits N={cfg['n']} "
                        f"Q={cfg['nq']} k={cfg['k']}",
            "d": cfg["d"], "N": cfg["n"], "Q": cfg["nq"], "k": cfg["k"],
            "l2": ("packed rows larger than L2 (126 MB); no flush"
                   if cfg["n"] * cfg["d"] / 8 > 126e6 else
                   "packed rows fit in L2 (the configuration's own size); no flush"),
        }
    return {
        "workload": f"{name}: k-means L2 N={cfg['n']} d={cfg['d']} K={cfg['K']} "
                    f"({cfg['niter']} Lloyd iterations; one per step)",
        "d": cfg["d"], "N": cfg["n"], "K": cfg["K"], "iterations": cfg["niter"],
        "l2": "points (5.1 GB) larger than L2; no flush",
    }


def metric_name(cfg):
    if cfg["kind"] == "ivf":
        return "IVFFlat queries/sec (list-scan HBM GB/s vs peak in roofline)"
    if cfg["kind"] == "flat":
        return "FlatIndex queries/sec (distance-GEMM tensor fraction in roofline)"
    if cfg["kind"] == "ivfpq":
        return "IVFPQ queries/sec (ADC code-scan bytes in roofline)"
    if cfg["kind"] == "binary":
        return "BinaryFlatIndex queries/sec (Hamming word operations in roofline)"
    return "k-means Lloyd iterations/sec (assignment GEMM tensor fraction in roofline)"


def host_threads():
    return len(os.sched_getaffinity(0))


class Timer:
    """Warm-up, then K steps between CUDA events on the launching stream, with
    a barrier and a synchronize on both sides and clocks sampled meanwhile;
    the max over ranks."""

    def __init__(self, device, world):
        self.device, self.world = device, world

    def run(self, step, steps, warmup):
        import torch.distributed as dist

        from metalfaiss_b200 import _native as nat

        dev = self.device
        for _ in range(warmup):
            step()
        torch.cuda.synchronize(dev)
        if self.world > 1:
            dist.barrier()
        sampler = ClockSampler(dev.index)
        sampler.start()
        launches0 = nat.launch_count()
        stream = torch.cuda.current_stream(dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        if self.world > 1:
            dist.barrier()
        # an NVTX range "timed" marks the timed steps for profilers' filters
        torch.cuda.nvtx.range_push("timed")
        ev0.record(stream)
        for _ in range(steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_pop()
        launches = nat.launch_count() - launches0
        ms = ev0.elapsed_time(ev1)
        clocks = sampler.stop()
        return self.max_over_ranks(ms), clocks, launches

    def max_over_ranks(self, ms):
        if self.world == 1:
            return ms
        import torch.distributed as dist

        t = torch.tensor([ms], device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def kernel_times(self, step, names, steps):
        """Per-kernel CUDA-event totals over a separate run of a few steps
        (the per-launch events stay out of the timed steps)."""
        from metalfaiss_b200 import _native as nat

        nat.timing_reset()
        nat.timing_enable(True)
        for _ in range(steps):
            step()
        torch.cuda.synchronize(self.device)
        nat.timing_enable(False)
        return {n: nat.timing_read(n) for n in names}


def end_to_end(timer, search, xq, k, device, steps):
    """The search end to end through the public API, over `steps` batches of
    the queries from pinned host memory, every batch copied in, searched and
    its (distances, labels) copied back to pinned host memory inside the
    timed region. Returns the total ms of
    * the pipelined run (metalfaiss_b200.pipeline.search_host_batches: batch
      i + 1's copy in and batch i - 1's copy out overlap batch i's search), and
    * the serial run (copy in, search, copy out, one stream),
    each the max over ranks. The pipelined results are checked against the
    device search."""
    from metalfaiss_b200.pipeline import search_host_batches

    xq_host = xq.cpu().pin_memory()
    r0 = search(xq)  # the results' shapes and types
    outs = [(torch.empty(r0.distances.shape, dtype=r0.distances.dtype).pin_memory(),
             torch.empty(r0.labels.shape, dtype=r0.labels.dtype).pin_memory())
            for _ in range(2)]
    del r0

    def serial_step():
        r = search(xq_host.to(device, non_blocking=True))
        outs[0][0].copy_(r.distances, non_blocking=True)
        outs[0][1].copy_(r.labels, non_blocking=True)

    serial_ms, _, _ = timer.run(serial_step, steps, 2)
    for D_h, I_h in outs:
        D_h.fill_(-1)
        I_h.fill_(-2)
    batches = [xq_host] * steps
    batch_outs = [outs[i % 2] for i in range(steps)]
    pipe_ms, _, _ = timer.run(lambda: search_host_batches(search, batches, batch_outs, device),
                              1, 1)
    ref = search(xq)
    torch.cuda.synchronize(device)
    for D_h, I_h in outs:
        if not (torch.equal(I_h, ref.labels.cpu()) and torch.equal(D_h, ref.distances.cpu())):
            raise RuntimeError("pipelined end-to-end results differ from the device search")
    return pipe_ms, serial_ms


def e2e_entry(nq, d, k, steps, pipe_ms, serial_ms, query_bytes=None):
    return {
        "value": round(nq * steps / (pipe_ms * 1e-3), 1),
        "unit": "queries/s",
        "h2d_bytes_per_step": int(nq * (d * 4 if query_bytes is None else query_bytes)),
        "d2h_bytes_per_step": int(nq * k * 12),
        "steps": steps,
        "mode": "pipelined: search_host_batches, each batch copied in from pinned host "
                "memory, searched and copied out, the copies overlapping the next and "
                "previous batches' searches",
        "serial_value": round(nq * steps / (serial_ms * 1e-3), 1),
    }


# ------------------------------------------------------------------- IVF arm
def build_index(cfg, device, seed=1234, rank=0, world=1):
    """The benchmark's IVF index. With world > 1 every rank trains on the same
    subsample (identical centroids), adds only the rows of the lists it owns
    (greedy LPT on the list sizes) and keeps the head bank (the first rows of
    every list, for the bound pass). Returns (index, queries, owners, heads)."""
    from metalfaiss_b200 import IVFFlatIndex, synthetic as syn
    from metalfaiss_b200.clustering import ClusteringParameters

    t0 = time.time()
    x, centres = syn.torch_mixture(cfg["n"], cfg["d"], cfg["nlist"], seed, device)
    params = ClusteringParameters(niter=cfg["niter"], seed=seed, max_points_per_centroid=256)
    idx = IVFFlatIndex(cfg["d"], cfg["nlist"], device=device, clustering=params)
    idx.train(x)
    torch.cuda.synchronize(device)
    t1 = time.time()
    owners = heads = None
    if world > 1:
        from metalfaiss_b200.sharding import add_owned_rows, empty_heads

        heads = empty_heads(idx)
        owners = add_owned_rows(idx, x, rank, world, heads=heads)
    else:
        idx.add(x)
    torch.cuda.synchronize(device)
    t2 = time.time()
    del x
    xq, _ = syn.torch_mixture(cfg["nq"], cfg["d"], cfg["nlist"], seed + 1, device, centres=centres)
    torch.cuda.empty_cache()
    log(f"[bench] built index: train {t1 - t0:.1f}s add {t2 - t1:.1f}s ntotal={idx.ntotal}")
    return idx, xq, owners, heads


# A list probed by at most this many queries is scanned by the few-query
# kernel; the others, in groups of up to 128 queries, by the tensor-core kernel.
SMALL_GROUP = 16


def scan_work(sizes, probes_np, d, k):
    """Work of one IVF scan over the probes (nq, P) of an index with these list sizes:
    * pairs: (query, row) distance evaluations in the tensor-core launch, i.e.
      over the lists probed by more than SMALL_GROUP queries (a list probed by
      at most SMALL_GROUP queries is scanned by the few-query kernel);
    * bytes: what the list-major scan must move once: every probed list's rows
      (vector + norm) read once, the query vectors read once and each
      (query, probe) pair's k partial results written once;
    * rows: distinct probed rows."""
    valid = probes_np[probes_np >= 0]
    probed = np.unique(valid)
    rows = int(sizes[probed].sum())
    qpl = np.bincount(valid, minlength=len(sizes))
    small = (qpl > 0) & (qpl <= SMALL_GROUP)
    pairs = int((sizes * np.where(small, 0, qpl)).sum())
    small_rows = int(sizes[small].sum())
    nq, P = probes_np.shape
    return pairs, rows * (4 * d + 4) + nq * d * 4 + nq * P * k * 12, rows, small_rows


def filter_work(sizes, probes_np, d, slots=20):
    """Work of the filter search's tensor-core pass over the probes (nq, P),
    over the lists probed by more than SMALL_GROUP queries (the others go to
    the exact few-query kernel, as in scan_work):
    * pairs: (query, row) fp16 distance evaluations (in groups of up to 128
      queries per list);
    * bytes: those lists' fp16 residual rows and their squared norms read once,
      the query rows and their list centroids read once per pair, and each
      pair's slots (value + row) written at most once;
    * rows: distinct rows of those lists."""
    valid = probes_np[probes_np >= 0]
    qpl = np.bincount(valid, minlength=len(sizes))
    big = qpl > SMALL_GROUP
    rows = int(sizes[big].sum())
    pairs = int((sizes * np.where(big, qpl, 0)).sum())
    npairs = int(qpl[big].sum())
    return pairs, rows * (2 * d + 4) + npairs * d * 8 + npairs * slots * 12, rows


def run_ivf(args, cfg, rank, world, device):
    from metalfaiss_b200 import _native as nat
    from metalfaiss_b200.sharding import ShardedIVF

    idx, xq, owners, heads = build_index(cfg, device, rank=rank, world=world)
    idx.nprobe = cfg["nprobe"]
    k, nq, d = cfg["k"], cfg["nq"], cfg["d"]
    sharded = ShardedIVF(idx, rank, world, owners=owners, heads=heads) if world > 1 else None
    search = (lambda q: sharded.search(q, k)) if sharded else (lambda q: idx.search(q, k))

    # probes (for the roofline bytes): the coarse step of this batch
    probes = idx.quantizer._search_padded(xq, min(cfg["nprobe"], cfg["nlist"]),
                                          map_ids=False).labels
    mine = sharded.local if sharded else idx
    filtered = mine._filter_ok(k)
    probes_np = probes.cpu().numpy()
    sizes = mine.list_sizes()
    pairs, alg_bytes, probed_rows, small_rows = scan_work(sizes, probes_np, d, k)
    if filtered:
        pairs, alg_bytes, probed_rows = filter_work(sizes, probes_np, d)
    logical_bytes = pairs * d * 4
    tf32_peak = gemm_peak(device, tf32=True) if rank == 0 else None

    timer = Timer(device, world)
    ms, clocks, launches = timer.run(lambda: search(xq), args.steps, args.warmup)
    names = ["scan_topk_ivf_filter" if filtered else "scan_topk_ivf", "scan_topk_ivf_small",
             "ivf_filter_refine"]
    kt = timer.kernel_times(lambda: search(xq), names, min(args.steps, 20))
    phases = None
    if sharded:
        # per-phase device times of a few more steps (events between the
        # phases; outside the timed steps), the max over ranks per phase
        sharded.phase_events = []
        n_ph = min(args.steps, 10)
        for _ in range(n_ph):
            search(xq)
        torch.cuda.synchronize(device)
        evs, sharded.phase_events = sharded.phase_events, None
        per = {}
        step_len = len(evs) // n_ph
        for i in range(n_ph):
            chunk = evs[i * step_len:(i + 1) * step_len]
            for (_, e0), (name, e1) in zip(chunk[:-1], chunk[1:]):
                per[name] = per.get(name, 0.0) + e0.elapsed_time(e1) / n_ph
        import torch.distributed as dist
        names_ph = list(per)
        t = torch.tensor([per[n] for n in names_ph], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        phases = {n: round(float(v), 4) for n, v in zip(names_ph, t.tolist())}
    scan_ms, scan_n = kt[names[0]]
    small_ms, small_n = kt["scan_topk_ivf_small"]
    refine_ms, refine_n = kt["ivf_filter_refine"]
    rescans = nat.filter_rescans(device.index, reset=True)

    # ---- end to end through the public API: pinned host queries in, results out
    e2e_steps = max(3, args.steps // 2)
    e2e_ms, e2e_serial_ms = end_to_end(timer, search, xq, k, device, e2e_steps)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_ivf(idx.centroids.cpu().numpy(), idx.list_offsets.cpu().numpy(),
                               idx._vecs, idx._ids, xq, cfg,
                               min(args.cpu_baseline_sample, nq))

    if rank == 0:
        hbm_peak, bf16_peak, peak_kind = measured_peaks()
        scan_avg_ms = scan_ms / max(scan_n, 1)
        scan_s = scan_avg_ms * 1e-3
        # 3xTF32: three tensor-core products (hi*hi, hi*lo, lo*hi) of 2d flops
        # per pair against the TF32 rate; the filter pass: one fp16 product
        # against the 16-bit rate (fp16 and bf16 run at the same dense rate;
        # the measured bf16 GEMM is the denominator)
        flops_pair = 2.0 * d if filtered else 6.0 * d
        # the few-query pass reads each row once: its fp16 filter residual and
        # residual norm (filter search), or its fp32 vector and norm
        small_row_bytes = (2 * d + 4) if filtered else (4 * d + 4)
        tc_peak = bf16_peak if filtered else tf32_peak
        tflops = flops_pair * pairs / scan_s / 1e12 if scan_n else None
        gbs = alg_bytes / scan_s / 1e9 if scan_n else None
        value = nq * args.steps / (ms * 1e-3)
        tkey = args.config + ("/filter" if filtered else "")
        line = line_head(args, cfg, world, value, ms)
        line.update({
            "dtype": "f32",
            "data": "synthetic (seeded Gaussian mixture, generated in HBM)",
            "parallelism": f"list-sharded x{world}" if world > 1 else "single GPU",
            "workload_facts": {"logical_scan_bytes_per_step": logical_bytes,
                               "probed_rows_per_step_tensor_pass": probed_rows},
            "roofline": {
                "bound": "tensor",
                "kernel": ("tq_scan_kernel<FLT> (IVF list-major fp16 tcgen05 filter over "
                           "scaled residuals + fused top-2k of upper bounds), lists probed by "
                           "more than 16 queries"
                           if filtered else
                           "tq_scan_kernel (IVF list-major 3xTF32 tcgen05 scan + fused top-k), "
                           "all-probes pass over lists probed by more than 16 queries"),
                "achieved": round(tflops, 2) if tflops else None,
                "peak": round(tc_peak, 1),
                "unit": "TFLOP/s",
                "frac": round(tflops / tc_peak, 4) if tflops else None,
                "peak_kind": (f"{peak_kind} bf16 (cuBLAS bf16 GEMM, burst; fp16 runs at the "
                              f"same dense rate); TF32 measured in "
                              f"this run {round(tf32_peak, 1)} TFLOP/s" if filtered else
                              "cuBLAS TF32 GEMM 8192^3 measured in this run (best of 10); "
                              f"{peak_kind} bf16 {bf16_peak} TFLOP/s for context"),
                "algorithmic_flops_per_launch": int(flops_pair * pairs),
                "pairs_per_launch": pairs,
                "avg_launch_ms": round(scan_avg_ms, 4),
                "traffic": (TRAFFIC[tkey]["bytes"] if tkey in TRAFFIC and world == 1 else None),
                "traffic_source": TRAFFIC[tkey]["source"] if tkey in TRAFFIC else None,
                "hbm": {
                    "algorithmic_bytes_per_launch": alg_bytes,
                    "achieved": round(gbs, 1) if gbs else None,
                    "peak": hbm_peak,
                    "unit": "GB/s",
                    "frac": round(gbs / hbm_peak, 4) if gbs else None,
                    "peak_kind": f"{peak_kind} hbm_gbs",
                    "logical_scan_GBps": round(logical_bytes / scan_s / 1e9, 1) if scan_n else None,
                },
                # the filter search's exact refinement (one warp per query)
                "refine": ({
                    "kernel": "filter_refine_kernel (exact fp32 distances of the kept rows)",
                    "avg_launch_ms": round(refine_ms / refine_n, 4) if refine_n else None,
                    "lists_rescanned": rescans,
                } if filtered else None),
                # the few-query groups' pass: bound by reading those lists' rows once
                "small_groups": {
                    "kernel": ("few_scan_kernel<FLT> (fp16 filter rows, lists probed by at most "
                               "16 queries)" if filtered else
                               "few_scan_kernel (lists probed by at most 16 queries)"),
                    "rows_per_launch": small_rows,
                    "bytes_per_row": small_row_bytes,
                    "bytes_per_launch": small_rows * small_row_bytes,
                    "avg_launch_ms": round(small_ms / small_n, 4) if small_n else None,
                    "achieved": (round(small_rows * small_row_bytes / (small_ms / small_n * 1e-3)
                                       / 1e9, 1) if small_n else None),
                    "peak": hbm_peak,
                    "unit": "GB/s",
                    "frac": (round(small_rows * small_row_bytes / (small_ms / small_n * 1e-3) / 1e9
                                   / hbm_peak, 4) if small_n else None),
                },
            },
            "e2e": e2e_entry(nq, d, k, e2e_steps, e2e_ms, e2e_serial_ms),
            "gpu_launches": int(launches),
            "clocks": clocks,
            "cpu_baseline": cpu,
        })
        if phases:
            line["phases_ms_max_over_ranks"] = phases
        print(json.dumps(line), flush=True)


def line_head(args, cfg, world, value, ms):
    return {
        "metric": metric_name(cfg),
        "value": round(value, 3),
        "unit": "iterations/s" if cfg["kind"] == "kmeans" else "queries/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "config": workload_config(args.config, cfg),
    }


def cpu_baseline_ivf(cents, offsets, vecs, ids, xq, cfg, sample, threads=None):
    """The oracle's C port of the reference's IVF search on the host cores,
    over `sample` queries of the batch: the coarse step over all centroids,
    then the exact top-k over the probed lists. Only the probed lists travel
    to the host (vecs / ids stay on the device until then)."""
    from oracle import cport

    nprobe, k, d = cfg["nprobe"], cfg["k"], cfg["d"]
    threads = threads or host_threads()
    q = xq[:sample, :d].cpu().numpy()
    probes = cport.coarse_probes(q, cents[:, :d], nprobe, threads=threads)
    lists = np.unique(probes)
    nlist = len(offsets) - 1
    sizes = np.zeros(nlist, np.int64)
    sizes[lists] = offsets[lists + 1] - offsets[lists]
    sub_off = np.zeros(nlist + 1, np.int64)
    np.cumsum(sizes, out=sub_off[1:])
    hv = np.empty((int(sub_off[-1]), d), np.float32)
    hi = np.empty(int(sub_off[-1]), np.int64)
    for l in lists:
        a, b = int(offsets[l]), int(offsets[l + 1])
        hv[sub_off[l]:sub_off[l + 1]] = vecs[a:b, :d].cpu().numpy()
        hi[sub_off[l]:sub_off[l + 1]] = ids[a:b].cpu().numpy()
    t0 = time.perf_counter()
    cport.ivf_search(q, cents[:, :d], sub_off, hv, hi, nprobe, k, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": round(sample / dt, 2), "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{sample} of the {cfg['nq']} queries (coarse + scan + top-k), same index"}


def _torch_assign(x, c, chunk=1 << 17):
    """argmin_j (|x|^2 + |c_j|^2 - 2 x.c_j) per row, fp32 (TF32 off), in chunks."""
    cn = (c * c).sum(1)
    out = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    for s in range(0, x.shape[0], chunk):
        xs = x[s:s + chunk]
        dist = (xs * xs).sum(1, keepdim=True) + cn[None, :]
        dist.addmm_(xs, c.t(), alpha=-2.0)
        out[s:s + chunk] = dist.argmin(1)
    return out


def _torch_update(x, labels, c, chunk=1 << 20):
    """Masked mean per cluster in fp64; an empty cluster keeps its centroid."""
    K = c.shape[0]
    sums = torch.zeros((K, x.shape[1]), dtype=torch.float64, device=x.device)
    for s in range(0, x.shape[0], chunk):
        sums.index_add_(0, labels[s:s + chunk], x[s:s + chunk].double())
    counts = torch.bincount(labels, minlength=K)
    nz = counts > 0
    out = c.clone()
    out[nz] = (sums[nz] / counts[nz, None].double()).float()
    return out


def reference_ivf_index(cfg, device, seed=1234):
    """The benchmark's IVF index built with plain torch operations (fp32
    distances with TF32 off, fp64 sums), never this library: the same
    mixture, the same 256-per-list training subsample and seeded initial
    centroids as the library's build, the same number of Lloyd iterations,
    then every row assigned to its nearest centroid and the rows grouped by
    list in input order (python/metalfaiss/index/ivf_flat_index.py:74-93)."""
    syn = _synthetic()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        n, d, nlist = cfg["n"], cfg["d"], cfg["nlist"]
        x, centres = syn.torch_mixture(n, d, nlist, seed, device)
        cap = 256 * nlist
        xt = x
        if n > cap:
            perm = np.random.Generator(np.random.PCG64(seed + 1)).permutation(n)[:cap]
            xt = x.index_select(0, torch.from_numpy(np.sort(perm)).to(device))
        init = np.random.Generator(np.random.PCG64(seed)).permutation(xt.shape[0])[:nlist]
        c = xt.index_select(0, torch.from_numpy(init).to(device)).contiguous()
        for _ in range(cfg["niter"]):
            c = _torch_update(xt, _torch_assign(xt, c), c)
        del xt
        lab = _torch_assign(x, c)
        order = torch.argsort(lab, stable=True)
        counts = torch.bincount(lab, minlength=nlist)
        offsets = torch.zeros(nlist + 1, dtype=torch.int64, device=device)
        offsets[1:] = torch.cumsum(counts, 0)
        vecs = x.index_select(0, order)
        del x
        xq, _ = syn.torch_mixture(cfg["nq"], d, nlist, seed + 1, device, centres=centres)
        return c.cpu().numpy(), offsets.cpu().numpy(), vecs, order, xq
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def run_reference_ivf(args, cfg, device):
    t0 = time.time()
    cents, offsets, vecs, ids, xq = reference_ivf_index(cfg, device)
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    log(f"[bench] reference arm: index built with torch ops in {time.time() - t0:.1f}s")
    threads = host_threads()
    sample = min(args.cpu_sample, cfg["nq"])
    for _ in range(args.warmup):
        cpu_baseline_ivf(cents, offsets, vecs, ids, xq, cfg, max(4, sample // 8), threads)
    vals = [cpu_baseline_ivf(cents, offsets, vecs, ids, xq, cfg, sample, threads)
            for _ in range(args.steps)]
    v = statistics.median(r["value"] for r in vals)
    return v, vals[0], sample / v * 1000.0, ("port: the oracle's C port of the reference IVF "
                                             "search; index built with plain torch operations")


# ------------------------------------------------------------------ flat arm
def flat_data(cfg, device):
    syn = _synthetic()
    if cfg["data"] == "unit":
        return syn.torch_unit_rows(cfg["n"], cfg["d"], 41, device), \
            syn.torch_unit_rows(cfg["nq"], cfg["d"], 42, device)
    return syn.torch_gaussian(cfg["n"], cfg["d"], 1, device), \
        syn.torch_gaussian(cfg["nq"], cfg["d"], 2, device)


def run_flat(args, cfg, rank, world, device):
    from metalfaiss_b200 import FlatIndex, MetricType
    from metalfaiss_b200 import _native as nat
    from metalfaiss_b200.sharding import ShardedFlat

    xb, xq = flat_data(cfg, device)
    n, d, nq, k, metric = cfg["n"], cfg["d"], cfg["nq"], cfg["k"], cfg["metric"]
    idx = FlatIndex(d, MetricType(metric), device=device)
    if world > 1:
        from metalfaiss_b200.sharding import row_shard

        b, e = row_shard(n, rank, world)
        idx.add(xb[b:e], torch.arange(b, e, dtype=torch.int64, device=device))
        sharded = ShardedFlat(idx, rank, world, local=True)
        search = lambda q: sharded.search(q, k)  # noqa: E731
    else:
        idx.add(xb)
        search = lambda q: idx.search(q, k)  # noqa: E731
    del xb
    torch.cuda.empty_cache()
    nloc = idx.ntotal
    tc = nat.load().mf_flat_engine(metric, d, k, nloc, 1) == 1
    peak = gemm_peak(device, tf32=tc) if rank == 0 else None
    timer = Timer(device, world)
    ms, clocks, launches = timer.run(lambda: search(xq), args.steps, args.warmup)
    kt = timer.kernel_times(lambda: search(xq), ["scan_topk_flat", "merge"], min(args.steps, 10))
    scan_ms, scan_n = kt["scan_topk_flat"]

    e2e_steps = max(3, args.steps // 2)
    e2e_ms, e2e_serial_ms = end_to_end(timer, search, xq, k, device, e2e_steps)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_flat(idx.xb, xq, cfg, args.flat_cpu_sample)
    if rank == 0:
        hbm_peak, _, peak_kind = measured_peaks()
        avg = scan_ms / max(scan_n, 1)
        # useful work of one launch: 2 d flops per (query, row) pair, computed
        # as three tf32 products on the tensor cores (6 d) or 2 d fp32 FMA flops
        pairs = nq * nloc
        flops = (6.0 if tc else 2.0) * d * pairs
        ach = flops / (avg * 1e-3) / 1e12 if scan_n else None
        line = line_head(args, cfg, world, nq * args.steps / (ms * 1e-3), ms)
        line.update({
            "dtype": "f32",
            "data": "synthetic (seeded, generated in HBM)",
            "parallelism": f"row-sharded x{world}" if world > 1 else "single GPU",
            "roofline": {
                "bound": "tensor" if tc else "fp32 FMA",
                "kernel": ("tq_scan_kernel (flat 3xTF32 tcgen05 distance tiles + fused top-k)"
                           if tc else "scan_kernel (flat SIMT fp32 distance tiles + fused "
                                      "warp top-k)"),
                "achieved": round(ach, 2) if ach else None,
                "peak": round(peak, 1),
                "unit": "TFLOP/s",
                "frac": round(ach / peak, 4) if ach else None,
                "peak_kind": ("cuBLAS TF32 GEMM 8192^3 measured in this run (3xTF32 counts "
                              "three products per useful one)" if tc else
                              "cuBLAS fp32 SGEMM (TF32 off) 8192^3 measured in this run"),
                "algorithmic_flops_per_launch": int(flops),
                "useful_tflops": round(2.0 * d * pairs / (avg * 1e-3) / 1e12, 2) if scan_n else None,
                "avg_launch_ms": round(avg, 4),
                "launches_per_step": round(scan_n / max(1, min(args.steps, 10)), 2),
                "hbm": {"database_bytes": int(nloc * d * 4 * (2 if tc else 1)),
                        "peak": hbm_peak, "peak_kind": f"{peak_kind} hbm_gbs"},
                "traffic": None,
            },
            "e2e": e2e_entry(nq, d, k, e2e_steps, e2e_ms, e2e_serial_ms),
            "gpu_launches": int(launches),
            "clocks": clocks,
            "cpu_baseline": cpu,
        })
        print(json.dumps(line), flush=True)


def cpu_baseline_flat(xb, xq, cfg, sample, xb_host=None):
    """The numpy restatement of FlatIndex.search (BLAS distances, full stable
    argsort per row, as python/metalfaiss/indexflat.py:88-110 with
    python/metalfaiss/utils/sorting.py:39-87 does) over `sample` queries."""
    from oracle import oracle

    d = cfg["d"]
    xbh = xb_host if xb_host is not None else xb[:, :d].cpu().numpy()
    q = xq[:sample, :d].cpu().numpy()
    t0 = time.perf_counter()
    oracle.flat_search(q, xbh, cfg["k"], cfg["metric"])
    dt = time.perf_counter() - t0
    return {"value": round(sample / dt, 4), "unit": "queries/s", "cores": host_threads(),
            "kind": "port", "sample": f"{sample} of the {cfg['nq']} queries, full database "
                                      f"(numpy BLAS threads for the distances; the sort is "
                                      f"single-threaded)"}


def run_reference_flat(args, cfg, device):
    xb, xq = flat_data(cfg, device)
    xbh = xb[:, :cfg["d"]].cpu().numpy()
    del xb
    sample = min(args.flat_cpu_sample, cfg["nq"])
    for _ in range(min(args.warmup, 1)):
        cpu_baseline_flat(None, xq, cfg, sample, xbh)
    vals = [cpu_baseline_flat(None, xq, cfg, sample, xbh) for _ in range(args.steps)]
    v = statistics.median(r["value"] for r in vals)
    return v, vals[0], sample / v * 1000.0, "port: numpy restatement of FlatIndex.search"


# ---------------------------------------------------------------- k-means arm
def kmeans_data(cfg, device):
    syn = _synthetic()
    x, _ = syn.torch_mixture(cfg["n"], cfg["d"], cfg["K"], 77, device)
    return x


def run_kmeans(args, cfg, rank, world, device):
    from metalfaiss_b200 import _native as nat
    from metalfaiss_b200.clustering import (ClusteringParameters, assign, compute_norms,
                                            init_centroids, kmeans_clustering, update)

    n, d, K = cfg["n"], cfg["d"], cfg["K"]
    x = kmeans_data(cfg, device)
    c = init_centroids(x, K, 77)
    cache = nat.Workspace(device)

    def step():
        labels, _ = assign(x, c, compute_norms(c), cache)
        update(x, labels, c, cache)

    tc = nat.load().mf_flat_engine(1, d, 1, K, 1) == 1
    peak = gemm_peak(device, tf32=tc)
    timer = Timer(device, 1)
    ms, clocks, launches = timer.run(step, args.steps, args.warmup)
    kt = timer.kernel_times(step, ["scan_topk_flat"], min(args.steps, 5))
    scan_ms, scan_n = kt["scan_topk_flat"]
    # end to end through the public API: the points from pinned host memory,
    # kmeans_clustering over `steps` iterations, the centroids back to the host
    xh = x[:, :d].cpu().pin_memory()
    del x
    torch.cuda.empty_cache()
    params = ClusteringParameters(niter=args.steps, seed=77, max_points_per_centroid=0)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    cents = kmeans_clustering(xh, d, K, params, device=device).cpu()
    e1.record()
    torch.cuda.synchronize(device)
    e2e_ms = e0.elapsed_time(e1)
    cpu = None if args.no_cpu_baseline else cpu_baseline_kmeans(xh.numpy(), cfg,
                                                                 args.kmeans_cpu_sample)
    hbm_peak, _, peak_kind = measured_peaks()
    avg = scan_ms / max(scan_n, 1)
    flops = (6.0 if tc else 2.0) * d * n * K
    ach = flops / (avg * 1e-3) / 1e12 if scan_n else None
    line = line_head(args, cfg, 1, args.steps / (ms * 1e-3), ms)
    line.update({
        "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture, generated in HBM)",
        "parallelism": "single GPU",
        "roofline": {
            "bound": "tensor" if tc else "fp32 FMA",
            "kernel": ("tq_scan_kernel (assignment: 3xTF32 tcgen05 distance tiles + fused "
                       "argmin, k=1)" if tc else "scan_kernel (assignment, SIMT fp32)"),
            "achieved": round(ach, 2) if ach else None,
            "peak": round(peak, 1),
            "unit": "TFLOP/s",
            "frac": round(ach / peak, 4) if ach else None,
            "peak_kind": "cuBLAS TF32 GEMM 8192^3 measured in this run (3xTF32 counts three "
                         "products per useful one)" if tc else "cuBLAS SGEMM measured",
            "algorithmic_flops_per_launch": int(flops),
            "useful_tflops": round(2.0 * d * n * K / (avg * 1e-3) / 1e12, 2) if scan_n else None,
            "avg_launch_ms": round(avg, 4),
            "update_ms": round(ms / args.steps - avg, 4),
            "traffic": None,
            "hbm": {"points_bytes": n * d * 4, "peak": hbm_peak,
                    "peak_kind": f"{peak_kind} hbm_gbs"},
        },
        "e2e": {"value": round(args.steps / (e2e_ms * 1e-3), 3), "unit": "iterations/s",
                "h2d_bytes_per_step": int(n * d * 4 / args.steps),
                "d2h_bytes_per_step": int(K * d * 4 / args.steps),
                "note": "kmeans_clustering from pinned host points: one copy in, `steps` "
                        "iterations, the centroids out"},
        "gpu_launches": int(launches),
        "clocks": clocks,
        "cpu_baseline": cpu,
    })
    print(json.dumps(line), flush=True)


def cpu_baseline_kmeans(xh, cfg, sample, seed=5):
    """One Lloyd iteration of the numpy restatement (fp32 BLAS distances by
    norm expansion, argmin, fp64 masked mean; an empty cluster keeps its
    centroid: python/metalfaiss/clustering/any_clustering.py:105-120) over
    `sample` points; iterations/s extrapolated to all N points."""
    from oracle import oracle

    n, K = cfg["n"], cfg["K"]
    rng = np.random.Generator(np.random.PCG64(seed))
    pts = np.asarray(xh[np.sort(rng.choice(n, sample, replace=False))], np.float32)
    c = np.asarray(xh[:K], np.float32)
    t0 = time.perf_counter()
    lab = np.argmin(oracle.pairwise_l2sqr_f32(pts, c), axis=1)
    oracle.kmeans_update(pts, lab, c)
    dt = time.perf_counter() - t0
    return {"value": round(sample / (n * dt), 6), "unit": "iterations/s", "cores": host_threads(),
            "kind": "port", "sample": f"one iteration over {sample} of the {n} points, "
                                      f"extrapolated to all (numpy BLAS threads)"}


def run_reference_kmeans(args, cfg, device):
    x = kmeans_data(cfg, device)
    xh = x[:, :cfg["d"]].cpu().numpy()
    del x
    vals = [cpu_baseline_kmeans(xh, cfg, args.kmeans_cpu_sample, seed=5 + i)
            for i in range(args.steps)]
    v = statistics.median(r["value"] for r in vals)
    return v, vals[0], 1000.0 / v, "port: numpy restatement of the k-means iteration"


# ------------------------------------------------------------ IVFPQ / binary
def training_sample(x, cap, seed):
    """The rows a build trains on: all of x up to `cap`, else a seeded sample
    of `cap` rows in input order."""
    if x.shape[0] <= cap:
        return x
    perm = np.random.Generator(np.random.PCG64(seed + 1)).permutation(x.shape[0])[:cap]
    return x.index_select(0, torch.from_numpy(np.sort(perm)).to(x.device))


def ivfpq_index(cfg, device, seed=1234):
    """The IVFPQ benchmark index through the library: coarse centroids and the
    PQ trained on 256 rows per list, then every row added."""
    from metalfaiss_b200 import IVFPQIndex, synthetic as syn

    x, centres = syn.torch_mixture(cfg["n"], cfg["d"], cfg["nlist"], seed, device)
    idx = IVFPQIndex(cfg["d"], cfg["nlist"], cfg["M"], device=device, seed=seed)
    idx.train(training_sample(x, 256 * cfg["nlist"], seed), niter=cfg["niter"])
    idx.add(x)
    del x
    xq, _ = syn.torch_mixture(cfg["nq"], cfg["d"], cfg["nlist"], seed + 1, device, centres=centres)
    idx.nprobe = cfg["nprobe"]
    return idx, xq


def cpu_baseline_ivfpq(cents, pqc, offsets, codes, ids, xq, cfg, sample):
    """The oracle's numpy restatement of IVFPQIndex.search (coarse step, then
    the per-list ADC tables and scores, python/metalfaiss/index/ivf_pq_index.py:127-186)
    over `sample` queries."""
    from oracle import oracle

    q = xq[:sample, :cfg["d"]].cpu().numpy()
    t0 = time.perf_counter()
    oracle.ivfpq_search(q, cents, pqc, offsets, codes, ids, cfg["nprobe"], cfg["k"])
    dt = time.perf_counter() - t0
    return {"value": round(sample / dt, 4), "unit": "queries/s", "cores": 1, "kind": "port",
            "sample": f"{sample} of the {cfg['nq']} queries, the whole index (numpy, one core "
                      f"for the per-list loop)"}


def run_ivfpq(args, cfg, device):
    idx, xq = ivfpq_index(cfg, device)
    k, nq, d = cfg["k"], cfg["nq"], cfg["d"]
    P = min(cfg["nprobe"], cfg["nlist"])
    search = lambda q: idx.search(q, k)  # noqa: E731
    probes = idx.quantizer._search_padded(xq, P, map_ids=False).labels.cpu().numpy()
    sizes = idx.list_sizes()
    valid = probes[probes >= 0]
    pitch = idx.pq.code_pitch
    pair_rows = int(sizes[valid].sum())  # (query, row) scores of one search
    distinct_rows = int(sizes[np.unique(valid)].sum())
    timer = Timer(device, 1)
    ms, clocks, launches = timer.run(lambda: search(xq), args.steps, args.warmup)
    kt = timer.kernel_times(lambda: search(xq), ["ivfpq_scan"], min(args.steps, 10))
    scan_ms, scan_n = kt["ivfpq_scan"]
    e2e_steps = max(3, args.steps // 2)
    e2e_ms, e2e_serial_ms = end_to_end(timer, search, xq, k, device, e2e_steps)
    cpu = None
    if not args.no_cpu_baseline:
        M = cfg["M"]
        cpu = cpu_baseline_ivfpq(idx.centroids[:, :d].cpu().numpy(),
                                 idx.pq.centroids.cpu().numpy(), idx._offsets.cpu().numpy(),
                                 idx._codes[:, :M].cpu().numpy(), idx._ids.cpu().numpy(), xq,
                                 cfg, min(args.pq_cpu_sample, nq))
    hbm_peak, _, peak_kind = measured_peaks()
    avg = scan_ms / max(scan_n, 1)
    logical = pair_rows * pitch
    line = line_head(args, cfg, 1, nq * args.steps / (ms * 1e-3), ms)
    line.update({
        "dtype": "u8 codes, f32 tables",
        "data": "synthetic (seeded Gaussian mixture, generated in HBM)",
        "parallelism": "single GPU",
        "roofline": {
            "bound": "hbm",
            "kernel": "ivfpq_adc_kernel (one block per (query, probe): the pair's ADC table in "
                      "shared memory, the list's codes once per probing query)",
            "achieved": round(logical / (avg * 1e-3) / 1e9, 1) if scan_n else None,
            "peak": hbm_peak, "unit": "GB/s",
            "frac": round(logical / (avg * 1e-3) / 1e9 / hbm_peak, 4) if scan_n else None,
            "peak_kind": f"{peak_kind} hbm_gbs",
            "traffic": None,
            "algorithmic_bytes_per_launch": int(logical),
            "bytes_note": "code bytes once per (query, probed row); the distinct probed rows' "
                          f"codes are {distinct_rows * pitch} bytes, the rest comes from L2",
            "scores_per_launch": pair_rows,
            "avg_launch_ms": round(avg, 4),
        },
        "e2e": e2e_entry(nq, d, k, e2e_steps, e2e_ms, e2e_serial_ms),
        "gpu_launches": int(launches),
        "clocks": clocks,
        "cpu_baseline": cpu,
    })
    print(json.dumps(line), flush=True)


def reference_ivfpq_index(cfg, device, seed=1234):
    """The IVFPQ benchmark index built with plain torch operations, never this
    library: the same mixture and training sample, seeded k-means for the
    coarse centroids and for each subspace's 256 codewords on the training
    rows' residuals, then every row's residual encoded and the rows grouped by
    list in input order (python/metalfaiss/index/ivf_pq_index.py:59-124)."""
    syn = _synthetic()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        n, d, nlist, M = cfg["n"], cfg["d"], cfg["nlist"], cfg["M"]
        dsub = d // M
        x, centres = syn.torch_mixture(n, d, nlist, seed, device)
        x = x[:, :d].contiguous()
        xt = training_sample(x, 256 * nlist, seed)

        def kmeans(v, K, s):
            init = np.random.Generator(np.random.PCG64(s)).permutation(v.shape[0])[:K]
            c = v.index_select(0, torch.from_numpy(init).to(v.device)).contiguous()
            for _ in range(cfg["niter"]):
                c = _torch_update(v, _torch_assign(v, c), c)
            return c

        c = kmeans(xt, nlist, seed)
        rt = xt - c.index_select(0, _torch_assign(xt, c))
        pqc = torch.stack([kmeans(rt[:, m * dsub:(m + 1) * dsub].contiguous(), 256,
                                  seed + 1 + m) for m in range(M)])
        del xt, rt
        lab = _torch_assign(x, c)
        res = x - c.index_select(0, lab)
        codes = torch.stack([_torch_assign(res[:, m * dsub:(m + 1) * dsub].contiguous(), pqc[m])
                             for m in range(M)], 1).to(torch.uint8)
        del res, x
        order = torch.argsort(lab, stable=True)
        offsets = torch.zeros(nlist + 1, dtype=torch.int64, device=device)
        offsets[1:] = torch.cumsum(torch.bincount(lab, minlength=nlist), 0)
        xq, _ = syn.torch_mixture(cfg["nq"], d, nlist, seed + 1, device, centres=centres)
        return (c.cpu().numpy(), pqc.cpu().numpy(), offsets.cpu().numpy(),
                codes.index_select(0, order).cpu().numpy(), order.cpu().numpy(), xq)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def run_reference_ivfpq(args, cfg, device):
    cents, pqc, offsets, codes, ids, xq = reference_ivfpq_index(cfg, device)
    sample = min(args.pq_cpu_sample, cfg["nq"])
    cpu_baseline_ivfpq(cents, pqc, offsets, codes, ids, xq, cfg, max(1, sample // 8))
    vals = [cpu_baseline_ivfpq(cents, pqc, offsets, codes, ids, xq, cfg, sample)
            for _ in range(args.steps)]
    v = statistics.median(r["value"] for r in vals)
    return v, vals[0], sample / v * 1000.0, ("port: the oracle's numpy IVFPQ search; index "
                                             "built with plain torch operations")


def binary_data(cfg, device, seed=91):
    """Uniform random 0/1 rows (n, d) and queries (nq, d), uint8, seeded."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    xb = torch.randint(0, 2, (cfg["n"], cfg["d"]), generator=g, dtype=torch.uint8, device=device)
    xq = torch.randint(0, 2, (cfg["nq"], cfg["d"]), generator=g, dtype=torch.uint8, device=device)
    return xb, xq


def cpu_baseline_binary(xb_words, xq, cfg, sample):
    """The oracle's Hamming search (popcount of XOR over packed 64-bit words,
    then the k smallest with ties to the lower row: BinaryFlatIndex.search,
    python/metalfaiss/index/binary_flat_index.py:50-92) over `sample` queries."""
    from oracle import oracle

    q = oracle.pack01_words(xq[:sample].cpu().numpy())
    t0 = time.perf_counter()
    oracle.hamming_search_packed(q, xb_words, cfg["k"])
    dt = time.perf_counter() - t0
    return {"value": round(sample / dt, 4), "unit": "queries/s", "cores": 1, "kind": "port",
            "sample": f"{sample} of the {cfg['nq']} queries, all rows (numpy, one core)"}


def run_binary(args, cfg, device):
    from metalfaiss_b200 import BinaryFlatIndex

    xb, xq = binary_data(cfg, device)
    n, d, nq, k = cfg["n"], cfg["d"], cfg["nq"], cfg["k"]
    idx = BinaryFlatIndex(d, device=device)
    idx.add(xb)
    del xb
    search = lambda q: idx.search(q, k)  # noqa: E731
    timer = Timer(device, 1)
    ms, clocks, launches = timer.run(lambda: search(xq), args.steps, args.warmup)
    kt = timer.kernel_times(lambda: search(xq), ["binary_topk"], min(args.steps, 10))
    scan_ms, scan_n = kt["binary_topk"]
    e2e_steps = max(3, args.steps // 2)
    e2e_ms, e2e_serial_ms = end_to_end(timer, search, xq, k, device, e2e_steps)
    cpu = None
    if not args.no_cpu_baseline:
        # the library's packed rows: bit j of a row is bit j % 64 of 64-bit word
        # j / 64, as pack01_words packs the queries
        words = idx.codes.cpu().numpy().view(np.uint64) if d % 64 == 0 else None
        if words is not None:
            cpu = cpu_baseline_binary(words, xq, cfg, min(args.bin_cpu_sample, nq))
    hbm_peak, _, peak_kind = measured_peaks()
    avg = scan_ms / max(scan_n, 1)
    W = (d + 31) // 32
    word_ops = nq * n * W  # xor + popc per 32-bit word of every (query, row) pair
    row_bytes = n * W * 4
    line = line_head(args, cfg, 1, nq * args.steps / (ms * 1e-3), ms)
    line.update({
        "dtype": "u32 words",
        "data": "synthetic (seeded uniform bits, generated in HBM)",
        "parallelism": "single GPU",
        "roofline": {
            "bound": "int",
            "kernel": "binary_topk_kernel (32-query tiles x 128-row tiles, xor + popc per word, "
                      "warp top-k)",
            "achieved": round(word_ops / (avg * 1e-3) / 1e12, 3) if scan_n else None,
            "peak": None, "unit": "T word-ops/s",
            "frac": None,
            "peak_kind": "no measured integer-pipe peak on this pool",
            "traffic": None,
            "hbm": {"row_bytes": row_bytes, "reads_per_launch": -(-nq // 32),
                    "achieved_distinct_GBps": (round(row_bytes / (avg * 1e-3) / 1e9, 1)
                                               if scan_n else None),
                    "peak": hbm_peak, "peak_kind": f"{peak_kind} hbm_gbs"},
            "avg_launch_ms": round(avg, 4),
        },
        "e2e": e2e_entry(nq, d, k, e2e_steps, e2e_ms, e2e_serial_ms, query_bytes=d),
        "gpu_launches": int(launches),
        "clocks": clocks,
        "cpu_baseline": cpu,
    })
    print(json.dumps(line), flush=True)


def run_reference_binary(args, cfg, device):
    from oracle import oracle

    xb, xq = binary_data(cfg, device)
    words = oracle.pack01_words(xb.cpu().numpy())
    del xb
    sample = min(args.bin_cpu_sample, cfg["nq"])
    cpu_baseline_binary(words, xq, cfg, 1)
    vals = [cpu_baseline_binary(words, xq, cfg, sample) for _ in range(args.steps)]
    v = statistics.median(r["value"] for r in vals)
    return v, vals[0], sample / v * 1000.0, "port: the oracle's packed Hamming search"


# ------------------------------------------------------------------ dispatch
def run_ours(args, cfg):
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    try:
        if cfg["kind"] == "ivf":
            run_ivf(args, cfg, rank, world, device)
        elif cfg["kind"] == "flat":
            run_flat(args, cfg, rank, world, device)
        elif cfg["kind"] in ("ivfpq", "binary"):
            if world > 1:
                raise SystemExit(f"{args.config} runs on one GPU")
            (run_ivfpq if cfg["kind"] == "ivfpq" else run_binary)(args, cfg, device)
        else:
            if world > 1:
                raise SystemExit("kmeans5m runs on one GPU")
            run_kmeans(args, cfg, rank, world, device)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


def run_reference(args, cfg):
    """Reference arm: rank 0 only; times the CPU implementation of the path.
    This library is never loaded here."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if torch.cuda.is_available():
        device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(device)
    else:  # the arm times host code; only its data preparation uses torch
        device = torch.device("cpu")
    fn = {"ivf": run_reference_ivf, "flat": run_reference_flat,
          "kmeans": run_reference_kmeans, "ivfpq": run_reference_ivfpq,
          "binary": run_reference_binary}[cfg["kind"]]
    v, base, ms_step, kind = fn(args, cfg, device)
    unit = "iterations/s" if cfg["kind"] == "kmeans" else "queries/s"
    line = {
        "impl": "reference",
        "metric": metric_name(cfg),
        "value": v, "unit": unit, "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": {"ivfpq": "u8 codes, f32 tables", "binary": "u32 words"}.get(cfg["kind"], "f32"),
        "data": "synthetic (seeded, the same draws as this arm's counterpart)",
        "config": workload_config(args.config, cfg),
        "cpu_baseline": {"value": v, "unit": unit, "cores": base["cores"], "kind": base["kind"],
                         "sample": base["sample"], "what": kind},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="ivf20m")
    ap.add_argument("--nprobe", type=int, default=None, help="override (ivf configurations)")
    ap.add_argument("--k", type=int, default=None, help="override")
    # queries per reference-arm step (each step a bounded sample, so that the
    # whole --steps K run ends within minutes)
    ap.add_argument("--cpu-sample", type=int, default=64)
    # queries of the ivf arm's cpu_baseline (about 10 s of host work)
    ap.add_argument("--cpu-baseline-sample", type=int, default=6144)
    # queries of the flat CPU baseline (a full-row argsort each)
    ap.add_argument("--flat-cpu-sample", type=int, default=2)
    # points of the k-means CPU baseline's iteration
    ap.add_argument("--kmeans-cpu-sample", type=int, default=20000)
    # queries of the IVFPQ and binary CPU baselines (per reference-arm step too)
    ap.add_argument("--pq-cpu-sample", type=int, default=64)
    ap.add_argument("--bin-cpu-sample", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.nprobe is not None:
        cfg["nprobe"] = args.nprobe
    if args.k is not None:
        cfg["k"] = args.k
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
