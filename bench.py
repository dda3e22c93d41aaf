#!/usr/bin/env python
"""IVFFlat search throughput on B200 (queries/sec), with the list-scan kernel's
HBM roofline and a CPU baseline.

Workload (default): IVFFlat L2, d=128, N=20M rows from a Gaussian mixture of
16384 clusters (centres ~ N(0, 4 I), sigma = 1), nlist=16384 trained by seeded
k-means on a 256*nlist subsample, Q=10000 queries from the same mixture,
nprobe=32, k=10. One step = one search of the Q-query batch. The database
(10.2 GB) is far larger than L2 (126 MB), so no flush is needed between steps.

N>1 GPUs (one process per GPU, NCCL): the inverted lists are partitioned over
the ranks by greedy LPT on list size; every rank runs the coarse step for all
queries, scans its own lists, and the (Q, k) partial results are merged after
an all-gather. The database is fixed as N grows (strong scaling).

--impl reference times the reference algorithm on the host cores: the coarse
step restated in numpy and the reference's list-scan kernel
(python/metalfaiss/faissmlx/kernels/ivf_kernels.py:21-122) run as the oracle's C
port, over a bounded sample of the same queries and index.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # The headline workload: IVFFlat L2 at d=128, N=20M, nlist=16384, Q=10000, nprobe=32, k=10.
    "ivf20m": dict(d=128, n=20_000_000, nlist=16384, nq=10_000, nprobe=32, k=10, niter=10),
    # The small IVF configuration (d=64, N=32768, nlist=128, Q=16), for quick runs.
    "ivf32k": dict(d=64, n=32768, nlist=128, nq=16, nprobe=8, k=10, niter=10),
    # Mid-size for development runs.
    "ivf2m": dict(d=128, n=2_000_000, nlist=2048, nq=10_000, nprobe=32, k=10, niter=5),
    # The headline's list count at a fifth of its rows (4 GB on the device with
    # residuals): lists probed by few queries dominate, as at full size; small
    # enough for multi-pass profiler captures.
    "ivf4m": dict(d=128, n=4_000_000, nlist=16384, nq=10_000, nprobe=32, k=10, niter=5),
}


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


def tf32_gemm_peak(device, n=8192, reps=10):
    """Dense TF32 tensor-core throughput of cuBLAS on this GPU (TFLOP/s, best of
    `reps` n^3 GEMMs, CUDA events): the denominator for the 3xTF32 scans."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
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

    def __init__(self, cuda_index: int, period_s: float = 0.02):
        self.cuda_index = cuda_index
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
                "samples": len(sm), "source": "NVML every 20 ms"}


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


def lpt_partition(sizes: np.ndarray, world: int) -> np.ndarray:
    """Owner rank of each list: greedy longest-processing-time on list sizes."""
    from metalfaiss_b200.sharding import lpt_partition as f

    return f(sizes, world)


def build_index(cfg, device, seed=1234):
    from metalfaiss_b200 import IVFFlatIndex, synthetic as syn
    from metalfaiss_b200.clustering import ClusteringParameters

    t0 = time.time()
    x, centres = syn.torch_mixture(cfg["n"], cfg["d"], cfg["nlist"], seed, device)
    params = ClusteringParameters(niter=cfg["niter"], seed=seed, max_points_per_centroid=256)
    idx = IVFFlatIndex(cfg["d"], cfg["nlist"], device=device, clustering=params)
    idx.train(x)
    torch.cuda.synchronize(device)
    t1 = time.time()
    idx.add(x)
    torch.cuda.synchronize(device)
    t2 = time.time()
    del x
    xq, _ = syn.torch_mixture(cfg["nq"], cfg["d"], cfg["nlist"], seed + 1, device, centres=centres)
    torch.cuda.empty_cache()
    log(f"[bench] built index: train {t1 - t0:.1f}s add {t2 - t1:.1f}s ntotal={idx.ntotal}")
    return idx, xq


# A list probed by at most this many queries is scanned by the few-query
# kernel; the others, in groups of up to 128 queries, by the tensor-core kernel.
SMALL_GROUP = 16


def scan_work(idx, probes_np, d, k):
    """Work of one IVF scan over the probes (nq, P) of this index:
    * pairs: (query, row) distance evaluations in the tensor-core launch, i.e.
      over the lists probed by more than SMALL_GROUP queries (a list probed by
      at most SMALL_GROUP queries is scanned by the few-query kernel);
    * bytes: what the list-major scan must move once: every probed list's rows
      (vector + norm) read once, the query vectors read once and each
      (query, probe) pair's k partial results written once;
    * rows: distinct probed rows."""
    sizes = idx.list_sizes()
    valid = probes_np[probes_np >= 0]
    probed = np.unique(valid)
    rows = int(sizes[probed].sum())
    qpl = np.bincount(valid, minlength=len(sizes))
    small = (qpl > 0) & (qpl <= SMALL_GROUP)
    pairs = int((sizes * np.where(small, 0, qpl)).sum())
    small_rows = int(sizes[small].sum())
    nq, P = probes_np.shape
    return pairs, rows * (4 * d + 4) + nq * d * 4 + nq * P * k * 12, rows, small_rows


def filter_work(idx, probes_np, d, slots=20):
    """Work of the filter search's tensor-core pass over the probes (nq, P),
    over the lists probed by more than SMALL_GROUP queries (the others go to
    the exact few-query kernel, as in scan_work):
    * pairs: (query, row) fp16 distance evaluations (in groups of up to 128
      queries per list);
    * bytes: those lists' fp16 residual rows and their squared norms read once,
      the query rows and their list centroids read once per pair, and each
      pair's slots (value + row) written at most once;
    * rows: distinct rows of those lists."""
    sizes = idx.list_sizes()
    valid = probes_np[probes_np >= 0]
    qpl = np.bincount(valid, minlength=len(sizes))
    big = qpl > SMALL_GROUP
    rows = int(sizes[big].sum())
    pairs = int((sizes * np.where(big, qpl, 0)).sum())
    npairs = int(qpl[big].sum())
    return pairs, rows * (2 * d + 4) + npairs * d * 8 + npairs * slots * 12, rows


def run_ours(args, cfg):
    import torch.distributed as dist

    from metalfaiss_b200 import _native as nat
    from metalfaiss_b200.sharding import ShardedIVF

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    idx, xq = build_index(cfg, device)
    idx.nprobe = cfg["nprobe"]
    k = cfg["k"]
    nq = cfg["nq"]
    d = cfg["d"]
    sharded = ShardedIVF(idx, rank, world) if world > 1 else None
    search = (lambda q: sharded.search(q, k)) if sharded else (lambda q: idx.search(q, k))

    # probes (for the roofline bytes): the coarse step of this batch
    probes = idx.quantizer._search_padded(xq, min(cfg["nprobe"], cfg["nlist"]), map_ids=False).labels
    local = sharded.local if sharded else idx
    filtered = local._filter_ok(k)
    probes_np = probes.cpu().numpy()
    pairs, alg_bytes, probed_rows, small_rows = scan_work(local, probes_np, d, k)
    if filtered:
        pairs, alg_bytes, probed_rows = filter_work(local, probes_np, d)
    logical_bytes = pairs * d * 4
    tf32_peak = tf32_gemm_peak(device) if rank == 0 else None

    nvtx = torch.cuda.nvtx
    nvtx.range_push("warmup")
    for _ in range(args.warmup):
        search(xq)
    nvtx.range_pop()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    launches0 = nat.launch_count()
    stream = torch.cuda.current_stream(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    nvtx.range_push("timed")
    ev0.record(stream)
    for _ in range(args.steps):
        res = search(xq)
    ev1.record(stream)
    nvtx.range_pop()
    torch.cuda.synchronize(device)
    launches = nat.launch_count() - launches0
    ms = ev0.elapsed_time(ev1)
    clocks = sampler.stop()
    # per-kernel CUDA-event times for the roofline, from a separate run of a few
    # steps (the per-launch events stay out of the timed steps above)
    nat.timing_reset()
    nat.timing_enable(True)
    for _ in range(min(args.steps, 20)):
        search(xq)
    torch.cuda.synchronize(device)
    nat.timing_enable(False)
    scan_ms, scan_n = nat.timing_read("scan_topk_ivf_filter" if filtered else "scan_topk_ivf")
    small_ms, small_n = nat.timing_read("scan_topk_ivf_small")
    refine_ms, refine_n = nat.timing_read("ivf_filter_refine")
    rescans = nat.filter_rescans(local.device.index, reset=True)
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # ---- end to end through the public API: pinned host queries in, results out
    # (every step copies its queries host -> device and its results device ->
    # host, in stream order, inside the timed region)
    xq_host = xq.cpu().pin_memory()
    D_host = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    I_host = torch.empty((nq, k), dtype=torch.int64).pin_memory()
    e2e_steps = max(3, args.steps // 2)
    for _ in range(2):
        r = search(xq_host.to(device, non_blocking=True))
        D_host.copy_(r.distances, non_blocking=True)
        I_host.copy_(r.labels, non_blocking=True)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        r = search(xq_host.to(device, non_blocking=True))
        D_host.copy_(r.distances, non_blocking=True)
        I_host.copy_(r.labels, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(idx, xq, cfg, min(args.cpu_baseline_sample, nq))

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
        line = {
            "metric": "IVFFlat queries/sec (list-scan HBM GB/s vs peak in roofline)",
            "value": round(value, 1),
            "unit": "queries/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded Gaussian mixture, generated in HBM)",
            "config": {
                "workload": f"{args.config}: IVFFlat L2 d={d} N={cfg['n']} nlist={cfg['nlist']} "
                            f"Q={nq} nprobe={cfg['nprobe']} k={k}",
                "d": d, "N": cfg["n"], "nlist": cfg["nlist"], "Q": nq, "nprobe": cfg["nprobe"],
                "k": k, "parallelism": f"list-sharded x{world}" if world > 1 else "single GPU",
                "l2": "database (>=10 GB) larger than L2; no flush",
                "logical_scan_bytes_per_step": logical_bytes,
                "probed_rows_per_step": probed_rows,
            },
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
                # the few-query groups' pass (one 4-warp block per item): bound by
                # reading those lists' rows (vector + norm) once
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
            "e2e": {
                "value": round(nq * e2e_steps / (e2e_ms * 1e-3), 1),
                "unit": "queries/s",
                "h2d_bytes_per_step": int(nq * d * 4),
                "d2h_bytes_per_step": int(nq * k * 12),
            },
            "gpu_launches": int(launches),
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def cpu_baseline(idx, xq, cfg, sample):
    """The oracle's C port of the reference's IVF search on the host cores, over
    `sample` queries of the same batch and the same index."""
    from oracle import cport

    nprobe, k, d = cfg["nprobe"], cfg["k"], cfg["d"]
    q = xq[:sample, :d].cpu().numpy()
    cents = idx.centroids.cpu().numpy()
    probes = cport.coarse_probes(q, cents, nprobe)
    # only the probed lists travel to the host
    lists = np.unique(probes)
    offsets = idx.list_offsets.cpu().numpy()
    sub_off = np.zeros(idx.nlist + 1, np.int64)
    sizes = np.zeros(idx.nlist, np.int64)
    sizes[lists] = offsets[lists + 1] - offsets[lists]
    np.cumsum(sizes, out=sub_off[1:])
    vecs = np.empty((int(sub_off[-1]), d), np.float32)
    ids = np.empty(int(sub_off[-1]), np.int64)
    for l in lists:
        a, b = int(offsets[l]), int(offsets[l + 1])
        vecs[sub_off[l]:sub_off[l + 1]] = idx._vecs[a:b, :d].cpu().numpy()
        ids[sub_off[l]:sub_off[l + 1]] = idx._ids[a:b].cpu().numpy()
    threads = len(os.sched_getaffinity(0))
    t0 = time.perf_counter()
    cport.ivf_search(q, cents, sub_off, vecs, ids, nprobe, k, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": round(sample / dt, 2), "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{sample} of the {cfg['nq']} queries (coarse + scan + top-k), same index"}


def run_reference(args, cfg):
    """Reference arm: rank 0 only; times the CPU implementation of the path."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    idx, xq = build_index(cfg, device)
    idx.nprobe = cfg["nprobe"]
    for _ in range(args.warmup):
        cpu_baseline(idx, xq, cfg, max(4, args.cpu_sample // 8))
    vals = []
    for _ in range(args.steps):
        vals.append(cpu_baseline(idx, xq, cfg, args.cpu_sample))
    v = statistics.median(r["value"] for r in vals)
    base = vals[0]
    line = {
        "impl": "reference",
        "metric": "IVFFlat queries/sec (list-scan HBM GB/s vs peak in roofline)",
        "value": v, "unit": "queries/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000.0 * args.cpu_sample / v, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture)",
        "config": {"workload": f"{args.config}: IVFFlat L2 d={cfg['d']} N={cfg['n']} nlist={cfg['nlist']} "
                               f"Q={cfg['nq']} nprobe={cfg['nprobe']} k={cfg['k']}"},
        "cpu_baseline": {"value": v, "unit": "queries/s", "cores": base["cores"], "kind": base["kind"],
                         "sample": base["sample"]},
        "e2e": {"value": v, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="ivf20m")
    # queries per reference-arm step (each step a bounded sample, so that the
    # whole --steps K run ends within minutes)
    ap.add_argument("--cpu-sample", type=int, default=64)
    # queries of this arm's cpu_baseline (about 10 s of host work)
    ap.add_argument("--cpu-baseline-sample", type=int, default=6144)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
