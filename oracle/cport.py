"""ctypes wrapper of the oracle's C port (oracle/c/ivf_oracle.c). Test
infrastructure and the timed CPU baseline only."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

_LIB = Path(__file__).resolve().parent / "_build" / "liboracle.so"
_lib = None


def _cpu_ok() -> bool:
    try:
        flags = Path("/proc/cpuinfo").read_text()
    except OSError:
        return True
    return " avx2" in flags and " fma" in flags


def lib():
    global _lib
    if _lib is None:
        if not _LIB.exists():
            from . import build_oracle

            build_oracle.build()
        if not _cpu_ok():
            raise RuntimeError("the oracle C port is built for x86-64-v3 (AVX2+FMA)")
        _lib = ctypes.CDLL(str(_LIB))
        P = ctypes.c_void_p
        I64, I32 = ctypes.c_int64, ctypes.c_int
        _lib.mfo_coarse.argtypes = [P, I64, P, I32, I32, I32, P, I32]
        _lib.mfo_ivf_scan.argtypes = [P, I64, P, I32, P, P, P, I32, I32, P, P, I32]
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def coarse_probes(xq, cents, nprobe, threads=1):
    xq = np.ascontiguousarray(xq, np.float32)
    cents = np.ascontiguousarray(cents, np.float32)
    P = min(nprobe, len(cents))
    out = np.empty((len(xq), P), np.int64)
    lib().mfo_coarse(_p(xq), len(xq), _p(cents), len(cents), xq.shape[1], P, _p(out), threads)
    return out


def ivf_search(xq, cents, offsets, vecs, ids, nprobe, k, threads=1, probes=None):
    xq = np.ascontiguousarray(xq, np.float32)
    if probes is None:
        probes = coarse_probes(xq, cents, nprobe, threads)
    probes = np.ascontiguousarray(probes, np.int64)
    offsets = np.ascontiguousarray(offsets, np.int64)
    vecs = np.ascontiguousarray(vecs, np.float32)
    ids = np.ascontiguousarray(ids, np.int64)
    D = np.empty((len(xq), k), np.float32)
    I = np.empty((len(xq), k), np.int64)
    lib().mfo_ivf_scan(_p(xq), len(xq), _p(probes), probes.shape[1], _p(offsets), _p(vecs),
                       _p(ids), xq.shape[1], k, _p(D), _p(I), threads)
    return D, I
