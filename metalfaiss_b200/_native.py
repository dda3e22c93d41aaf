"""ctypes binding of libmetalfaiss_b200.so (the C-ABI in include/metalfaiss_b200.h).

There is no fallback: if the library is missing or CUDA is unavailable, every
compute call raises. torch supplies device buffers and the current stream only.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

from .errors import CudaError, check_error

_LIB_PATH = Path(__file__).resolve().with_name("libmetalfaiss_b200.so")
_lock = threading.Lock()
_lib = None

P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_int64
SZ = ctypes.c_size_t
F32 = ctypes.c_float
PSZ = ctypes.POINTER(ctypes.c_size_t)
PI64 = ctypes.POINTER(ctypes.c_int64)

_SIGNATURES = {
    "mf_version": ([], I32),
    "mf_last_error": ([], ctypes.c_char_p),
    "mf_max_k": ([], I32),
    "mf_vector_norms": ([I32, P, P, I64, I32, P], I32),
    "mf_tf32_residual": ([I32, P, P, I64, I32, P], I32),
    "mf_flat_search_workspace_size": ([I64, I64, I32, I32, I32, PSZ], I32),
    "mf_flat_search": ([I32, P, P, I64, P, P, P, I64, I32, I32, I32, P, P, P, P, SZ], I32),
    "mf_flat_search_noalloc": ([I32, P, P, I64, P, P, P, I64, I32, I32, I32, P, P, P], I32),
    "mf_flat_search_bounded": ([I32, P, P, I64, P, P, P, I64, I32, I32, I32, P, P, P, P, P, SZ], I32),
    "mf_ivf_search_workspace_size": ([I64, I32, I32, I32, I32, I32, PSZ], I32),
    "mf_ivf_search": ([I32, P, P, I64, P, P, I32, I32, P, P, P, P, P, I64, P, I32, I32, I32, P, P, P, SZ], I32),
    "mf_ivf_search_preassigned_workspace_size": ([I64, I32, I32, I32, I32, I32, PSZ], I32),
    "mf_ivf_search_preassigned": ([I32, P, P, I64, P, I32, I32, P, P, P, P, P, I64, P, I32, I32, I32, P, P, P, SZ], I32),
    "mf_ivf_probe_bound": ([I32, P, P, I64, P, I32, I32, P, P, P, P, P, I64, P, I32, I32, I32, P, P, SZ], I32),
    "mf_ivf_search_bounded": ([I32, P, P, I64, P, I32, I32, P, P, P, P, P, I64, P, I32, I32, I32, P, P, P, P, SZ], I32),
    "mf_ivf_filter_eligible": ([I32, I32, I64], I32),
    "mf_ivf_filter_bank": ([I32, P, I32, I32, P, P, P, P, I64, P, P, P, P], I32),
    "mf_ivf_search_filtered_workspace_size": ([I64, I32, I32, I32, I32, PSZ], I32),
    "mf_ivf_search_filtered": ([I32, P, P, I64, P, P, I32, I32, P, P, P, P, P, I64, P, P, P, P, P, I32, I32, P, P, P, SZ], I32),
    "mf_ivf_search_bounded_filtered_workspace_size": ([I64, I32, I32, I32, I32, PSZ], I32),
    "mf_ivf_search_bounded_filtered": ([I32, P, P, I64, P, I32, I32, P, P, P, P, I64, P, P, P, P, P, P, I32, I32, P, P, P, P, SZ], I32),
    "mf_ivf_filter_rescans": ([I32, PI64, I32], I32),
    "mf_topk_merge": ([I32, P, P, P, I64, I32, I32, I32, P, P], I32),
    "mf_topk_merge_strided": ([I32, P, P, I64, I64, P, I64, I64, I64, I32, I32, I32, P, P], I32),
    "mf_ivf_bound_rows": ([], I32),
    "mf_kmeans_assign_workspace_size": ([I64, I32, I32, PSZ], I32),
    "mf_kmeans_assign": ([I32, P, P, I64, P, P, I32, I32, P, P, P, SZ], I32),
    "mf_kmeans_update_workspace_size": ([I64, I32, I32, PSZ], I32),
    "mf_kmeans_update": ([I32, P, P, I64, I32, P, I32, P, P, P, SZ], I32),
    "mf_kmeans_sums": ([I32, P, P, I64, I32, P, I32, P, P, P, SZ], I32),
    "mf_kmeans_apply": ([I32, P, P, P, I32, I32, P], I32),
    "mf_ivf_add_workspace_size": ([I64, I64, I32, PSZ], I32),
    "mf_ivf_add": ([I32, P, I32, I32, P, P, P, P, I64, P, P, P, P, I64, P, P, P, P, P, SZ], I32),
    "mf_flat_range_workspace_size": ([I64, I64, I32, PSZ], I32),
    "mf_flat_range_count": ([I32, P, P, I64, P, P, I64, I32, I32, F32, P, PI64, P, SZ], I32),
    "mf_flat_range_fill": ([I32, P, P, I64, P, P, I64, I32, I32, F32, P, P, P, P, P, SZ], I32),
    "mf_ivf_range_workspace_size": ([I64, I32, I32, I32, PSZ], I32),
    "mf_ivf_range_count": ([I32, P, P, I64, P, P, I32, I32, P, P, P, I32, I32, F32, P, PI64, P, SZ], I32),
    "mf_ivf_range_fill": ([I32, P, P, I64, P, P, I32, I32, P, P, P, P, I32, I32, F32, P, P, P, P, SZ], I32),
    "mf_timing_enable": ([I32], I32),
    "mf_timing_reset": ([], I32),
    "mf_launch_count": ([], I64),
    "mf_diag_f16_dot": ([I32, P, I32, P, P, I32, P], I32),
    "mf_binary_pack": ([I32, P, P, I64, I32, P], I32),
    "mf_binary_unpack": ([I32, P, P, I64, I32, P], I32),
    "mf_binary_flat_search_workspace_size": ([I64, I64, I32, I32, PSZ], I32),
    "mf_binary_flat_search": ([I32, P, P, I64, P, I64, I32, I32, P, P, P, P, SZ], I32),
    "mf_binary_range_workspace_size": ([I64, I64, I32, PSZ], I32),
    "mf_binary_range_count": ([I32, P, P, I64, P, I64, I32, I32, P, PI64, P, SZ], I32),
    "mf_binary_range_fill": ([I32, P, P, I64, P, I64, I32, I32, P, P, P, P, P, SZ], I32),
    "mf_binary_ivf_search_workspace_size": ([I64, I32, I32, PSZ], I32),
    "mf_binary_ivf_search": ([I32, P, P, I64, P, I32, I32, P, P, I32, P, I32, I32, P, P, P, SZ],
                             I32),
    "mf_pq_encode": ([I32, P, P, I64, I32, I32, I32, I32, P, P, P, P, I32], I32),
    "mf_ivfpq_search_workspace_size": ([I64, I32, I32, PSZ], I32),
    "mf_ivfpq_search_preassigned": ([I32, P, P, I64, I32, I32, P, I32, I32, P, P, I32, I32, P, P,
                                     I32, P, I32, P, P, P, SZ], I32),
    "mf_flat_engine": ([I32, I32, I32, I64, I32], I32),
    "mf_set_scan_engine": ([I32], I32),
    "mf_set_filter_groups": ([I32], I32),
    "mf_set_filter_small_group": ([I32], I32),
    "mf_device_error": ([I32, ctypes.POINTER(ctypes.c_int)], I32),
    "mf_timing_read": ([ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), PI64], I32),
}


def library_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Loads (once) and returns the library; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _LIB_PATH.exists():
            raise CudaError(
                f"{_LIB_PATH.name} is not built; run `python -m metalfaiss_b200._build` "
                "(the CUDA path has no CPU fallback)")
        lib = ctypes.CDLL(str(_LIB_PATH))
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def call(name: str, *args) -> None:
    lib = load()
    status = getattr(lib, name)(*args)
    if status != 0:
        msg = lib.mf_last_error().decode(errors="replace")
        check_error(status, f"{name}: {msg}")


def workspace_size(name: str, *args) -> int:
    out = ctypes.c_size_t(0)
    call(name, *args, ctypes.byref(out))
    return int(out.value)


def require_cuda(device: torch.device) -> None:
    if device.type != "cuda" or not torch.cuda.is_available():
        raise CudaError(
            "metalfaiss_b200 runs on a CUDA device only (no CPU fallback); "
            f"got device {device}")
    load()


def stream_of(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


class Workspace:
    """Grow-only device scratch buffer reused across calls on one device and stream."""

    def __init__(self, device: torch.device):
        self.device = device
        self.buf = None

    def get(self, nbytes: int) -> torch.Tensor:
        nbytes = max(int(nbytes), 256)
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.empty(nbytes + (nbytes >> 3), dtype=torch.uint8, device=self.device)
        return self.buf


def timing_enable(on: bool) -> None:
    call("mf_timing_enable", 1 if on else 0)


def timing_reset() -> None:
    call("mf_timing_reset")


def timing_read(kernel: str):
    """(total milliseconds, launches) recorded for `kernel` since the last reset."""
    t = ctypes.c_double(0.0)
    n = ctypes.c_int64(0)
    call("mf_timing_read", kernel.encode(), ctypes.byref(t), ctypes.byref(n))
    return float(t.value), int(n.value)


def set_scan_engine(engine: int) -> None:
    """0 automatic, 1 SIMT only, 2 tensor cores where eligible, 3 = 2 with the
    query tile streamed through shared memory (process-wide)."""
    call("mf_set_scan_engine", int(engine))


def device_error(device_index: int) -> int:
    """Reads and clears the device-side error word (0 = none)."""
    c = ctypes.c_int(0)
    call("mf_device_error", int(device_index), ctypes.byref(c))
    return int(c.value)


def filter_rescans(device_index: int, reset: bool = False) -> int:
    """Lists the IVF filter search rescanned exactly on this device since the
    last reset (mf_ivf_filter_rescans)."""
    c = ctypes.c_int64(0)
    call("mf_ivf_filter_rescans", int(device_index), ctypes.byref(c), 1 if reset else 0)
    return int(c.value)


def launch_count() -> int:
    return int(load().mf_launch_count())


def env_flag(name: str) -> bool:
    return os.environ.get(name, "").strip().lower() in {"1", "true", "yes", "on"}
