"""The C-ABI library loads and exports every entry point include/*.h declares
(CPU-only: no compute calls, only size queries and argument errors)."""
import ctypes
import re
from pathlib import Path

import pytest

from metalfaiss_b200 import _native as nat
from metalfaiss_b200.errors import ErrorCode

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names.update(re.findall(r"^MF_API\s+[\w\s\*]+?\b(mf_\w+)\s*\(", h.read_text(), re.M))
    return sorted(names)


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "mf_flat_search" in syms and "mf_ivf_search" in syms and len(syms) >= 20


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(nat.library_path()))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_table_covers_header():
    assert sorted(nat.exported_symbols()) == declared_symbols()


def test_version_and_limits():
    lib = nat.load()
    assert lib.mf_version() >= 100
    assert lib.mf_max_k() == 256
    assert lib.mf_ivf_bound_rows() == 128


def test_workspace_queries_without_gpu():
    assert nat.workspace_size("mf_flat_search_workspace_size", 16, 32768, 64, 1, 10) > 0
    assert nat.workspace_size("mf_ivf_search_workspace_size", 10000, 16384, 32, 128, 1, 10) > 10000 * 32 * 10 * 12
    assert nat.workspace_size("mf_kmeans_update_workspace_size", 1000, 10, 64) > 0
    with pytest.raises(ValueError):
        nat.workspace_size("mf_flat_search_workspace_size", 16, 100, 63, 1, 10)  # d % 4 != 0
    with pytest.raises(ValueError):
        nat.workspace_size("mf_flat_search_workspace_size", 16, 100, 64, 1, 257)  # k too large
    from metalfaiss_b200.errors import MetricError
    with pytest.raises(MetricError):
        nat.workspace_size("mf_flat_search_workspace_size", 16, 100, 64, 7, 10)


def test_compute_call_reports_status_not_crash():
    """A compute call on a machine without a usable device returns a status."""
    import torch

    lib = nat.load()
    status = lib.mf_vector_norms(0, None, None, 4, 4, None)
    if not torch.cuda.is_available():
        assert status == ErrorCode.INVALID_ARGS
        assert b"device" in lib.mf_last_error()
    else:
        assert status == ErrorCode.INVALID_ARGS  # NULL pointers rejected before launch


def test_strided_merge_rejects_bad_layout_before_launch():
    """mf_topk_merge_strided returns a status for a negative stride (or, with
    no usable device, for the device) and launches nothing."""
    lib = nat.load()
    status = lib.mf_topk_merge_strided(0, None, None, 10, -1, None, 10, 10, 4, 2, 10, 10, None,
                                       None)
    assert status == ErrorCode.INVALID_ARGS
    assert lib.mf_last_error()


def test_engine_and_filter_eligibility_queries_without_gpu():
    """The host-side dispatch queries: the tensor-core flat scan takes L2 and
    inner product at 32 <= d <= 1024; the filter search 64 <= d <= 128 with d
    a multiple of 8 and k <= 16."""
    lib = nat.load()
    L2, IP, L1 = 1, 0, 2
    assert lib.mf_flat_engine(L2, 128, 10, 1_000_000, 1) == 1
    assert lib.mf_flat_engine(IP, 128, 10, 1_000_000, 0) == 1
    assert lib.mf_flat_engine(L1, 128, 10, 1_000_000, 1) == 0
    assert lib.mf_flat_engine(L2, 16, 10, 1_000_000, 1) == 0      # d < 32
    assert lib.mf_flat_engine(L2, 128, 10, 100, 1) == 0           # tiny bank
    for d in (64, 72, 96, 128):
        assert lib.mf_ivf_filter_eligible(d, 10, 100_000) == 1
    for d in (32, 56, 60, 132, 136, 256):
        assert lib.mf_ivf_filter_eligible(d, 10, 100_000) == 0
    assert lib.mf_ivf_filter_eligible(128, 17, 100_000) == 0
