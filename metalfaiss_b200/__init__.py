"""metalfaiss_b200 — the MetalFaiss search hot path, rebuilt for NVIDIA B200 (sm_100a).

Drop-in surface of the reference package (python/metalfaiss/__init__.py:27-87):
FlatIndex, IVFFlatIndex, MetricType, SearchResult, SearchRangeResult,
kmeans_clustering / ClusteringParameters, write_index / read_index and the
error model. Compute runs in
hand-written CUDA kernels behind the C-ABI of include/metalfaiss_b200.h
(libmetalfaiss_b200.so, loaded with ctypes); torch provides device buffers and
streams. There is no CPU fallback: without a CUDA device every compute call raises.
"""
from .clustering import ClusteringParameters, KMeans, kmeans_clustering
from .errors import (BadStateError, CudaError, ErrorCode, FormatError, InvalidArgumentError,
                     IOFaissError, MetalFaissError, NotImplementedFaissError, check_error,
                     clear_last_error, get_last_error)
from .index_binary_flat import BinaryFlatIndex, BinaryIVFIndex
from .index_flat import FlatIndex
from .index_io import read_index, write_index
from .index_ivf_flat import IVFFlatIndex
from .index_ivfpq import IVFPQIndex, ProductQuantizer
from .metric_type import MetricType
from .search_result import SearchRangeResult, SearchResult

__version__ = "0.1.0"

__all__ = [
    "FlatIndex", "IVFFlatIndex", "BinaryFlatIndex", "BinaryIVFIndex", "IVFPQIndex", "ProductQuantizer", "MetricType", "SearchResult", "SearchRangeResult",
    "ClusteringParameters", "KMeans", "kmeans_clustering", "ErrorCode", "MetalFaissError",
    "InvalidArgumentError", "BadStateError", "NotImplementedFaissError", "CudaError",
    "check_error", "get_last_error", "clear_last_error", "IOFaissError", "FormatError",
    "write_index", "read_index",
]
