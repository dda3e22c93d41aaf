"""k-means on the B200: the assignment step (fused distance + argmin) and the
deterministic centroid update, python/metalfaiss/clustering/ of the reference.

The reference's AnyClustering cannot be constructed (it calls
BaseClustering.__init__ without (d, k) and reads a missing `max_points`,
python/metalfaiss/clustering/any_clustering.py:41,101), so this module restates
the algorithm it and IVFPQIndex._kmeans (python/metalfaiss/index/ivf_pq_index.py:59-78)
describe: a seeded permutation picks k distinct rows as the initial centroids,
then a fixed number of Lloyd iterations with no early stop; an empty cluster
keeps its previous centroid.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _native as nat
from ._tensors import as_matrix, default_device, padded_dim
from .errors import InvalidArgumentError


@dataclass
class ClusteringParameters:
    """Defaults of python/metalfaiss/clustering/clustering_parameters.py:11-51."""

    niter: int = 25
    nredo: int = 1
    is_verbose: bool = False
    is_spherical: bool = False
    min_points_per_centroid: int = 39
    max_points_per_centroid: int = 256
    seed: int = 1234

    @classmethod
    def default(cls) -> "ClusteringParameters":
        return cls()


def _ws(device, nbytes, cache):
    if cache is None:
        cache = nat.Workspace(device)
    return cache.get(nbytes), cache


def compute_norms(x: torch.Tensor) -> torch.Tensor:
    n, dp = x.shape
    out = torch.empty(n, dtype=torch.float32, device=x.device)
    if n:
        nat.call("mf_vector_norms", x.device.index, nat.stream_of(x.device), nat.ptr(x), n, dp,
                 nat.ptr(out))
    return out


def assign(x: torch.Tensor, centroids: torch.Tensor, centroid_norms: Optional[torch.Tensor] = None,
           workspace=None):
    """labels (n,) int64 and squared distances (n,) of each row's nearest
    centroid; x and centroids are padded fp32 device matrices."""
    dev = x.device
    n, dp = x.shape
    nc = centroids.shape[0]
    if centroid_norms is None:
        centroid_norms = compute_norms(centroids)
    labels = torch.empty(n, dtype=torch.int64, device=dev)
    dists = torch.empty(n, dtype=torch.float32, device=dev)
    if n == 0:
        return labels, dists
    nbytes = nat.workspace_size("mf_kmeans_assign_workspace_size", n, nc, dp)
    ws, _ = _ws(dev, nbytes, workspace)
    nat.call("mf_kmeans_assign", dev.index, nat.stream_of(dev), nat.ptr(x), n, nat.ptr(centroids),
             nat.ptr(centroid_norms), nc, dp, nat.ptr(labels), nat.ptr(dists), nat.ptr(ws),
             ws.numel())
    return labels, dists


def update(x: torch.Tensor, labels: torch.Tensor, centroids: torch.Tensor, workspace=None):
    """In-place centroid update; returns the cluster sizes (int64)."""
    dev = x.device
    n, dp = x.shape
    nc = centroids.shape[0]
    counts = torch.empty(nc, dtype=torch.int64, device=dev)
    nbytes = nat.workspace_size("mf_kmeans_update_workspace_size", n, nc, dp)
    ws, _ = _ws(dev, nbytes, workspace)
    nat.call("mf_kmeans_update", dev.index, nat.stream_of(dev), nat.ptr(x), n, dp, nat.ptr(labels),
             nc, nat.ptr(centroids), nat.ptr(counts), nat.ptr(ws), ws.numel())
    return counts


def cluster_sums(x: torch.Tensor, labels: torch.Tensor, nc: int, workspace=None):
    """Per-cluster fp64 sums (nc, d) and sizes of this device's points
    (mf_kmeans_sums): the update's reduction, before any division."""
    dev = x.device
    n, dp = x.shape
    sums = torch.empty((nc, dp), dtype=torch.float64, device=dev)
    counts = torch.empty(nc, dtype=torch.int64, device=dev)
    nbytes = nat.workspace_size("mf_kmeans_update_workspace_size", n, nc, dp)
    ws, _ = _ws(dev, nbytes, workspace)
    nat.call("mf_kmeans_sums", dev.index, nat.stream_of(dev), nat.ptr(x), n, dp, nat.ptr(labels),
             nc, nat.ptr(sums), nat.ptr(counts), nat.ptr(ws), ws.numel())
    return sums, counts


def apply_sums(sums: torch.Tensor, counts: torch.Tensor, centroids: torch.Tensor) -> None:
    """centroids[j] = sums[j] / counts[j] in place; empty clusters keep theirs
    (mf_kmeans_apply)."""
    dev = centroids.device
    nc, dp = centroids.shape
    nat.call("mf_kmeans_apply", dev.index, nat.stream_of(dev), nat.ptr(sums), nat.ptr(counts), nc,
             dp, nat.ptr(centroids))


def init_centroids(x: torch.Tensor, k: int, seed: int) -> torch.Tensor:
    """k distinct rows chosen by a seeded permutation (python/metalfaiss/index/ivf_pq_index.py:63;
    numpy PCG64 stands in for MLX's PRNG)."""
    n = x.shape[0]
    if k > n:
        raise InvalidArgumentError(f"need at least k={k} training points, got {n}")
    perm = np.random.Generator(np.random.PCG64(seed)).permutation(n)[:k]
    idx = torch.from_numpy(perm.astype(np.int64)).to(x.device)
    return x.index_select(0, idx).contiguous()


def subsample(x: torch.Tensor, k: int, params: ClusteringParameters) -> torch.Tensor:
    """Caps the training set at max_points_per_centroid * k rows (seeded)."""
    cap = params.max_points_per_centroid * k
    n = x.shape[0]
    if params.max_points_per_centroid <= 0 or n <= cap:
        return x
    perm = np.random.Generator(np.random.PCG64(params.seed + 1)).permutation(n)[:cap]
    idx = torch.from_numpy(np.sort(perm).astype(np.int64)).to(x.device)
    return x.index_select(0, idx).contiguous()


def train_kmeans(x: torch.Tensor, k: int, niter: int, seed: int,
                 init: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Lloyd's k-means on a padded device matrix; returns (k, padded d) centroids."""
    c = init_centroids(x, k, seed) if init is None else init.clone().contiguous()
    cache = nat.Workspace(x.device)
    for _ in range(int(niter)):
        cn = compute_norms(c)
        labels, _ = assign(x, c, cn, cache)
        update(x, labels, c, cache)
    return c


class KMeans:
    """Stateful wrapper: KMeans(d, k).train(x) then .centroids / .assign(x)."""

    def __init__(self, d: int, k: int, parameters: Optional[ClusteringParameters] = None,
                 device=None):
        self.d = int(d)
        self.k = int(k)
        self.parameters = parameters or ClusteringParameters()
        self.device = default_device(device)
        self._centroids: Optional[torch.Tensor] = None

    def train(self, xs) -> None:
        nat.require_cuda(self.device)
        x = as_matrix(xs, self.d, self.device, "training data")
        if x.shape[0] == 0:
            raise InvalidArgumentError("Empty training data")
        x = subsample(x, self.k, self.parameters)
        self._centroids = train_kmeans(x, self.k, self.parameters.niter, self.parameters.seed)

    @property
    def centroids(self) -> torch.Tensor:
        if self._centroids is None:
            raise RuntimeError("Clustering not trained")
        return self._centroids[:, : self.d]

    def assign(self, xs):
        x = as_matrix(xs, self.d, self.device)
        return assign(x, self._centroids)


def kmeans_clustering(xs, d: int, k: int, params: Optional[ClusteringParameters] = None,
                      device=None) -> torch.Tensor:
    """python/metalfaiss/clustering/any_clustering.py:136-145: returns (k, d) centroids."""
    km = KMeans(d, k, params, device)
    km.train(xs)
    return km.centroids


__all__ = ["ClusteringParameters", "KMeans", "kmeans_clustering", "assign", "update",
           "train_kmeans", "init_centroids", "compute_norms", "padded_dim"]
