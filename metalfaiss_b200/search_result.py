"""Result containers, python/metalfaiss/utils/search_result.py:9-80 of the reference.

Arrays are torch tensors on the index's device (the reference returns MLX
arrays). `labels` aliases `indices` (:38-40) and a SearchResult unpacks as
`D, I = result` the way the reference's tests use it
(python/metalfaiss/unittest/test_index_factory.py:160).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class SearchResult:
    distances: torch.Tensor
    indices: torch.Tensor

    def __post_init__(self):
        if tuple(self.distances.shape) != tuple(self.indices.shape):
            raise ValueError("Distances and indices must have same shape")

    @property
    def labels(self) -> torch.Tensor:
        return self.indices

    def __len__(self) -> int:
        return int(self.distances.shape[0])

    def __iter__(self):
        yield self.distances
        yield self.indices

    def __getitem__(self, idx) -> "SearchResult":
        return SearchResult(distances=self.distances[idx], indices=self.indices[idx])

    def numpy(self):
        return self.distances.cpu().numpy(), self.indices.cpu().numpy()


@dataclass
class SearchRangeResult:
    """Flat CSR layout: query q's hits are [lims[q], lims[q+1])."""

    distances: torch.Tensor
    indices: torch.Tensor
    lims: torch.Tensor

    def __post_init__(self):
        if tuple(self.distances.shape) != tuple(self.indices.shape):
            raise ValueError("Must have same number of distance and index entries")
        if self.lims.dim() != 1 or self.lims.numel() < 1:
            raise ValueError("Lims array must have length n_queries + 1")

    @property
    def labels(self) -> torch.Tensor:
        return self.indices

    def __len__(self) -> int:
        return int(self.lims.numel() - 1)

    def __getitem__(self, q: int):
        lims = self.lims.cpu()
        a, b = int(lims[q]), int(lims[q + 1])
        return self.distances[a:b], self.indices[a:b]

    def get_total_size(self) -> int:
        return int(self.lims[-1])

    def numpy(self):
        return self.lims.cpu().numpy(), self.distances.cpu().numpy(), self.indices.cpu().numpy()
