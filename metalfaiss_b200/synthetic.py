"""Seeded synthetic inputs with the shapes and distributions of the benchmark
configurations (no public dataset is involved).

* gaussian: i.i.d. N(0, 1) rows.
* unit_rows: N(0, 1) rows normalised to unit L2 length.
* mixture: isotropic Gaussian mixture; centres ~ N(0, 4 I) (variance 4, i.e.
  standard deviation 2) and points = centre + N(0, sigma^2 I), sigma = 1.

numpy generators (PCG64) are used for sizes the CPU oracle handles; the torch
generators produce the same distributions directly in HBM for the full-size
benchmark workloads (different streams of random numbers, same law).
"""
from __future__ import annotations

import numpy as np
import torch

CENTRE_STD = 2.0
SIGMA = 1.0


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def gaussian(n: int, d: int, seed: int) -> np.ndarray:
    return rng(seed).standard_normal((n, d), dtype=np.float32)


def unit_rows(n: int, d: int, seed: int) -> np.ndarray:
    x = gaussian(n, d, seed)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x


def mixture_centres(n_centres: int, d: int, seed: int) -> np.ndarray:
    return (rng(seed).standard_normal((n_centres, d), dtype=np.float32) * CENTRE_STD).astype(np.float32)


def mixture(n: int, d: int, n_centres: int, seed: int, centres: np.ndarray | None = None):
    """Returns (points, centres, component index of each point)."""
    g = rng(seed)
    if centres is None:
        centres = mixture_centres(n_centres, d, seed + 7919)
    comp = g.integers(0, n_centres, size=n)
    x = centres[comp] + g.standard_normal((n, d), dtype=np.float32) * SIGMA
    return x.astype(np.float32), centres, comp


# ------------------------------------------------------------- on the device
def torch_gaussian(n: int, d: int, seed: int, device) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn((n, d), generator=g, device=device, dtype=torch.float32)


def torch_unit_rows(n: int, d: int, seed: int, device, chunk: int = 1 << 22) -> torch.Tensor:
    x = torch_gaussian(n, d, seed, device)
    for s in range(0, n, chunk):
        blk = x[s:s + chunk]
        blk.div_(torch.linalg.vector_norm(blk, dim=1, keepdim=True))
    return x


def torch_mixture(n: int, d: int, n_centres: int, seed: int, device, centres: torch.Tensor | None = None,
                  chunk: int = 1 << 22):
    """Mixture built in place in HBM, chunk by chunk (no host copy)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    if centres is None:
        centres = torch.randn((n_centres, d), generator=g, device=device) * CENTRE_STD
    x = torch.empty((n, d), dtype=torch.float32, device=device)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        comp = torch.randint(0, n_centres, (m,), generator=g, device=device)
        x[s:s + m] = torch.randn((m, d), generator=g, device=device) * SIGMA
        x[s:s + m] += centres.index_select(0, comp)
    return x, centres
