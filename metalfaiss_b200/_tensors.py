"""Input/output buffer helpers (torch is used for buffers and copies only)."""
from __future__ import annotations

import numpy as np
import torch

from .errors import InvalidArgumentError


def default_device(device=None) -> torch.device:
    if device is None:
        idx = torch.cuda.current_device() if torch.cuda.is_available() else 0
        return torch.device("cuda", idx)
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device() if torch.cuda.is_available() else 0)
    return dev


def padded_dim(d: int) -> int:
    """Rows are stored with a length that is a multiple of 4 (16-byte vector loads)."""
    return (d + 3) // 4 * 4


# Up to this padded dimension the tensor-core scan can derive the rows' tf32
# residuals itself; above it they must be stored (mf_tf32_residual at add
# time). Loading stored residuals is faster, so indexes store them unless
# asked to save the memory (residuals=False), which halves their footprint.
RESIDUAL_FREE_MAX_D = 128


def stores_residuals(dp: int, wanted: bool = True) -> bool:
    return wanted or dp > RESIDUAL_FREE_MAX_D


def as_matrix(xs, d: int, device: torch.device, name: str = "xs") -> torch.Tensor:
    """(n, d) input of any array-like → contiguous fp32 (n, padded_dim(d)) on `device`."""
    if torch.is_tensor(xs):
        t = xs
    else:
        arr = np.asarray(xs, dtype=np.float32)
        if arr.dtype != np.float32:
            arr = arr.astype(np.float32)
        t = torch.from_numpy(np.ascontiguousarray(arr))
    if t.dim() == 1:
        t = t.reshape(1, -1) if t.numel() else t.reshape(0, d)
    if t.dim() != 2:
        raise InvalidArgumentError(f"{name} must be 2-D (n, d); got shape {tuple(t.shape)}")
    if t.shape[1] != d:
        raise InvalidArgumentError(
            f"{name} dimension {t.shape[1]} does not match index dimension {d}")
    t = t.to(device=device, dtype=torch.float32)
    dp = padded_dim(d)
    if dp != d:
        out = torch.zeros((t.shape[0], dp), dtype=torch.float32, device=device)
        out[:, :d] = t
        return out
    return t.contiguous()


def as_ids(ids, n: int, device: torch.device) -> torch.Tensor:
    if torch.is_tensor(ids):
        t = ids.to(device=device, dtype=torch.int64)
    else:
        t = torch.from_numpy(np.ascontiguousarray(np.asarray(ids, dtype=np.int64))).to(device)
    t = t.reshape(-1).contiguous()
    if t.numel() != n:
        raise InvalidArgumentError(f"got {t.numel()} ids for {n} vectors")
    return t


class GrowBuffer:
    """Capacity-doubling device array (rows × row_shape) so repeated add() calls
    append in amortised O(new rows) instead of re-concatenating the whole bank
    (the reference concatenates on every add, python/metalfaiss/indexflat.py:56,64)."""

    def __init__(self, row_shape, dtype, device):
        self.row_shape = tuple(row_shape)
        self.dtype = dtype
        self.device = device
        self.buf = None
        self.n = 0

    def append(self, rows: torch.Tensor) -> None:
        m = rows.shape[0]
        need = self.n + m
        if self.buf is None or self.buf.shape[0] < need:
            cap = max(need, 2 * (self.buf.shape[0] if self.buf is not None else 0), 1024)
            nb = torch.empty((cap, *self.row_shape), dtype=self.dtype, device=self.device)
            if self.n:
                nb[: self.n].copy_(self.buf[: self.n])
            self.buf = nb
        self.buf[self.n:need].copy_(rows)
        self.n = need

    def view(self) -> torch.Tensor:
        if self.buf is None:
            return torch.empty((0, *self.row_shape), dtype=self.dtype, device=self.device)
        return self.buf[: self.n]

    def reset(self) -> None:
        self.buf = None
        self.n = 0
