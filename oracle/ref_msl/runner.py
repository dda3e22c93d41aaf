"""Launches the CPU build of the reference's Metal kernels (oracle only)."""
from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np

_OUT = Path(__file__).resolve().parent.parent / "_ref"
_lib = None
_meta = None
_NP = {"float": np.float32, "int": np.int32, "uint": np.uint32}


def _load():
    global _lib, _meta
    if _lib is None:
        _lib = ctypes.CDLL(str(_OUT / "libivf_kernels_ref.so"))
        _meta = {k["name"]: k for k in json.loads((_OUT / "kernels.json").read_text())}
    return _lib, _meta


def available() -> bool:
    return (_OUT / "libivf_kernels_ref.so").exists()


def run(name, inputs, outputs, grid, threadgroup):
    """inputs/outputs: contiguous numpy arrays in the kernel's buffer order."""
    from .build_ref import CTYPES

    lib, meta = _load()
    m = meta[name]
    names = m["inputs"] + m["outputs"]
    bufs = list(inputs) + list(outputs)
    for nm, b in zip(names, bufs):
        want = _NP[CTYPES[nm]]
        if b.dtype != want:
            raise TypeError(f"{name}.{nm}: dtype {b.dtype}, kernel expects {np.dtype(want)}")
        if not b.flags.c_contiguous:
            raise ValueError(f"{name}.{nm} must be contiguous")
    arr = (ctypes.c_void_p * len(bufs))(*[b.ctypes.data for b in bufs])
    fn = getattr(lib, f"run_{name}")
    fn.argtypes = [ctypes.c_void_p, ctypes.c_uint, ctypes.c_uint]
    fn(arr, int(grid[0]), int(threadgroup[0]))
