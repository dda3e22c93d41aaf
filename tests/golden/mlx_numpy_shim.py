"""A numpy stand-in for the `mlx.core` API, enough to import and run the
reference's own search-path modules on the CPU of this container (MLX is not
installable here). Used only by make_golden.py to produce the committed
golden vectors; nothing at test or run time imports it.

What it reproduces: the reference's composition logic (which ops, in which
order, on which arrays). What it does not: MLX's floating-point kernels
(matmul blocking, reduction order) and MLX's PRNG; argsort is numpy's stable
sort. `fast.metal_kernel` runs the Metal source strings through the C++ build
of oracle/ref_msl (dispatchThreads semantics: `grid` counts threads).
"""
from __future__ import annotations

import sys
import types

import numpy as np

float32, float16, int32, int64, uint32, uint8, bool_ = (np.float32, np.float16, np.int32, np.int64,
                                                       np.uint32, np.uint8, np.bool_)
int8, int16, uint16, uint64, float64 = np.int8, np.int16, np.uint16, np.uint64, np.float64


class array(np.ndarray):
    def __new__(cls, data, dtype=None):
        return np.asarray(data, dtype=dtype).view(cls)

    def item(self):  # noqa: D401 - mirrors mx.array.item
        return np.ndarray.item(self)

    def astype(self, dtype, *a, **k):
        return np.ndarray.astype(self, dtype).view(array)


def _a(x):
    return np.asarray(x).view(array) if not isinstance(x, array) else x


def _wrap(fn):
    def f(*args, **kw):
        out = fn(*args, **kw)
        return _a(out) if isinstance(out, np.ndarray) or np.isscalar(out) else out
    return f


sum = _wrap(lambda x, axis=None, keepdims=False, dtype=None:
            np.sum(x, axis=axis, keepdims=keepdims, dtype=dtype))
max = _wrap(lambda x, axis=None, keepdims=False: np.max(x, axis=axis, keepdims=keepdims))
min = _wrap(lambda x, axis=None, keepdims=False: np.min(x, axis=axis, keepdims=keepdims))
mean = _wrap(lambda x, axis=None, keepdims=False: np.mean(x, axis=axis, keepdims=keepdims))
square = _wrap(np.square)
sqrt = _wrap(np.sqrt)
abs = _wrap(np.abs)
log = _wrap(np.log)
negative = _wrap(np.negative)
subtract = _wrap(np.subtract)
add = _wrap(np.add)
multiply = _wrap(np.multiply)
divide = _wrap(lambda a, b: np.divide(a, b))
maximum = _wrap(np.maximum)
minimum = _wrap(np.minimum)
matmul = _wrap(np.matmul)
dot = _wrap(np.dot)
transpose = _wrap(lambda x, axes=None: np.transpose(x, axes))
where = _wrap(np.where)
greater = _wrap(np.greater)
less_equal = _wrap(np.less_equal)
equal = _wrap(np.equal)
zeros_like = _wrap(np.zeros_like)
ones_like = _wrap(np.ones_like)
zeros = _wrap(lambda shape, dtype=np.float32: np.zeros(shape, dtype))
ones = _wrap(lambda shape, dtype=np.float32: np.ones(shape, dtype))
arange = _wrap(lambda *a, dtype=None: np.arange(*a, dtype=dtype))
concatenate = _wrap(lambda xs, axis=0: np.concatenate(xs, axis=axis))
stack = _wrap(lambda xs, axis=0: np.stack(xs, axis=axis))
argmin = _wrap(lambda x, axis=None: np.argmin(x, axis=axis).astype(np.uint32))
argsort = _wrap(lambda x, axis=-1: np.argsort(x, axis=axis, kind="stable").astype(np.uint32))
take = _wrap(lambda x, idx, axis=None: np.take(x, np.asarray(idx).astype(np.int64), axis=axis))
take_along_axis = _wrap(lambda x, idx, axis: np.take_along_axis(x, np.asarray(idx).astype(np.int64), axis))
reshape = _wrap(lambda x, shape: np.reshape(x, shape))
copy = _wrap(np.copy)
topk = _wrap(lambda x, k, axis=-1: np.sort(x, axis=axis)[..., -k:])
not_equal = _wrap(np.not_equal)
less = _wrap(np.less)
greater_equal = _wrap(np.greater_equal)
all = _wrap(lambda x, axis=None: np.all(x, axis=axis))  # noqa: A001 - MLX's name
any = _wrap(lambda x, axis=None: np.any(x, axis=axis))  # noqa: A001 - MLX's name
bitwise_and = _wrap(lambda a, b: np.bitwise_and(a, np.asarray(b, np.asarray(a).dtype)))
bitwise_or = _wrap(lambda a, b: np.bitwise_or(a, np.asarray(b, np.asarray(a).dtype)))
bitwise_xor = _wrap(lambda a, b: np.bitwise_xor(a, np.asarray(b, np.asarray(a).dtype)))
right_shift = _wrap(lambda a, b: np.right_shift(a, np.asarray(b, np.asarray(a).dtype)))
left_shift = _wrap(lambda a, b: np.left_shift(a, np.asarray(b, np.asarray(a).dtype)))


def _scatter(a, indices, updates, axis=0):
    out = np.array(a, copy=True)
    idx = np.asarray(indices).astype(np.int64)
    sl = [slice(None)] * out.ndim
    sl[axis] = idx
    out[tuple(sl)] = np.asarray(updates)
    return out


scatter = _wrap(_scatter)
broadcast_to = _wrap(lambda x, shape: np.broadcast_to(np.asarray(x), shape).copy())


def eval(*arrays):  # noqa: A001 - MLX's name
    return None


def compile(fn=None, **kw):  # noqa: A001 - MLX's name
    return fn if fn is not None else (lambda f: f)


def save(*a, **k):
    raise NotImplementedError("mx.save is outside the golden-vector generator")


class _Device:
    def __init__(self, kind):
        self.kind = kind

    def __repr__(self):
        return f"Device({self.kind}, 0)"


gpu = _Device("gpu")
cpu = _Device("cpu")
_default = [gpu]


def default_device():
    return _default[0]


def set_default_device(dev):
    _default[0] = dev


class stream:
    def __init__(self, *a, **k):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


# ------------------------------------------------------------------ random
class _Random(types.SimpleNamespace):
    pass


random = _Random()
random._gen = np.random.Generator(np.random.PCG64(0))
random.log = []  # (call, result) of every draw, for replay in the oracle


def _seed(s):
    random._gen = np.random.Generator(np.random.PCG64(int(s)))


def _perm(n, key=None):
    p = random._gen.permutation(int(n)).astype(np.uint32)
    random.log.append(("permutation", p.copy()))
    return _a(p)


def _randint(low, high, shape=(1,), dtype=np.int32, key=None):
    r = random._gen.integers(int(low), int(high), size=shape).astype(dtype)
    random.log.append(("randint", r.copy()))
    return _a(r)


def _normal(shape=(1,), dtype=np.float32, loc=0.0, scale=1.0, key=None):
    r = (random._gen.standard_normal(size=shape) * scale + loc).astype(dtype or np.float32)
    random.log.append(("normal", r.copy()))
    return _a(r)


random.seed = _seed
random.permutation = _perm
random.randint = _randint
random.normal = _normal
random.key = lambda s: s


# -------------------------------------------------------------------- fast
class _Fast(types.SimpleNamespace):
    pass


fast = _Fast()


def _metal_kernel(name, input_names, output_names, source, header="", ensure_row_contiguous=True,
                  **kw):
    from oracle.ref_msl import runner

    def call(inputs, output_shapes, output_dtypes, grid, threadgroup, **kw2):
        ins = [np.ascontiguousarray(np.asarray(x)) for x in inputs]
        outs = [np.zeros(s, dtype=np.dtype(t)) for s, t in zip(output_shapes, output_dtypes)]
        runner.run(name, ins, outs, grid, threadgroup)
        return [_a(o) for o in outs]

    return call


fast.metal_kernel = _metal_kernel


def install():
    """Registers this module as `mlx` / `mlx.core` in sys.modules."""
    pkg = types.ModuleType("mlx")
    pkg.__path__ = []
    pkg.core = sys.modules[__name__]
    sys.modules["mlx"] = pkg
    sys.modules["mlx.core"] = sys.modules[__name__]
