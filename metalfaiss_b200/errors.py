"""Error model mirroring python/metalfaiss/errors.py:13-163 of the reference.

Every C-ABI status maps to one exception class. Classes that the reference
raises as built-in exceptions (ValueError for bad arguments, RuntimeError for
bad state, python/metalfaiss/indexflat.py:84,123 and
python/metalfaiss/index/ivf_flat_index.py:81-82) also derive from those, so
callers written against the reference keep catching them.
"""
from __future__ import annotations

from enum import IntEnum
from typing import Optional


class ErrorCode(IntEnum):
    """FAISS-like codes, python/metalfaiss/errors.py:13-29, plus two device codes."""

    SUCCESS = 0
    READONLY = 1
    MEMORY = 2
    IO = 3
    RUNTIME = 4
    NOT_IMPLEMENTED = 5
    INVALID_ARGS = 6
    BAD_STATE = 7
    ASSERTION = 8
    METRIC = 9
    INDEX = 10
    THREAD = 11
    FILE_NOT_FOUND = 12
    PERMISSION = 13
    FORMAT = 14
    CUDA = 100
    TIMEOUT = 101


class MetalFaissError(Exception):
    """Base class; carries the code (python/metalfaiss/errors.py:31-50)."""

    def __init__(self, message: str, code: ErrorCode = ErrorCode.RUNTIME):
        super().__init__(message)
        self.code = code
        self.message = message

    def __str__(self) -> str:
        return f"[Error {self.code.name}] {self.message}"


class ReadOnlyError(MetalFaissError, RuntimeError):
    def __init__(self, message: str):
        super().__init__(message, ErrorCode.READONLY)


class MemoryError(MetalFaissError):  # noqa: A001 - mirrors the reference's name
    def __init__(self, message: str):
        super().__init__(message, ErrorCode.MEMORY)


class RuntimeFaissError(MetalFaissError, RuntimeError):
    def __init__(self, message: str):
        super().__init__(message, ErrorCode.RUNTIME)


class NotImplementedFaissError(MetalFaissError, NotImplementedError):
    def __init__(self, message: str):
        super().__init__(message, ErrorCode.NOT_IMPLEMENTED)


class InvalidArgumentError(MetalFaissError, ValueError):
    def __init__(self, message: str):
        super().__init__(message, ErrorCode.INVALID_ARGS)


class BadStateError(MetalFaissError, RuntimeError):
    def __init__(self, message: str):
        super().__init__(message, ErrorCode.BAD_STATE)


class MetricError(MetalFaissError, ValueError):
    def __init__(self, message: str):
        super().__init__(message, ErrorCode.METRIC)


class CudaError(MetalFaissError, RuntimeError):
    def __init__(self, message: str):
        super().__init__(message, ErrorCode.CUDA)


class IOFaissError(MetalFaissError, OSError):
    """python/metalfaiss/errors.py:64-68 (IOError there)."""

    def __init__(self, message: str):
        super().__init__(message, ErrorCode.IO)


class FormatError(MetalFaissError, ValueError):
    """python/metalfaiss/errors.py:124-128: a file that is not a valid index."""

    def __init__(self, message: str):
        super().__init__(message, ErrorCode.FORMAT)


class DeviceTimeoutError(MetalFaissError, TimeoutError):
    def __init__(self, message: str):
        super().__init__(message, ErrorCode.TIMEOUT)


_BY_CODE = {
    ErrorCode.READONLY: ReadOnlyError,
    ErrorCode.MEMORY: MemoryError,
    ErrorCode.RUNTIME: RuntimeFaissError,
    ErrorCode.NOT_IMPLEMENTED: NotImplementedFaissError,
    ErrorCode.INVALID_ARGS: InvalidArgumentError,
    ErrorCode.BAD_STATE: BadStateError,
    ErrorCode.METRIC: MetricError,
    ErrorCode.CUDA: CudaError,
    ErrorCode.TIMEOUT: DeviceTimeoutError,
    ErrorCode.IO: IOFaissError,
    ErrorCode.FORMAT: FormatError,
}

_last_error: Optional[MetalFaissError] = None


def error_for(code: int, message: str) -> MetalFaissError:
    try:
        ec = ErrorCode(code)
    except ValueError:
        return MetalFaissError(f"{message} (status {code})", ErrorCode.RUNTIME)
    cls = _BY_CODE.get(ec)
    if cls is None:
        return MetalFaissError(message, ec)
    return cls(message)


def set_last_error(error: MetalFaissError) -> None:
    """python/metalfaiss/errors.py:133-136."""
    global _last_error
    _last_error = error


def get_last_error() -> Optional[MetalFaissError]:
    """python/metalfaiss/errors.py:138-140."""
    return _last_error


def clear_last_error() -> None:
    """python/metalfaiss/errors.py:142-145."""
    global _last_error
    _last_error = None


def check_error(code: int, message: str = "") -> None:
    """Raise the mapped exception for a non-zero status (python/metalfaiss/errors.py:147-163)."""
    if code != ErrorCode.SUCCESS:
        err = error_for(code, message or f"operation failed with status {code}")
        set_last_error(err)
        raise err
