"""Error taxonomy of the reference (src/error.rs:24-36) and svl_status codes.

Every C-ABI call returns an ``svl_status``; :func:`raise_for_status` turns a
non-zero code into the matching exception so Python callers see the same
variants the Rust ``Result<T, Error>`` carries.
"""

from __future__ import annotations

OK = 0
USAGE = 1
IO = 2
CORRUPT = 3
LIMIT_EXCEEDED = 4
UNSUPPORTED = 5
INTERNAL = 6


class SvlError(Exception):
    """Base class; ``code`` is the svl_status value."""

    code = INTERNAL


class UsageError(SvlError):
    code = USAGE


class IoError(SvlError):
    code = IO


class CorruptError(SvlError):
    code = CORRUPT


class LimitExceededError(SvlError):
    code = LIMIT_EXCEEDED


class UnsupportedError(SvlError):
    code = UNSUPPORTED


class InternalError(SvlError):
    code = INTERNAL


_BY_CODE = {
    USAGE: UsageError,
    IO: IoError,
    CORRUPT: CorruptError,
    LIMIT_EXCEEDED: LimitExceededError,
    UNSUPPORTED: UnsupportedError,
    INTERNAL: InternalError,
}


def error_for(code: int, message: str) -> SvlError:
    return _BY_CODE.get(code, InternalError)(message)


def raise_for_status(code: int, message: str = "") -> None:
    if code != OK:
        raise error_for(code, message or f"status {code}")
