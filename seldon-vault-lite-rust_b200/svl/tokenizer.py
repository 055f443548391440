"""Frozen-model BPE tokenizer (src/model/tokenizer.rs) over the C ABI of
include/svl_tokenizer.h.

Same names, argument meanings and error variants as the reference:
``Tokenizer.load`` / ``from_json_str`` (tokenizer.rs:85-103) raise
CorruptError for an inconsistent document, UnsupportedError for another
pipeline and LimitExceededError past a cap; ``encode`` (:392-434) and
``decode`` (:441-466) follow the reference's pipeline exactly (the C++ side
runs it; there is no Python fallback).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

from . import errors
from ._abi import ErrBuf, load_library

MAX_TOKENIZER_FILE_BYTES = 64 * 1024 * 1024  # tokenizer.rs:25
MAX_INPUT_BYTES = 1024 * 1024                 # tokenizer.rs:37
MAX_TOKENS = 262_144                          # tokenizer.rs:43

c_size = ctypes.c_size_t
c_u32 = ctypes.c_uint32
c_ptr = ctypes.c_void_p


class SvlTokenizerInfo(ctypes.Structure):
    _fields_ = [
        ("vocab_size", ctypes.c_uint64),
        ("max_token_id", c_u32),
        ("bos_id", c_u32),
        ("eos_id", c_u32),
        ("unk_id", c_u32),
        ("pad_id", c_u32),
        ("has_pad", c_u32),
    ]


# name -> (restype, argtypes) for include/svl_tokenizer.h
PROTOTYPES = {
    "svl_tokenizer_create": (ctypes.c_int, [ctypes.c_char_p, c_size, ctypes.POINTER(c_ptr), ctypes.c_char_p, c_size]),
    "svl_tokenizer_destroy": (None, [c_ptr]),
    "svl_tokenizer_encode": (ctypes.c_int, [c_ptr, ctypes.c_char_p, c_size, ctypes.c_int, c_ptr, c_size,
                                            ctypes.POINTER(c_size), ctypes.c_char_p, c_size]),
    "svl_tokenizer_encode_batch": (ctypes.c_int, [c_ptr, c_ptr, c_ptr, ctypes.c_uint64, ctypes.c_int, c_u32, c_ptr,
                                                  ctypes.c_uint64, c_ptr, ctypes.POINTER(ctypes.c_uint64),
                                                  ctypes.c_char_p, c_size]),
    "svl_tokenizer_decode": (ctypes.c_int, [c_ptr, c_ptr, c_size, ctypes.c_int, c_ptr, c_size,
                                            ctypes.POINTER(c_size), ctypes.c_char_p, c_size]),
    "svl_tokenizer_token_id": (ctypes.c_int, [c_ptr, ctypes.c_char_p, c_size, ctypes.POINTER(c_u32)]),
    "svl_tokenizer_token": (ctypes.c_int, [c_ptr, c_u32, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(c_size)]),
    "svl_tokenizer_is_special": (ctypes.c_int, [c_ptr, c_u32]),
    "svl_tokenizer_get_info": (ctypes.c_int, [c_ptr, ctypes.POINTER(SvlTokenizerInfo)]),
}


def _lib():
    lib = load_library()
    if not getattr(lib, "_svl_tokenizer_bound", False):
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        lib._svl_tokenizer_bound = True
    return lib


class Tokenizer:
    """tokenizer.rs ``Tokenizer``: immutable once built, safe to share."""

    def __init__(self, handle, lib):
        self._h = handle
        self._lib = lib
        info = SvlTokenizerInfo()
        errors.raise_for_status(lib.svl_tokenizer_get_info(handle, ctypes.byref(info)), "tokenizer info")
        self._info = info

    # -- construction (tokenizer.rs:85-103)
    @classmethod
    def load(cls, path: str | os.PathLike) -> "Tokenizer":
        p = Path(path)
        size = p.stat().st_size
        if size > MAX_TOKENIZER_FILE_BYTES:
            raise errors.LimitExceededError(
                f"{p} is {size} bytes, above the {MAX_TOKENIZER_FILE_BYTES}-byte cap")
        return cls.from_json_bytes(p.read_bytes())

    @classmethod
    def from_files(cls, files) -> "Tokenizer":
        """Tokenizer::from_files (tokenizer.rs:92-96): tokenizer.json of a model
        directory or a parsed bundle (svl.bundle.ModelFiles)."""
        return cls.from_json_bytes(bytes(files.read("tokenizer.json", MAX_TOKENIZER_FILE_BYTES)))

    @classmethod
    def from_json_str(cls, text: str) -> "Tokenizer":
        return cls.from_json_bytes(text.encode("utf-8"))

    @classmethod
    def from_json_bytes(cls, data: bytes) -> "Tokenizer":
        lib = _lib()
        h = c_ptr()
        eb = ErrBuf()
        eb.check(lib.svl_tokenizer_create(data, len(data), ctypes.byref(h), *eb.args))
        return cls(h, lib)

    def close(self) -> None:
        if self._h:
            self._lib.svl_tokenizer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- encode / decode (tokenizer.rs:392-466)
    def encode(self, text: str, add_special_tokens: bool) -> list[int]:
        return self.encode_array(text, add_special_tokens).tolist()

    def encode_array(self, text: str, add_special_tokens: bool) -> np.ndarray:
        """``encode`` as a uint32 array (what ``TextModel.embed_ids`` takes)."""
        data = text.encode("utf-8")
        if len(data) > MAX_INPUT_BYTES:
            raise errors.LimitExceededError(
                f"tokenizer input is {len(data)} bytes, above the {MAX_INPUT_BYTES}-byte cap")
        out = np.empty(len(data) + 2, np.uint32)  # at most one token per byte, plus <bos> / <eos>
        n = c_size()
        eb = ErrBuf()
        eb.check(self._lib.svl_tokenizer_encode(self._h, data, len(data), int(bool(add_special_tokens)),
                                                out.ctypes.data, out.size, ctypes.byref(n), *eb.args))
        return out[: n.value].copy()

    def encode_batch(self, texts, add_special_tokens: bool, threads: int = 0):
        """``encode`` of many texts in one call on up to ``threads`` host
        threads (0: all of them).  Returns (ids uint32[T], cu_seqlens
        uint64[n + 1]), the packed layout ``TextModel.embed_packed`` takes;
        the same ids as per-text ``encode`` calls, whatever the thread count."""
        data = [t.encode("utf-8") for t in texts]
        offsets = np.zeros(len(data) + 1, np.uint64)
        np.cumsum([len(d) for d in data], out=offsets[1:])
        blob = b"".join(data)
        cap = int(offsets[-1]) + 2 * len(data)
        ids = np.empty(max(cap, 1), np.uint32)
        cu = np.zeros(len(data) + 1, np.uint64)
        failed = ctypes.c_uint64()
        eb = ErrBuf()
        eb.check(self._lib.svl_tokenizer_encode_batch(self._h, blob, offsets.ctypes.data, len(data),
                                                      int(bool(add_special_tokens)), threads, ids.ctypes.data, cap,
                                                      cu.ctypes.data, ctypes.byref(failed), *eb.args))
        return ids[: int(cu[-1])].copy(), cu

    def decode(self, ids, skip_special_tokens: bool) -> str:
        arr = np.ascontiguousarray(np.asarray(ids, dtype=np.int64))
        if arr.size and (arr.min() < 0 or arr.max() > 0xFFFFFFFF):
            bad = int(arr[(arr < 0) | (arr > 0xFFFFFFFF)][0])
            raise errors.CorruptError(f"cannot decode unknown token id {bad}")
        ids32 = arr.astype(np.uint32)
        n = c_size()
        eb = ErrBuf()
        skip = int(bool(skip_special_tokens))
        eb.check(self._lib.svl_tokenizer_decode(self._h, ids32.ctypes.data, ids32.size, skip, None, 0,
                                                ctypes.byref(n), *eb.args))
        buf = ctypes.create_string_buffer(max(n.value, 1))
        eb.check(self._lib.svl_tokenizer_decode(self._h, ids32.ctypes.data, ids32.size, skip, buf, n.value,
                                                ctypes.byref(n), *eb.args))
        return buf.raw[: n.value].decode("utf-8")

    # -- accessors (tokenizer.rs:469-516)
    def token_id(self, token: str) -> int | None:
        data = token.encode("utf-8")
        out = c_u32()
        return out.value if self._lib.svl_tokenizer_token_id(self._h, data, len(data), ctypes.byref(out)) else None

    def token(self, id: int) -> str | None:
        if not 0 <= id <= 0xFFFFFFFF:
            return None
        p = ctypes.c_char_p()
        n = c_size()
        if not self._lib.svl_tokenizer_token(self._h, id, ctypes.byref(p), ctypes.byref(n)):
            return None
        return ctypes.string_at(p, n.value).decode("utf-8")

    def vocab_size(self) -> int:
        return int(self._info.vocab_size)

    def max_token_id(self) -> int:
        return int(self._info.max_token_id)

    def bos_id(self) -> int:
        return int(self._info.bos_id)

    def eos_id(self) -> int:
        return int(self._info.eos_id)

    def unk_id(self) -> int:
        return int(self._info.unk_id)

    def pad_id(self) -> int | None:
        return int(self._info.pad_id) if self._info.has_pad else None

    def is_special_id(self, id: int) -> bool:
        return 0 <= id <= 0xFFFFFFFF and bool(self._lib.svl_tokenizer_is_special(self._h, id))
