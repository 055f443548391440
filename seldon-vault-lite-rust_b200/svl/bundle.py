"""`.svlm` model bundles and bundle-or-directory model sources
(src/bundle/mod.rs, src/model/source.rs) over the C ABI of include/svl_bundle.h.

``Bundle.parse`` checks the structure, header CRC-32 and catalog digest;
``verify`` checks every section's SHA-256; ``Bundle.build`` writes the
deterministic bundle of a set of sections (the packer's format).
``load_text_model`` / ``load_text_embedder`` / ``load_tokenizer`` take either a
model directory or a bundle file, as the reference's loaders do: a file is
read, parsed and fully verified once, then the model is built from its
sections (``model.safetensors`` BF16 weights are widened to FP32 on the GPU by
``svl_model_create``).  Errors are the reference's variants.
"""

from __future__ import annotations

import ctypes
import enum
import os
from dataclasses import dataclass
from pathlib import Path

from . import errors
from ._abi import ErrBuf, load_library

MAX_BUNDLE_BYTES = 1 << 33                  # bundle/mod.rs:33
MAX_CONFIG_BYTES = 1024 * 1024              # config.rs:20
MAX_MODEL_FILE_BYTES = 4 * 1024 * 1024 * 1024  # weights.rs:25
MAX_TOKENIZER_FILE_BYTES = 64 * 1024 * 1024    # tokenizer.rs:25

c_u64 = ctypes.c_uint64
c_ptr = ctypes.c_void_p
c_size = ctypes.c_size_t


class SectionRole(enum.IntEnum):
    """bundle/mod.rs:49-58 (stable on-disk role bytes)."""

    Manifest = 0
    Config = 1
    Tokenizer = 2
    Processor = 3
    Weights = 4
    Other = 5


class SvlBundleSection(ctypes.Structure):
    _fields_ = [
        ("path", ctypes.c_void_p),
        ("path_len", c_u64),
        ("role", ctypes.c_uint32),
        ("reserved", ctypes.c_uint32),
        ("offset", c_u64),
        ("length", c_u64),
        ("sha256", ctypes.c_uint8 * 32),
        ("data", ctypes.c_void_p),
    ]


class SvlBundleInput(ctypes.Structure):
    _fields_ = [
        ("path", ctypes.c_char_p),
        ("path_len", c_u64),
        ("role", ctypes.c_uint32),
        ("reserved", ctypes.c_uint32),
        ("data", ctypes.c_void_p),
        ("length", c_u64),
    ]


# name -> (restype, argtypes) for include/svl_bundle.h
PROTOTYPES = {
    "svl_bundle_parse": (ctypes.c_int, [c_ptr, c_u64, ctypes.POINTER(c_ptr), ctypes.c_char_p, c_size]),
    "svl_bundle_destroy": (None, [c_ptr]),
    "svl_bundle_verify": (ctypes.c_int, [c_ptr, ctypes.c_char_p, c_size]),
    "svl_bundle_header_len": (c_u64, [c_ptr]),
    "svl_bundle_section_count": (c_u64, [c_ptr]),
    "svl_bundle_section_at": (ctypes.c_int, [c_ptr, c_u64, ctypes.POINTER(SvlBundleSection)]),
    "svl_bundle_find": (ctypes.c_int, [c_ptr, ctypes.c_char_p, c_u64, ctypes.POINTER(c_u64)]),
    "svl_bundle_build": (ctypes.c_int, [ctypes.POINTER(SvlBundleInput), c_u64, c_ptr, c_u64, ctypes.POINTER(c_u64),
                                        ctypes.c_char_p, c_size]),
    "svl_sha256": (None, [c_ptr, c_u64, ctypes.POINTER(ctypes.c_uint8 * 32)]),
    "svl_crc32": (ctypes.c_uint32, [c_ptr, c_u64]),
}


def _lib():
    lib = load_library()
    if not getattr(lib, "_svl_bundle_bound", False):
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        lib._svl_bundle_bound = True
    return lib


def sha256(data) -> bytes:
    """FIPS 180-4 SHA-256 (src/binary/sha256.rs) from the library."""
    b = bytes(data) if not isinstance(data, bytes) else data
    out = (ctypes.c_uint8 * 32)()
    _lib().svl_sha256(b, len(b), ctypes.byref(out))
    return bytes(out)


def crc32(data) -> int:
    """IEEE CRC-32 (src/binary/crc32.rs) from the library."""
    b = bytes(data) if not isinstance(data, bytes) else data
    return int(_lib().svl_crc32(b, len(b)))


@dataclass(frozen=True)
class SectionInput:
    """bundle/mod.rs ``SectionInput``: one section to build."""

    path: str
    role: SectionRole
    data: bytes


@dataclass(frozen=True)
class BundleSection:
    """bundle/mod.rs ``BundleSection``: one parsed section (data borrows the bundle)."""

    path: str
    role: SectionRole
    sha256: bytes
    offset: int
    data: memoryview

    def __len__(self) -> int:
        return len(self.data)


class Bundle:
    """bundle/mod.rs ``Bundle``: a parsed bundle over bytes it keeps alive."""

    def __init__(self, data: bytes, handle, lib):
        self._data = data
        self._h = handle
        self._lib = lib
        view = memoryview(data)
        self._sections = []
        for i in range(int(lib.svl_bundle_section_count(handle))):
            s = SvlBundleSection()
            errors.raise_for_status(lib.svl_bundle_section_at(handle, i, ctypes.byref(s)), "bundle section")
            path = ctypes.string_at(s.path, s.path_len).decode("utf-8")
            self._sections.append(BundleSection(path, SectionRole(s.role), bytes(s.sha256), int(s.offset),
                                                view[s.offset:s.offset + s.length]))

    @classmethod
    def parse(cls, data: bytes) -> "Bundle":
        data = bytes(data)
        lib = _lib()
        h = c_ptr()
        eb = ErrBuf()
        eb.check(lib.svl_bundle_parse(data, len(data), ctypes.byref(h), *eb.args))
        return cls(data, h, lib)

    @staticmethod
    def build(sections) -> bytes:
        """bundle/mod.rs ``Bundle::build`` (sorted by path, duplicates -> UsageError)."""
        lib = _lib()
        items = list(sections)
        keep = []
        arr = (SvlBundleInput * max(len(items), 1))()
        for i, s in enumerate(items):
            p = s.path.encode("utf-8")
            d = bytes(s.data)
            keep += [p, d]
            arr[i] = SvlBundleInput(p, len(p), int(s.role), 0, ctypes.cast(ctypes.c_char_p(d), c_ptr), len(d))
        n = c_u64()
        eb = ErrBuf()
        eb.check(lib.svl_bundle_build(arr, len(items), None, 0, ctypes.byref(n), *eb.args))
        out = ctypes.create_string_buffer(n.value)
        eb.check(lib.svl_bundle_build(arr, len(items), out, n.value, ctypes.byref(n), *eb.args))
        del keep
        return out.raw[: n.value]

    def close(self) -> None:
        if self._h:
            self._lib.svl_bundle_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def verify(self) -> None:
        eb = ErrBuf()
        eb.check(self._lib.svl_bundle_verify(self._h, *eb.args))

    def header_len(self) -> int:
        return int(self._lib.svl_bundle_header_len(self._h))

    def sections(self) -> list[BundleSection]:
        return list(self._sections)

    def section(self, path: str) -> BundleSection | None:
        p = path.encode("utf-8")
        idx = c_u64()
        if not self._lib.svl_bundle_find(self._h, p, len(p), ctypes.byref(idx)):
            return None
        return self._sections[idx.value]

    def data(self, path: str) -> memoryview | None:
        s = self.section(path)
        return None if s is None else s.data


def _safe_relative(path: str) -> bool:
    if not path or path.startswith("/") or "\\" in path or "\0" in path:
        return False
    return all(c not in ("", ".", "..") for c in path.split("/"))


class ModelFiles:
    """source.rs ``ModelFiles``: a model directory or a parsed bundle."""

    def __init__(self, directory: Path | None = None, bundle: Bundle | None = None):
        self._dir = directory
        self._bundle = bundle

    @classmethod
    def directory(cls, path) -> "ModelFiles":
        return cls(directory=Path(path))

    @classmethod
    def from_bundle(cls, bundle: Bundle) -> "ModelFiles":
        return cls(bundle=bundle)

    def read(self, path: str, cap: int):
        if not _safe_relative(path):
            raise errors.InternalError(f"model file path {path} is not a safe relative path")
        if self._bundle is None:
            p = self._dir / path
            try:
                size = p.stat().st_size
            except FileNotFoundError:
                raise errors.CorruptError(f"model file {path} is missing") from None
            if size > cap:
                raise errors.LimitExceededError(f"{path} is {size} bytes, above the {cap}-byte cap")
            return p.read_bytes()
        data = self._bundle.data(path)
        if data is None:
            raise errors.CorruptError(f"model bundle has no section {path}")
        if len(data) > cap:
            raise errors.LimitExceededError(f"bundle section {path} is {len(data)} bytes, above the {cap}-byte cap")
        return data

    def read_utf8(self, path: str, cap: int) -> str:
        try:
            return bytes(self.read(path, cap)).decode("utf-8")
        except UnicodeDecodeError:
            raise errors.CorruptError(f"{path} is not valid UTF-8") from None

    def section_sha256(self, path: str) -> bytes | None:
        if self._bundle is None:
            return None
        s = self._bundle.section(path)
        return None if s is None else s.sha256

    def contains(self, path: str) -> bool:
        if not _safe_relative(path):
            return False
        return (self._dir / path).is_file() if self._bundle is None else self._bundle.section(path) is not None


def with_source(path, load):
    """source.rs ``with_source``: a regular file is a bundle (read, parsed,
    every section verified); anything else a model directory."""
    p = Path(path)
    if p.is_file():
        size = p.stat().st_size
        if size > MAX_BUNDLE_BYTES:
            raise errors.LimitExceededError(f"{p} is {size} bytes, above the {MAX_BUNDLE_BYTES}-byte cap")
        bundle = Bundle.parse(p.read_bytes())
        bundle.verify()
        return load(ModelFiles.from_bundle(bundle))
    return load(ModelFiles.directory(p))


def load_text_model(path: str | os.PathLike, device: int = 0):
    """source.rs ``load_text_model``."""
    from .text import TextModel

    return with_source(path, lambda files: TextModel.from_files(files, device))


def load_text_embedder(path: str | os.PathLike, device: int = 0):
    """source.rs ``load_text_embedder``."""
    from .text import TextEmbedder

    return with_source(path, lambda files: TextEmbedder.from_files(files, device))


def load_tokenizer(path: str | os.PathLike):
    """``Tokenizer::from_files`` over a directory or bundle file."""
    from .tokenizer import Tokenizer

    return with_source(path, Tokenizer.from_files)
