"""The C-ABI library loads without a GPU and exports every function the
public headers declare (include/svl_gpu.h, include/svl_gpu_testing.h,
include/svl_tokenizer.h, include/svl_bundle.h)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared(header):
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / header).read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(svl_[a-z0-9_]+)\s*\(", text)))


@pytest.mark.parametrize("header", ["svl_gpu.h", "svl_gpu_testing.h", "svl_tokenizer.h", "svl_bundle.h"])
def test_library_exports_every_declared_symbol(header):
    from svl._abi import LIBRARY_PATH

    lib = ctypes.CDLL(str(LIBRARY_PATH))
    names = declared(header)
    assert len(names) >= 2
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_python_prototypes_cover_the_public_header():
    from svl._abi import PROTOTYPES

    assert set(declared("svl_gpu.h")) == set(PROTOTYPES)


def test_python_prototypes_cover_the_tokenizer_header():
    from svl.tokenizer import PROTOTYPES

    assert set(declared("svl_tokenizer.h")) == set(PROTOTYPES)


def test_python_prototypes_cover_the_bundle_header():
    from svl.bundle import PROTOTYPES

    assert set(declared("svl_bundle.h")) == set(PROTOTYPES)


def test_abi_version_without_a_gpu():
    from svl._abi import load_library

    assert load_library().svl_abi_version() == 1


def _c_arity(headers):
    """Argument count of every svl_* prototype in the public headers."""
    out = {}
    for h in headers:
        text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / h).read_text(), flags=re.S)
        for name, args in re.findall(r"\b(svl_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
            args = args.strip()
            out[name] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def test_integration_rust_bindings_match_the_headers():
    """INTEGRATION.md's Rust `extern "C"` blocks declare every public entry
    point with the C prototype's number of arguments."""
    # array types ([u8; 32]) hold a ';' of their own
    doc = re.sub(r"\[(\w+);\s*(\d+)\]", r"[\1 x \2]", (ROOT / "INTEGRATION.md").read_text())
    rust = {}
    for name, args in re.findall(r"pub fn (svl_[a-z0-9_]+)\s*\(([^;]*?)\)\s*(?:->\s*[\w:]+)?\s*;", doc, flags=re.S):
        args = re.sub(r"/\*.*?\*/", "", args).strip()
        rust[name] = 0 if not args else args.count(",") + 1
    c = _c_arity(["svl_gpu.h", "svl_tokenizer.h", "svl_bundle.h"])
    assert set(rust) == set(c), (sorted(set(c) - set(rust)), sorted(set(rust) - set(c)))
    wrong = {n: (rust[n], c[n]) for n in c if rust[n] != c[n]}
    assert not wrong, wrong


@pytest.mark.parametrize("header,module", [("svl_gpu.h", "svl._abi"), ("svl_tokenizer.h", "svl.tokenizer"),
                                           ("svl_bundle.h", "svl.bundle")])
def test_python_prototypes_have_the_c_arities(header, module):
    """Each ctypes prototype passes as many arguments as its C prototype takes."""
    import importlib

    protos = importlib.import_module(module).PROTOTYPES
    c = _c_arity([header])
    wrong = {n: (len(args), c[n]) for n, (_, args) in protos.items() if len(args) != c[n]}
    assert not wrong, wrong
