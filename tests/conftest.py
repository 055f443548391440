"""Shared pytest setup: the `gpu` marker, import paths and golden fixtures."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "seldon-vault-lite-rust_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def tiny_config():
    from svl.config import TextConfig

    return TextConfig.from_file(GOLDEN / "tiny_text" / "config.json")


@pytest.fixture(scope="session")
def tiny_tensors():
    from svl import safetensors

    return safetensors.load(GOLDEN / "tiny_text" / "model.safetensors")


@pytest.fixture(scope="session")
def tiny_golden():
    return json.loads((GOLDEN / "tiny_text" / "golden.json").read_text())
