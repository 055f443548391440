"""Weight ingress from `.svlm` bundles on the B200 (src/model/source.rs,
tests/bundle_loading.rs): a model loaded from a bundle file is the model
loaded from its directory (same fingerprint, parameters and embeddings, bit
for bit), and BF16 weights in a bundle, widened on the device by
svl_model_create, embed exactly as the same values widened to FP32 on the
host (src/binary/bf16.rs:40: the widening is exact)."""

from __future__ import annotations

import json
import struct

import numpy as np
import pytest

from conftest import GOLDEN
from svl import bundle, errors, safetensors
from svl.bundle import Bundle, SectionInput, SectionRole
from svl.text import TextModel

pytestmark = pytest.mark.gpu

TINY = GOLDEN / "tiny_text"
IDS = [2, 5, 6, 7, 1]


def _tiny_bundle(path, weights: bytes, extra=()):
    path.write_bytes(Bundle.build([
        SectionInput("config.json", SectionRole.Config, (TINY / "config.json").read_bytes()),
        SectionInput("model.safetensors", SectionRole.Weights, weights),
        *extra,
    ]))
    return path


def _bf16_safetensors(tensors) -> tuple[bytes, dict]:
    """The tensors rounded to BF16 (nearest even) as a safetensors file, and
    the same BF16 values widened back to FP32."""
    header, blobs, widened, off = {}, [], {}, 0
    for name, entry in tensors.items():
        f = np.ascontiguousarray(entry.to_f32(), np.float32)
        u = f.view(np.uint32).astype(np.uint64)
        bits = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        raw = bits.tobytes()
        header[name] = {"dtype": "BF16", "shape": list(f.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
        widened[name] = (bits.astype(np.uint32) << 16).view(np.float32).reshape(f.shape)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    return struct.pack("<Q", len(h)) + h + b"".join(blobs), widened


def test_text_model_from_bundle_matches_the_directory(tmp_path):
    """tests/bundle_loading.rs:46-77 and :99-114."""
    path = _tiny_bundle(tmp_path / "tiny.svlm", (TINY / "model.safetensors").read_bytes())
    from_bundle = bundle.load_text_model(path)
    from_directory = TextModel.load(TINY)
    assert from_bundle.config().vocab_size == from_directory.config().vocab_size
    assert from_bundle.config().hidden_size == from_directory.config().hidden_size
    assert from_bundle.fingerprint_hex() == from_directory.fingerprint_hex() is not None
    assert from_bundle.parameters() == from_directory.parameters()
    assert np.array_equal(from_bundle.embed_ids(IDS, 8), from_directory.embed_ids(IDS, 8))
    # and the directory path through the same loader
    assert np.array_equal(bundle.load_text_model(TINY).embed_ids(IDS, 8), from_directory.embed_ids(IDS, 8))


def test_bf16_weights_in_a_bundle_are_widened_exactly_on_the_device(tmp_path):
    tensors = safetensors.load(TINY / "model.safetensors")
    raw, widened = _bf16_safetensors(tensors)
    path = _tiny_bundle(tmp_path / "tiny_bf16.svlm", raw)
    from_bundle = bundle.load_text_model(path)
    cfg = from_bundle.config()
    host = TextModel(cfg, widened)
    for dim in (8, 4):
        assert np.array_equal(from_bundle.embed_ids(IDS, dim), host.embed_ids(IDS, dim))
    b = Bundle.parse(path.read_bytes())
    assert from_bundle.fingerprint_hex() == b.section("model.safetensors").sha256.hex()


def test_embedder_bundle_with_a_mismatched_tokenizer_is_corrupt(tmp_path):
    """TextEmbedder::from_files (text.rs:584-595): the tokenizer's vocabulary
    must match the model's (the reduced tokenizer's 694 entries do not match
    the tiny model's)."""
    tok = SectionInput("tokenizer.json", SectionRole.Tokenizer,
                       (GOLDEN / "tokenizer" / "mini_tokenizer.json").read_bytes())
    path = _tiny_bundle(tmp_path / "tiny_tok.svlm", (TINY / "model.safetensors").read_bytes(), (tok,))
    with pytest.raises(errors.CorruptError, match="vocabulary"):
        bundle.load_text_embedder(path)
