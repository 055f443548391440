"""Seeded synthetic models and inputs for the benchmark configurations.

No public dataset or checkpoint is involved: the production encoder's shapes
come from the frozen manifest (text_config of the reference's
fixtures/model/manifest.json, with the per-layer-input width 512 of
docs/adr/0004-text-embeddings.md and the manifest's special ids pad 0,
eos 1, bos 2), the weights are random N(0, 0.02), and token ids are uniform.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from .config import TextConfig

SEARCH_QUERY_PREFIX_IDS = [2, 8071, 236787, 3927, 1354, 1109, 7609, 236787]  # <bos> + "task: search result | query: "
EOS_ID = 1


def manifest_config_dict() -> dict:
    here = Path(__file__).resolve().parent
    # the package ships a copy of the manifest's text_config next to this file
    d = json.loads((here / "manifest_text_config.json").read_text())
    d = dict(d)
    d.setdefault("hidden_size_per_layer_input", 512)
    d.setdefault("pad_token_id", 0)
    d.setdefault("eos_token_id", 1)
    d.setdefault("bos_token_id", 2)
    return d


def manifest_config(num_layers: int | None = None, vocab_size: int | None = None) -> TextConfig:
    """The production encoder shape; optionally fewer layers / a smaller vocab
    (the last layer stays full attention, as config.rs requires)."""
    d = manifest_config_dict()
    if num_layers is not None:
        types = d["layer_types"][:num_layers]
        types[-1] = "full_attention"
        d["layer_types"] = types
        d["num_hidden_layers"] = num_layers
        plc = {}
        for i, t in enumerate(types):
            if t == "full_attention":
                plc[str(i)] = {"head_dim": 512, "num_key_value_heads": 1}
        d["per_layer_config"] = plc
    if vocab_size is not None:
        d["vocab_size"] = vocab_size
    return TextConfig.from_json_value(d)


def random_weights(config: TextConfig, seed: int = 1234, std: float = 0.02, unit_norms: bool = False) -> dict:
    """Every tensor of config.tensor_shapes() ~ N(0, std), float32, drawn in
    inventory order from default_rng(seed).  With unit_norms, norm weights and
    layer scalars are 1 + N(0, std) instead (a stress model whose attention
    logits and activations are unit scale)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in config.tensor_shapes():
        a = rng.standard_normal(int(np.prod(shape)), dtype=np.float32).reshape(shape)
        a *= np.float32(std)
        if unit_norms and (name.endswith("norm.weight") or name.endswith("layer_scalar")):
            a += np.float32(1.0)
        out[name] = a
    return out


def config1_ids(seed: int = 0, length: int = 32, vocab: int = 262144) -> np.ndarray:
    """the SearchQuery prefix ids, uniform ids in
    [2, vocab), then eos."""
    rng = np.random.default_rng(seed)
    body = rng.integers(2, vocab, size=length - len(SEARCH_QUERY_PREFIX_IDS) - 1, dtype=np.int64)
    return np.concatenate([SEARCH_QUERY_PREFIX_IDS, body, [EOS_ID]]).astype(np.uint32)


def config2_batch(seed: int = 2, batch: int = 64, lo: int = 64, hi: int = 512, vocab: int = 262144):
    """lengths ~ U[lo, hi], ids ~ U[2, vocab)."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(lo, hi + 1, size=batch)
    return [rng.integers(2, vocab, size=int(n), dtype=np.int64).astype(np.uint32) for n in lengths]


def config3_batch(seed: int = 3, batch: int = 8, length: int = 2048, vocab: int = 262144):
    rng = np.random.default_rng(seed)
    return [rng.integers(2, vocab, size=length, dtype=np.int64).astype(np.uint32) for _ in range(batch)]


def config5_lengths(seed: int = 5, n: int = 65536) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.clip(np.rint(rng.lognormal(np.log(200.0), 0.8, size=n)), 8, 2048).astype(np.int64)


def unit_rows(rng, n: int, dim: int) -> np.ndarray:
    x = rng.standard_normal((n, dim), dtype=np.float32)
    x /= np.linalg.norm(x.astype(np.float64), axis=1, keepdims=True).astype(np.float32)
    return x
