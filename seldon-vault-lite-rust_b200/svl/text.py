"""TextModel / ForwardOutput over libsvl_gpu.so -- the reference's text API
(src/model/text.rs:38-554) with its bodies on the B200.

Same names, argument meanings and error variants as the Rust types:

* ``TextModel.load(dir)`` / ``TextModel(config, tensors)``   (text.rs:93-126)
* ``forward(ids, capture_hidden)`` -> ``ForwardOutput``        (text.rs:150)
* ``forward_with_features(ids, features, start, count, ...)`` (text.rs:167)
* ``embed_ids(ids, dimension)``                                 (text.rs:546)
* ``ForwardOutput.embedding(dimension)``                        (text.rs:72)

plus batch entry points (``forward_batch``, ``embed_batch``,
``embed_batch_device``) that pack many sequences into one device call; the
reference has no batching (it embeds one sequence per call).

There is no CPU path: every call goes through the CUDA library, and a missing
library raises.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import errors, safetensors
from ._abi import PRECISION_FAST, PRECISION_SPLIT, ErrBuf, SvlModelOptions, load_library, tensor_views
from .config import MAX_TEXT_TOKENS, TextConfig

_P = ctypes.c_void_p


def _ptr(a):
    return None if a is None else a.ctypes.data


def pack(sequences) -> tuple[np.ndarray, np.ndarray]:
    """Packs a list of id sequences into (ids uint32[T], cu_seqlens uint64[B+1])."""
    seqs = [np.ascontiguousarray(s, dtype=np.uint32).ravel() for s in sequences]
    cu = np.zeros(len(seqs) + 1, np.uint64)
    np.cumsum([s.size for s in seqs], out=cu[1:])
    ids = np.concatenate(seqs) if seqs else np.zeros(0, np.uint32)
    return np.ascontiguousarray(ids, dtype=np.uint32), cu


@dataclass
class ForwardOutput:
    """Result of one forward pass (text.rs:38-75)."""

    _projected: np.ndarray
    _pooled: np.ndarray
    _normalized: np.ndarray
    _hidden_states: list

    def projected(self) -> np.ndarray:
        return self._projected

    def pooled(self) -> np.ndarray:
        return self._pooled

    def normalized(self) -> np.ndarray:
        return self._normalized

    def hidden_states(self) -> list:
        return self._hidden_states

    def embedding(self, dimension: int) -> np.ndarray:
        """truncate_and_normalize (kernels.rs:916-927): the leading dims, L2 again."""
        v = self._normalized
        if dimension == 0:
            raise errors.InternalError("embedding dimension must be positive")
        if dimension > v.size:
            raise errors.InternalError(f"cannot truncate {v.size} elements to {dimension}")
        head = v[:dimension].astype(np.float32)
        s = np.float32(0.0)
        for x in head:
            s = np.float32(s + x * x)
        if not np.isfinite(s) or s <= 0:
            raise errors.InternalError("cannot normalize a zero or non-finite vector")
        return (head * (np.float32(1.0) / np.sqrt(s))).astype(np.float32)


class TextModel:
    """FP32 EmbeddingGemma-2 text encoder resident on one B200."""

    def __init__(self, config: TextConfig, tensors: dict, device: int = 0, precision: str | None = None):
        """precision: None (the library default: "fast", or "split" when the
        SVL_PRECISION environment variable says so), "fast" (11-bit-significand
        tensor-core operands) or "split" (hi/lo-split TF32 products and FP32
        attention, ~22-bit products; see svl_precision in svl_gpu.h)."""
        self._lib = load_library()
        self._config = config
        cfg, keep_cfg = config.to_c()
        views, keep = tensor_views(tensors)
        handle = _P()
        eb = ErrBuf()
        if precision is None:
            eb.check(self._lib.svl_model_create(ctypes.byref(cfg), views, len(tensors), device, ctypes.byref(handle),
                                                *eb.args))
        else:
            if precision not in ("fast", "split"):
                raise errors.UsageError(f"unknown precision {precision!r} (fast or split)")
            opts = SvlModelOptions(PRECISION_SPLIT if precision == "split" else PRECISION_FAST)
            eb.check(self._lib.svl_model_create_ex(ctypes.byref(cfg), views, len(tensors), device,
                                                   ctypes.byref(opts), ctypes.byref(handle), *eb.args))
        self._h = handle
        self.device = device
        del keep, keep_cfg

    @classmethod
    def load(cls, model_dir, device: int = 0) -> "TextModel":
        """TextModel::load (text.rs:93): config.json + model.safetensors."""
        from .bundle import ModelFiles

        return cls.from_files(ModelFiles.directory(model_dir), device)

    @classmethod
    def from_files(cls, files, device: int = 0) -> "TextModel":
        """TextModel::from_files (text.rs:104-108) over a model directory or a
        parsed bundle (svl.bundle.ModelFiles).  The weights fingerprint is the
        SHA-256 recorded in the bundle header, or that of the directory's
        model.safetensors (weights.rs:80-96)."""
        from . import bundle

        config = TextConfig.from_json_str(files.read_utf8("config.json", bundle.MAX_CONFIG_BYTES))
        data = files.read("model.safetensors", bundle.MAX_MODEL_FILE_BYTES)
        digest = files.section_sha256("model.safetensors")
        if digest is None:
            digest = bundle.sha256(data)
        model = cls(config, safetensors.parse(data), device)
        model._fingerprint = digest.hex()
        return model

    def fingerprint_hex(self) -> str | None:
        """SHA-256 of the weights file this model was loaded from (text.rs:133-136);
        None for a model built from in-memory tensors."""
        return getattr(self, "_fingerprint", None)

    def close(self):
        if getattr(self, "_h", None):
            self._lib.svl_model_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def config(self) -> TextConfig:
        return self._config

    def precision(self) -> str:
        """"fast" or "split" (svl_model_precision)."""
        out = ctypes.c_uint32()
        self._lib.svl_model_precision(self._h, ctypes.byref(out))
        return "split" if out.value == PRECISION_SPLIT else "fast"

    def parameters(self) -> int:
        out = ctypes.c_uint64()
        self._lib.svl_model_parameters(self._h, ctypes.byref(out))
        return out.value

    # ------------------------------------------------------------- forward
    def forward_batch(self, sequences, capture_hidden=False, projected=False, features=None):
        """Forward over many sequences in one call.  Returns a dict with
        normalized [B, E], pooled [B, E], and optionally projected [T, E] and
        hidden_states [L+1, T, H]."""
        from ._abi import SvlFeatureSpan

        c = self._config
        ids, cu = pack(sequences)
        B = cu.size - 1
        T = int(cu[-1])
        normalized = np.empty((B, c.embedding_dim), np.float32)
        pooled = np.empty((B, c.embedding_dim), np.float32)
        proj = np.empty((T, c.embedding_dim), np.float32) if projected else None
        hidden = np.empty((c.num_hidden_layers + 1, T, c.hidden_size), np.float32) if capture_hidden else None
        feats = spans = None
        n_spans = 0
        if features:
            flat = []
            spans = (SvlFeatureSpan * len(features))()
            off = 0
            for i, (seq, start, rows) in enumerate(features):
                rows = np.ascontiguousarray(rows, np.float32).reshape(-1, c.hidden_size)
                spans[i] = SvlFeatureSpan(seq, start, rows.shape[0], 0, off)
                flat.append(rows.ravel())
                off += rows.size
            feats = np.ascontiguousarray(np.concatenate(flat), np.float32)
            n_spans = len(features)
        eb = ErrBuf()
        eb.check(self._lib.svl_forward_batch(self._h, _ptr(ids), _ptr(cu), B, _ptr(feats), spans, n_spans,
                                             _ptr(normalized), _ptr(pooled), _ptr(proj), _ptr(hidden), *eb.args))
        return {"normalized": normalized, "pooled": pooled, "projected": proj, "hidden_states": hidden, "cu": cu}

    def forward(self, input_ids, capture_hidden: bool = False) -> ForwardOutput:
        return self._forward_one(input_ids, capture_hidden, None)

    def forward_with_features(self, input_ids, features, feature_start: int, feature_count: int,
                              capture_hidden: bool = False) -> ForwardOutput:
        c = self._config
        features = np.ascontiguousarray(features, np.float32).ravel()
        if feature_count == 0:
            raise errors.CorruptError("multimodal feature replacement requires at least one token")
        if features.size != feature_count * c.hidden_size:
            raise errors.CorruptError(
                f"multimodal features have {features.size} values, expected {feature_count * c.hidden_size}")
        if feature_start + feature_count > len(input_ids):
            raise errors.CorruptError("multimodal feature range is outside the sequence")
        return self._forward_one(input_ids, capture_hidden, [(0, feature_start, features)])

    def _forward_one(self, input_ids, capture_hidden, features) -> ForwardOutput:
        ids = np.ascontiguousarray(input_ids, np.uint32).ravel()
        out = self.forward_batch([ids], capture_hidden=capture_hidden, projected=True, features=features)
        hidden = list(out["hidden_states"]) if capture_hidden else []
        return ForwardOutput(out["projected"], out["pooled"][0], out["normalized"][0], hidden)

    def embed_ids(self, input_ids, dimension: int) -> np.ndarray:
        return self.embed_batch([input_ids], dimension)[0]

    def embed_batch(self, sequences, dimension: int) -> np.ndarray:
        ids, cu = pack(sequences)
        return self.embed_packed(ids, cu, dimension)

    def embed_packed(self, ids: np.ndarray, cu: np.ndarray, dimension: int, out: np.ndarray | None = None) -> np.ndarray:
        """Host buffers in, host buffers out (pinned buffers avoid a staging copy)."""
        B = cu.size - 1
        if out is None:
            out = np.empty((B, dimension), np.float32)
        eb = ErrBuf()
        eb.check(self._lib.svl_embed_batch(self._h, _ptr(ids), _ptr(cu), B, dimension, _ptr(out), *eb.args))
        return out

    def embed_batch_device(self, d_ids_ptr: int, cu: np.ndarray, dimension: int, d_out_ptr: int, stream: int = 0):
        """Device ids / output (raw CUDA pointers), host cu_seqlens; asynchronous."""
        cu = np.ascontiguousarray(cu, np.uint64)
        eb = ErrBuf()
        eb.check(self._lib.svl_embed_batch_device(self._h, d_ids_ptr, _ptr(cu), cu.size - 1, dimension, d_out_ptr,
                                                  stream or None, *eb.args))

    def check(self):
        eb = ErrBuf()
        eb.check(self._lib.svl_model_check(self._h, *eb.args))


def validate_text_length(ids) -> None:
    """TextEmbedder::embed's length check (text.rs:619-624)."""
    if len(ids) > MAX_TEXT_TOKENS:
        raise errors.LimitExceededError(
            f"tokenized input has {len(ids)} tokens, above the {MAX_TEXT_TOKENS}-token context")


class TextEmbedder:
    """text.rs ``TextEmbedder`` (:590-626): the frozen tokenizer in front of a
    ``TextModel``.  ``embed`` applies the prompt prefix to the raw text,
    tokenises it with <bos> / <eos>, checks the context length and embeds the
    ids; ``embed_many`` does the same for many texts in one batched forward."""

    def __init__(self, model: "TextModel", tokenizer):
        self._model = model
        self._tokenizer = tokenizer

    @classmethod
    def from_parts(cls, model: "TextModel", tokenizer) -> "TextEmbedder":
        return cls(model, tokenizer)

    @classmethod
    def from_files(cls, files, device: int = 0) -> "TextEmbedder":
        """TextEmbedder::from_files (text.rs:584-595): the model and its
        tokenizer.json, whose vocabulary must match the model's."""
        from .tokenizer import Tokenizer

        model = TextModel.from_files(files, device)
        tokenizer = Tokenizer.from_files(files)
        if tokenizer.vocab_size() != model.config().vocab_size:
            raise errors.CorruptError(
                f"tokenizer vocabulary has {tokenizer.vocab_size()} entries, model declares "
                f"{model.config().vocab_size}")
        return cls(model, tokenizer)

    def model(self) -> "TextModel":
        return self._model

    def tokenizer(self):
        return self._tokenizer

    def token_ids(self, text: str, prompt) -> np.ndarray:
        from . import prompt as prompts

        ids = self._tokenizer.encode_array(prompts.apply(prompt, text), True)
        validate_text_length(ids)
        return ids

    def embed(self, text: str, prompt, dimension: int) -> np.ndarray:
        return self._model.embed_ids(self.token_ids(text, prompt), dimension)

    def token_ids_many(self, texts, prompt):
        """``token_ids`` of many texts, tokenised in one call on all host
        threads: (ids, cu_seqlens) packed for ``TextModel.embed_packed``."""
        from . import prompt as prompts

        ids, cu = self._tokenizer.encode_batch([prompts.apply(prompt, t) for t in texts], True)
        longest = int(np.diff(cu).max()) if cu.size > 1 else 0
        if longest > MAX_TEXT_TOKENS:  # text.rs:619-624, for each text
            raise errors.LimitExceededError(
                f"tokenized input has {longest} tokens, above the {MAX_TEXT_TOKENS}-token context")
        return ids, cu

    def embed_many(self, texts, prompt, dimension: int) -> np.ndarray:
        ids, cu = self.token_ids_many(texts, prompt)
        return self._model.embed_packed(ids, cu, dimension)

    def ingest(self, index, texts, chunk_ids, prompt=None) -> None:
        """Chunk texts (with the Document prompt unless another is given)
        embedded and appended to a device ``VectorIndex`` without a host copy
        of the embeddings (``VectorIndex.ingest``)."""
        from . import prompt as prompts

        p = prompts.Prompt.Document if prompt is None else prompt
        ids, cu = self.token_ids_many(texts, p)
        index.ingest(self._model, [ids[cu[i]:cu[i + 1]] for i in range(cu.size - 1)], chunk_ids)
