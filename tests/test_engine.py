"""Engine::embed_tokens / embed_text (src/api/engine.rs:205-260) on the CPU:
the engine's own checks and error variants, in the reference's order, before
the model is called (a recording stand-in for the model here; the GPU test in
tests/test_gpu_encoder.py runs the real one)."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

from svl import errors
from svl.engine import Engine
from svl.prompt import Prompt, apply


class RecordingModel:
    def __init__(self, embedding_dim=768, vocab_size=4096):
        self.cfg = SimpleNamespace(embedding_dim=embedding_dim, vocab_size=vocab_size)
        self.calls = []

    def config(self):
        return self.cfg

    def embed_ids(self, ids, dimension):
        self.calls.append((list(np.asarray(ids).tolist()), dimension))
        return np.zeros(dimension, np.float32)


class FakeTokenizer:
    def __init__(self, vocab_size=4096, n_ids=None):
        self.vocab = vocab_size
        self.n_ids = n_ids
        self.seen = []

    def vocab_size(self):
        return self.vocab

    def encode_array(self, text, add_special_tokens):
        self.seen.append((text, add_special_tokens))
        n = self.n_ids if self.n_ids is not None else len(text.split()) + 2
        return np.arange(2, 2 + n, dtype=np.uint32)


def test_dimensions_and_matryoshka_set():
    e = Engine(RecordingModel())
    assert e.embedding_dimension() == 768
    assert e.matryoshka_dimensions() == [768, 512, 256, 128]
    assert Engine(RecordingModel(embedding_dim=300)).matryoshka_dimensions() == [256, 128]
    assert not e.text_input_available() and Engine(RecordingModel(), FakeTokenizer()).text_input_available()


@pytest.mark.parametrize("dim", [0, 769])
def test_dimension_outside_one_to_the_model_width_is_a_usage_error(dim):
    m = RecordingModel()
    with pytest.raises(errors.UsageError, match=f"dimension {dim} is outside 1..=768"):
        Engine(m).embed_tokens([5, 6], dim)
    with pytest.raises(errors.UsageError, match="is outside"):
        Engine(m, FakeTokenizer()).embed_text("hello", Prompt.SearchQuery, dim)
    assert m.calls == []


def test_embed_tokens_checks_then_calls_the_model():
    m = RecordingModel()
    e = Engine(m)
    with pytest.raises(errors.UsageError, match="token id input must not be empty"):
        e.embed_tokens([], 256)
    with pytest.raises(errors.UsageError, match="is outside"):  # the dimension is checked first
        e.embed_tokens([], 0)
    with pytest.raises(errors.LimitExceededError, match="8193 ids, above the 8192-token context"):
        e.embed_tokens([7] * 8193, 256)
    assert m.calls == []
    out = e.embed_tokens([7] * 8192, 128)
    assert out.shape == (128,) and m.calls == [([7] * 8192, 128)]


def test_embed_text_applies_the_prompt_and_the_specials():
    m, t = RecordingModel(), FakeTokenizer()
    e = Engine(m, t)
    e.embed_text("what is a vault", Prompt.SearchQuery, 512)
    assert t.seen == [(apply(Prompt.SearchQuery, "what is a vault"), True)]
    ids, dim = m.calls[0]
    assert dim == 512 and ids == list(range(2, 2 + len(t.seen[0][0].split()) + 2))


def test_embed_text_without_a_tokenizer_is_unsupported():
    with pytest.raises(errors.UnsupportedError, match="no tokenizer.json"):
        Engine(RecordingModel()).embed_text("hello", Prompt.SearchQuery, 768)


def test_embed_text_over_the_context_is_limit_exceeded():
    m = RecordingModel()
    with pytest.raises(errors.LimitExceededError, match="8193 tokens, above the 8192-token context"):
        Engine(m, FakeTokenizer(n_ids=8193)).embed_text("long", Prompt.Document, 768)
    assert m.calls == []


def test_a_tokenizer_for_another_vocabulary_is_corrupt():
    with pytest.raises(errors.CorruptError, match="tokenizer vocabulary has 100 entries, model declares 4096"):
        Engine(RecordingModel(), FakeTokenizer(vocab_size=100))
