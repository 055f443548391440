"""The text half of the reference's ``Engine`` (src/api/engine.rs): the entry
points the CLI and the HTTP server call, ``embed_tokens`` (:222) and
``embed_text`` (:243), with their own argument checks in front of the model.

They differ from ``TextModel.embed_ids`` (text.rs:546-554) in the error the
caller sees: the engine checks the dimension first and reports it as a usage
error (the model reports a bad dimension as internal), an empty id list as a
usage error (the model: corrupt), and an over-long input as limit exceeded
before the model is called.  The vision and audio towers behind the same
struct are out of scope."""

from __future__ import annotations

from . import errors
from . import prompt as prompts
from .config import MAX_TEXT_TOKENS

MATRYOSHKA_DIMENSIONS = (768, 512, 256, 128)  # engine.rs:104-107


class Engine:
    """``Engine`` over a loaded ``TextModel`` and, when the model directory has
    one, its tokenizer (engine.rs:69-121: the vocabulary check at :95-101)."""

    def __init__(self, model, tokenizer=None):
        if tokenizer is not None and tokenizer.vocab_size() != model.config().vocab_size:
            raise errors.CorruptError(
                f"tokenizer vocabulary has {tokenizer.vocab_size()} entries, model declares "
                f"{model.config().vocab_size}")
        self._model = model
        self._tokenizer = tokenizer
        self._dimension = model.config().embedding_dim

    def embedding_dimension(self) -> int:
        return self._dimension

    def matryoshka_dimensions(self) -> list[int]:
        return [d for d in MATRYOSHKA_DIMENSIONS if d <= self._dimension]

    def text_input_available(self) -> bool:
        return self._tokenizer is not None

    def validate_dimension(self, dimension: int) -> None:
        """engine.rs:205-213"""
        if dimension == 0 or dimension > self._dimension:
            raise errors.UsageError(f"dimension {dimension} is outside 1..={self._dimension}")

    def embed_tokens(self, ids, dimension: int):
        """engine.rs:222-234: explicit token ids, no tokenizer, no prompt."""
        self.validate_dimension(dimension)
        n = len(ids)
        if n == 0:
            raise errors.UsageError("token id input must not be empty")
        if n > MAX_TEXT_TOKENS:
            raise errors.LimitExceededError(
                f"token id input has {n} ids, above the {MAX_TEXT_TOKENS}-token context")
        return self._model.embed_ids(ids, dimension)

    def embed_text(self, text: str, prompt, dimension: int):
        """engine.rs:243-260: the prompt prefix, the tokenizer with <bos> /
        <eos>, the context check, then the model."""
        self.validate_dimension(dimension)
        if self._tokenizer is None:
            raise errors.UnsupportedError(
                "this model directory has no tokenizer.json; use the token-id input type")
        ids = self._tokenizer.encode_array(prompts.apply(prompt, text), True)
        if len(ids) > MAX_TEXT_TOKENS:
            raise errors.LimitExceededError(
                f"tokenized input has {len(ids)} tokens, above the {MAX_TEXT_TOKENS}-token context")
        return self._model.embed_ids(ids, dimension)
