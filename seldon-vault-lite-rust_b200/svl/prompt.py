"""Task prompt prefixes of the frozen model (src/model/prompt.rs).

The prefix is prepended to the raw text before tokenisation
(``TextEmbedder.embed``, text.rs:616-626), so a query and a document never
share an accidental embedding.
"""

from __future__ import annotations

import enum

SEARCH_QUERY = "task: search result | query: "
DOCUMENT = "title: none | text: "
CLASSIFICATION = "task: classification | query: "
CLUSTERING = "task: clustering | query: "
CODE_RETRIEVAL = "task: code retrieval | query: "
FACT_CHECKING = "task: fact checking | query: "
SENTENCE_SIMILARITY = "task: sentence similarity | query: "
QUESTION_ANSWERING = "task: question answering | query: "


class Prompt(enum.Enum):
    """prompt.rs ``Prompt``: the official prompt roles and their prefixes."""

    SearchQuery = SEARCH_QUERY
    Document = DOCUMENT
    Classification = CLASSIFICATION
    Clustering = CLUSTERING
    CodeRetrieval = CODE_RETRIEVAL
    FactChecking = FACT_CHECKING
    SentenceSimilarity = SENTENCE_SIMILARITY
    QuestionAnswering = QUESTION_ANSWERING

    def prefix(self) -> str:
        return self.value

    def is_query(self) -> bool:
        return self is not Prompt.Document

    @classmethod
    def from_name(cls, name: str) -> "Prompt | None":
        """The exact (case-sensitive) official name, else None."""
        return cls.__members__.get(name)


def apply(prompt: Prompt, text: str) -> str:
    return prompt.prefix() + text
