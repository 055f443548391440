"""Exact cosine vector search on the B200 behind the reference's search API.

* ``VectorIndex``      -- a device-resident shard of unit-norm rows with chunk
                          ids (the in-memory view Index::build_from builds,
                          src/index/mod.rs:271-308; rows normalised as
                          Chunk::new does, src/storage/model.rs:546-581).
* ``rank``             -- vector::rank (src/index/vector.rs:17-97): the
                          ranking of every row that passes the filter.
* ``Index.search``     -- Index::search in vector mode
                          (src/index/mod.rs:325-388): validate, rank,
                          skip(offset).take(limit).
* ``fuse``             -- hybrid::fuse (src/index/hybrid.rs:29-68): RRF of a
                          caller's lexical ranking and ``rank``'s full
                          vector ranking.

Scores are the reference's f64 cosines, bit for bit; ties are ordered by
ascending chunk id.  Every call runs on the GPU.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import errors
from ._abi import ErrBuf, load_library

MAX_SEARCH_LIMIT = 1000  # index/mod.rs:21
MAX_SEARCH_OFFSET = 1_000_000  # index/mod.rs:23
MAX_EMBEDDING_DIMENSION = 8192  # storage/model.rs:35

_P = ctypes.c_void_p


def _ptr(a):
    return None if a is None else a.ctypes.data


class VectorIndex:
    def __init__(self, dim: int, capacity: int, device: int = 0):
        self._lib = load_library()
        h = _P()
        eb = ErrBuf()
        eb.check(self._lib.svl_index_create(device, dim, capacity, ctypes.byref(h), *eb.args))
        self._h = h
        self.device = device

    def close(self):
        if getattr(self, "_h", None):
            self._lib.svl_index_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __len__(self):
        return int(self._lib.svl_index_len(self._h))

    @property
    def dim(self) -> int:
        return int(self._lib.svl_index_dim(self._h))

    @property
    def handle(self):
        return self._h

    def append(self, rows, chunk_ids) -> None:
        rows = np.ascontiguousarray(rows, np.float32)
        ids = np.ascontiguousarray(chunk_ids, np.uint64)
        if rows.ndim != 2 or rows.shape[0] != ids.size:
            raise errors.UsageError("rows and chunk ids disagree")
        if rows.shape[1] != self.dim:
            raise errors.UsageError(f"embedding dimension {rows.shape[1]} does not match the index dimension {self.dim}")
        eb = ErrBuf()
        eb.check(self._lib.svl_index_append(self._h, _ptr(rows), _ptr(ids), ids.size, *eb.args))

    def append_device(self, d_rows_ptr: int, d_chunk_ids_ptr: int, n: int, stream: int = 0) -> None:
        eb = ErrBuf()
        eb.check(self._lib.svl_index_append_device(self._h, d_rows_ptr, d_chunk_ids_ptr, n, stream or None, *eb.args))

    def ingest(self, model, sequences, chunk_ids) -> None:
        """Embeds token-id sequences with ``model`` (a ``TextModel`` on the
        same GPU) at this index's dimension and appends them with their chunk
        ids, the embeddings never leaving the GPU (``svl_ingest_batch``: the
        chunk embedding of Store::put_document, then Chunk::new's
        normalisation and the append)."""
        from .text import pack

        ids, cu = pack(sequences)
        chunk = np.ascontiguousarray(chunk_ids, np.uint64)
        if chunk.size != cu.size - 1:
            raise errors.UsageError("sequences and chunk ids disagree")
        eb = ErrBuf()
        eb.check(self._lib.svl_ingest_batch(model._h, self._h, _ptr(ids), _ptr(cu), cu.size - 1, _ptr(chunk),
                                            *eb.args))

    def search(self, queries, k: int, row_mask=None):
        """Top-k of vector::rank for each query.  Returns (rows, chunk_ids,
        scores, counts) with shapes [Q, k], [Q, k], [Q, k], [Q]."""
        q = np.ascontiguousarray(queries, np.float32)
        if q.ndim == 1:
            q = q[None, :]
        nq, dim = q.shape
        rows = np.zeros((nq, k), np.uint64)
        chunk = np.zeros((nq, k), np.uint64)
        scores = np.zeros((nq, k), np.float64)
        counts = np.zeros(nq, np.uint32)
        mask = None if row_mask is None else np.ascontiguousarray(row_mask, np.uint8)
        eb = ErrBuf()
        eb.check(self._lib.svl_index_search(self._h, _ptr(q), nq, dim, _ptr(mask), k, _ptr(rows), _ptr(chunk),
                                            _ptr(scores), _ptr(counts), *eb.args))
        return rows, chunk, scores, counts

    def search_device(self, d_queries_ptr, nq, k, d_rows_ptr, d_chunk_ptr, d_scores_ptr, d_counts_ptr,
                      d_mask_ptr=None, stream: int = 0) -> None:
        eb = ErrBuf()
        eb.check(self._lib.svl_index_search_device(self._h, d_queries_ptr, nq, d_mask_ptr, k, d_rows_ptr, d_chunk_ptr,
                                                   d_scores_ptr, d_counts_ptr, stream or None, *eb.args))

    def check(self):
        eb = ErrBuf()
        eb.check(self._lib.svl_index_check(self._h, *eb.args))


def rank(query, index: VectorIndex, row_mask=None, dimension: int | None = None):
    """vector::rank: every surviving row as (row, f64 score), best first."""
    q = np.ascontiguousarray(query, np.float32).ravel()
    if dimension is not None and q.size != dimension and q.size > 0:
        # the reference validates finiteness and norm before the dimension
        _validate_query(q)
        raise errors.UsageError(f"query embedding dimension {q.size} does not match the index dimension {dimension}")
    n = len(index)
    if n == 0:
        _validate_query(q)
        return []
    rows, _, scores, counts = index.search(q[None, :], n, row_mask)
    c = int(counts[0])
    return list(zip(rows[0, :c].tolist(), scores[0, :c].tolist()))


RRF_K = 60.0  # hybrid.rs:13


@dataclass
class Fused:
    """hybrid.rs ``Fused``: one candidate of the reciprocal-rank fusion."""

    index: int
    score: float
    lexical_rank: int | None = None
    vector_rank: int | None = None


def fuse(lexical, vector, chunk_ids) -> list[Fused]:
    """hybrid::fuse (hybrid.rs:29-68): reciprocal-rank fusion of a lexical and
    a vector ranking, each a best-first list of (row, score).  A row's score
    is the sum of 1 / (60 + rank) over the lists that hold it (one-based
    ranks; the lexical term is added first, as in the reference, so the f64
    sums are the same); ties go to the lower chunk id (``chunk_ids[row]``).
    The vector list is normally ``rank(query, index)``, the GPU's complete
    ranking; BM25 stays with the caller."""
    fused: dict[int, Fused] = {}
    for pos, (row, _) in enumerate(lexical):
        f = fused.setdefault(int(row), Fused(int(row), 0.0))
        f.score += 1.0 / (RRF_K + (pos + 1))
        f.lexical_rank = pos + 1
    for pos, (row, _) in enumerate(vector):
        f = fused.setdefault(int(row), Fused(int(row), 0.0))
        f.score += 1.0 / (RRF_K + (pos + 1))
        f.vector_rank = pos + 1
    ids = np.asarray(chunk_ids, np.uint64)
    return sorted(fused.values(), key=lambda f: (-f.score, int(ids[f.index])))


def _validate_query(q):
    if q.size == 0:
        raise errors.UsageError("query embedding must have at least one dimension")
    if q.size > MAX_EMBEDDING_DIMENSION:
        raise errors.LimitExceededError("query embedding above the 8192-dimension cap")
    if not np.isfinite(q).all():
        raise errors.UsageError("query embedding contains a non-finite value")
    s = float(np.sum(q.astype(np.float64) ** 2))
    if not np.isfinite(s) or s <= 0:
        raise errors.UsageError("query embedding norm is zero or non-finite; cosine similarity is undefined")


@dataclass
class SearchHit:
    chunk_id: int
    row: int
    score: float
    vector_rank: int


@dataclass
class SearchRequest:
    """The vector-mode fields of SearchRequest (index/mod.rs:143-201)."""

    embedding: np.ndarray
    limit: int = 10
    offset: int = 0
    row_mask: np.ndarray | None = field(default=None)

    def validate(self):
        if self.limit == 0 or self.limit > MAX_SEARCH_LIMIT:
            raise errors.UsageError(f"search limit must be between 1 and {MAX_SEARCH_LIMIT}")
        if self.offset > MAX_SEARCH_OFFSET:
            raise errors.UsageError(f"search offset must not exceed {MAX_SEARCH_OFFSET}")
        e = np.asarray(self.embedding)
        if e.size == 0:
            raise errors.UsageError("query embedding must have at least one dimension")
        if e.size > MAX_EMBEDDING_DIMENSION:
            raise errors.LimitExceededError("query embedding above the 8192-dimension cap")
        if not np.isfinite(e).all():
            raise errors.UsageError("query embedding contains a non-finite value")


class Index:
    """Vector-mode Index::search over a VectorIndex."""

    def __init__(self, vectors: VectorIndex):
        self.vectors = vectors

    def search(self, request: SearchRequest) -> list[SearchHit]:
        request.validate()
        k = request.offset + request.limit
        n = len(self.vectors)
        kk = max(1, min(k, n)) if n else 1
        rows, chunks, scores, counts = self.vectors.search(request.embedding, kk, request.row_mask)
        c = int(counts[0])
        hits = []
        for pos in range(request.offset, min(c, k)):
            hits.append(SearchHit(int(chunks[0, pos]), int(rows[0, pos]), float(scores[0, pos]), pos + 1))
        return hits
