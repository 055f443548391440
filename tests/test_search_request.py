"""SearchRequest::validate (src/index/mod.rs:143-201, vector mode) on the CPU:
the limit and offset caps (mod.rs:21-23) and the query-embedding checks raise
the reference's error variants before any device work."""

from __future__ import annotations

import numpy as np
import pytest

from svl import errors
from svl.index import MAX_EMBEDDING_DIMENSION, MAX_SEARCH_LIMIT, MAX_SEARCH_OFFSET, SearchRequest


def _q(n=8):
    return np.ones(n, np.float32)


def test_the_reference_caps():
    assert (MAX_SEARCH_LIMIT, MAX_SEARCH_OFFSET, MAX_EMBEDDING_DIMENSION) == (1000, 1_000_000, 8192)


@pytest.mark.parametrize("limit,offset", [(1, 0), (MAX_SEARCH_LIMIT, 0), (10, MAX_SEARCH_OFFSET)])
def test_requests_at_the_caps_are_accepted(limit, offset):
    SearchRequest(_q(), limit=limit, offset=offset).validate()


@pytest.mark.parametrize("limit", [0, MAX_SEARCH_LIMIT + 1])
def test_limit_outside_one_to_the_cap_is_a_usage_error(limit):
    with pytest.raises(errors.UsageError, match="search limit must be between 1 and 1000"):
        SearchRequest(_q(), limit=limit).validate()


def test_offset_above_the_cap_is_a_usage_error():
    with pytest.raises(errors.UsageError, match="search offset must not exceed 1000000"):
        SearchRequest(_q(), offset=MAX_SEARCH_OFFSET + 1).validate()


def test_query_embedding_checks():
    with pytest.raises(errors.UsageError, match="at least one dimension"):
        SearchRequest(np.zeros(0, np.float32)).validate()
    SearchRequest(_q(MAX_EMBEDDING_DIMENSION)).validate()
    with pytest.raises(errors.LimitExceededError):
        SearchRequest(_q(MAX_EMBEDDING_DIMENSION + 1)).validate()
    for bad in (np.nan, np.inf, -np.inf):
        e = _q()
        e[3] = bad
        with pytest.raises(errors.UsageError, match="non-finite"):
            SearchRequest(e).validate()


def test_limit_is_checked_before_the_embedding():
    """mod.rs:144-153 come first: a bad limit is reported even with a bad query."""
    with pytest.raises(errors.UsageError, match="search limit"):
        SearchRequest(np.zeros(0, np.float32), limit=0).validate()
