"""svl_search_noalloc: the allocation-free search entry point.

Some callers cannot let the library call cudaMalloc (a fixed, pre-carved
device memory budget, or a thread that may not take the allocation lock).
For them svl_search_noalloc runs the exact search with its scratch in one
static device array.  This test calls it through the C ABI, twice in a row on
the same inputs (the scratch keeps the first call's contents, which must not
leak into the second), and requires the same answer as svl_index_search --
the existing entry point -- exactly: identical rows and chunk ids and
bit-identical f64 scores.  It also covers a row filter (against the CPU
oracle of vector::rank), an empty corpus, a NULL chunk-id output, a
misaligned rows pointer, near-ties that the allocation-free screen cannot
settle (SVL_UNSUPPORTED, counts 0) and oversized requests.

The file is named so that pytest collects it last; it passes on its own in a
fresh process (where its first call performs the one-time set-up) and after
the rest of the suite.
"""

import ctypes

import numpy as np
import pytest

from svl import errors
from svl._abi import ErrBuf, load_library
from svl.index import VectorIndex

pytestmark = pytest.mark.gpu


def _call(lib, rows, ids, queries, k, mask=None, chunk_out=True, rows_offset=0, counts_out=None, n_rows=None):
    """One svl_search_noalloc call on device tensors.  rows_offset shifts the
    rows pointer by that many bytes (the misaligned-pointer case, refused on
    the host before any launch); counts_out receives the counts even when
    the call raises."""
    import torch

    nq, dim = queries.shape
    out_rows = torch.full((nq, k), -1, dtype=torch.int64, device="cuda")
    out_chunk = torch.full((nq, k), -1, dtype=torch.int64, device="cuda")
    out_scores = torch.full((nq, k), float("nan"), dtype=torch.float64, device="cuda")
    out_counts = torch.full((nq,), -1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    eb = ErrBuf()
    n = rows.shape[0] if n_rows is None else n_rows
    rc = lib.svl_search_noalloc(rows.data_ptr() + rows_offset, ids.data_ptr(), n, dim,
                                queries.data_ptr(), nq, None if mask is None else mask.data_ptr(), k,
                                out_rows.data_ptr(), out_chunk.data_ptr() if chunk_out else None,
                                out_scores.data_ptr(), out_counts.data_ptr(), None, *eb.args)
    if counts_out is not None:
        counts_out[:] = out_counts.cpu().numpy()
    eb.check(rc)
    return (out_rows.cpu().numpy().astype(np.uint64), out_chunk.cpu().numpy().astype(np.uint64),
            out_scores.cpu().numpy(), out_counts.cpu().numpy().astype(np.uint32))


def _stored(raw):
    """The unit-norm rows the index stores: Chunk::new's f64 sum of squares in
    dimension order, then (f64 value / norm) rounded to f32."""
    x = raw.astype(np.float64)
    sumsq = np.zeros(raw.shape[0], np.float64)
    for d in range(raw.shape[1]):
        sumsq += x[:, d] * x[:, d]
    return (x / np.sqrt(sumsq)[:, None]).astype(np.float32)


def test_noalloc_search_matches_the_index_search_on_two_calls():
    import torch

    lib = load_library()
    rng = np.random.default_rng(31)
    n, dim, k = 30000, 768, 10
    raw = rng.standard_normal((n, dim), dtype=np.float32)
    ids = rng.permutation(n).astype(np.uint64) + 7
    index = VectorIndex(dim, n)
    index.append(raw, ids)
    stored = _stored(raw)
    d_rows = torch.from_numpy(stored).cuda()
    d_ids = torch.from_numpy(ids.astype(np.int64)).cuda()
    for trial in range(2):
        q = rng.standard_normal((100, dim), dtype=np.float32)
        want = index.search(q, k)
        for _ in range(2):  # two calls in a row share the scratch
            got = _call(lib, d_rows, d_ids, torch.from_numpy(q).cuda(), k)
            assert np.array_equal(got[3], want[3])
            assert np.array_equal(got[0], want[0])
            assert np.array_equal(got[1], want[1])
            assert np.array_equal(got[2], want[2])


def test_noalloc_search_refuses_oversized_requests():
    import torch

    lib = load_library()
    rows = torch.zeros((16, 8), device="cuda")
    ids = torch.zeros((16,), dtype=torch.int64, device="cuda")
    with pytest.raises(errors.LimitExceededError):
        _call(lib, rows, ids, torch.ones((129, 8), device="cuda"), 5)
    with pytest.raises(errors.LimitExceededError):
        _call(lib, rows, ids, torch.ones((4, 8), device="cuda"), 33)
    big = torch.zeros((4, 1028), device="cuda")
    with pytest.raises(errors.LimitExceededError):
        _call(lib, torch.zeros((16, 1028), device="cuda"), ids, big, 5)


def test_noalloc_search_with_a_row_filter_matches_the_oracle():
    """A row mask (vector.rs:57-60 filters before ranking) on two calls in a
    row: the same answer as svl_index_search under the same filter, and as
    the CPU oracle of vector::rank for every query."""
    import torch

    import oracle

    lib = load_library()
    rng = np.random.default_rng(41)
    n, dim, k = 12000, 256, 12
    raw = rng.standard_normal((n, dim), dtype=np.float32)
    ids = np.arange(n, dtype=np.uint64) * 3 + 1
    index = VectorIndex(dim, n)
    index.append(raw, ids)
    stored = _stored(raw)
    mask = (rng.random(n) < 0.3).astype(np.uint8)
    q = rng.standard_normal((24, dim), dtype=np.float32)
    want = index.search(q, k, row_mask=mask)
    d_rows, d_ids = torch.from_numpy(stored).cuda(), torch.from_numpy(ids.astype(np.int64)).cuda()
    d_mask, d_q = torch.from_numpy(mask).cuda(), torch.from_numpy(q).cuda()
    for _ in range(2):
        got = _call(lib, d_rows, d_ids, d_q, k, mask=d_mask)
        for a, b in zip(got, want):
            assert np.array_equal(a, b)
    for qi in range(q.shape[0]):
        r, s = oracle.vector_rank(q[qi], stored, chunk_ids=ids, row_mask=mask)
        assert got[3][qi] == min(k, r.size)
        assert np.array_equal(got[0][qi], r[:k]) and np.array_equal(got[2][qi], s[:k])
        assert np.array_equal(got[1][qi], ids[r[:k].astype(np.int64)])


def test_noalloc_search_on_an_empty_corpus_and_without_chunk_ids():
    import torch

    lib = load_library()
    rng = np.random.default_rng(43)
    q = torch.from_numpy(rng.standard_normal((3, 64), dtype=np.float32)).cuda()
    # n_rows = 0 over valid (non-null) buffers: an empty corpus has no hits (vector.rs:202)
    none_rows = torch.zeros((1, 64), device="cuda")
    none_ids = torch.zeros((1,), dtype=torch.int64, device="cuda")
    for _ in range(2):
        got = _call(lib, none_rows, none_ids, q, 5, n_rows=0)
        assert (got[3] == 0).all()
    raw = rng.standard_normal((500, 64), dtype=np.float32)
    ids = np.arange(500, dtype=np.uint64) + 100
    index = VectorIndex(64, 500)
    index.append(raw, ids)
    d_rows, d_ids = torch.from_numpy(_stored(raw)).cuda(), torch.from_numpy(ids.astype(np.int64)).cuda()
    want = index.search(q.cpu().numpy(), 7)
    got = _call(lib, d_rows, d_ids, q, 7, chunk_out=False)  # d_out_chunk_ids may be NULL
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[2], want[2]) and np.array_equal(got[3], want[3])


def test_noalloc_search_refuses_a_misaligned_rows_pointer():
    """Checked on the host before anything is launched: SVL_USAGE."""
    import torch

    lib = load_library()
    rows = torch.zeros((17, 8), device="cuda")
    ids = torch.zeros((16,), dtype=torch.int64, device="cuda")
    with pytest.raises(errors.UsageError):
        _call(lib, rows[:16], ids, torch.ones((2, 8), device="cuda"), 3, rows_offset=4)


def test_noalloc_search_reports_near_ties_it_cannot_settle():
    """Hundreds of rows identical to the query fill every candidate list of
    the screen with the same score, so the allocation-free path cannot prove
    its top-k: SVL_UNSUPPORTED, and the tied query's count is 0.  The
    allocating entry point answers the same query exactly (full path)."""
    import torch

    import oracle

    lib = load_library()
    rng = np.random.default_rng(47)
    dim = 128
    q = rng.standard_normal(dim, dtype=np.float32)
    far = rng.standard_normal((20000, dim), dtype=np.float32)
    raw = np.concatenate([far[:9000], np.repeat(q[None, :], 600, axis=0), far[9000:]])
    ids = np.arange(raw.shape[0], dtype=np.uint64)
    stored = _stored(raw)
    d_rows, d_ids = torch.from_numpy(stored).cuda(), torch.from_numpy(ids.astype(np.int64)).cuda()
    counts = np.full(1, -1, np.int64)
    with pytest.raises(errors.UnsupportedError):
        _call(lib, d_rows, d_ids, torch.from_numpy(q[None, :]).cuda(), 10, counts_out=counts)
    assert counts[0] == 0
    index = VectorIndex(dim, raw.shape[0])
    index.append(raw, ids)
    rows, _, scores, cnt = index.search(q[None, :], 10)
    r, s = oracle.vector_rank(q, stored, chunk_ids=ids)
    assert cnt[0] == 10 and np.array_equal(rows[0], r[:10]) and np.array_equal(scores[0], s[:10])
