"""Exact vector search parity on the B200 against the CPU oracle of
vector::rank (src/index/vector.rs:17-97).

The bar is exact: identical row ids, identical chunk ids and bit-identical
f64 scores (the GPU rescoring performs the reference's own f64 operations in
the same order), ties broken by ascending chunk id.
"""

import numpy as np
import pytest

import oracle
from svl import errors, synth
from svl.index import Index, SearchRequest, VectorIndex, rank

pytestmark = pytest.mark.gpu


def stored(rows):
    return np.stack([oracle.normalize_embedding(r) for r in rows])


def check_topk(index, corpus_stored, chunk_ids, queries, k, mask=None):
    rows, chunks, scores, counts = index.search(queries, k, row_mask=mask)
    if mask is None:
        ref_rows, ref_scores = oracle.vector_topk(queries, corpus_stored, k, chunk_ids=chunk_ids)
        n = min(k, corpus_stored.shape[0])
        assert (counts == n).all()
        assert np.array_equal(rows[:, :n], ref_rows[:, :n])
        assert np.array_equal(scores[:, :n], ref_scores[:, :n])
        assert np.array_equal(chunks[:, :n], np.asarray(chunk_ids, np.uint64)[ref_rows[:, :n].astype(np.int64)])
    else:
        for qi in range(queries.shape[0]):
            r, s = oracle.vector_rank(queries[qi], corpus_stored, chunk_ids=chunk_ids, row_mask=mask)
            n = min(k, r.size)
            assert counts[qi] == n
            assert np.array_equal(rows[qi, :n], r[:n])
            assert np.array_equal(scores[qi, :n], s[:n])


@pytest.fixture(scope="module")
def corpus768():
    rng = np.random.default_rng(3)
    raw = rng.standard_normal((20000, 768), dtype=np.float32)
    ids = rng.permutation(20000).astype(np.uint64) + 1000
    idx = VectorIndex(768, 20000)
    idx.append(raw, ids)
    return idx, stored(raw), ids


@pytest.mark.parametrize("nq,k", [(1, 10), (37, 10), (130, 1), (64, 32)])
def test_fast_path_matches_oracle(corpus768, nq, k):
    idx, st, ids = corpus768
    q = np.random.default_rng(nq + k).standard_normal((nq, 768), dtype=np.float32)
    check_topk(idx, st, ids, q, k)


def test_full_ranking_path_for_large_k(corpus768):
    idx, st, ids = corpus768
    q = np.random.default_rng(8).standard_normal((3, 768), dtype=np.float32)
    check_topk(idx, st, ids, q, 100)


def test_rank_returns_the_whole_ordering():
    rng = np.random.default_rng(2)
    raw = rng.standard_normal((300, 64), dtype=np.float32)
    ids = np.arange(300, dtype=np.uint64)
    idx = VectorIndex(64, 300)
    idx.append(raw, ids)
    q = rng.standard_normal(64, dtype=np.float32)
    got = rank(q, idx)
    r, s = oracle.vector_rank(q, stored(raw), chunk_ids=ids)
    assert [g[0] for g in got] == r.tolist()
    assert [g[1] for g in got] == s.tolist()


@pytest.mark.parametrize("dim", [77, 100, 131])
def test_rank_with_ragged_dimensions_and_a_row_mask(dim):
    """The full path stages 32 dimensions per step with 16-byte copies when
    dim % 4 == 0 and 4-byte copies otherwise; a last step narrower than 32,
    a row count that is not a multiple of the 128-row block and masked rows
    must still give the oracle's whole ordering with bit-identical f64
    scores (vector::rank, src/index/vector.rs:17-97)."""
    rng = np.random.default_rng(dim)
    n = 1000
    raw = rng.standard_normal((n, dim), dtype=np.float32)
    ids = (rng.permutation(n) * 7).astype(np.uint64)
    idx = VectorIndex(dim, n)
    idx.append(raw, ids)
    q = rng.standard_normal(dim, dtype=np.float32)
    mask = rng.random(n) < 0.8
    got = rank(q, idx, row_mask=mask)
    r, s = oracle.vector_rank(q, stored(raw), chunk_ids=ids, row_mask=mask)
    assert [g[0] for g in got] == r.tolist()
    assert [g[1] for g in got] == s.tolist()


def test_matryoshka_256_index():
    rng = np.random.default_rng(4)
    raw = rng.standard_normal((5000, 768), dtype=np.float32)
    trunc = raw[:, :256]
    ids = np.arange(5000, dtype=np.uint64)
    idx = VectorIndex(256, 5000)
    idx.append(trunc, ids)
    q = rng.standard_normal((16, 256), dtype=np.float32)
    check_topk(idx, stored(trunc), ids, q, 10)


def test_filters_exclude_rows(corpus768):
    idx, st, ids = corpus768
    rng = np.random.default_rng(5)
    mask = (rng.random(st.shape[0]) < 0.3).astype(np.uint8)
    q = rng.standard_normal((4, 768), dtype=np.float32)
    check_topk(idx, st, ids, q, 10, mask=mask)


def test_ties_are_ordered_by_ascending_chunk_id():
    rng = np.random.default_rng(6)
    base = rng.standard_normal((50, 32), dtype=np.float32)
    raw = np.concatenate([base, base, base])  # every vector three times
    ids = rng.permutation(150).astype(np.uint64)
    idx = VectorIndex(32, 150)
    idx.append(raw, ids)
    q = base[:5] + 0.01 * rng.standard_normal((5, 32), dtype=np.float32)
    check_topk(idx, stored(raw), ids, q, 9)
    check_topk(idx, stored(raw), ids, q, 60)


def test_near_ties_take_the_exact_fallback():
    """Hundreds of rows within 1e-4 of each other defeat the screen's error
    margin; the answer must still be exact."""
    rng = np.random.default_rng(7)
    q = rng.standard_normal(128, dtype=np.float32)
    q /= np.linalg.norm(q)
    near = q[None, :] + 1e-3 * rng.standard_normal((400, 128), dtype=np.float32)
    far = rng.standard_normal((30000, 128), dtype=np.float32)
    raw = np.concatenate([far[:15000], near, far[15000:]])
    ids = np.arange(raw.shape[0], dtype=np.uint64)
    idx = VectorIndex(128, raw.shape[0])
    idx.append(raw, ids)
    check_topk(idx, stored(raw), ids, q[None, :], 10)


def test_edge_cases():
    idx = VectorIndex(2, 8)
    rows, _, _, counts = idx.search(np.array([[1.0, 0.0]], np.float32), 5)
    assert counts[0] == 0  # empty index -> no hits (vector.rs:202)
    idx.append(np.array([[1, 0], [0, 1], [1, 1]], np.float32), np.array([1, 2, 3], np.uint64))
    got = rank(np.array([1.0, 0.0], np.float32), idx)
    assert [g[0] for g in got] == [0, 2, 1]  # vector.rs:140
    assert abs(got[0][1] - 1.0) < 1e-9 and abs(got[1][1] - 2 ** -0.5) < 1e-6
    for bad in ([0.0, 0.0], [np.nan, 1.0], [np.inf, 0.0]):
        with pytest.raises(errors.UsageError):
            idx.search(np.array([bad], np.float32), 1)
    with pytest.raises(errors.UsageError):
        idx.search(np.array([[1.0, 0.0, 0.0]], np.float32), 1)
    with pytest.raises(errors.UsageError):
        idx.append(np.zeros((1, 2), np.float32), np.array([9], np.uint64))
    rows, _, _, counts = idx.search(np.array([[1.0, 0.0]], np.float32), 10)
    assert counts[0] == 3


def test_concurrent_searches_from_threads_match_sequential_searches(corpus768):
    """One index searched from several host threads at once (the handle's
    mutex serialises the overlapping C calls; index/mod.rs:692 asks for
    deterministic searches) returns what sequential searches return."""
    import threading

    idx, _, _ = corpus768
    qs = [np.random.default_rng(40 + i).standard_normal((8, 768), dtype=np.float32) for i in range(4)]
    want = [idx.search(q, 10) for q in qs]
    got = [None] * 6
    failures = []

    def run(t):
        try:
            got[t] = [idx.search(qs[(t + j) % len(qs)], 10) for j in range(len(qs))]
        except Exception as e:  # reported below, on the main thread
            failures.append(repr(e))

    threads = [threading.Thread(target=run, args=(t,)) for t in range(len(got))]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=120)
    assert not failures, failures
    assert not any(th.is_alive() for th in threads)
    for t, out in enumerate(got):
        for j, res in enumerate(out):
            for a, b in zip(res, want[(t + j) % len(qs)]):
                assert np.array_equal(a, b), (t, j)


def test_index_search_paginates_the_ranking(corpus768):
    idx, st, ids = corpus768
    q = np.random.default_rng(9).standard_normal(768, dtype=np.float32)
    full = Index(idx).search(SearchRequest(q, limit=20, offset=0))
    page = Index(idx).search(SearchRequest(q, limit=5, offset=10))
    assert [h.chunk_id for h in page] == [h.chunk_id for h in full[10:15]]
    assert [h.vector_rank for h in page] == [11, 12, 13, 14, 15]
    with pytest.raises(errors.UsageError):
        Index(idx).search(SearchRequest(q, limit=0))


def test_merge_of_shard_lists_matches_a_global_search():
    import torch

    from svl import dist

    rng = np.random.default_rng(10)
    raw = rng.standard_normal((6000, 96), dtype=np.float32)
    ids = rng.permutation(6000).astype(np.uint64)
    q = rng.standard_normal((7, 96), dtype=np.float32)
    k = 10
    shards = np.array_split(np.arange(6000), 3)
    lists = []
    for sh in shards:
        idx = VectorIndex(96, sh.size)
        idx.append(raw[sh], ids[sh])
        r, c, s, n = idx.search(q, k)
        lists.append((s, c, r + sh[0], n))
    scores = torch.from_numpy(np.stack([l[0] for l in lists])).cuda()
    chunks = torch.from_numpy(np.stack([l[1] for l in lists]).astype(np.int64)).cuda()
    rows = torch.from_numpy(np.stack([l[2] for l in lists]).astype(np.int64)).cuda()
    counts = torch.from_numpy(np.stack([l[3] for l in lists]).astype(np.int32)).cuda()
    ms, mc, mr, mshard, mn = dist.merge_topk_device(scores, chunks, rows, counts, k)
    ref_rows, ref_scores = oracle.vector_topk(q, stored(raw), k, chunk_ids=ids)
    assert np.array_equal(ms.cpu().numpy(), ref_scores)
    assert np.array_equal(mc.cpu().numpy().astype(np.uint64), ids[ref_rows.astype(np.int64)])
    assert np.array_equal(mr.cpu().numpy().astype(np.uint64), ref_rows)


def test_tf32_screen_matches_oracle():
    """SVL_SEARCH_TF32=1 at creation: no FP16 screening copy, the FP32 rows
    screened in TF32 -- the same exact results."""
    import os

    rng = np.random.default_rng(21)
    raw = rng.standard_normal((5000, 256), dtype=np.float32)
    ids = rng.permutation(5000).astype(np.uint64) + 7
    os.environ["SVL_SEARCH_TF32"] = "1"
    try:
        idx = VectorIndex(256, 5000)
    finally:
        os.environ.pop("SVL_SEARCH_TF32", None)
    idx.append(raw, ids)
    q = rng.standard_normal((40, 256), dtype=np.float32)
    check_topk(idx, stored(raw), ids, q, 10)


def test_dimension_not_a_multiple_of_8_screens_in_tf32():
    """dim % 8 != 0 (FP16 rows would not fill whole 16-byte units): the index
    keeps no FP16 copy and screens its FP32 rows in TF32."""
    rng = np.random.default_rng(22)
    raw = rng.standard_normal((3000, 76), dtype=np.float32)
    ids = np.arange(3000, dtype=np.uint64)
    idx = VectorIndex(76, 3000)
    idx.append(raw, ids)
    q = rng.standard_normal((9, 76), dtype=np.float32)
    check_topk(idx, stored(raw), ids, q, 5)


def test_indexes_on_two_devices_in_one_process():
    """Kernel shared-memory opt-ins apply per device: an index on device 1
    created after one on device 0 (same process, same kernels) must search
    exactly too.  Needs two GPUs."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    rng = np.random.default_rng(53)
    raw = rng.standard_normal((5000, 256), dtype=np.float32)
    ids = np.arange(5000, dtype=np.uint64)
    q = rng.standard_normal((300, 256), dtype=np.float32)
    want = None
    for dev in (0, 1):
        idx = VectorIndex(256, 5000, device=dev)
        idx.append(raw, ids)
        got = idx.search(q, 10)
        if want is None:
            want = got
            check_topk(idx, stored(raw), ids, q[:4], 10)
        for a, b in zip(got, want):
            assert np.array_equal(a, b)
