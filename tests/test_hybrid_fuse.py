"""Reciprocal-rank fusion of a lexical and a vector ranking (svl.index.fuse,
src/index/hybrid.rs:29-68), on the CPU: the reference's unit cases
(hybrid.rs:98-164) and a seeded comparison with a literal restatement of the
reference's accumulation (a BTreeMap keyed by row, lexical terms first,
sorted by f64 score descending then chunk id)."""

from __future__ import annotations

import random

from svl.index import RRF_K, fuse


def test_fuses_ranks_with_the_standard_constant():
    fused = fuse([(0, 2.0), (1, 1.0), (2, 0.5)], [(2, 0.9), (0, 0.8), (1, 0.7)], [1, 2, 3])
    assert [f.index for f in fused] == [0, 2, 1]
    assert fused[0].lexical_rank == 1 and fused[0].vector_rank == 2
    assert abs(fused[0].score - (1.0 / 61.0 + 1.0 / 62.0)) < 1e-12


def test_a_single_list_preserves_its_order():
    fused = fuse([(1, 1.0), (0, 0.5)], [], [1, 2])
    assert [f.index for f in fused] == [1, 0]
    assert fused[0].lexical_rank == 1 and fused[0].vector_rank is None


def test_equal_scores_break_ties_by_chunk_id():
    assert [f.index for f in fuse([(0, 1.0)], [(0, 1.0)], [2, 1])] == [0]
    # rows 0 and 1 both at 1 / 61: the lower chunk id (row 1's) comes first
    assert [f.index for f in fuse([(0, 1.0)], [(1, 1.0)], [9, 4])] == [1, 0]


def test_matches_a_literal_restatement_on_random_lists():
    rnd = random.Random(3)
    for _ in range(50):
        n = rnd.randint(1, 60)
        chunk_ids = rnd.sample(range(10_000), n)
        lex = [(r, 0.0) for r in rnd.sample(range(n), rnd.randint(0, n))]
        vec = [(r, 0.0) for r in rnd.sample(range(n), rnd.randint(0, n))]
        acc = {}
        for pos, (r, _) in enumerate(lex):
            acc[r] = acc.get(r, 0.0) + 1.0 / (RRF_K + (pos + 1))
        for pos, (r, _) in enumerate(vec):
            acc[r] = acc.get(r, 0.0) + 1.0 / (RRF_K + (pos + 1))
        want = sorted(acc, key=lambda r: (-acc[r], chunk_ids[r]))
        got = fuse(lex, vec, chunk_ids)
        assert [f.index for f in got] == want
        assert [f.score for f in got] == [acc[r] for r in want]
