"""The reference's own kernel and vector-search known-answer tests, replayed on
the CPU oracle (src/tensor/kernels.rs:1150-1580, src/index/vector.rs:139-205,
src/index/mod.rs:496-700).  Each test names the reference test it restates."""

import math

import numpy as np
import pytest

import oracle


def close(a, e, tol):
    np.testing.assert_allclose(np.asarray(a, np.float32), np.asarray(e, np.float32), atol=tol, rtol=0)


def test_matmul_is_correct():  # kernels.rs:1198
    out = oracle.matmul(np.array([[1, 2, 3], [4, 5, 6]]), np.array([[7, 8], [9, 10], [11, 12]]))
    assert out.ravel().tolist() == [58.0, 64.0, 139.0, 154.0]


def test_matmul_identity_is_identity():  # kernels.rs:1206
    v = np.array([[2.0, 3.0], [4.0, 5.0]])
    assert np.array_equal(oracle.matmul(v, np.eye(2)), v.astype(np.float32))


def test_linear_projects_rows_against_weight_rows():  # kernels.rs:1390
    out = oracle.linear(np.array([[1, 2, 3], [4, 5, 6]]), np.array([[1, 0, -1], [0, 1, 1]]))
    assert out.ravel().tolist() == [-2.0, 5.0, -2.0, 11.0]


def test_softmax_sums_to_one_and_preserves_order():  # kernels.rs:1229
    out = oracle.softmax([1.0, 2.0, 3.0])
    assert abs(out.sum() - 1.0) < 1e-6 and out[0] < out[1] < out[2]


def test_softmax_is_stable_for_large_values():  # kernels.rs:1238
    out = oracle.softmax([1000.0, 1001.0])
    assert np.isfinite(out).all() and abs(out.sum() - 1.0) < 1e-6


def test_softmax_handles_infinities():  # kernels.rs:1245
    assert oracle.softmax([math.inf, 1.0]).tolist() == [1.0, 0.0]
    with pytest.raises(oracle.OracleError):
        oracle.softmax([-math.inf, -math.inf])
    with pytest.raises(oracle.OracleError):
        oracle.softmax([1.0, math.nan])


def test_rms_norm_is_correct():  # kernels.rs:1267
    close(oracle.rms_norm_rows([3.0, 4.0], [1.0, 1.0], 2, 0.0), [0.848528, 1.131371], 1e-5)
    close(oracle.rms_norm_rows([3.0, 4.0], [2.0, 2.0], 2, 0.0), [1.697056, 2.262741], 1e-5)
    assert oracle.rms_norm_rows([0.0, 0.0], [1.0, 1.0], 2, 1e-6).tolist() == [0.0, 0.0]


def test_rms_norm_rows_normalizes_each_row():  # kernels.rs:1418
    close(oracle.rms_norm_rows([3, 4, 0, 2], [1, 1], 2, 0.0), [0.848528, 1.131371, 0.0, math.sqrt(2)], 1e-5)
    close(oracle.rms_norm_rows([3, 4], None, 2, 0.0), [0.848528, 1.131371], 1e-5)
    with pytest.raises(oracle.OracleError):
        oracle.rms_norm_rows([math.nan], [1.0], 1, 0.0)
    with pytest.raises(oracle.OracleError):
        oracle.rms_norm_rows([1.0], [1.0], 1, -1.0)


def test_gelu_is_correct_at_reference_points():  # kernels.rs:1301
    close([oracle.gelu_tanh_value(0.0)], [0.0], 1e-7)
    close([oracle.gelu_tanh_value(1.0)], [0.841192], 1e-5)
    close([oracle.gelu_tanh_value(-1.0)], [-0.158808], 1e-5)
    close([oracle.gelu_tanh_value(10.0)], [10.0], 1e-4)


def test_geglu_multiplies_the_activated_gate():  # kernels.rs:1309
    close(oracle.geglu([1.0, 0.0], [2.0, 3.0]), [1.682384, 0.0], 1e-5)


def test_l2_normalization_produces_unit_vectors():  # kernels.rs:1319
    out = oracle.l2_normalize([3.0, 4.0])
    close(out, [0.6, 0.8], 1e-7)
    for bad in ([0.0, 0.0], [math.nan, 1.0]):
        with pytest.raises(oracle.OracleError):
            oracle.l2_normalize(bad)


def test_rope_rotates_and_preserves_the_norm():  # kernels.rs:1351, 1494
    inv = oracle.rope_inv_freq(2, 10000.0)
    assert inv.tolist() == [1.0]
    out = oracle.rope([1.0, 0.0], 1, 1, 2, inv, offset=1)
    close(out, [0.540302, 0.841471], 1e-5)
    assert abs(float((out * out).sum()) - 1.0) < 1e-6
    ident = oracle.rope([1.0, 2.0, 3.0, 4.0], 1, 1, 4, oracle.rope_inv_freq(4, 10000.0), offset=0)
    close(ident, [1, 2, 3, 4], 1e-6)


def test_mean_pool_averages_rows():  # kernels.rs:1466
    assert oracle.mean_pool([1.0, 2.0, 3.0, 4.0], 2, 2).tolist() == [2.0, 3.0]


def test_truncation_renormalizes_the_slice():  # kernels.rs:1480
    close(oracle.truncate_and_normalize([3.0, 4.0, 12.0], 2), [0.6, 0.8], 1e-7)
    with pytest.raises(oracle.OracleError):
        oracle.truncate_and_normalize([1.0], 2)
    with pytest.raises(oracle.OracleError):
        oracle.truncate_and_normalize([1.0], 0)


def test_bidirectional_attention_matches_full_attention():  # kernels.rs:1529
    close(oracle.attention([1, 1], [1, 0], [10, 20], 2, 1, 1, 1), [12.6894, 12.6894], 1e-4)


def test_sliding_window_restricts_each_position_to_its_neighbourhood():  # kernels.rs:1540
    q, k, v = [1, 1, 1], [1, 0, 0], [10, 20, 30]
    assert oracle.attention(q, k, v, 3, 1, 1, 1, window=0).tolist() == [10.0, 20.0, 30.0]
    close(oracle.attention(q, k, v, 3, 1, 1, 1, window=1), [12.6894, 16.3582, 25.0], 1e-4)


def test_grouped_query_attention_repeats_key_value_heads_in_order():  # kernels.rs:1556
    close(oracle.attention([1, 1, 0, 0], [1, 0], [5, 7], 1, 4, 2, 1), [5, 5, 7, 7], 1e-6)


def test_bidirectional_attention_rejects_invalid_shapes():  # kernels.rs:1565
    with pytest.raises(oracle.OracleError):
        oracle.attention([1], [1], [1], 1, 3, 2, 1)
    with pytest.raises(oracle.OracleError):
        oracle.attention([1], [1], [1], 1, 1, 1, 1, scale=math.nan)


def _store(rows):
    return np.stack([oracle.normalize_embedding(np.asarray(r, np.float32)) for r in rows])


def test_ranks_by_cosine_similarity():  # vector.rs:140
    rows, scores = oracle.vector_rank([1.0, 0.0], _store([[1, 0], [0, 1], [1, 1]]), chunk_ids=[1, 2, 3])
    assert rows.tolist() == [0, 2, 1]
    assert abs(scores[0] - 1.0) < 1e-9
    assert abs(scores[1] - math.sqrt(0.5)) < 1e-6
    assert abs(scores[2]) < 1e-9


def test_filters_exclude_documents():  # vector.rs:159
    rows, _ = oracle.vector_rank([1.0, 0.0], _store([[1, 0], [1, 0]]), chunk_ids=[1, 2], row_mask=[0, 1])
    assert rows.tolist() == [1]


def test_zero_and_non_finite_queries_are_rejected():  # vector.rs:190
    corpus = _store([[1, 0]])
    for q in ([0.0, 0.0], [math.nan, 1.0], [math.inf, 0.0]):
        with pytest.raises(oracle.OracleError) as e:
            oracle.vector_rank(q, corpus)
        assert e.value.code == 1  # Usage


def test_empty_index_yields_no_hits():  # vector.rs:202
    rows, scores = oracle.vector_rank([1.0, 0.0], np.zeros((0, 2), np.float32))
    assert rows.size == 0


def test_ties_order_by_ascending_chunk_id():  # vector.rs:90-95, index/mod.rs:692
    corpus = _store([[1, 0], [1, 0], [1, 0]])
    rows, scores = oracle.vector_rank([1.0, 0.0], corpus, chunk_ids=[30, 10, 20])
    assert rows.tolist() == [1, 2, 0]


def test_topk_equals_the_head_of_the_full_ranking():
    rng = np.random.default_rng(7)
    corpus = np.stack([oracle.normalize_embedding(r) for r in rng.standard_normal((500, 24)).astype(np.float32)])
    queries = rng.standard_normal((5, 24)).astype(np.float32)
    ids = rng.permutation(500).astype(np.uint64)
    rows_k, scores_k = oracle.vector_topk(queries, corpus, 17, chunk_ids=ids)
    for qi in range(5):
        rows, scores = oracle.vector_rank(queries[qi], corpus, chunk_ids=ids)
        assert rows[:17].tolist() == rows_k[qi].tolist()
        assert np.array_equal(scores[:17], scores_k[qi])


def test_stored_rows_are_normalised_in_f64():  # storage/model.rs:546-581
    v = np.array([3.0, 4.0], np.float32)
    assert oracle.normalize_embedding(v).tolist() == [np.float32(0.6), np.float32(0.8)]
    with pytest.raises(oracle.OracleError):
        oracle.normalize_embedding(np.zeros(3, np.float32))
