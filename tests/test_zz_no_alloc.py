"""svl_search_noalloc: the allocation-free search entry point.

Some callers cannot let the library call cudaMalloc (a fixed, pre-carved
device memory budget, or a thread that may not take the allocation lock).
For them svl_search_noalloc runs the exact search with its scratch in one
static device array.  This test calls it through the C ABI, twice in a row on
the same inputs (the scratch keeps the first call's contents, which must not
leak into the second), and requires the same answer as svl_index_search --
the existing entry point -- exactly: identical rows and chunk ids and
bit-identical f64 scores.  It also checks that oversized requests are refused.

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


def _call(lib, rows, ids, queries, k, mask=None):
    import torch

    nq, dim = queries.shape
    out_rows = torch.full((nq, k), -1, dtype=torch.int64, device="cuda")
    out_chunk = torch.full((nq, k), -1, dtype=torch.int64, device="cuda")
    out_scores = torch.full((nq, k), float("nan"), dtype=torch.float64, device="cuda")
    out_counts = torch.full((nq,), -1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    eb = ErrBuf()
    rc = lib.svl_search_noalloc(rows.data_ptr(), ids.data_ptr(), rows.shape[0], dim, queries.data_ptr(), nq,
                                None if mask is None else mask.data_ptr(), k, out_rows.data_ptr(),
                                out_chunk.data_ptr(), out_scores.data_ptr(), out_counts.data_ptr(), None, *eb.args)
    eb.check(rc)
    return (out_rows.cpu().numpy().astype(np.uint64), out_chunk.cpu().numpy().astype(np.uint64),
            out_scores.cpu().numpy(), out_counts.cpu().numpy().astype(np.uint32))


def test_noalloc_search_matches_the_index_search_on_two_calls():
    import torch

    lib = load_library()
    rng = np.random.default_rng(31)
    n, dim, k = 30000, 768, 10
    raw = rng.standard_normal((n, dim), dtype=np.float32)
    ids = rng.permutation(n).astype(np.uint64) + 7
    index = VectorIndex(dim, n)
    index.append(raw, ids)
    # the same unit-norm rows the index stores: Chunk::new's f64 sum of squares
    # in dimension order, then (f64 value / norm) rounded to f32
    x = raw.astype(np.float64)
    sumsq = np.zeros(n, np.float64)
    for d in range(dim):
        sumsq += x[:, d] * x[:, d]
    stored = (x / np.sqrt(sumsq)[:, None]).astype(np.float32)
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
