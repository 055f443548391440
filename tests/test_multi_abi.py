"""Host side of the multi-GPU C ABI (include/svl_gpu.h, "multi-GPU"), on CPU:
NCCL is opened at run time and its unique id made without a GPU; argument
errors come back as the reference's error variants before any device or
collective work; the ingest-then-query partition helpers."""

import ctypes

import numpy as np
import pytest

from svl import dist as sdist
from svl import errors
from svl._abi import ErrBuf, load_library


def test_nccl_unique_id_is_128_bytes():
    a, b = sdist.NcclComm.unique_id(), sdist.NcclComm.unique_id()
    assert len(a) == len(b) == 128 and a != b


def test_sharded_search_rejects_bad_arguments_before_any_work():
    lib = load_library()
    eb = ErrBuf()
    dummy = ctypes.c_void_p(16)  # never dereferenced: every check below precedes any use
    args = (dummy, dummy, 0, dummy, 4)
    with pytest.raises(errors.UsageError):
        eb.check(lib.svl_sharded_search(None, dummy, 0, dummy, 4, 10, dummy, None, dummy, dummy, None, *eb.args))
    with pytest.raises(errors.UsageError):
        eb.check(lib.svl_sharded_search(*args, 0, dummy, None, dummy, dummy, None, *eb.args))
    with pytest.raises(errors.LimitExceededError):
        eb.check(lib.svl_sharded_search(*args, 4097, dummy, None, dummy, dummy, None, *eb.args))
    with pytest.raises(errors.UsageError):
        eb.check(lib.svl_nccl_comm_create(0, 2, 2, dummy, ctypes.byref(ctypes.c_void_p()), *eb.args))
    with pytest.raises(errors.UsageError):
        eb.check(lib.svl_allgather_rows(None, dummy, 4, 8, dummy, None, *eb.args))
    with pytest.raises(errors.UsageError):
        sdist.NcclComm(0, 2, 0, b"short")


def test_documents_are_assigned_once_and_queries_split_evenly():
    rng = np.random.default_rng(0)
    costs = rng.lognormal(5, 1, size=1000)
    for world in (1, 2, 3, 8):
        parts = sdist.assign_documents(costs, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(1000))
        loads = [costs[p].sum() for p in parts]
        assert max(loads) - min(loads) <= costs.max()  # LPT: within one item
        spans = [sdist.query_slice(4096, world, r) for r in range(world)] if 4096 % world == 0 else []
        if spans:
            assert spans[0][0] == 0 and spans[-1][1] == 4096
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(errors.UsageError):
        sdist.query_slice(4096, 3, 0)
