"""The multi-GPU C ABI on B200s: svl_nccl_comm_create, svl_allgather_rows and
svl_sharded_search (one NCCL all-gather of packed per-shard lists, merged on
every rank).

On one GPU a one-rank communicator runs the whole path (search, packing,
all-gather, merge); its answer must equal svl_index_search exactly --
identical rows, chunk ids and bit-identical f64 scores -- including k past
the fast path's 32 and a query whose near-ties need the exact full path.
With two GPUs, two processes (one per GPU) each hold half of a corpus and
must both return the oracle's global top-k (vector::rank,
src/index/vector.rs:17-97)."""

import os
import socket
import time

import numpy as np
import pytest

import oracle
from svl import dist as sdist
from svl.index import VectorIndex

pytestmark = pytest.mark.gpu


def _stored(raw):
    return np.stack([oracle.normalize_embedding(r) for r in raw])


@pytest.fixture(scope="module")
def comm1():
    import torch

    torch.cuda.set_device(0)
    c = sdist.NcclComm(0, 1, 0, sdist.NcclComm.unique_id())
    yield c
    c.close()


def test_one_rank_allgather_is_the_identity(comm1):
    import torch

    x = torch.randn((37, 24), device="cuda")
    y = comm1.allgather_rows(x)
    torch.cuda.synchronize()
    assert torch.equal(x, y)


@pytest.mark.parametrize("k", [10, 100])
def test_one_rank_sharded_search_equals_the_index_search(comm1, k):
    import torch

    rng = np.random.default_rng(61)
    n, dim = 20000, 256
    raw = rng.standard_normal((n, dim), dtype=np.float32)
    ids = rng.permutation(n).astype(np.uint64) * 5 + 3
    idx = VectorIndex(dim, n)
    idx.append(raw, ids)
    q = rng.standard_normal((50, dim), dtype=np.float32)
    want = idx.search(q, k)
    for _ in range(2):
        sc, ch, rw, cn = sdist.ShardedIndex(idx, 1000, comm1).search(torch.from_numpy(q).cuda(), k)
        torch.cuda.synchronize()
        idx.check()
        assert np.array_equal(cn.cpu().numpy().astype(np.uint32), want[3])
        assert np.array_equal(rw.cpu().numpy().astype(np.uint64), want[0] + 1000)
        assert np.array_equal(ch.cpu().numpy().astype(np.uint64), want[1])
        assert np.array_equal(sc.cpu().numpy(), want[2])


def test_one_rank_sharded_search_resolves_near_ties(comm1):
    """400 rows within 1e-3 of the query defeat the screen's margin: the
    exact full path answers them inside svl_sharded_search."""
    import torch

    rng = np.random.default_rng(7)
    q = rng.standard_normal(128, dtype=np.float32)
    q /= np.linalg.norm(q)
    near = q[None, :] + 1e-3 * rng.standard_normal((400, 128), dtype=np.float32)
    far = rng.standard_normal((30000, 128), dtype=np.float32)
    raw = np.concatenate([far[:15000], near, far[15000:]])
    ids = np.arange(raw.shape[0], dtype=np.uint64)
    idx = VectorIndex(128, raw.shape[0])
    idx.append(raw, ids)
    sc, ch, rw, cn = sdist.ShardedIndex(idx, 0, comm1).search(torch.from_numpy(q[None, :]).cuda(), 10)
    torch.cuda.synchronize()
    idx.check()
    r, s = oracle.vector_rank(q, _stored(raw), chunk_ids=ids)
    assert int(cn[0]) == 10
    assert np.array_equal(rw[0].cpu().numpy().astype(np.uint64), r[:10])
    assert np.array_equal(sc[0].cpu().numpy(), s[:10])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    # gloo carries the 128-byte NCCL id; the search's collective is the library's own
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    comm = sdist.NcclComm.from_torch(rank)
    rng = np.random.default_rng(71)
    n, dim, k, nq = 12000, 128, 12, 24
    raw = rng.standard_normal((n, dim), dtype=np.float32)
    ids = rng.permutation(n).astype(np.uint64) * 2
    q = rng.standard_normal((nq, dim), dtype=np.float32)
    r0, r1 = sdist.shard_range(n, world, rank)
    idx = VectorIndex(dim, r1 - r0, device=rank)
    idx.append(raw[r0:r1], ids[r0:r1])
    local_q = torch.from_numpy(q[rank * nq // world:(rank + 1) * nq // world]).cuda()
    all_q = comm.allgather_rows(local_q)
    sc, ch, rw, cn = sdist.ShardedIndex(idx, r0, comm).search(all_q, k)
    torch.cuda.synchronize()
    idx.check()
    stored = _stored(raw)
    ref_rows, ref_scores = oracle.vector_topk(q, stored, k, chunk_ids=ids)
    ok = (np.array_equal(all_q.cpu().numpy(), q) and (cn.cpu().numpy() == k).all()
          and np.array_equal(rw.cpu().numpy().astype(np.uint64), ref_rows)
          and np.array_equal(sc.cpu().numpy(), ref_scores)
          and np.array_equal(ch.cpu().numpy().astype(np.uint64), ids[ref_rows.astype(np.int64)]))
    with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
        f.write("ok" if ok else "mismatch")
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


def test_two_gpus_sharded_search_matches_the_oracle(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.start_processes(_two_gpu_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.time() + 180
    while not ctx.join(timeout=5):
        if time.time() > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail("two-GPU sharded search did not finish in 180 s")
    for r in range(2):
        assert (tmp_path / f"rank{r}").read_text() == "ok"
