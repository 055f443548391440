"""Multi-process host logic of the multi-GPU path, on CPU with the gloo
backend (world size 2): the data-parallel split of the encoder batch and the
row-sharded search whose per-shard top-k lists are all-gathered and merged.

The per-shard search and the per-rank forward are the CPU oracle here (a
stand-in for each rank's GPU); what is under test is the sharding, the
gathered layout and the merge order (score desc, chunk id asc), which must
reproduce the single-process answer exactly.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from svl import dist as sdist


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _merge_host(scores, chunk_ids, rows, counts, k):
    S, Q, _ = scores.shape
    out = []
    for q in range(Q):
        e = [(-float(scores[s, q, i]), int(chunk_ids[s, q, i]), int(rows[s, q, i]))
             for s in range(S) for i in range(int(counts[s, q]))]
        e.sort()
        out.append(e[:k])
    return out


def _search_worker(rank, world, port, result_path):
    import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(0)
    n, dim, k, nq = 3000, 48, 7, 5
    raw = rng.standard_normal((n, dim), dtype=np.float32)
    corpus = np.stack([oracle.normalize_embedding(r) for r in raw])
    ids = rng.permutation(n).astype(np.uint64) * 3
    q = rng.standard_normal((nq, dim), dtype=np.float32)
    r0, r1 = sdist.shard_range(n, world, rank)
    rows, scores = oracle.vector_topk(q, corpus[r0:r1], k, chunk_ids=ids[r0:r1])
    rows = rows.astype(np.int64) + r0
    chunks = ids[rows].astype(np.int64)
    counts = np.full(nq, k, np.int32)
    g = sdist.all_gather_lists(torch.from_numpy(scores), torch.from_numpy(chunks), torch.from_numpy(rows),
                               torch.from_numpy(counts))
    merged = _merge_host(*(t.numpy() for t in g), k)
    if rank == 0:
        ref_rows, ref_scores = oracle.vector_topk(q, corpus, k, chunk_ids=ids)
        ok = all([r for (_, _, r) in merged[qi]] == ref_rows[qi].tolist() and
                 [-s for (s, _, _) in merged[qi]] == ref_scores[qi].tolist() for qi in range(nq))
        with open(result_path, "w") as f:
            f.write("ok" if ok else "mismatch")
    dist.barrier()
    dist.destroy_process_group()


def _encoder_worker(rank, world, port, result_path):
    import json

    import oracle
    from svl import safetensors
    from svl.config import TextConfig
    from svl.text import pack

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    here = os.path.join(os.path.dirname(__file__), "golden", "tiny_text")
    cfg = TextConfig.from_file(os.path.join(here, "config.json"))
    model = oracle.OracleModel(cfg, safetensors.load(os.path.join(here, "model.safetensors")))
    rng = np.random.default_rng(1)
    seqs = [rng.integers(0, cfg.vocab_size, size=int(L)).astype(np.uint32) for L in rng.integers(1, 40, size=11)]
    parts = sdist.balance([cfg.flops_per_sequence(s.size) for s in seqs], world)
    mine = parts[rank]
    ids, cu = pack([seqs[i] for i in mine])
    emb = model.embed_many(ids, cu, cfg.embedding_dim, threads=1)
    # gather (index, embedding) pairs from every rank
    width = max(len(p) for p in parts)
    buf = np.full((width, 1 + cfg.embedding_dim), -1.0, np.float32)
    buf[: len(mine), 0] = mine
    buf[: len(mine), 1:] = emb
    out = [torch.empty_like(torch.from_numpy(buf)) for _ in range(world)]
    dist.all_gather(out, torch.from_numpy(buf))
    if rank == 0:
        got = {}
        for t in out:
            for row in t.numpy():
                if row[0] >= 0:
                    got[int(row[0])] = row[1:]
        ids1, cu1 = pack(seqs)
        ref = model.embed_many(ids1, cu1, cfg.embedding_dim, threads=1)
        ok = sorted(got) == list(range(len(seqs))) and all(np.array_equal(got[i], ref[i]) for i in got)
        with open(result_path, "w") as f:
            f.write(json.dumps({"ok": ok, "parts": parts}))
    dist.barrier()
    dist.destroy_process_group()


def _ingest_then_query_worker(rank, world, port, result_path):
    """BASELINE configs[4]'s orchestration with CPU stand-ins for the GPUs:
    documents assigned by assign_documents (each rank's rows appended to its
    own shard, chunk id = document index), each rank embedding its
    query_slice, the query rows all-gathered rank-major, every shard searched
    with all the queries, the lists all-gathered and merged.  The merged
    top-k must equal one index holding every document."""
    import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    n_docs, dim, nq, k = 700, 40, 12, 9
    lengths = np.clip(np.rint(np.random.default_rng(5).lognormal(np.log(200.0), 0.8, size=n_docs)), 8, 2048)

    def embed(key):  # the stand-in encoder: a deterministic vector per key
        return np.random.default_rng(1000 + key).standard_normal(dim, dtype=np.float32)

    mine = sdist.assign_documents(list(lengths), world)[rank]
    shard = np.stack([oracle.normalize_embedding(embed(d)) for d in mine])
    a, b = sdist.query_slice(nq, world, rank)
    local_q = torch.from_numpy(np.stack([embed(100000 + i) for i in range(a, b)]))
    parts = [torch.empty_like(local_q) for _ in range(world)]
    dist.all_gather(parts, local_q)
    queries = torch.cat(parts).numpy()
    rows, scores = oracle.vector_topk(queries, shard, k, chunk_ids=np.asarray(mine, np.uint64))
    chunks = np.asarray(mine, np.int64)[rows.astype(np.int64)]
    counts = np.full(nq, min(k, len(mine)), np.int32)
    g = sdist.all_gather_lists(torch.from_numpy(scores), torch.from_numpy(chunks),
                               torch.from_numpy(rows.astype(np.int64)), torch.from_numpy(counts))
    merged = _merge_host(*(t.numpy() for t in g), k)
    if rank == 0:
        everything = np.stack([oracle.normalize_embedding(embed(d)) for d in range(n_docs)])
        all_q = np.stack([embed(100000 + i) for i in range(nq)])
        ref_rows, ref_scores = oracle.vector_topk(all_q, everything, k)
        ok = np.array_equal(queries, all_q) and all(
            [c for (_, c, _) in merged[qi]] == ref_rows[qi].tolist() and
            [-s for (s, _, _) in merged[qi]] == ref_scores[qi].tolist() for qi in range(nq))
        with open(result_path, "w") as f:
            f.write("ok" if ok else "mismatch")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("worker,expect", [(_search_worker, "ok"), (_encoder_worker, None),
                                           (_ingest_then_query_worker, "ok")])
def test_two_rank_gloo(tmp_path, worker, expect):
    path = str(tmp_path / "result")
    mp.start_processes(worker, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    text = open(path).read()
    if expect:
        assert text == expect
    else:
        import json

        r = json.loads(text)
        assert r["ok"]
        assert sorted(i for p in r["parts"] for i in p) == list(range(11))


def test_balance_is_deterministic_and_balanced():
    costs = [5, 3, 8, 1, 1, 9, 2, 7]
    a = sdist.balance(costs, 3)
    assert a == sdist.balance(costs, 3)
    assert sorted(i for p in a for i in p) == list(range(len(costs)))
    loads = [sum(costs[i] for i in p) for p in a]
    assert max(loads) - min(loads) <= max(costs)


def test_shard_ranges_tile_the_corpus():
    for n in (0, 1, 7, 10_000_000):
        for world in (1, 2, 3, 8):
            ranges = [sdist.shard_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
