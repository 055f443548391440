"""Multi-GPU plumbing: one process per GPU, torch.distributed for the
collectives (NCCL over NVLink on the B200 box, gloo on CPU in tests).

* Encoder: independent sequences shard with no collective.  ``balance`` assigns
  sequences to ranks by longest-processing-time on the forward's cost model
  (FLOPs linear + quadratic in length), weights are replicated.
* Search: the corpus is row-sharded; each rank returns its local top-k per
  query, one all-gather brings every shard's (score, chunk id, row) lists to
  every rank, and ``merge_topk_device`` merges them on the GPU in the
  reference's order (score desc, chunk id asc; vector.rs:90-95).
"""

from __future__ import annotations

import ctypes
import heapq

import numpy as np

from ._abi import ErrBuf, load_library


def balance(costs, world: int) -> list[list[int]]:
    """LPT: items sorted by cost descending, each to the least-loaded rank.
    Deterministic (ties by item index, then rank index)."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(world)]
    parts = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + float(costs[i]), r))
    return [sorted(p) for p in parts]


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous row range of `rank` in an n-row corpus."""
    return n * rank // world, n * (rank + 1) // world


def merge_topk_device(scores, chunk_ids, rows, counts, k: int, stream: int = 0):
    """Merges shard-major lists ([S, Q, k] f64 scores / int64 chunk ids / int64
    rows, [S, Q] int32 counts; CUDA torch tensors) into the global top-k.
    Returns (scores [Q,k], chunk_ids [Q,k], rows [Q,k], shard [Q,k], counts [Q])."""
    import torch

    lib = load_library()
    S, Q, kk = scores.shape
    assert kk == k
    dev = scores.device
    out_s = torch.empty((Q, k), dtype=torch.float64, device=dev)
    out_c = torch.empty((Q, k), dtype=torch.int64, device=dev)
    out_r = torch.empty((Q, k), dtype=torch.int64, device=dev)
    out_sh = torch.empty((Q, k), dtype=torch.int32, device=dev)
    out_n = torch.empty((Q,), dtype=torch.int32, device=dev)
    eb = ErrBuf()
    eb.check(lib.svl_merge_topk_device(dev.index or 0, scores.data_ptr(), chunk_ids.data_ptr(),
                                       rows.data_ptr() if rows is not None else None, counts.data_ptr(), S, Q, k,
                                       out_s.data_ptr(), out_c.data_ptr(), out_r.data_ptr(), out_sh.data_ptr(),
                                       out_n.data_ptr(), stream or None, *eb.args))
    return out_s, out_c, out_r, out_sh, out_n


def all_gather_lists(scores, chunk_ids, rows, counts, group=None):
    """All-gathers per-shard lists into shard-major tensors on every rank."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    outs = []
    for t in (scores, chunk_ids, rows, counts):
        t = t.contiguous()
        if t.is_cuda:
            o = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(o, t, group=group)
        else:  # gloo on CPU tensors
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t, group=group)
            o = torch.stack(parts)
        outs.append(o)
    return outs


class ShardedSearch:
    """This rank's shard of a row-sharded exact index plus the global merge."""

    def __init__(self, index, row_offset: int, group=None):
        self.index = index
        self.row_offset = row_offset
        self.group = group

    def search(self, d_queries, k: int, stream: int = 0):
        """d_queries: CUDA float32 [Q, dim] on this rank (all ranks pass the same
        queries).  Returns the merged global (scores, chunk_ids, rows, counts)."""
        import torch

        Q = d_queries.shape[0]
        dev = d_queries.device
        rows = torch.empty((Q, k), dtype=torch.int64, device=dev)
        chunks = torch.empty((Q, k), dtype=torch.int64, device=dev)
        scores = torch.empty((Q, k), dtype=torch.float64, device=dev)
        counts = torch.empty((Q,), dtype=torch.int32, device=dev)
        self.index.search_device(d_queries.data_ptr(), Q, k, rows.data_ptr(), chunks.data_ptr(), scores.data_ptr(),
                                 counts.data_ptr(), stream=stream)
        rows += self.row_offset
        g = all_gather_lists(scores, chunks, rows, counts, self.group)
        ms, mc, mr, _, mn = merge_topk_device(*g, k, stream=stream)
        return ms, mc, mr, mn
