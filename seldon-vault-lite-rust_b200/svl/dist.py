"""Multi-GPU plumbing: one process per GPU, torch.distributed for the
collectives (NCCL over NVLink on the B200 box, gloo on CPU in tests).

* Encoder: independent sequences shard with no collective.  ``balance`` assigns
  sequences to ranks by longest-processing-time on the forward's cost model
  (FLOPs linear + quadratic in length), weights are replicated.
* Search: the corpus is row-sharded; each rank returns its local top-k per
  query, one all-gather brings every shard's (score, chunk id, row) lists to
  every rank, and the lists are merged on the GPU in the reference's order
  (score desc, chunk id asc; vector.rs:90-95).  ``ShardedIndex`` does it all
  in the C ABI (``svl_sharded_search``: one NCCL all-gather of packed records)
  over an ``NcclComm``; ``ShardedSearch`` is the same over torch.distributed
  (four all-gathers and ``merge_topk_device``; any backend, gloo included).
* Ingest then query: ``assign_documents`` spreads the
  documents over the ranks (each rank appends its own to its own shard, no
  exchange), ``query_slice`` gives each rank its slice of the queries, and
  ``NcclComm.allgather_rows`` gives every rank every query embedding.
"""

from __future__ import annotations

import ctypes
import heapq

import numpy as np

from . import errors
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


def assign_documents(costs, world: int) -> list[list[int]]:
    """Document indices of each rank for data-parallel ingest (LPT on the
    forward's cost, like ``balance``); a document keeps its global index as
    its chunk id, so the shards together hold every document exactly once."""
    return balance(costs, world)


def query_slice(n_queries: int, world: int, rank: int) -> tuple[int, int]:
    """The contiguous slice of the queries rank `rank` embeds (equal sizes:
    n_queries must be a multiple of world, as the row all-gather needs)."""
    if n_queries % world:
        raise errors.UsageError(f"{n_queries} queries do not split evenly over {world} ranks")
    per = n_queries // world
    return rank * per, (rank + 1) * per


class NcclComm:
    """An NCCL communicator made by the library (svl_nccl_comm_create)."""

    ID_BYTES = 128

    def __init__(self, device: int, world: int, rank: int, unique_id: bytes):
        self._lib = load_library()
        if len(unique_id) != self.ID_BYTES:
            raise errors.UsageError("an NCCL unique id is 128 bytes")
        h = ctypes.c_void_p()
        eb = ErrBuf()
        buf = ctypes.create_string_buffer(bytes(unique_id), self.ID_BYTES)
        eb.check(self._lib.svl_nccl_comm_create(device, world, rank, buf, ctypes.byref(h), *eb.args))
        self.handle, self.device, self.world, self.rank = h, device, world, rank

    @staticmethod
    def unique_id() -> bytes:
        lib = load_library()
        buf = ctypes.create_string_buffer(NcclComm.ID_BYTES)
        eb = ErrBuf()
        eb.check(lib.svl_nccl_unique_id(buf, *eb.args))
        return buf.raw

    @classmethod
    def from_torch(cls, device: int, group=None) -> "NcclComm":
        """Every rank of a torch.distributed group joins one communicator; rank
        0's id travels over the group (any backend)."""
        import torch.distributed as dist

        obj = [cls.unique_id() if dist.get_rank(group) == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(device, dist.get_world_size(group), dist.get_rank(group), obj[0])

    def close(self, abort: bool = False):
        if getattr(self, "handle", None):
            self._lib.svl_nccl_comm_destroy(self.handle, 1 if abort else 0)
            self.handle = None

    def __del__(self):
        self.close()

    def allgather_rows(self, d_local, stream: int = 0):
        """d_local: CUDA float32 [n, dim] (same n on every rank) -> [world * n,
        dim], rank-major, on every rank (svl_allgather_rows)."""
        import torch

        n, dim = d_local.shape
        out = torch.empty((self.world * n, dim), dtype=torch.float32, device=d_local.device)
        eb = ErrBuf()
        eb.check(self._lib.svl_allgather_rows(self.handle, d_local.data_ptr(), n, dim, out.data_ptr(),
                                              stream or None, *eb.args))
        return out


class ShardedIndex:
    """This rank's shard of a row-sharded index, searched with
    svl_sharded_search: the global exact top-k on every rank, one NCCL
    all-gather of packed per-shard lists."""

    def __init__(self, index, row_offset: int, comm: NcclComm):
        self.index, self.row_offset, self.comm = index, row_offset, comm

    def search(self, d_queries, k: int, stream: int = 0):
        """d_queries: CUDA float32 [Q, dim], the same on every rank.  Returns
        (scores f64, chunk_ids i64, global rows i64, counts i32) CUDA tensors."""
        import torch

        Q = d_queries.shape[0]
        dev = d_queries.device
        rows = torch.empty((Q, k), dtype=torch.int64, device=dev)
        chunks = torch.empty((Q, k), dtype=torch.int64, device=dev)
        scores = torch.empty((Q, k), dtype=torch.float64, device=dev)
        counts = torch.empty((Q,), dtype=torch.int32, device=dev)
        eb = ErrBuf()
        eb.check(self.index._lib.svl_sharded_search(self.comm.handle, self.index.handle, self.row_offset,
                                                    d_queries.data_ptr(), Q, k, rows.data_ptr(), chunks.data_ptr(),
                                                    scores.data_ptr(), counts.data_ptr(), stream or None, *eb.args))
        return scores, chunks, rows, counts
