// multi.cu -- the multi-GPU entry points: one process per GPU, NCCL over
// NVLink / NVSwitch.
//
// The reference is a single-process program (no collective anywhere); these
// calls exist for the row-sharded index of the B200 build:
//   * svl_nccl_unique_id / svl_nccl_comm_create / svl_nccl_comm_destroy: a
//     communicator over the ranks, so a host without its own NCCL binding (the
//     std-only Rust crate) can set one up; the 128-byte id travels between
//     the processes by whatever means the host has;
//   * svl_allgather_rows: the query stage of ingest-then-query (BASELINE
//     configs[4]) -- each rank embeds its slice of the queries, one all-gather
//     gives every rank every query so that each shard scores all of them;
//   * svl_sharded_search: vector::rank's top-k over the union of the ranks'
//     shards (src/index/vector.rs:17-97): each rank searches its shard, the
//     per-shard lists travel in ONE all-gather of packed (score, chunk id,
//     global row) records with the counts and the rank's status in the same
//     block, and every rank merges them on its GPU in the reference's order
//     (score descending, chunk id ascending).
// NCCL is not linked: libnccl.so.2 is opened at run time the first time one
// of these calls needs it, which binds to the copy already loaded in the
// process when there is one (a communicator only works with the library that
// created it).  No TMA multicast and no peer-memory loads are involved.

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "../../include/svl_gpu.h"
#include "common.cuh"
#include "model.cuh"
#include "search.cuh"

namespace svl {

namespace {

// The NCCL entry points these calls use, resolved from the shared library.
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string load_error;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      api.load_error = std::string("cannot load libnccl.so.2: ") + (e ? e : "not found");
      return;
    }
    bool ok = true;
    auto sym = [&](const char* name, auto* fn) {
      void* p = dlsym(h, name);
      if (!p) ok = false;
      *fn = reinterpret_cast<std::remove_reference_t<decltype(*fn)>>(p);
    };
    sym("ncclGetUniqueId", &api.get_unique_id);
    sym("ncclCommInitRank", &api.comm_init_rank);
    sym("ncclCommDestroy", &api.comm_destroy);
    sym("ncclCommAbort", &api.comm_abort);
    sym("ncclCommCount", &api.comm_count);
    sym("ncclCommUserRank", &api.comm_user_rank);
    sym("ncclAllGather", &api.all_gather);
    sym("ncclGetErrorString", &api.error_string);
    if (!ok) {
      api = NcclApi{};
      api.load_error = "libnccl.so.2 lacks an entry point this library needs";
    }
  });
  return api;
}

bool nccl_ready(std::string* msg) {
  const NcclApi& a = nccl();
  if (!a.all_gather) {
    *msg = a.load_error;
    return false;
  }
  return true;
}

std::string nccl_msg(const char* what, ncclResult_t r) {
  const NcclApi& a = nccl();
  return std::string(what) + " failed: " + (a.error_string ? a.error_string(r) : "NCCL error");
}

// One shard's result record in the exchanged block.
struct ShardHit {
  double score;
  uint64_t chunk_id;
  uint64_t row;  // global row: the shard's row offset + its local row
};

// Exchanged block of one rank: n_queries * k records, then n_queries counts,
// then the rank's status (svl_status), padded to 8 bytes.
size_t block_bytes(uint32_t nq, uint32_t k) {
  return (size_t)nq * k * sizeof(ShardHit) + (((size_t)nq + 1) * 4 + 7) / 8 * 8;
}

__global__ void pack_hits_kernel(const double* __restrict__ scores, const uint64_t* __restrict__ chunks,
                                 const uint64_t* __restrict__ rows, const uint32_t* __restrict__ counts,
                                 uint64_t row_offset, uint32_t nq, uint32_t k, uint32_t status, uint8_t* block) {
  ShardHit* rec = (ShardHit*)block;
  uint32_t* cnt = (uint32_t*)(block + (size_t)nq * k * sizeof(ShardHit));
  const size_t n = (size_t)nq * k;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t q = (uint32_t)(i / k), j = (uint32_t)(i - (size_t)q * k);
    const uint32_t c = status ? 0u : counts[q];
    ShardHit h{0.0, 0, 0};
    if (j < c) h = ShardHit{scores[i], chunks[i], rows[i] + row_offset};
    rec[i] = h;
    if (j == 0) cnt[q] = c;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) cnt[nq] = status;
}

// k-way merge of the gathered blocks, one thread per query; blocks whose
// rank reported a failure are skipped and flagged in the error word.
__global__ void merge_blocks_kernel(const uint8_t* __restrict__ gathered, size_t blk, uint32_t n_shards, uint32_t nq,
                                    uint32_t k, double* out_scores, uint64_t* out_chunk_ids, uint64_t* out_rows,
                                    uint32_t* out_counts, uint32_t* err) {
  const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const size_t cnt_off = (size_t)nq * k * sizeof(ShardHit);
  uint32_t head[64], cnt[64];
  bool peer_failed = false;
  for (uint32_t s = 0; s < n_shards; ++s) {
    const uint32_t* c = (const uint32_t*)(gathered + s * blk + cnt_off);
    const bool bad = c[nq] != 0;
    peer_failed |= bad;
    head[s] = 0;
    cnt[s] = bad ? 0u : (c[q] < k ? c[q] : k);
  }
  if (peer_failed && q == 0) atomicOr(err, SVL_DEVERR_PEER);
  uint32_t n = 0;
  for (; n < k; ++n) {
    int best = -1;
    ShardHit b{0.0, 0, 0};
    for (uint32_t s = 0; s < n_shards; ++s) {
      if (head[s] >= cnt[s]) continue;
      const ShardHit h = ((const ShardHit*)(gathered + s * blk))[(size_t)q * k + head[s]];
      if (best < 0 || h.score > b.score || (h.score == b.score && h.chunk_id < b.chunk_id)) {
        best = (int)s;
        b = h;
      }
    }
    if (best < 0) break;
    const size_t o = (size_t)q * k + n;
    out_scores[o] = b.score;
    if (out_chunk_ids) out_chunk_ids[o] = b.chunk_id;
    out_rows[o] = b.row;
    ++head[best];
  }
  out_counts[q] = n;
}

}  // namespace

}  // namespace svl

using svl::drain_device_error;
using svl::set_err;

extern "C" {

int svl_nccl_unique_id(void* id_out, char* err, size_t err_len) {
  std::string msg;
  if (!id_out) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  if (!svl::nccl_ready(&msg)) {
    set_err(err, err_len, msg);
    return SVL_UNSUPPORTED;
  }
  ncclUniqueId id;
  ncclResult_t r = svl::nccl().get_unique_id(&id);
  if (r != ncclSuccess) {
    set_err(err, err_len, svl::nccl_msg("ncclGetUniqueId", r));
    return SVL_INTERNAL;
  }
  std::memcpy(id_out, &id, sizeof(id));
  return SVL_OK;
}

int svl_nccl_comm_create(int device, int n_ranks, int rank, const void* id, void** comm_out, char* err,
                         size_t err_len) {
  std::string msg;
  if (!id || !comm_out || n_ranks < 1 || rank < 0 || rank >= n_ranks) {
    set_err(err, err_len, "invalid communicator arguments");
    return SVL_USAGE;
  }
  *comm_out = nullptr;
  if (n_ranks > 64) {
    set_err(err, err_len, "at most 64 ranks");
    return SVL_LIMIT_EXCEEDED;
  }
  if (!svl::nccl_ready(&msg)) {
    set_err(err, err_len, msg);
    return SVL_UNSUPPORTED;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    set_err(err, err_len, "cannot select CUDA device " + std::to_string(device));
    return SVL_INTERNAL;
  }
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t comm = nullptr;
  ncclResult_t r = svl::nccl().comm_init_rank(&comm, n_ranks, uid, rank);
  if (r != ncclSuccess) {
    set_err(err, err_len, svl::nccl_msg("ncclCommInitRank", r));
    return SVL_INTERNAL;
  }
  *comm_out = comm;
  return SVL_OK;
}

int svl_nccl_comm_destroy(void* comm, int abort) {
  if (!comm) return SVL_OK;
  std::string msg;
  if (!svl::nccl_ready(&msg)) return SVL_UNSUPPORTED;
  const svl::NcclApi& a = svl::nccl();
  ncclResult_t r = abort ? a.comm_abort((ncclComm_t)comm) : a.comm_destroy((ncclComm_t)comm);
  return r == ncclSuccess ? SVL_OK : SVL_INTERNAL;
}

int svl_allgather_rows(void* comm, const float* d_local, uint64_t n_local, uint32_t dim, float* d_all, void* stream,
                       char* err, size_t err_len) {
  std::string msg;
  if (!comm || (!d_local && n_local) || (!d_all && n_local) || !dim) {
    set_err(err, err_len, "null or empty argument");
    return SVL_USAGE;
  }
  if (!svl::nccl_ready(&msg)) {
    set_err(err, err_len, msg);
    return SVL_UNSUPPORTED;
  }
  ncclResult_t r = svl::nccl().all_gather(d_local, d_all, (size_t)n_local * dim, ncclFloat32, (ncclComm_t)comm,
                                          (cudaStream_t)stream);
  if (r != ncclSuccess) {
    set_err(err, err_len, svl::nccl_msg("ncclAllGather", r));
    return SVL_INTERNAL;
  }
  return SVL_OK;
}

int svl_sharded_search(void* comm, svl_index* shard, uint64_t row_offset, const float* d_queries, uint32_t n_queries,
                       uint32_t k, uint64_t* d_out_rows, uint64_t* d_out_chunk_ids, double* d_out_scores,
                       uint32_t* d_out_counts, void* stream, char* err, size_t err_len) {
  std::string msg;
  if (!comm || !shard || !d_queries || !d_out_rows || !d_out_scores || !d_out_counts) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  if (k == 0) {
    set_err(err, err_len, "k must be at least 1");
    return SVL_USAGE;
  }
  if (k > SVL_SHARDED_MAX_K) {
    set_err(err, err_len, "svl_sharded_search takes k up to " + std::to_string(SVL_SHARDED_MAX_K));
    return SVL_LIMIT_EXCEEDED;
  }
  if (!svl::nccl_ready(&msg)) {
    set_err(err, err_len, msg);
    return SVL_UNSUPPORTED;
  }
  const svl::NcclApi& api = svl::nccl();
  int world = 0;
  ncclResult_t r = api.comm_count((ncclComm_t)comm, &world);
  if (r != ncclSuccess || world < 1 || world > 64) {
    set_err(err, err_len, r != ncclSuccess ? svl::nccl_msg("ncclCommCount", r) : "1..64 ranks");
    return SVL_INTERNAL;
  }
  if (n_queries == 0) return SVL_OK;
  svl::Index& x = shard->x;
  std::lock_guard<std::mutex> lock(x.mu);
  cudaSetDevice(x.device);
  cudaStream_t st = stream ? (cudaStream_t)stream : x.stream;
  const size_t nq = n_queries;
  const size_t blk = svl::block_bytes(n_queries, k);
  uint64_t* l_rows = (uint64_t*)x.workspace("shard_rows", nq * k * 8);
  uint64_t* l_chunk = (uint64_t*)x.workspace("shard_chunk", nq * k * 8);
  double* l_scores = (double*)x.workspace("shard_scores", nq * k * 8);
  uint32_t* l_counts = (uint32_t*)x.workspace("shard_counts", nq * 4);
  uint8_t* send = (uint8_t*)x.workspace("shard_send", blk);
  uint8_t* recv = (uint8_t*)x.workspace("shard_recv", blk * world);
  if (!send || !recv) {
    // nothing to exchange: the other ranks' all-gather cannot complete; the
    // caller aborts the communicator on every rank
    set_err(err, err_len, "out of device memory for the exchange buffers; abort the communicator");
    return SVL_LIMIT_EXCEEDED;
  }
  // local search; a failure still takes part in the exchange, with its status
  int local = SVL_OK;
  if (!l_rows || !l_chunk || !l_scores || !l_counts) {
    local = SVL_LIMIT_EXCEEDED;
    msg = "out of device memory for the shard search";
  }
  std::vector<uint8_t> fb(nq, 0);
  if (local == SVL_OK)
    local = x.search_device(d_queries, n_queries, nullptr, k, l_rows, l_chunk, l_scores, l_counts, st, fb.data(), &msg);
  if (cudaStreamSynchronize(st) != cudaSuccess && local == SVL_OK) {
    local = SVL_INTERNAL;
    msg = "CUDA error in the shard search";
  }
  if (local == SVL_OK)
    local = x.resolve_fallbacks(d_queries, n_queries, fb.data(), nullptr, k, l_rows, l_chunk, l_scores, l_counts, st,
                                &msg);
  if (local == SVL_OK) local = drain_device_error(x.err_d, x.err_h, st, &msg);
  svl::pack_hits_kernel<<<(unsigned)std::min<size_t>((nq * k + 255) / 256, 1184), 256, 0, st>>>(
      l_scores, l_chunk, l_rows, l_counts, row_offset, n_queries, k, (uint32_t)local, send);
  r = api.all_gather(send, recv, blk / 8, ncclUint64, (ncclComm_t)comm, st);
  if (r != ncclSuccess) {
    set_err(err, err_len, svl::nccl_msg("ncclAllGather", r));
    return SVL_INTERNAL;
  }
  svl::merge_blocks_kernel<<<(n_queries + 127) / 128, 128, 0, st>>>(recv, blk, (uint32_t)world, n_queries, k,
                                                                     d_out_scores, d_out_chunk_ids, d_out_rows,
                                                                     d_out_counts, x.err_d);
  if (cudaGetLastError() != cudaSuccess && local == SVL_OK) {
    local = SVL_INTERNAL;
    msg = "merge launch failed";
  }
  if (local != SVL_OK) set_err(err, err_len, msg);
  return local;
}

}  // extern "C"
