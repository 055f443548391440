// search.cuh -- device-resident exact cosine index behind svl_index.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <string>

#include "profiler.cuh"

namespace svl {

constexpr uint32_t kMaxEmbeddingDimension = 8192;  // storage/model.rs:35
constexpr int kMaxFastK = 32;                      // larger k takes the full-ranking path

struct ScreenParams {
  int n_queries;
  uint64_t n_rows;
  int dim;
  const uint8_t* mask;
  int n_qb, n_ranges;
  int n_lists;        // candidate lists per query: 2 per corpus range (one per column half)
  float* cand_score;  // [nq][n_lists][kc]
  uint32_t* cand_row;
  float* tau;         // [nq][n_lists]
  uint32_t* err;
};

struct RescoreParams {
  const float* queries;
  const double* qnorm;
  const float* rows;
  const uint64_t* chunk_ids;
  int dim, n_lists, kc, k;
  const float* cand_score;
  const uint32_t* cand_row;
  const float* tau;
  uint64_t* out_rows;
  uint64_t* out_chunk_ids;
  double* out_scores;
  uint32_t* out_count;
  uint8_t* fallback;
  uint32_t* err;
};

struct Index {
  int device = -1;
  cudaStream_t stream = nullptr;
  uint32_t dim = 0;
  uint64_t capacity = 0, len = 0;
  float* rows = nullptr;         // [capacity][dim], unit norm (Chunk::new)
  uint16_t* rows16 = nullptr;    // [capacity][dim] FP16 copy the screen reads (null: TF32 screen of `rows`)
  uint64_t* chunk_ids = nullptr;  // [capacity]
  uint64_t* order = nullptr;      // rows by ascending chunk id (full path)
  bool order_valid = false;
  uint64_t fallbacks = 0;         // queries answered by the full path after the fast-path check
  struct Buf {
    void* ptr = nullptr;
    size_t bytes = 0;
  };
  std::map<std::string, Buf> ws;
  uint32_t* err_d = nullptr;
  uint32_t* err_h = nullptr;
  Profiler prof;
  std::mutex mu;

  ~Index();
  int create(int dev, uint32_t dim, uint64_t capacity, std::string* msg);
  void* workspace(const char* name, size_t bytes);
  int append_device(const float* d_rows, const uint64_t* d_ids, uint64_t n, cudaStream_t st, bool ids_on_host,
                    const uint64_t* h_ids, std::string* msg);
  int ensure_order(cudaStream_t st);
  int search_full_one(const float* d_query, double qn, const uint8_t* d_mask, uint32_t k, uint64_t* d_rows,
                      uint64_t* d_chunk, double* d_scores, uint32_t* d_count, cudaStream_t st);
  int search_device(const float* d_queries, uint32_t nq, const uint8_t* d_mask, uint32_t k, uint64_t* d_rows,
                    uint64_t* d_chunk, double* d_scores, uint32_t* d_counts, cudaStream_t st, uint8_t* fallback_h,
                    std::string* msg);
  int resolve_fallbacks(const float* d_queries, uint32_t nq, const uint8_t* fallback_h, const uint8_t* d_mask,
                        uint32_t k, uint64_t* d_rows, uint64_t* d_chunk, double* d_scores, uint32_t* d_counts,
                        cudaStream_t st, std::string* msg);
};

int merge_topk_device(const double* scores, const uint64_t* chunk_ids, const uint64_t* rows, const uint32_t* counts,
                      uint32_t n_shards, uint32_t nq, uint32_t k, double* out_scores, uint64_t* out_chunk_ids,
                      uint64_t* out_rows, uint32_t* out_shard, uint32_t* out_counts, cudaStream_t st);

}  // namespace svl

struct svl_index {
  svl::Index x;
};
