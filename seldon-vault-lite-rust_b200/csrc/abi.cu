// abi.cu -- the extern "C" entry points of include/svl_gpu.h and
// include/svl_gpu_testing.h.  No exception or C++ type crosses this file's
// boundary; every failure becomes an svl_status plus a message.

#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/svl_gpu.h"
#include "../../include/svl_gpu_testing.h"
#include "common.cuh"
#include "attention_f16.cuh"
#include "attention_tc.cuh"
#include "encoder_kernels.cuh"
#include "gemm_tc.cuh"
#include "model.cuh"
#include "search.cuh"

using svl::drain_device_error;
using svl::set_err;

namespace {


struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  bool alloc(size_t n) { return cudaMalloc(&p, n ? n : 1) == cudaSuccess; }
};

}  // namespace

extern "C" {

uint32_t svl_abi_version(void) { return SVL_ABI_VERSION; }

int svl_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return -1;
  return n;
}

int svl_model_create(const svl_text_config* config, const svl_tensor_view* tensors, size_t n_tensors, int device,
                     svl_model** out, char* err, size_t err_len) {
  svl_model_options opts{};
  const char* e = std::getenv("SVL_PRECISION");
  opts.precision = e && std::strcmp(e, "split") == 0 ? SVL_PRECISION_SPLIT : SVL_PRECISION_FAST;
  return svl_model_create_ex(config, tensors, n_tensors, device, &opts, out, err, err_len);
}

int svl_model_precision(const svl_model* model, uint32_t* out) {
  if (!model || !out) return SVL_USAGE;
  *out = model->m.split ? SVL_PRECISION_SPLIT : SVL_PRECISION_FAST;
  return SVL_OK;
}

int svl_model_create_ex(const svl_text_config* config, const svl_tensor_view* tensors, size_t n_tensors, int device,
                        const svl_model_options* options, svl_model** out, char* err, size_t err_len) {
  if (!config || !out || (!tensors && n_tensors) || !config->layers) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  *out = nullptr;
  const uint32_t precision = options ? options->precision : SVL_PRECISION_FAST;
  if (options)
    for (uint32_t r : options->reserved)
      if (r) {
        set_err(err, err_len, "svl_model_options.reserved must be zero");
        return SVL_USAGE;
      }
  svl_model* m = new (std::nothrow) svl_model();
  if (!m) return SVL_INTERNAL;
  std::string msg;
  int rc = m->m.create(config, tensors, n_tensors, device, precision, &msg);
  if (rc != SVL_OK) {
    set_err(err, err_len, msg);
    delete m;
    return rc;
  }
  *out = m;
  return SVL_OK;
}

void svl_model_destroy(svl_model* model) { delete model; }

int svl_model_parameters(const svl_model* model, uint64_t* out) {
  if (!model || !out) return SVL_USAGE;
  *out = model->m.parameters;
  return SVL_OK;
}

static int forward_host(svl_model* model, const uint32_t* ids, const uint64_t* cu, uint32_t batch,
                        const float* features, const svl_feature_span* spans, uint32_t n_spans, uint32_t dim,
                        float* out, float* normalized, float* pooled, float* projected, float* hidden_states,
                        char* err, size_t err_len) {
  if (!model || !ids || !cu) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  svl::Model& m = model->m;
  std::lock_guard<std::mutex> lock(m.mu);
  std::string msg;
  int rc = m.validate_batch(ids, cu, batch, &msg);
  if (rc) {
    set_err(err, err_len, msg);
    return rc;
  }
  const uint64_t T = cu[batch];
  const size_t H = m.cfg.hidden_size, E = m.cfg.embedding_dim, L = m.cfg.num_hidden_layers;
  svl::FeatureRows frows;
  if (n_spans) {  // text.rs:226-275
    if (!features || !spans) {
      set_err(err, err_len, "multimodal features are missing");
      return SVL_CORRUPT;
    }
    if (m.cfg.pad_token_id < 0) {
      set_err(err, err_len, "model has no padding token for multimodal inputs");
      return SVL_UNSUPPORTED;
    }
    for (uint32_t i = 0; i < n_spans; ++i) {
      const svl_feature_span& s = spans[i];
      if (s.count == 0) {
        set_err(err, err_len, "multimodal feature replacement requires at least one token");
        return SVL_CORRUPT;
      }
      if (s.sequence >= batch || (uint64_t)s.start + s.count > cu[s.sequence + 1] - cu[s.sequence]) {
        set_err(err, err_len, "multimodal feature range is outside the sequence");
        return SVL_CORRUPT;
      }
      for (uint32_t r = 0; r < s.count; ++r) {
        const float* row = features + s.feature_offset + (size_t)r * H;
        for (size_t c = 0; c < H; ++c)
          if (!std::isfinite(row[c])) {
            set_err(err, err_len, "multimodal features contain a non-finite activation");
            return SVL_INTERNAL;
          }
        frows.rows.emplace_back(cu[s.sequence] + s.start + r, row);
      }
    }
  }
  cudaSetDevice(m.device);
  cudaStream_t st = m.stream;
  uint32_t* d_ids = (uint32_t*)m.workspace("io_ids", T * 4);
  uint64_t* d_cu = (uint64_t*)m.workspace("io_cu", (batch + 1) * 8);
  float* d_out = out ? (float*)m.workspace("io_out", (size_t)batch * dim * 4) : nullptr;
  float* d_norm = normalized ? (float*)m.workspace("io_norm", (size_t)batch * E * 4) : nullptr;
  float* d_pool = pooled ? (float*)m.workspace("io_pool", (size_t)batch * E * 4) : nullptr;
  float* d_proj = projected ? (float*)m.workspace("io_proj", T * E * 4) : nullptr;
  float* d_hid = hidden_states ? (float*)m.workspace("io_hidden", (L + 1) * T * H * 4) : nullptr;
  if (!d_ids || !d_cu || (out && !d_out) || (normalized && !d_norm) || (pooled && !d_pool) || (projected && !d_proj) ||
      (hidden_states && !d_hid)) {
    set_err(err, err_len, "out of device memory");
    return SVL_LIMIT_EXCEEDED;
  }
  cudaMemsetAsync(m.err_d, 0, 4, st);
  cudaMemcpyAsync(d_ids, ids, T * 4, cudaMemcpyHostToDevice, st);
  cudaMemcpyAsync(d_cu, cu, (batch + 1) * 8, cudaMemcpyHostToDevice, st);
  rc = m.forward(d_ids, cu, batch, d_cu, n_spans ? &frows : nullptr, out ? dim : (uint32_t)E, d_out, d_pool, d_norm,
                 d_proj, d_hid, st, &msg);
  if (rc) {
    set_err(err, err_len, msg);
    cudaStreamSynchronize(st);
    return rc;
  }
  if (out) cudaMemcpyAsync(out, d_out, (size_t)batch * dim * 4, cudaMemcpyDeviceToHost, st);
  if (normalized) cudaMemcpyAsync(normalized, d_norm, (size_t)batch * E * 4, cudaMemcpyDeviceToHost, st);
  if (pooled) cudaMemcpyAsync(pooled, d_pool, (size_t)batch * E * 4, cudaMemcpyDeviceToHost, st);
  if (projected) cudaMemcpyAsync(projected, d_proj, T * E * 4, cudaMemcpyDeviceToHost, st);
  if (hidden_states) cudaMemcpyAsync(hidden_states, d_hid, (L + 1) * T * H * 4, cudaMemcpyDeviceToHost, st);
  rc = drain_device_error(m.err_d, m.err_h, st, &msg);
  if (rc) set_err(err, err_len, msg);
  return rc;
}

int svl_forward_batch(svl_model* model, const uint32_t* ids, const uint64_t* cu_seqlens, uint32_t batch,
                      const float* features, const svl_feature_span* spans, uint32_t n_spans, float* normalized,
                      float* pooled, float* projected, float* hidden_states, char* err, size_t err_len) {
  if (!normalized) {
    set_err(err, err_len, "normalized output is required");
    return SVL_USAGE;
  }
  return forward_host(model, ids, cu_seqlens, batch, features, spans, n_spans, 0, nullptr, normalized, pooled,
                      projected, hidden_states, err, err_len);
}

int svl_embed_batch(svl_model* model, const uint32_t* ids, const uint64_t* cu_seqlens, uint32_t batch,
                    uint32_t dimension, float* out, char* err, size_t err_len) {
  if (!model || !out) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  if (dimension == 0 || dimension > model->m.cfg.embedding_dim) {  // text.rs:547-552
    set_err(err, err_len, "embedding dimension " + std::to_string(dimension) + " is outside 1..=" +
                              std::to_string(model->m.cfg.embedding_dim));
    return SVL_INTERNAL;
  }
  return forward_host(model, ids, cu_seqlens, batch, nullptr, nullptr, 0, dimension, out, nullptr, nullptr, nullptr,
                      nullptr, err, err_len);
}

int svl_embed_batch_device(svl_model* model, const uint32_t* d_ids, const uint64_t* cu_seqlens, uint32_t batch,
                           uint32_t dimension, float* d_out, void* stream, char* err, size_t err_len) {
  if (!model || !d_ids || !cu_seqlens || !d_out) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  svl::Model& m = model->m;
  if (dimension == 0 || dimension > m.cfg.embedding_dim) {
    set_err(err, err_len, "embedding dimension is outside 1..=embedding_dim");
    return SVL_INTERNAL;
  }
  std::lock_guard<std::mutex> lock(m.mu);
  std::string msg;
  int rc = m.validate_batch(nullptr, cu_seqlens, batch, &msg);
  if (rc) {
    set_err(err, err_len, msg);
    return rc;
  }
  cudaSetDevice(m.device);
  cudaStream_t st = stream ? (cudaStream_t)stream : m.stream;
  uint64_t* d_cu = (uint64_t*)m.workspace("dev_cu", (batch + 1) * 8);
  if (!d_cu) {
    set_err(err, err_len, "out of device memory");
    return SVL_LIMIT_EXCEEDED;
  }
  cudaMemcpyAsync(d_cu, cu_seqlens, (batch + 1) * 8, cudaMemcpyHostToDevice, st);
  rc = m.forward(d_ids, cu_seqlens, batch, d_cu, nullptr, dimension, d_out, nullptr, nullptr, nullptr, nullptr, st,
                 &msg);
  if (rc) set_err(err, err_len, msg);
  return rc;
}

int svl_model_check(svl_model* model, char* err, size_t err_len) {
  if (!model) return SVL_USAGE;
  svl::Model& m = model->m;
  std::lock_guard<std::mutex> lock(m.mu);
  cudaSetDevice(m.device);
  cudaDeviceSynchronize();
  std::string msg;
  int rc = drain_device_error(m.err_d, m.err_h, m.stream, &msg);
  if (rc) set_err(err, err_len, msg);
  return rc;
}

// ---------------------------------------------------------------- index --

int svl_index_create(int device, uint32_t dim, uint64_t capacity, svl_index** out, char* err, size_t err_len) {
  if (!out) return SVL_USAGE;
  *out = nullptr;
  svl_index* x = new (std::nothrow) svl_index();
  if (!x) return SVL_INTERNAL;
  std::string msg;
  int rc = x->x.create(device, dim, capacity, &msg);
  if (rc) {
    set_err(err, err_len, msg);
    delete x;
    return rc;
  }
  *out = x;
  return SVL_OK;
}

void svl_index_destroy(svl_index* index) { delete index; }

uint64_t svl_index_len(const svl_index* index) { return index ? index->x.len : 0; }

uint32_t svl_index_dim(const svl_index* index) { return index ? index->x.dim : 0; }

int svl_index_append(svl_index* index, const float* rows, const uint64_t* chunk_ids, uint64_t n, char* err,
                     size_t err_len) {
  if (!index || (n && (!rows || !chunk_ids))) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  svl::Index& x = index->x;
  std::lock_guard<std::mutex> lock(x.mu);
  // host-side check first, matching Chunk::new's Usage errors
  for (uint64_t r = 0; r < n; ++r) {
    double sum = 0.0;
    for (uint32_t d = 0; d < x.dim; ++d) {
      const float v = rows[r * x.dim + d];
      if (!std::isfinite(v)) {
        set_err(err, err_len, "embedding contains a non-finite value");
        return SVL_USAGE;
      }
      sum += (double)v * (double)v;
    }
    if (!(sum > 0.0) || !std::isfinite(sum)) {
      set_err(err, err_len, "embedding norm is zero or non-finite; cosine similarity is undefined");
      return SVL_USAGE;
    }
  }
  cudaSetDevice(x.device);
  std::string msg;
  int rc = x.append_device(rows, nullptr, n, x.stream, true, chunk_ids, &msg);
  if (rc) {
    set_err(err, err_len, msg);
    return rc;
  }
  rc = drain_device_error(x.err_d, x.err_h, x.stream, &msg);
  if (rc) set_err(err, err_len, msg);
  return rc;
}

int svl_index_append_device(svl_index* index, const float* d_rows, const uint64_t* d_chunk_ids, uint64_t n,
                            void* stream, char* err, size_t err_len) {
  if (!index || (n && (!d_rows || !d_chunk_ids))) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  svl::Index& x = index->x;
  std::lock_guard<std::mutex> lock(x.mu);
  cudaSetDevice(x.device);
  std::string msg;
  int rc = x.append_device(d_rows, d_chunk_ids, n, stream ? (cudaStream_t)stream : x.stream, false, nullptr, &msg);
  if (rc) set_err(err, err_len, msg);
  return rc;
}

int svl_ingest_batch(svl_model* model, svl_index* index, const uint32_t* ids, const uint64_t* cu_seqlens,
                     uint32_t batch, const uint64_t* chunk_ids, char* err, size_t err_len) {
  if (!model || !index || !ids || !cu_seqlens || (batch && !chunk_ids)) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  svl::Model& m = model->m;
  svl::Index& x = index->x;
  if (m.device != x.device) {
    set_err(err, err_len, "model and index are on different GPUs");
    return SVL_USAGE;
  }
  const uint32_t dim = x.dim;
  if (dim == 0 || dim > m.cfg.embedding_dim) {
    set_err(err, err_len, "index dimension is outside 1..=embedding_dim of the model");
    return SVL_USAGE;
  }
  std::scoped_lock lock(m.mu, x.mu);
  std::string msg;
  int rc = m.validate_batch(ids, cu_seqlens, batch, &msg);
  if (rc) {
    set_err(err, err_len, msg);
    return rc;
  }
  if (x.len + batch > x.capacity) {
    set_err(err, err_len, "index capacity exceeded");
    return SVL_LIMIT_EXCEEDED;
  }
  cudaSetDevice(m.device);
  cudaStream_t st = m.stream;
  const uint64_t T = cu_seqlens[batch];
  uint32_t* d_ids = (uint32_t*)m.workspace("io_ids", T * 4);
  uint64_t* d_cu = (uint64_t*)m.workspace("io_cu", (batch + 1) * 8);
  float* d_out = (float*)m.workspace("ingest_out", (size_t)batch * dim * 4);
  if (!d_ids || !d_cu || !d_out) {
    set_err(err, err_len, "out of device memory");
    return SVL_LIMIT_EXCEEDED;
  }
  cudaMemsetAsync(m.err_d, 0, 4, st);
  cudaMemcpyAsync(d_ids, ids, T * 4, cudaMemcpyHostToDevice, st);
  cudaMemcpyAsync(d_cu, cu_seqlens, (batch + 1) * 8, cudaMemcpyHostToDevice, st);
  rc = m.forward(d_ids, cu_seqlens, batch, d_cu, nullptr, dim, d_out, nullptr, nullptr, nullptr, nullptr, st, &msg);
  if (rc == SVL_OK) rc = drain_device_error(m.err_d, m.err_h, st, &msg);  // nothing is appended after a failure
  else cudaStreamSynchronize(st);
  if (rc) {
    set_err(err, err_len, msg);
    return rc;
  }
  // the rows stay on the device: copied into the index, normalised there in f64
  rc = x.append_device(d_out, nullptr, batch, st, true, chunk_ids, &msg);
  if (rc == SVL_OK) rc = drain_device_error(x.err_d, x.err_h, st, &msg);
  if (rc) set_err(err, err_len, msg);
  return rc;
}

int svl_index_search(svl_index* index, const float* queries, uint32_t n_queries, uint32_t dim,
                     const uint8_t* row_mask, uint32_t k, uint64_t* out_rows, uint64_t* out_chunk_ids,
                     double* out_scores, uint32_t* out_counts, char* err, size_t err_len) {
  if (!index || !queries || !out_rows || !out_scores || !out_counts) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  svl::Index& x = index->x;
  // vector.rs:23-55, per query, before any device work
  if (dim == 0) {
    set_err(err, err_len, "query embedding must have at least one dimension");
    return SVL_USAGE;
  }
  if (dim > svl::kMaxEmbeddingDimension) {
    set_err(err, err_len, "query embedding above the 8192-dimension cap");
    return SVL_LIMIT_EXCEEDED;
  }
  for (uint32_t q = 0; q < n_queries; ++q) {
    double sum = 0.0;
    for (uint32_t d = 0; d < dim; ++d) {
      const float v = queries[(size_t)q * dim + d];
      if (!std::isfinite(v)) {
        set_err(err, err_len, "query embedding contains a non-finite value");
        return SVL_USAGE;
      }
      sum += (double)v * (double)v;
    }
    if (!std::isfinite(sum) || sum <= 0.0) {
      set_err(err, err_len, "query embedding norm is zero or non-finite; cosine similarity is undefined");
      return SVL_USAGE;
    }
  }
  if (dim != x.dim) {
    set_err(err, err_len, "query embedding dimension " + std::to_string(dim) + " does not match the index dimension " +
                              std::to_string(x.dim));
    return SVL_USAGE;
  }
  if (k == 0) {
    set_err(err, err_len, "k must be at least 1");
    return SVL_USAGE;
  }
  std::lock_guard<std::mutex> lock(x.mu);
  cudaSetDevice(x.device);
  cudaStream_t st = x.stream;
  const size_t nq = n_queries;
  float* d_q = (float*)x.workspace("io_q", nq * dim * 4);
  uint8_t* d_mask = row_mask ? (uint8_t*)x.workspace("io_mask", x.len ? x.len : 1) : nullptr;
  uint64_t* d_rows = (uint64_t*)x.workspace("io_rows", nq * k * 8);
  uint64_t* d_chunk = (uint64_t*)x.workspace("io_chunk", nq * k * 8);
  double* d_scores = (double*)x.workspace("io_scores", nq * k * 8);
  uint32_t* d_counts = (uint32_t*)x.workspace("io_counts", nq * 4);
  if (!d_q || (row_mask && !d_mask) || !d_rows || !d_chunk || !d_scores || !d_counts) {
    set_err(err, err_len, "out of device memory");
    return SVL_LIMIT_EXCEEDED;
  }
  cudaMemcpyAsync(d_q, queries, nq * dim * 4, cudaMemcpyHostToDevice, st);
  if (row_mask && x.len) cudaMemcpyAsync(d_mask, row_mask, x.len, cudaMemcpyHostToDevice, st);
  std::vector<uint8_t> fb(nq ? nq : 1, 0);
  std::string msg;
  int rc = x.search_device(d_q, n_queries, d_mask, k, d_rows, d_chunk, d_scores, d_counts, st, fb.data(), &msg);
  if (rc == SVL_OK) {
    cudaStreamSynchronize(st);
    rc = x.resolve_fallbacks(d_q, n_queries, fb.data(), d_mask, k, d_rows, d_chunk, d_scores, d_counts, st, &msg);
  }
  if (rc) {
    set_err(err, err_len, msg);
    cudaStreamSynchronize(st);
    return rc;
  }
  cudaMemcpyAsync(out_rows, d_rows, nq * k * 8, cudaMemcpyDeviceToHost, st);
  if (out_chunk_ids) cudaMemcpyAsync(out_chunk_ids, d_chunk, nq * k * 8, cudaMemcpyDeviceToHost, st);
  cudaMemcpyAsync(out_scores, d_scores, nq * k * 8, cudaMemcpyDeviceToHost, st);
  cudaMemcpyAsync(out_counts, d_counts, nq * 4, cudaMemcpyDeviceToHost, st);
  rc = drain_device_error(x.err_d, x.err_h, st, &msg);
  if (rc) set_err(err, err_len, msg);
  return rc;
}

int svl_index_search_device(svl_index* index, const float* d_queries, uint32_t n_queries,
                            const uint8_t* d_row_mask, uint32_t k, uint64_t* d_out_rows, uint64_t* d_out_chunk_ids,
                            double* d_out_scores, uint32_t* d_out_counts, void* stream, char* err, size_t err_len) {
  if (!index || !d_queries || !d_out_rows || !d_out_scores || !d_out_counts) {
    set_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  svl::Index& x = index->x;
  std::lock_guard<std::mutex> lock(x.mu);
  cudaSetDevice(x.device);
  std::string msg;
  int rc = x.search_device(d_queries, n_queries, d_row_mask, k, d_out_rows, d_out_chunk_ids, d_out_scores,
                           d_out_counts, stream ? (cudaStream_t)stream : x.stream, nullptr, &msg);
  if (rc) set_err(err, err_len, msg);
  return rc;
}

int svl_index_check(svl_index* index, char* err, size_t err_len) {
  if (!index) return SVL_USAGE;
  svl::Index& x = index->x;
  std::lock_guard<std::mutex> lock(x.mu);
  cudaSetDevice(x.device);
  cudaDeviceSynchronize();
  std::string msg;
  int rc = drain_device_error(x.err_d, x.err_h, x.stream, &msg);
  if (rc) set_err(err, err_len, msg);
  return rc;
}

int svl_merge_topk_device(int device, const double* d_scores, const uint64_t* d_chunk_ids, const uint64_t* d_rows,
                          const uint32_t* d_counts, uint32_t n_shards, uint32_t n_queries, uint32_t k,
                          double* d_out_scores, uint64_t* d_out_chunk_ids, uint64_t* d_out_rows,
                          uint32_t* d_out_shard, uint32_t* d_out_counts, void* stream, char* err, size_t err_len) {
  if (!d_scores || !d_chunk_ids || !d_counts || !d_out_scores || !d_out_chunk_ids || !d_out_counts || !n_shards ||
      !k) {
    set_err(err, err_len, "null or empty argument");
    return SVL_USAGE;
  }
  if (n_shards > 64) {
    set_err(err, err_len, "at most 64 shards");
    return SVL_LIMIT_EXCEEDED;
  }
  cudaSetDevice(device);
  int rc = svl::merge_topk_device(d_scores, d_chunk_ids, d_rows, d_counts, n_shards, n_queries, k, d_out_scores,
                                  d_out_chunk_ids, d_out_rows, d_out_shard, d_out_counts, (cudaStream_t)stream);
  if (rc) set_err(err, err_len, "merge kernel launch failed");
  return rc;
}

// ------------------------------------------------------------- testing --

// FP16 operands as the encoder builds them: A rows with power-of-two row
// scales, B with one power-of-two scale for the whole matrix (K padded to a
// multiple of 8 with zeros).  Returns false when a buffer cannot be had.
static bool test_f16_operands(svl::GemmParams* p, const float* A, int lda, const float* B, int ldb, int M, int N,
                              int K, DevBuf* a16, DevBuf* b16, DevBuf* ainv, DevBuf* bscale, DevBuf* b32,
                              cudaStream_t st) {
  const int ka = (K + 7) / 8 * 8;
  if (!a16->alloc((size_t)M * ka * 2) || !b16->alloc((size_t)N * ka * 2) || !ainv->alloc((size_t)M * 4) ||
      !bscale->alloc(8) || !b32->alloc((size_t)N * ka * 4))
    return false;
  cudaMemset(a16->p, 0, (size_t)M * ka * 2);
  cudaMemset(b32->p, 0, (size_t)N * ka * 4);
  svl::launch_rows_to_f16(A, lda, (uint16_t*)a16->p, ka, M, K, (float*)ainv->p, nullptr, st);
  cudaMemcpy2DAsync(b32->p, (size_t)ka * 4, B, (size_t)ldb * 4, (size_t)K * 4, N, cudaMemcpyDeviceToDevice, st);
  svl::launch_matrix_to_f16((const float*)b32->p, (size_t)N * ka, (uint16_t*)b16->p, (float*)bscale->p,
                            (uint32_t*)bscale->p + 1, st);
  p->f16 = 1;
  p->A = a16->p;
  p->B = b16->p;
  p->lda = p->ldb = ka;
  p->K = ka;
  p->a_inv = (const float*)ainv->p;
  p->b_scale = (const float*)bscale->p;
  return true;
}

int svl_test_gemm_tf32(const float* A, int lda, const float* B, int ldb, float* C, int ldc, int M, int N, int K,
                       int epilogue, float alpha, const float* aux, int ld_aux, int round_out, int n_out,
                       int tf32_tma, void* stream) {
  svl::GemmParams p{};
  p.A = A;
  p.lda = lda;
  p.B = B;
  p.ldb = ldb;
  p.C = C;
  p.ldc = ldc;
  p.M = M;
  p.N = N;
  p.K = K;
  p.n_out = n_out;
  p.epilogue = epilogue;
  p.alpha = alpha;
  p.aux = aux;
  p.ld_aux = ld_aux;
  p.round_out = round_out;
  p.tf32_tma = tf32_tma & 1;
  p.single_cta = (tf32_tma >> 1) & 1;
  DevBuf e, a16, b16, ainv, bscale, b32;
  if (!e.alloc(4)) return SVL_INTERNAL;
  cudaMemset(e.p, 0, 4);
  p.err = (uint32_t*)e.p;
  if (((tf32_tma >> 2) & 1) &&
      !test_f16_operands(&p, A, lda, B, ldb, M, N, K, &a16, &b16, &ainv, &bscale, &b32, (cudaStream_t)stream))
    return SVL_INTERNAL;
  if (svl::gemm_tf32(p, (cudaStream_t)stream) != cudaSuccess) return SVL_USAGE;
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return SVL_INTERNAL;
  uint32_t w = 0;
  cudaMemcpy(&w, e.p, 4, cudaMemcpyDeviceToHost);
  return w ? SVL_INTERNAL : SVL_OK;
}

int svl_test_gemm_grouped(const float* A, int lda, const float* B, int ldb, uint16_t* C16, int ldc, int M, int N,
                          int K, float alpha, float* group_inv, float* row_ss, int group_stride, int single_cta,
                          void* stream) {
  svl::GemmParams p{};
  p.C = (float*)C16;
  p.ldc = ldc;
  p.M = M;
  p.N = N;
  p.epilogue = svl::kEpiStore;
  p.alpha = alpha;
  p.out_f16 = 1;
  p.group_inv = group_inv;
  p.row_ss = row_ss;
  p.row_ss_stride = group_stride;
  p.single_cta = single_cta;
  DevBuf e, a16, b16, ainv, bscale, b32;
  if (!e.alloc(4)) return SVL_INTERNAL;
  cudaMemset(e.p, 0, 4);
  p.err = (uint32_t*)e.p;
  if (!test_f16_operands(&p, A, lda, B, ldb, M, N, K, &a16, &b16, &ainv, &bscale, &b32, (cudaStream_t)stream))
    return SVL_INTERNAL;
  if (svl::gemm_tf32(p, (cudaStream_t)stream) != cudaSuccess) return SVL_USAGE;
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return SVL_INTERNAL;
  uint32_t w = 0;
  cudaMemcpy(&w, e.p, 4, cudaMemcpyDeviceToHost);
  return w ? SVL_INTERNAL : SVL_OK;
}

int svl_test_attention(const float* qkv, int ld, int T, int nh, int kvh, int hd, const uint64_t* d_cu,
                       const uint64_t* h_cu, int batch, int window, int impl, float* out, int ld_out, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  DevBuf e, seq, pos, items;
  if (!e.alloc(4) || !seq.alloc((size_t)T * 4) || !pos.alloc((size_t)T * 4)) return SVL_INTERNAL;
  cudaMemsetAsync(e.p, 0, 4, st);
  if (impl == 1 || impl == 2) {
    if (!svl::attention_tc_supported(hd)) return SVL_UNSUPPORTED;
    const size_t bytes = svl::attention_tc_items_bytes(h_cu, batch, nh) + 16;
    if (!items.alloc(bytes)) return SVL_INTERNAL;
    svl::AttnParams ap{};
    ap.qkv = qkv;
    ap.ld = ld;
    ap.T = T;
    ap.nh = nh;
    ap.kvh = kvh;
    ap.hd = hd;
    ap.window = window;
    ap.out = out;
    ap.ld_out = ld_out;
    ap.round_out = 0;
    ap.single_cta = impl == 2;
    ap.err = (uint32_t*)e.p;
    if (svl::launch_attention_tc(ap, h_cu, batch, items.p, bytes, st) != cudaSuccess) return SVL_INTERNAL;
  } else if (impl == 3) {
    if (!svl::attention_f16_supported(hd, nh, kvh)) return SVL_UNSUPPORTED;
    std::vector<uint32_t> sched;
    const int pairs = svl::attention_f16_schedule(h_cu, batch, nh, hd, window, &sched);
    if (pairs < 0) return SVL_INTERNAL;
    DevBuf half;
    if (!items.alloc(sched.size() * 4 + 16) || !half.alloc((size_t)T * ld * 2)) return SVL_INTERNAL;
    if (!sched.empty() && cudaMemcpy(items.p, sched.data(), sched.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return SVL_INTERNAL;
    svl::launch_f32_to_f16(qkv, (uint16_t*)half.p, (size_t)T * ld, st);
    svl::AttnF16Params ap{};
    ap.qkv = (const uint16_t*)half.p;
    ap.ld = ld;
    ap.T = T;
    ap.nh = nh;
    ap.kvh = kvh;
    ap.hd = hd;
    ap.window = window;
    ap.out = out;
    ap.ld_out = ld_out;
    ap.round_out = 0;
    ap.err = (uint32_t*)e.p;
    if (svl::launch_attention_f16(ap, (const uint32_t*)items.p, pairs, st) != cudaSuccess) return SVL_INTERNAL;
    if (cudaStreamSynchronize(st) != cudaSuccess) return SVL_INTERNAL;
  } else {
    svl::launch_positions(d_cu, (uint32_t)batch, (uint32_t*)seq.p, (uint32_t*)pos.p, st);
    if (!svl::launch_attention_simt(qkv, ld, T, nh, kvh, hd, d_cu, (uint32_t*)seq.p, (uint32_t*)pos.p, window, out,
                                    ld_out, 0, (uint32_t*)e.p, st))
      return SVL_UNSUPPORTED;
  }
  if (cudaStreamSynchronize(st) != cudaSuccess) return SVL_INTERNAL;
  uint32_t w = 0;
  cudaMemcpy(&w, e.p, 4, cudaMemcpyDeviceToHost);
  return w ? SVL_INTERNAL : SVL_OK;
}

int svl_model_profile(svl_model* model, int enable) {
  if (!model) return SVL_USAGE;
  std::lock_guard<std::mutex> lock(model->m.mu);
  model->m.prof.enabled = enable != 0;
  return SVL_OK;
}

int svl_model_profile_read(svl_model* model, double* ms, uint64_t* launches) {
  if (!model) return SVL_USAGE;
  svl::Model& m = model->m;
  std::lock_guard<std::mutex> lock(m.mu);
  cudaSetDevice(m.device);
  cudaDeviceSynchronize();
  m.prof.read(ms, launches);
  return SVL_OK;
}

int svl_index_profile(svl_index* index, int enable) {
  if (!index) return SVL_USAGE;
  std::lock_guard<std::mutex> lock(index->x.mu);
  index->x.prof.enabled = enable != 0;
  return SVL_OK;
}

int svl_index_profile_read(svl_index* index, double* ms, uint64_t* launches) {
  if (!index) return SVL_USAGE;
  svl::Index& x = index->x;
  std::lock_guard<std::mutex> lock(x.mu);
  cudaSetDevice(x.device);
  cudaDeviceSynchronize();
  x.prof.read(ms, launches);
  return SVL_OK;
}

}  // extern "C"
