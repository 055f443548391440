// model.cuh -- the device-resident text encoder behind svl_model.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "../../include/svl_gpu.h"
#include "profiler.cuh"

namespace svl {

void set_err(char* err, size_t len, const std::string& msg);
// Maps the device error word to an svl_status (and a message).
int status_from_device(uint32_t word, std::string* msg);

struct LayerDev {
  float *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr, *wpg = nullptr, *wpp = nullptr;
  float *in_ln = nullptr, *post_attn = nullptr, *pre_ff = nullptr, *post_ff = nullptr, *post_ple = nullptr;
  float *q_norm = nullptr, *k_norm = nullptr;
  float layer_scalar = 1.0f;
  int hd = 0, kvh = 0, full = 0, qd = 0, kvd = 0, ld_qkv = 0;
};

// Soft-token rows (forward_with_features): (packed row, host pointer to H floats).
struct FeatureRows {
  std::vector<std::pair<uint64_t, const float*>> rows;
};

struct Model {
  int device = -1;
  cudaStream_t stream = nullptr;
  svl_text_config cfg{};
  std::vector<svl_layer_config> layer_cfg;
  uint64_t parameters = 0;
  int F_pad = 0;
  float *embed = nullptr, *wemb = nullptr, *final_norm = nullptr, *wple = nullptr, *ple_norm = nullptr;
  float *full_inv = nullptr, *sliding_inv = nullptr;
  float2 *full_rope = nullptr, *sliding_rope = nullptr;      // [position][hd / 2] (cos, sin)
  float2 *full_rope_t = nullptr, *sliding_rope_t = nullptr;  // [hd / 2][position]
  int rope_positions = 0;
  // attention operands in FP16 (default); SVL_ATTENTION_TF32=1 at creation
  // keeps them in FP32 for the TF32 kernels
  bool attn_f16 = true;
  std::vector<LayerDev> layers;
  std::vector<void*> allocations;
  struct Buf {
    void* ptr = nullptr;
    size_t bytes = 0;
  };
  std::map<std::string, Buf> ws;
  uint32_t* err_d = nullptr;
  uint32_t* err_h = nullptr;
  Profiler prof;
  std::mutex mu;

  ~Model();
  int create(const svl_text_config* config, const svl_tensor_view* tensors, size_t n_tensors, int dev,
             std::string* msg);
  int validate_batch(const uint32_t* ids, const uint64_t* cu, uint32_t batch, std::string* msg) const;
  int forward(const uint32_t* d_ids, const uint64_t* cu, uint32_t batch, const uint64_t* d_cu,
              const FeatureRows* features, uint32_t dim, float* d_out, float* d_pooled, float* d_normalized,
              float* d_projected, float* d_hidden, cudaStream_t st, std::string* msg);

  // Pinned staging for small per-forward uploads (the attention schedules):
  // the copy is asynchronous, and the event keeps the next forward from
  // overwriting the staging before the previous copy has run.
  uint32_t* pinned = nullptr;
  size_t pinned_bytes = 0;
  cudaEvent_t pinned_done = nullptr;
  bool upload_pinned(const void* src, size_t bytes, void* dst, cudaStream_t st);

  float* dalloc(size_t n);
  void* workspace(const char* name, size_t bytes);
  int gemm(const float* A, int lda, const float* B, int ldb, float* C, int ldc, int M, int N, int K, int epi,
           float alpha, const float* aux, int ld_aux, int round_out, int n_out, cudaStream_t st);
};

}  // namespace svl

struct svl_model {
  svl::Model m;
};
