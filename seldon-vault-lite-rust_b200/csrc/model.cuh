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
// Reads and clears a handle's device error word after synchronising `st`.
int drain_device_error(uint32_t* err_d, uint32_t* err_h, cudaStream_t st, std::string* msg);

// A GEMM weight: FP32 (TF32-rounded) and, when the FP16 operand path is on,
// an FP16 copy with one power-of-two scale for the matrix (inv = device
// scalar holding the inverse scale).
struct Weight {
  float* f32 = nullptr;
  uint16_t* f16 = nullptr;
  float* inv = nullptr;
};

struct LayerDev {
  float *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr, *wpg = nullptr, *wpp = nullptr;
  Weight qkv16, o16, gu16, pg16, down16, pp16;  // FP16 copies (with the FP16 operand path)
  // largest row L2 norms of the gate, up and PLE-gate weights: the bounds
  // behind the FP16 row scales of the GeGLU and PLE-gate outputs
  float g_max = 0.0f, u_max = 0.0f, pg_max = 0.0f;
  float *in_ln = nullptr, *post_attn = nullptr, *pre_ff = nullptr, *post_ff = nullptr, *post_ple = nullptr;
  float *q_norm = nullptr, *k_norm = nullptr;
  float layer_scalar = 1.0f;
  int hd = 0, kvh = 0, full = 0, qd = 0, kvd = 0, ld_qkv = 0;
};

// One FP16 attention work schedule of a forward (per head dim and window).
struct AttnSched {
  int hd, window, pairs;
  size_t word;  // offset in the forward's uploaded words
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
  Weight ple16, emb16;
  float *full_inv = nullptr, *sliding_inv = nullptr;
  float2 *full_rope = nullptr, *sliding_rope = nullptr;      // [position][hd / 2] (cos, sin)
  float2 *full_rope_t = nullptr, *sliding_rope_t = nullptr;  // [hd / 2][position]
  int rope_positions = 0;
  // attention operands in FP16 (default); SVL_ATTENTION_TF32=1 at creation
  // keeps them in FP32 for the TF32 kernels
  bool attn_f16 = true;
  // GEMM operands in FP16 with power-of-two row scales (default) for the
  // projections whose inputs are produced row by row; SVL_GEMM_TF32=1 at
  // creation keeps every GEMM on FP32 operands (TF32 products)
  bool gemm_f16 = true;
  // per-head norms and RoPE fused into the QKV GEMM's epilogue for 256-wide
  // heads (default) or a separate kernel; SVL_QKV_EPILOGUE=1 / 0 forces one
  bool qkv_fused = true;
  // split precision (SVL_PRECISION_SPLIT): every GEMM weight is stored as
  // [hi | lo | hi] over 3K columns and every GEMM input expanded to
  // [hi | hi | lo] just before its GEMM, so each TF32 product carries ~22
  // significant bits; producers write exact FP32 and attention runs in FP32
  // on the CUDA cores.  Off by default (the FP16 / TF32 paths above).
  bool split = false;
  // row-fused kernels (row_fused.cu) at hidden width 512 with FP16 operands
  // (default; SVL_ROW_FUSED=0 at creation keeps the separate GEMMs and
  // residual kernels): the o and down projections with their residual steps
  // (row_fused), the per-layer-input block (ple_fused, per-layer width 512)
  bool row_fused = false;
  bool ple_fused = false;
  std::vector<LayerDev> layers;
  std::vector<void*> allocations;
  struct Buf {
    void* ptr = nullptr;
    size_t bytes = 0;
  };
  std::map<std::string, Buf> ws;
  std::mutex ws_mu;  // workspace() callers need not hold the model mutex
  uint32_t* err_d = nullptr;
  uint32_t* err_h = nullptr;
  Profiler prof;
  std::mutex mu;

  ~Model();
  int create(const svl_text_config* config, const svl_tensor_view* tensors, size_t n_tensors, int dev,
             uint32_t precision, std::string* msg);
  int validate_batch(const uint32_t* ids, const uint64_t* cu, uint32_t batch, std::string* msg) const;
  int forward(const uint32_t* d_ids, const uint64_t* cu, uint32_t batch, const uint64_t* d_cu,
              const FeatureRows* features, uint32_t dim, float* d_out, float* d_pooled, float* d_normalized,
              float* d_projected, float* d_hidden, cudaStream_t st, std::string* msg);
  // One group of sequences (the whole batch, or one half run on its own
  // stream): cu / d_cu are the group's own offsets, outputs point at its rows,
  // `tag` suffixes its workspace names, scheds / d_sched its attention work.
  int forward_part(const std::string& tag, const uint32_t* d_ids, const uint64_t* cu, uint32_t batch,
                   const uint64_t* d_cu, const FeatureRows* features, uint32_t dim, float* d_out, float* d_pooled,
                   float* d_normalized, float* d_projected, float* d_hidden, const std::vector<AttnSched>& scheds,
                   const uint32_t* d_sched, cudaStream_t st, std::string* msg);
  int attention_schedules(const uint64_t* cu, uint32_t batch, std::vector<AttnSched>* scheds,
                          std::vector<uint32_t>* words, std::string* msg);
  // second stream for the other half of a split batch, and its fork / join events
  cudaStream_t stream2 = nullptr;
  cudaEvent_t fork_ev = nullptr, join_ev = nullptr;

  // Pinned staging for small per-forward uploads (the attention schedules):
  // the copy is asynchronous, and the event keeps the next forward from
  // overwriting the staging before the previous copy has run.
  uint32_t* pinned = nullptr;
  size_t pinned_bytes = 0;
  cudaEvent_t pinned_done = nullptr;
  double sequence_cost(uint64_t L) const;
  bool upload_pinned(const void* src, size_t bytes, void* dst, cudaStream_t st);

  float* dalloc(size_t n);
  void* workspace(const char* name, size_t bytes);
  void* workspace(const std::string& name, size_t bytes) { return workspace(name.c_str(), bytes); }
  int gemm(const float* A, int lda, const float* B, int ldb, float* C, int ldc, int M, int N, int K, int epi,
           float alpha, const float* aux, int ld_aux, int round_out, int n_out, cudaStream_t st);
  // FP16 operands: A rows scaled by a_inv (NULL = 1), weight rows by w.inv.
  int gemm16(const uint16_t* A, int lda, const float* a_inv, const Weight& w, int ldb, float* C, int ldc, int M, int N,
             int K, int epi, float alpha, const float* aux, int ld_aux, int round_out, int n_out, cudaStream_t st,
             const float* out_inv = nullptr, const float* aux_row_inv = nullptr, int aux_row_stride = 0,
             const float* aux_col_w = nullptr, float* row_ss = nullptr, int row_ss_stride = 0,
             float* group_inv = nullptr);
  bool make_f16(const float* w, size_t rows, size_t cols, Weight* out);
  // Replaces the FP32 weight *w ([rows, cols]) by its split form [rows, 3 cols].
  bool make_split(float** w, size_t rows, size_t cols);
  // A GEMM in split precision: expands A ([M, K], row pitch lda) into the
  // workspace `x3` and runs the TF32 GEMM over 3K against the split weight W3.
  int gemm_split(const float* A, int lda, float* x3, const float* W3, float* C, int ldc, int M, int N, int K, int epi,
                 float alpha, const float* aux, int ld_aux, int n_out, cudaStream_t st);
};

}  // namespace svl

struct svl_model {
  svl::Model m;
};
