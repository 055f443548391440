// model.cu -- svl_model: device-resident EmbeddingGemma-2 text encoder.
//
// Host side of TextModel (src/model/text.rs) over the sm_100a kernels:
//   * svl_model_create checks the tensor inventory the way
//     TextWeights::decode does (src/model/weights.rs:125-189) and uploads the
//     weights once, in FP32, into fused layouts: [q; k; v] projections
//     concatenated, gate/up interleaved in 128-row blocks for the GeGLU
//     epilogue, GEMM weights pre-rounded to the TF32 grid;
//   * forward() is text.rs:182-538 for a packed batch of sequences, one
//     kernel per fused step, all on the model's stream.
// Attention operands (normalised q, k, v) are written in FP16 -- the TF32
// significand in half the bytes -- for the CTA-pair kernel of
// attention_f16.cu; SVL_ATTENTION_TF32=1 in the environment at model creation
// keeps them in FP32 for the TF32 kernels instead.
// Activations live in a per-model workspace that grows to the largest token
// count seen; calls on one model are serialised by its mutex.

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "common.cuh"
#include "attention_f16.cuh"
#include "attention_tc.cuh"
#include "encoder_kernels.cuh"
#include "gemm_tc.cuh"
#include "model.cuh"
#include "row_fused.cuh"

namespace svl {

namespace {

constexpr size_t kMaxTextTokens = 8192;                     // config.rs:27
constexpr size_t kMaxActivationElements = size_t(1) << 28;  // text.rs:34

std::string layer_prefix(size_t l) { return "language_model.layers." + std::to_string(l) + "."; }

}  // namespace

void set_err(char* err, size_t len, const std::string& msg) {
  if (err && len) {
    size_t n = msg.size() < len - 1 ? msg.size() : len - 1;
    std::memcpy(err, msg.data(), n);
    err[n] = 0;
  }
}

int status_from_device(uint32_t word, std::string* msg) {
  if (word & SVL_DEVERR_BAD_TOKEN) {
    *msg = "a token id is outside the vocabulary";
    return SVL_CORRUPT;
  }
  if (word & SVL_DEVERR_BAD_QUERY) {
    *msg = "query embedding norm is zero or non-finite; cosine similarity is undefined";
    return SVL_USAGE;
  }
  if (word & SVL_DEVERR_BAD_ROW) {
    *msg = "embedding norm is zero or non-finite; cosine similarity is undefined";
    return SVL_USAGE;
  }
  if (word & SVL_DEVERR_TIMEOUT) {
    *msg = "a device wait timed out";
    return SVL_INTERNAL;
  }
  if (word & SVL_DEVERR_OVERFLOW) {
    *msg = "a device candidate buffer overflowed";
    return SVL_INTERNAL;
  }
  if (word & SVL_DEVERR_NONFINITE) {
    *msg = "the forward pass produced a non-finite value";
    return SVL_INTERNAL;
  }
  if (word & SVL_DEVERR_PEER) {
    *msg = "another rank's shard search failed";
    return SVL_INTERNAL;
  }
  return SVL_OK;
}

// Reads and clears a handle's device error word after synchronising `st`.
int drain_device_error(uint32_t* err_d, uint32_t* err_h, cudaStream_t st, std::string* msg) {
  cudaMemcpyAsync(err_h, err_d, 4, cudaMemcpyDeviceToHost, st);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    *msg = std::string("CUDA error: ") + cudaGetErrorString(e);
    return SVL_INTERNAL;
  }
  const uint32_t word = *err_h;
  if (word) {
    cudaMemsetAsync(err_d, 0, 4, st);
    cudaStreamSynchronize(st);
  }
  return status_from_device(word, msg);
}

Model::~Model() {
  if (device >= 0) cudaSetDevice(device);
  for (void* p : allocations) cudaFree(p);
  for (auto& kv : ws) cudaFree(kv.second.ptr);
  if (err_d) cudaFree(err_d);
  if (err_h) cudaFreeHost(err_h);
  if (pinned_done) {
    cudaEventSynchronize(pinned_done);
    cudaEventDestroy(pinned_done);
  }
  if (pinned) cudaFreeHost(pinned);
  if (stream2) cudaStreamDestroy(stream2);
  if (fork_ev) cudaEventDestroy(fork_ev);
  if (join_ev) cudaEventDestroy(join_ev);
  if (stream) cudaStreamDestroy(stream);
}

bool Model::upload_pinned(const void* src, size_t bytes, void* dst, cudaStream_t st) {
  if (pinned_done) {
    if (cudaEventSynchronize(pinned_done) != cudaSuccess) return false;  // the last copy has read the staging
  } else if (cudaEventCreateWithFlags(&pinned_done, cudaEventDisableTiming) != cudaSuccess) {
    return false;
  }
  if (bytes > pinned_bytes) {
    if (pinned) cudaFreeHost(pinned);
    pinned = nullptr;
    pinned_bytes = 0;
    const size_t cap = bytes < 65536 ? 65536 : bytes * 2;
    if (cudaMallocHost((void**)&pinned, cap) != cudaSuccess) return false;
    pinned_bytes = cap;
  }
  std::memcpy(pinned, src, bytes);
  return cudaMemcpyAsync(dst, pinned, bytes, cudaMemcpyHostToDevice, st) == cudaSuccess &&
         cudaEventRecord(pinned_done, st) == cudaSuccess;
}

float* Model::dalloc(size_t n) {
  void* p = nullptr;
  if (cudaMalloc(&p, n * sizeof(float)) != cudaSuccess) return nullptr;
  allocations.push_back(p);
  return (float*)p;
}

void* Model::workspace(const char* name, size_t bytes) {
  std::lock_guard<std::mutex> lock(ws_mu);
  Buf& b = ws[name];
  if (b.bytes >= bytes) return b.ptr;
  if (b.ptr) cudaFree(b.ptr);
  b.ptr = nullptr;
  b.bytes = 0;
  const size_t rounded = (bytes + (size_t(1) << 20) - 1) & ~((size_t(1) << 20) - 1);
  if (cudaMalloc(&b.ptr, rounded) != cudaSuccess) return nullptr;
  b.bytes = rounded;
  return b.ptr;
}

namespace {

struct HostTensor {
  const svl_tensor_view* view = nullptr;
  size_t numel = 0;
};

// Converts one tensor view to FP32 (BF16 widened exactly), checking finiteness.
bool to_f32(const svl_tensor_view* v, size_t numel, std::vector<float>& out) {
  out.resize(numel);
  if (v->dtype == SVL_DTYPE_BF16) {
    const uint16_t* s = (const uint16_t*)v->data;
    for (size_t i = 0; i < numel; ++i) {
      uint32_t u = (uint32_t)s[i] << 16;
      std::memcpy(&out[i], &u, 4);
    }
  } else {
    std::memcpy(out.data(), v->data, numel * 4);
  }
  for (size_t i = 0; i < numel; ++i)
    if (!std::isfinite(out[i])) return false;
  return true;
}

}  // namespace

int Model::create(const svl_text_config* config, const svl_tensor_view* tensors, size_t n_tensors, int dev,
                  uint32_t precision, std::string* msg) {
  device = dev;
  cfg = *config;
  if (precision != SVL_PRECISION_FAST && precision != SVL_PRECISION_SPLIT) {
    *msg = "unknown precision mode " + std::to_string(precision);
    return SVL_USAGE;
  }
  split = precision == SVL_PRECISION_SPLIT;
  {
    const char* e = std::getenv("SVL_ATTENTION_TF32");
    attn_f16 = !(e && e[0] == '1');
    const char* g = std::getenv("SVL_GEMM_TF32");
    // the row producers of FP16 operands are the vectorised kernels (width a
    // multiple of 128 up to 1024); TMA needs FP16 rows of 16-byte multiples
    const size_t hh = config->hidden_size;
    gemm_f16 = !(g && g[0] == '1') && hh % 128 == 0 && hh <= 1024;
    // The fused norm/RoPE epilogue writes FP16 q/k/v once instead of FP32
    // rows that a separate kernel reads back (measured faster with both
    // operand types); SVL_QKV_EPILOGUE=0/1 overrides.
    const char* q = std::getenv("SVL_QKV_EPILOGUE");
    qkv_fused = q && (q[0] == '0' || q[0] == '1') ? q[0] == '1' : true;
    // the row-fused kernels (row_fused.cu: FP16 GEMM operands, hidden width
    // 512): the o and down projections with the residual step after them,
    // the per-layer-input block (per-layer width 512 too); SVL_ROW_FUSED=0
    // runs the separate GEMMs and residual kernels instead
    const char* f = std::getenv("SVL_ROW_FUSED");
    row_fused = gemm_f16 && !(f && f[0] == '0') && config->hidden_size == 512;
    ple_fused = row_fused && ple_block_supported((int)config->hidden_size, (int)config->hidden_size_per_layer_input);
    if (split) {  // exact FP32 producers, split TF32 GEMMs, FP32 attention
      attn_f16 = gemm_f16 = qkv_fused = ple_fused = row_fused = false;
    }
  }
  layer_cfg.assign(config->layers, config->layers + config->num_hidden_layers);
  cfg.layers = layer_cfg.data();
  const size_t H = cfg.hidden_size, P = cfg.hidden_size_per_layer_input, F = cfg.intermediate_size,
               L = cfg.num_hidden_layers, NH = cfg.num_attention_heads, E = cfg.embedding_dim;
  if (!H || !P || !F || !L || !NH || !E || !cfg.vocab_size) {
    *msg = "configuration has a zero dimension";
    return SVL_CORRUPT;
  }
  // The tensor-core GEMMs need every reduction width to be a multiple of 4
  // FP32 elements (16-byte TMA rows).
  if (H % 4 || P % 4 || F % 4) {
    *msg = "hidden, per-layer and intermediate sizes must be multiples of 4 on this device";
    return SVL_UNSUPPORTED;
  }
  for (size_t l = 0; l < L; ++l) {
    const auto& lc = layer_cfg[l];
    if (!lc.head_dim || lc.head_dim % 2 || !lc.num_key_value_heads || NH % lc.num_key_value_heads) {
      *msg = "invalid head layout in layer " + std::to_string(l);
      return SVL_CORRUPT;
    }
    if ((NH * lc.head_dim) % 4 || lc.head_dim > 1024) {
      *msg = "head layout unsupported on this device in layer " + std::to_string(l);
      return SVL_UNSUPPORTED;
    }
  }
  // Expected inventory (config.rs:394-484).
  std::map<std::string, size_t> expected;
  expected["language_model.embed_tokens.weight"] = (size_t)cfg.vocab_size * H;
  expected["language_model.embedding_projection.weight"] = E * H;
  expected["language_model.norm.weight"] = H;
  expected["language_model.ple.per_layer_model_projection.weight"] = L * P * H;
  expected["language_model.ple.per_layer_projection_norm.weight"] = P;
  for (size_t l = 0; l < L; ++l) {
    const std::string pre = layer_prefix(l);
    const size_t hd = layer_cfg[l].head_dim, kvh = layer_cfg[l].num_key_value_heads;
    for (const char* n : {"input_layernorm.weight", "post_attention_layernorm.weight",
                          "pre_feedforward_layernorm.weight", "post_feedforward_layernorm.weight",
                          "ple_block.post_per_layer_input_norm.weight"})
      expected[pre + n] = H;
    expected[pre + "layer_scalar"] = 1;
    expected[pre + "mlp.gate_proj.weight"] = F * H;
    expected[pre + "mlp.up_proj.weight"] = F * H;
    expected[pre + "mlp.down_proj.weight"] = H * F;
    expected[pre + "ple_block.per_layer_input_gate.weight"] = P * H;
    expected[pre + "ple_block.per_layer_projection.weight"] = H * P;
    expected[pre + "self_attn.q_proj.weight"] = NH * hd * H;
    expected[pre + "self_attn.k_proj.weight"] = kvh * hd * H;
    expected[pre + "self_attn.v_proj.weight"] = kvh * hd * H;
    expected[pre + "self_attn.o_proj.weight"] = H * NH * hd;
    expected[pre + "self_attn.q_norm.weight"] = hd;
    expected[pre + "self_attn.k_norm.weight"] = hd;
  }
  std::map<std::string, HostTensor> found;
  for (size_t i = 0; i < n_tensors; ++i) {
    const svl_tensor_view* v = &tensors[i];
    if (!v->name || !v->data) {
      *msg = "tensor view without a name or data";
      return SVL_CORRUPT;
    }
    const std::string name = v->name;
    if (name.rfind("language_model.", 0) != 0) continue;  // audio / vision tensors are ignored
    auto it = expected.find(name);
    if (it == expected.end()) {
      *msg = "unexpected text tensor " + name + " in the weight file";
      return SVL_CORRUPT;
    }
    if (v->dtype != SVL_DTYPE_F32 && v->dtype != SVL_DTYPE_BF16) {
      *msg = "text weight " + name + " has an unsupported dtype";
      return SVL_UNSUPPORTED;
    }
    size_t numel = 1;
    if (v->ndim == 0 || v->ndim > 4) {
      *msg = "text weight " + name + " has an invalid rank";
      return SVL_CORRUPT;
    }
    for (uint32_t d = 0; d < v->ndim; ++d) numel *= v->shape[d];
    if (numel != it->second) {
      *msg = "text weight " + name + " has the wrong shape";
      return SVL_CORRUPT;
    }
    found[name] = HostTensor{v, numel};
  }
  for (auto& kv : expected)
    if (!found.count(kv.first)) {
      *msg = "text weight " + kv.first + " is missing from the Safetensors file";
      return SVL_CORRUPT;
    }
  parameters = 0;
  for (auto& kv : expected) parameters += kv.second;

  if (cudaSetDevice(device) != cudaSuccess) {
    *msg = "cannot select CUDA device " + std::to_string(device);
    return SVL_INTERNAL;
  }
  if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&stream2, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&fork_ev, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&join_ev, cudaEventDisableTiming) != cudaSuccess ||
      cudaMalloc(&err_d, sizeof(uint32_t)) != cudaSuccess || cudaMallocHost(&err_h, sizeof(uint32_t)) != cudaSuccess) {
    *msg = "CUDA initialisation failed";
    return SVL_INTERNAL;
  }
  cudaMemsetAsync(err_d, 0, sizeof(uint32_t), stream);

  std::vector<float> host;
  bool ok = true;
  // Uploads tensor `name` (rows x cols) into dst with row pitch ld (floats).
  auto upload = [&](const std::string& name, float* dst, size_t rows, size_t cols, size_t ld) -> bool {
    const HostTensor& t = found[name];
    if (!to_f32(t.view, t.numel, host)) {
      *msg = "text weight " + name + " contains a non-finite value";
      ok = false;
      return false;
    }
    if (cudaMemcpy2D(dst, ld * 4, host.data(), cols * 4, cols * 4, rows, cudaMemcpyHostToDevice) != cudaSuccess) {
      *msg = "weight upload failed";
      ok = false;
      return false;
    }
    return true;
  };
  auto single = [&](const std::string& name, size_t n) -> float* {
    float* d = dalloc(n);
    if (!d) {
      *msg = "out of device memory for weights";
      ok = false;
      return nullptr;
    }
    if (!upload(name, d, 1, n, n)) return nullptr;
    return d;
  };
  // GEMM weights: TF32-rounded in place, or (split precision) kept exact
  // here and replaced by their split form below
  auto round_dev = [&](float* p, size_t n) {
    if (p && !split) launch_round_tf32(p, n, stream);
  };

  embed = single("language_model.embed_tokens.weight", (size_t)cfg.vocab_size * H);
  wemb = single("language_model.embedding_projection.weight", E * H);
  final_norm = single("language_model.norm.weight", H);
  wple = single("language_model.ple.per_layer_model_projection.weight", L * P * H);
  ple_norm = single("language_model.ple.per_layer_projection_norm.weight", P);
  if (!ok) return SVL_CORRUPT;
  round_dev(wemb, E * H);
  round_dev(wple, L * P * H);

  F_pad = (int)((F + 127) / 128 * 128);
  layers.resize(L);
  for (size_t l = 0; l < L && ok; ++l) {
    const std::string pre = layer_prefix(l);
    LayerDev& ly = layers[l];
    ly.hd = (int)layer_cfg[l].head_dim;
    ly.kvh = (int)layer_cfg[l].num_key_value_heads;
    ly.full = layer_cfg[l].layer_type == SVL_LAYER_FULL;
    ly.qd = (int)NH * ly.hd;
    ly.kvd = ly.kvh * ly.hd;
    ly.ld_qkv = ly.qd + 2 * ly.kvd;
    ly.wqkv = dalloc((size_t)ly.ld_qkv * H);
    if (!ly.wqkv) {
      *msg = "out of device memory for weights";
      return SVL_INTERNAL;
    }
    upload(pre + "self_attn.q_proj.weight", ly.wqkv, ly.qd, H, H);
    upload(pre + "self_attn.k_proj.weight", ly.wqkv + (size_t)ly.qd * H, ly.kvd, H, H);
    upload(pre + "self_attn.v_proj.weight", ly.wqkv + (size_t)(ly.qd + ly.kvd) * H, ly.kvd, H, H);
    ly.wo = single(pre + "self_attn.o_proj.weight", H * ly.qd);
    // gate/up interleaved: block b = [gate rows 128b..128b+127 | up rows], zero padded to F_pad
    ly.wgu = dalloc((size_t)2 * F_pad * H);
    if (!ly.wgu) {
      *msg = "out of device memory for weights";
      return SVL_INTERNAL;
    }
    cudaMemset(ly.wgu, 0, (size_t)2 * F_pad * H * 4);
    for (int half = 0; half < 2 && ok; ++half) {
      const std::string name = pre + (half ? "mlp.up_proj.weight" : "mlp.gate_proj.weight");
      const HostTensor& t = found[name];
      if (!to_f32(t.view, t.numel, host)) {
        *msg = "text weight " + name + " contains a non-finite value";
        return SVL_CORRUPT;
      }
      for (size_t b = 0; b * 128 < F; ++b) {
        const size_t rows = F - b * 128 < 128 ? F - b * 128 : 128;
        float* dst = ly.wgu + (b * 256 + half * 128) * H;
        cudaMemcpy(dst, host.data() + b * 128 * H, rows * H * 4, cudaMemcpyHostToDevice);
      }
    }
    ly.wdown = single(pre + "mlp.down_proj.weight", H * F);
    ly.wpg = single(pre + "ple_block.per_layer_input_gate.weight", P * H);
    ly.wpp = single(pre + "ple_block.per_layer_projection.weight", H * P);
    ly.in_ln = single(pre + "input_layernorm.weight", H);
    ly.post_attn = single(pre + "post_attention_layernorm.weight", H);
    ly.pre_ff = single(pre + "pre_feedforward_layernorm.weight", H);
    ly.post_ff = single(pre + "post_feedforward_layernorm.weight", H);
    ly.post_ple = single(pre + "ple_block.post_per_layer_input_norm.weight", H);
    ly.q_norm = single(pre + "self_attn.q_norm.weight", ly.hd);
    ly.k_norm = single(pre + "self_attn.k_norm.weight", ly.hd);
    {
      const HostTensor& t = found[pre + "layer_scalar"];
      if (!to_f32(t.view, 1, host)) {
        *msg = pre + "layer_scalar is not finite";
        return SVL_CORRUPT;
      }
      ly.layer_scalar = host[0];
    }
    if (!ok) break;
    round_dev(ly.wqkv, (size_t)ly.ld_qkv * H);
    round_dev(ly.wo, H * ly.qd);
    round_dev(ly.wgu, (size_t)2 * F_pad * H);
    round_dev(ly.wdown, H * F);
    round_dev(ly.wpg, P * H);
    round_dev(ly.wpp, H * P);
    if (split && (!make_split(&ly.wqkv, ly.ld_qkv, H) || !make_split(&ly.wo, H, ly.qd) ||
                  !make_split(&ly.wgu, 2 * F_pad, H) || !make_split(&ly.wdown, H, F) ||
                  !make_split(&ly.wpg, P, H) || !make_split(&ly.wpp, H, P))) {
      *msg = "out of device memory for split-precision weights";
      return SVL_INTERNAL;
    }
    if (gemm_f16 && (!make_f16(ly.wqkv, ly.ld_qkv, H, &ly.qkv16) || !make_f16(ly.wo, H, ly.qd, &ly.o16) ||
                     !make_f16(ly.wgu, 2 * F_pad, H, &ly.gu16) || !make_f16(ly.wpg, P, H, &ly.pg16) ||
                     !make_f16(ly.wdown, H, F, &ly.down16) || !make_f16(ly.wpp, H, P, &ly.pp16))) {
      *msg = "out of device memory for FP16 weights";
      return SVL_INTERNAL;
    }
    if (gemm_f16) {
      // row-norm maxima: gate rows (128-row blocks at even positions) and up
      // rows of the interleaved gate/up weight, and the PLE-gate rows
      uint32_t* nm = (uint32_t*)dalloc(4);
      uint32_t host_nm[4] = {0, 0, 0, 0};
      if (!nm) return SVL_INTERNAL;
      cudaMemsetAsync(nm, 0, 16, stream);
      launch_row_norm_max(ly.wgu, (int)(2 * F_pad), (int)H, 128, nm, stream);
      launch_row_norm_max(ly.wpg, (int)P, (int)H, 0, nm + 2, stream);
      if (cudaMemcpyAsync(host_nm, nm, 16, cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
          cudaStreamSynchronize(stream) != cudaSuccess)
        return SVL_INTERNAL;
      std::memcpy(&ly.g_max, &host_nm[0], 4);
      std::memcpy(&ly.u_max, &host_nm[1], 4);
      std::memcpy(&ly.pg_max, &host_nm[2], 4);
    }
  }
  if (!ok) return SVL_CORRUPT;
  if (split && (!make_split(&wple, L * P, H) || !make_split(&wemb, E, H))) {
    *msg = "out of device memory for split-precision weights";
    return SVL_INTERNAL;
  }
  if (gemm_f16 && (!make_f16(wple, L * P, H, &ple16) || !make_f16(wemb, E, H, &emb16))) {
    *msg = "out of device memory for FP16 weights";
    return SVL_INTERNAL;
  }

  // RoPE inverse frequencies per layer type (config.rs:366-373 ->
  // kernels.rs:991-1010), computed on the host with the same f32 powf.
  for (int full = 0; full < 2; ++full) {
    size_t hd = 0;
    for (size_t l = 0; l < L; ++l)
      if ((layer_cfg[l].layer_type == SVL_LAYER_FULL) == (full == 1)) {
        hd = layer_cfg[l].head_dim;
        break;
      }
    if (!hd) continue;
    const float base = full ? cfg.full_rope_theta : cfg.sliding_rope_theta;
    if (!std::isfinite(base) || base <= 1.0f) {
      *msg = "RoPE theta must be finite and greater than one";
      return SVL_CORRUPT;
    }
    std::vector<float> inv(hd / 2);
    for (size_t p = 0; p < hd / 2; ++p) inv[p] = 1.0f / std::pow(base, (float)(2 * p) / (float)hd);
    float* d = dalloc(hd / 2);
    if (!d) return SVL_INTERNAL;
    cudaMemcpy(d, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice);
    (full ? full_inv : sliding_inv) = d;
    // (cos, sin) for every position a sequence may have (<= 8192 tokens)
    const int n_pos = (int)(cfg.max_position_embeddings < kMaxTextTokens ? cfg.max_position_embeddings : kMaxTextTokens);
    float2* table = (float2*)dalloc((size_t)n_pos * hd);
    if (!table) {
      *msg = "out of device memory for the RoPE table";
      return SVL_INTERNAL;
    }
    launch_rope_table(d, (int)(hd / 2), n_pos, 1, table, stream);
    (full ? full_rope : sliding_rope) = table;
    float2* table_t = (float2*)dalloc((size_t)n_pos * hd);  // [p][position] for the fused QKV epilogue
    if (!table_t) {
      *msg = "out of device memory for the RoPE table";
      return SVL_INTERNAL;
    }
    launch_rope_table(d, (int)(hd / 2), n_pos, 0, table_t, stream);
    (full ? full_rope_t : sliding_rope_t) = table_t;
    rope_positions = n_pos;
  }
  if (cudaStreamSynchronize(stream) != cudaSuccess || cudaGetLastError() != cudaSuccess) {
    *msg = "weight preparation failed on the device";
    return SVL_INTERNAL;
  }
  return SVL_OK;
}

// Host-side validation of a packed batch (text.rs:188-202, 211-218).
int Model::validate_batch(const uint32_t* ids, const uint64_t* cu, uint32_t batch, std::string* msg) const {
  if (batch == 0) {
    *msg = "cannot embed an empty batch";
    return SVL_CORRUPT;
  }
  if (cu[0] != 0) {
    *msg = "cu_seqlens[0] must be 0";
    return SVL_CORRUPT;
  }
  for (uint32_t b = 0; b < batch; ++b) {
    if (cu[b + 1] < cu[b]) {
      *msg = "cu_seqlens must be non-decreasing";
      return SVL_CORRUPT;
    }
    const uint64_t n = cu[b + 1] - cu[b];
    if (n == 0) {
      *msg = "cannot embed an empty token sequence";
      return SVL_CORRUPT;
    }
    if (n > kMaxTextTokens) {
      *msg = "sequence has " + std::to_string(n) + " tokens, above the 8192-token context";
      return SVL_LIMIT_EXCEEDED;
    }
    if (n > cfg.max_position_embeddings) {
      *msg = "sequence has " + std::to_string(n) + " tokens, above the declared positions";
      return SVL_LIMIT_EXCEEDED;
    }
  }
  const uint64_t T = cu[batch];
  if (T * (uint64_t)cfg.num_hidden_layers * cfg.hidden_size_per_layer_input > (uint64_t)1 << 40 ||
      T > (uint64_t)1 << 30) {
    *msg = "batch too large";
    return SVL_LIMIT_EXCEEDED;
  }
  (void)kMaxActivationElements;
  if (ids) {
    for (uint64_t t = 0; t < T; ++t)
      if (ids[t] >= cfg.vocab_size) {
        *msg = "token id " + std::to_string(ids[t]) + " is outside the vocabulary of " +
               std::to_string(cfg.vocab_size) + " entries";
        return SVL_CORRUPT;
      }
  }
  return SVL_OK;
}

int Model::gemm(const float* A, int lda, const float* B, int ldb, float* C, int ldc, int M, int N, int K, int epi,
                float alpha, const float* aux, int ld_aux, int round_out, int n_out, cudaStream_t st) {
  GemmParams p{};
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
  p.epilogue = epi;
  p.alpha = alpha;
  p.aux = aux;
  p.ld_aux = ld_aux;
  p.round_out = round_out;
  p.err = err_d;
  p.tf32_tma = 0;
  Profiler::Scope scope(&prof, kProfGemm, st);
  return gemm_tf32(p, st) == cudaSuccess ? SVL_OK : SVL_INTERNAL;
}

int Model::gemm16(const uint16_t* A, int lda, const float* a_inv, const Weight& w, int ldb, float* C, int ldc, int M,
                  int N, int K, int epi, float alpha, const float* aux, int ld_aux, int round_out, int n_out,
                  cudaStream_t st, const float* out_inv, const float* aux_row_inv, int aux_row_stride,
                  const float* aux_col_w, float* row_ss, int row_ss_stride, float* group_inv) {
  GemmParams p{};
  p.A = A;
  p.lda = lda;
  p.B = w.f16;
  p.ldb = ldb;
  p.C = C;
  p.ldc = ldc;
  p.M = M;
  p.N = N;
  p.K = K;
  p.n_out = n_out;
  p.epilogue = epi;
  p.alpha = alpha;
  p.aux = aux;
  p.ld_aux = ld_aux;
  p.round_out = round_out;
  p.err = err_d;
  p.f16 = 1;
  p.a_inv = a_inv;
  p.b_scale = w.inv;
  p.out_f16 = out_inv != nullptr || group_inv != nullptr;  // FP16 output rows (scaled)
  p.out_inv = out_inv;
  p.aux_row_inv = aux_row_inv;
  p.aux_row_stride = aux_row_stride;
  p.aux_col_w = aux_col_w;
  p.row_ss = row_ss;
  p.row_ss_stride = row_ss_stride;
  p.group_inv = group_inv;
  Profiler::Scope scope(&prof, kProfGemm, st);
  return gemm_tf32(p, st) == cudaSuccess ? SVL_OK : SVL_INTERNAL;
}

// FP16 copy of a [rows, cols] weight with one power-of-two scale for the
// whole matrix (inv: a device scalar, the GEMM's b_scale).
bool Model::make_f16(const float* w, size_t rows, size_t cols, Weight* out) {
  out->f32 = const_cast<float*>(w);
  out->f16 = (uint16_t*)dalloc((rows * cols + 1) / 2);
  out->inv = dalloc(2);  // [inverse scale, reduction scratch]
  if (!out->f16 || !out->inv) return false;
  launch_matrix_to_f16(w, rows * cols, out->f16, out->inv, (uint32_t*)(out->inv + 1), stream);
  return cudaGetLastError() == cudaSuccess;
}

bool Model::make_split(float** w, size_t rows, size_t cols) {
  float* w3 = dalloc(rows * cols * 3);
  if (!w3) return false;
  launch_split3(*w, (int)cols, w3, (int)rows, (int)cols, 1, stream);
  if (cudaStreamSynchronize(stream) != cudaSuccess) return false;
  // the exact copy is no longer needed
  for (auto it = allocations.begin(); it != allocations.end(); ++it)
    if (*it == (void*)*w) {
      cudaFree(*it);
      allocations.erase(it);
      break;
    }
  *w = w3;
  return true;
}

int Model::gemm_split(const float* A, int lda, float* x3, const float* W3, float* C, int ldc, int M, int N, int K,
                      int epi, float alpha, const float* aux, int ld_aux, int n_out, cudaStream_t st) {
  {
    Profiler::Scope scope(&prof, kProfOther, st);
    launch_split3(A, lda, x3, M, K, 0, st);
  }
  return gemm(x3, 3 * K, W3, 3 * K, C, ldc, M, N, 3 * K, epi, alpha, aux, ld_aux, 0, n_out, st);
}

// text.rs:182-538 for a packed batch.  d_ids / d_cu on the device, cu on the
// host (schedule).  Outputs are device pointers (nullable except one of
// d_out / d_normalized).
int Model::forward_part(const std::string& tag, const uint32_t* d_ids, const uint64_t* cu, uint32_t batch,
                        const uint64_t* d_cu, const FeatureRows* features, uint32_t dim, float* d_out,
                        float* d_pooled, float* d_normalized, float* d_projected, float* d_hidden,
                        const std::vector<AttnSched>& scheds, const uint32_t* d_sched, cudaStream_t st,
                        std::string* msg) {
  const int H = (int)cfg.hidden_size, P = (int)cfg.hidden_size_per_layer_input, F = (int)cfg.intermediate_size,
            L = (int)cfg.num_hidden_layers, NH = (int)cfg.num_attention_heads, E = (int)cfg.embedding_dim;
  const int T = (int)cu[batch];
  const float eps = cfg.rms_norm_eps;
  int max_qkv = 0, max_q = 0;
  for (auto& ly : layers) {
    max_qkv = ly.ld_qkv > max_qkv ? ly.ld_qkv : max_qkv;
    max_q = ly.qd > max_q ? ly.qd : max_q;
  }
  uint32_t* seq_of = (uint32_t*)workspace(tag + "seq_of", (size_t)T * 4);
  uint32_t* pos_of = (uint32_t*)workspace(tag + "pos_of", (size_t)T * 4);
  float* hidden = (float*)workspace(tag + "hidden", (size_t)T * H * 4);
  float* xn = (float*)workspace(tag + "xn", (size_t)T * H * 4);
  float* tmp = (float*)workspace(tag + "tmp", (size_t)T * H * 4);
  float* per_layer = (float*)workspace(tag + "per_layer", (size_t)T * L * P * 4);
  float* qkv = (float*)workspace(tag + "qkv", (size_t)T * max_qkv * 4);
  // the grouped FP16 projection's scales and partial sums of squares
  float* qkv_gi = gemm_f16 ? (float*)workspace(tag + "qkv_gi", (size_t)T * (max_qkv / 128 + 1) * 4) : nullptr;
  float* qkv_ss = gemm_f16 ? (float*)workspace(tag + "qkv_ss", (size_t)T * (max_qkv / 128 + 1) * 4) : nullptr;
  float* attn = (float*)workspace(tag + "attn", (size_t)T * max_q * 4);
  float* ffn = (float*)workspace(tag + "ffn", (size_t)T * F * 4);
  float* gated = (float*)workspace(tag + "gated", (size_t)T * P * 4);
  float* projected = d_projected ? d_projected : (float*)workspace(tag + "projected", (size_t)T * E * 4);
  uint16_t* qkv16 = attn_f16 ? (uint16_t*)workspace(tag + "qkv16", (size_t)T * max_qkv * 2) : nullptr;
  // FP16 GEMM operands: xn16 / xn_inv replace xn (row-scaled), attn16 the
  // attention output (|O| <= max |v|, no scale needed)
  uint16_t* xn16 = gemm_f16 ? (uint16_t*)workspace(tag + "xn16", (size_t)T * H * 2) : nullptr;
  float* xn_inv = gemm_f16 ? (float*)workspace(tag + "xn_inv", (size_t)T * 4) : nullptr;
  uint16_t* attn16 = gemm_f16 && attn_f16 ? (uint16_t*)workspace(tag + "attn16", (size_t)T * max_q * 2) : nullptr;
  // FP16 GeGLU / PLE-gate outputs (the down and PLE-projection operands) with
  // bound-derived row scales, and the per-(token, layer) largest |per_layer|
  uint16_t* ffn16 = gemm_f16 ? (uint16_t*)workspace(tag + "ffn16", (size_t)T * F * 2) : nullptr;
  uint16_t* gated16 = gemm_f16 ? (uint16_t*)workspace(tag + "gated16", (size_t)T * P * 2) : nullptr;
  float* ffn_inv = gemm_f16 ? (float*)workspace(tag + "ffn_inv", (size_t)T * 4) : nullptr;
  float* gated_inv = gemm_f16 ? (float*)workspace(tag + "gated_inv", (size_t)T * 4) : nullptr;
  float* pmax = gemm_f16 ? (float*)workspace(tag + "pmax", (size_t)T * L * 4) : nullptr;
  // with FP16 GEMMs (and a vectorised per-layer width) per_layer stays
  // un-normalised: pinv holds each (token, layer) row's 1 / rms and the
  // PLE-gate epilogue applies the norm
  const bool ple_stats = gemm_f16 && P % 128 == 0 && P <= 1024;
  float* pinv = ple_stats ? (float*)workspace(tag + "pinv", (size_t)T * L * 4) : nullptr;
  // with the fused per-layer-input block, the PLE projection's epilogue writes
  // the [T, 24 x 512] table in FP16 with a power-of-two scale per (token,
  // 128-column part) and each part's sum of squares; the block forms 1 / rms
  // itself, so the table is half the bytes and never read back for its
  // statistics
  const bool ple_partials = ple_fused && ple_stats && P == 512 && (L * P) % 128 == 0;
  float* pss = ple_partials ? (float*)workspace(tag + "pss", (size_t)T * (L * P / 128) * 4) : nullptr;
  float* pgi = ple_partials ? (float*)workspace(tag + "pgi", (size_t)T * (L * P / 128) * 4) : nullptr;
  // split precision: the expanded [hi | hi | lo] operand of the next GEMM
  const int max_k = std::max(std::max(H, max_q), std::max(F, P));
  float* x3 = split ? (float*)workspace(tag + "x3", (size_t)T * 3 * max_k * 4) : nullptr;
  const size_t items_bytes = attention_tc_items_bytes(cu, (int)batch, NH) + 16;
  void* attn_items = workspace(tag + "attn_items", items_bytes);
  if (!seq_of || !pos_of || !hidden || !xn || !tmp || !per_layer || !qkv || !attn || !ffn || !gated || !projected ||
      !attn_items || (attn_f16 && !qkv16) || (gemm_f16 && (!xn16 || !xn_inv)) || (gemm_f16 && attn_f16 && !attn16) ||
      (gemm_f16 && (!ffn16 || !gated16 || !ffn_inv || !gated_inv || !pmax)) || (ple_stats && !pinv) || (ple_partials && (!pss || !pgi)) || (gemm_f16 && (!qkv_gi || !qkv_ss)) ||
      (split && !x3)) {
    *msg = "out of device memory for activations";
    return SVL_LIMIT_EXCEEDED;
  }
  int st_code = SVL_OK;
#define SVL_G(...)                                  \
  do {                                              \
    if ((st_code = gemm(__VA_ARGS__)) != SVL_OK) {  \
      *msg = "GEMM launch failed";                  \
      return st_code;                               \
    }                                               \
  } while (0)
  // A split-precision GEMM (A expanded into x3 first)
#define SVL_GS(...)                                               \
  do {                                                            \
    if ((st_code = gemm_split(__VA_ARGS__, st)) != SVL_OK) {      \
      *msg = "GEMM launch failed";                                \
      return st_code;                                             \
    }                                                             \
  } while (0)
  const int exact = split ? kResExact : 0;  // producers of split GEMM inputs write exact FP32

  {
    Profiler::Scope s1(&prof, kProfOther, st);
    launch_positions(d_cu, batch, seq_of, pos_of, st);
  }
  {
    Profiler::Scope s2(&prof, kProfOther, st);
    launch_embed(d_ids, T, embed, H, cfg.vocab_size, cfg.embedding_scale, hidden, err_d, st);
  }
  if (features)
    for (const auto& f : features->rows)
      cudaMemcpyAsync(hidden + (size_t)f.first * H, f.second, (size_t)H * 4, cudaMemcpyHostToDevice, st);
  if (d_hidden) cudaMemcpyAsync(d_hidden, hidden, (size_t)T * H * 4, cudaMemcpyDeviceToDevice, st);

  // A GEMM on the xn operand: FP16 row-scaled (xn16 / xn_inv) or FP32.
#define SVL_GX(W16, W32, ...)                                                                     \
  do {                                                                                            \
    if ((st_code = gemm_f16 ? gemm16(xn16, H, xn_inv, W16, H, __VA_ARGS__, st)                    \
                            : gemm(xn, H, W32, H, __VA_ARGS__, st)) != SVL_OK) {                  \
      *msg = "GEMM launch failed";                                                                \
      return st_code;                                                                             \
    }                                                                                             \
  } while (0)

  // PLE (text.rs:282-306): per_layer = rmsnorm(linear(hidden) * ple_scale)
  // the GEMM operand is a copy of the scaled embeddings (FP16 row-scaled, or
  // TF32-rounded)
  if (split) {
    SVL_GS(hidden, H, x3, wple, per_layer, L * P, T, L * P, H, kEpiStore, cfg.ple_scale, nullptr, 0, 0);
  } else {
    if (gemm_f16) {
      Profiler::Scope s3(&prof, kProfOther, st);
      launch_rows_to_f16(hidden, H, xn16, H, T, H, xn_inv, err_d, st);
    } else {
      cudaMemcpyAsync(xn, hidden, (size_t)T * H * 4, cudaMemcpyDeviceToDevice, st);
      Profiler::Scope s3(&prof, kProfOther, st);
      launch_round_tf32(xn, (size_t)T * H, st);
    }
    if (ple_partials) {
      // the FP16 table reuses the FP32 table's buffer (half of it)
      if ((st_code = gemm16(xn16, H, xn_inv, ple16, H, per_layer, L * P, T, L * P, H, kEpiStore, cfg.ple_scale,
                            nullptr, 0, 0, 0, st, nullptr, nullptr, 0, nullptr, pss, L * P / 128, pgi)) != SVL_OK) {
        *msg = "GEMM launch failed";
        return st_code;
      }
    } else {
      SVL_GX(ple16, wple, per_layer, L * P, T, L * P, H, kEpiStore, cfg.ple_scale, nullptr, 0, 0, 0);
    }
  }
  if (!ple_partials) {
    Profiler::Scope s4(&prof, kProfNorm, st);
    if (ple_stats) {
      // statistics only (1 / rms and the normalised row's largest |value|):
      // the 4 B per value write and re-read of the normalised copy are saved
      launch_rmsnorm_rows(per_layer, P, nullptr, P, T * L, P, ple_norm, 1.0f, eps, 0, err_d, st, nullptr, nullptr,
                          pmax, pinv);
    } else {
      launch_rmsnorm_rows(per_layer, P, per_layer, P, T * L, P, ple_norm, 1.0f, eps, 0, err_d, st, nullptr, nullptr,
                          pmax);
    }
  }
  {
    Profiler::Scope s5(&prof, kProfNorm, st);
    launch_rmsnorm_rows(hidden, H, xn, H, T, H, layers[0].in_ln, 1.0f, eps, split ? 0 : 1, err_d, st, xn16, xn_inv);
  }

  for (int l = 0; l < L; ++l) {
    const LayerDev& ly = layers[l];
    // attention block (text.rs:345-433)
    const float2* rope = ly.full ? full_rope : sliding_rope;
    // FP16 attention operands (same significand as TF32) for the CTA-pair kernel
    bool f16 = attn_f16 && rope && attention_f16_supported(ly.hd, NH, ly.kvh);
    if (ly.hd == 256 && rope && qkv_fused) {
      // per-head norms and RoPE fused into the projection's epilogue
      GemmParams gp{};
      gp.A = xn;
      gp.lda = H;
      gp.B = ly.wqkv;
      gp.ldb = H;
      if (gemm_f16) {
        gp.f16 = 1;
        gp.A = xn16;
        gp.a_inv = xn_inv;
        gp.B = ly.qkv16.f16;
        gp.b_scale = ly.qkv16.inv;
      }
      gp.C = qkv;
      gp.ldc = ly.ld_qkv;
      gp.M = T;
      gp.N = ly.ld_qkv;
      gp.K = H;
      gp.epilogue = kEpiQkv;
      gp.alpha = 1.0f;
      gp.err = err_d;
      gp.nh = NH;
      gp.kvh = ly.kvh;
      gp.q_norm = ly.q_norm;
      gp.k_norm = ly.k_norm;
      gp.rope = ly.full ? full_rope_t : sliding_rope_t;
      gp.rope_stride = rope_positions;
      gp.pos_of = pos_of;
      gp.eps = eps;
      if (f16) {
        gp.C = (float*)qkv16;
        gp.out_f16 = 1;
      }
      Profiler::Scope sq(&prof, kProfGemm, st);
      if (gemm_tf32(gp, st) != cudaSuccess) {
        *msg = "GEMM launch failed";
        return SVL_INTERNAL;
      }
    } else {
      // FP16 operands and attention: the projection stored in FP16 with
      // per-(token, 128-column) scales and partial sums of squares, the
      // norms and RoPE applied from those (half the bytes each way)
      const bool grouped = f16 && gemm_f16 && !split && ly.hd % 128 == 0 && ly.ld_qkv % 128 == 0 && ly.ld_qkv > 128;
      if (split) {
        SVL_GS(xn, H, x3, ly.wqkv, qkv, ly.ld_qkv, T, ly.ld_qkv, H, kEpiStore, 1.0f, nullptr, 0, 0);
      } else if (grouped) {
        if ((st_code = gemm16(xn16, H, xn_inv, ly.qkv16, H, qkv, ly.ld_qkv, T, ly.ld_qkv, H, kEpiStore, 1.0f, nullptr,
                              0, 0, 0, st, nullptr, nullptr, 0, nullptr, qkv_ss, max_qkv / 128, qkv_gi)) != SVL_OK) {
          *msg = "GEMM launch failed";
          return st_code;
        }
      } else {
        SVL_GX(ly.qkv16, ly.wqkv, qkv, ly.ld_qkv, T, ly.ld_qkv, H, kEpiStore, 1.0f, nullptr, 0, 0, 0);
      }
      Profiler::Scope s6(&prof, kProfNorm, st);
      const float* inv = ly.full ? full_inv : sliding_inv;
      if (grouped && launch_qkv_post16((const uint16_t*)qkv, qkv_gi, qkv_ss, max_qkv / 128, ly.ld_qkv, T, NH, ly.kvh,
                                       ly.hd, ly.q_norm, ly.k_norm, rope, pos_of, eps, qkv16, err_d, st)) {
        // done
      } else if (grouped) {
        *msg = "q/k/v post-processing launch failed";
        return SVL_INTERNAL;
      } else if (!f16 || !launch_qkv_post(qkv, ly.ld_qkv, T, NH, ly.kvh, ly.hd, ly.q_norm, ly.k_norm, inv, rope, pos_of,
                                          eps, 1, qkv16, err_d, st)) {
        f16 = false;
        launch_qkv_post(qkv, ly.ld_qkv, T, NH, ly.kvh, ly.hd, ly.q_norm, ly.k_norm, inv, rope, pos_of, eps,
                        split ? 0 : 1, nullptr, err_d, st);
      }
    }
    Profiler::Scope* s7 = new Profiler::Scope(&prof, kProfAttention, st);
    const int window = ly.full ? -1 : (int)cfg.sliding_window;
    bool launched;
    if (f16) {
      AttnF16Params ap{};
      ap.qkv = qkv16;
      ap.ld = ly.ld_qkv;
      ap.T = T;
      ap.nh = NH;
      ap.kvh = ly.kvh;
      ap.hd = ly.hd;
      ap.window = window;
      ap.out = attn;
      ap.ld_out = ly.qd;
      ap.round_out = 1;
      ap.out16 = attn16;  // FP16 operand of the o projection (when GEMM operands are FP16)
      ap.err = err_d;
      const AttnSched* sc = nullptr;
      for (const AttnSched& x : scheds)
        if (x.hd == ly.hd && x.window == window) sc = &x;
      launched = sc && launch_attention_f16(ap, d_sched + sc->word, sc->pairs, st) == cudaSuccess;
    } else if (!split && attention_tc_supported(ly.hd)) {
      AttnParams ap{};
      ap.qkv = qkv;
      ap.ld = ly.ld_qkv;
      ap.T = T;
      ap.nh = NH;
      ap.kvh = ly.kvh;
      ap.hd = ly.hd;
      ap.window = window;
      ap.out = attn;
      ap.ld_out = ly.qd;
      ap.round_out = 1;
      ap.err = err_d;
      launched = launch_attention_tc(ap, cu, (int)batch, attn_items, items_bytes, st) == cudaSuccess;
    } else {
      // FP32 on the CUDA cores (head dims the tensor-core kernels do not
      // take, and split precision)
      launched = launch_attention_simt(qkv, ly.ld_qkv, T, NH, ly.kvh, ly.hd, d_cu, seq_of, pos_of, window, attn, ly.qd,
                                       split ? 0 : 1, err_d, st);
    }
    delete s7;
    if (!launched) {
      *msg = "attention launch failed";
      return SVL_INTERNAL;
    }
    // the o projection and the residual step after it as one row-fused kernel
    const bool o_fused = row_fused && f16 && attn16 && gemm_residual_supported(H, ly.qd);
    if (o_fused) {
      GemmResidualLaunch g{};
      g.K = ly.qd;
      g.a16 = attn16;
      g.lda = ly.qd;
      g.a_inv = nullptr;
      g.w16 = ly.o16.f16;
      g.w_inv = ly.o16.inv;
      g.out16 = xn16;
      g.out = kOutNormNextBound;
      g.res.T = T;
      g.res.hidden = hidden;
      g.res.w_post = ly.post_attn;
      g.res.layer_scalar = 1.0f;
      g.res.apply_scalar = 0;
      g.res.w_next = ly.pre_ff;
      g.res.eps = eps;
      g.res.xn_inv_out = xn_inv;
      g.res.bound_inv = ffn_inv;
      g.res.bound_a = ly.g_max;
      g.res.bound_b = ly.u_max;
      g.res.err = err_d;
      Profiler::Scope so(&prof, kProfGemm, st);
      if (launch_gemm_residual(g, st) != cudaSuccess) {
        *msg = "fused o projection launch failed";
        return SVL_INTERNAL;
      }
    } else if (f16 && attn16) {
      if ((st_code = gemm16(attn16, ly.qd, nullptr, ly.o16, ly.qd, tmp, H, T, H, ly.qd, kEpiStore, 1.0f, nullptr, 0, 0,
                            0, st)) != SVL_OK) {
        *msg = "GEMM launch failed";
        return st_code;
      }
    } else if (split) {
      SVL_GS(attn, ly.qd, x3, ly.wo, tmp, H, T, H, ly.qd, kEpiStore, 1.0f, nullptr, 0, 0);
    } else {
      SVL_G(attn, ly.qd, ly.wo, ly.qd, tmp, H, T, H, ly.qd, kEpiStore, 1.0f, nullptr, 0, 0, 0, st);
    }
    BoundScale ffn_bound, gated_bound;
    if (gemm_f16) {
      ffn_bound.inv = ffn_inv;
      ffn_bound.a_max = ly.g_max;
      ffn_bound.b_max = ly.u_max;
      gated_bound.inv = gated_inv;
      gated_bound.a_max = ly.pg_max;
      gated_bound.row_max = pmax + l;
      gated_bound.stride = L;
    }
    {
      Profiler::Scope s8(&prof, kProfNorm, st);
      if (!o_fused)
        launch_residual_norm(hidden, tmp, T, H, ly.post_attn, 1.0f, 0, ly.pre_ff, xn, kResNormNext | exact, eps, err_d,
                             st, xn16, xn_inv, gemm_f16 ? &ffn_bound : nullptr);
    }
    // feed-forward block (text.rs:435-472); with FP16 operands the GeGLU
    // output is written FP16 with the bound-derived row scale for down
    // with the fused PLE block after it, the down projection and its
    // residual step (the stream's FP16 copy) run as one row-fused kernel
    const bool down_fused = ple_fused && ple_stats && gemm_residual_supported(H, F);
    if (gemm_f16) {
      if ((st_code = gemm16(xn16, H, xn_inv, ly.gu16, H, (float*)ffn16, F, T, 2 * F_pad, H, kEpiGeglu, 1.0f, nullptr,
                            0, 0, F, st, ffn_inv)) != SVL_OK ||
          (!down_fused && (st_code = gemm16(ffn16, F, ffn_inv, ly.down16, F, tmp, H, T, H, F, kEpiStore, 1.0f, nullptr,
                                            0, 0, 0, st)) != SVL_OK)) {
        *msg = "GEMM launch failed";
        return st_code;
      }
      if (down_fused) {
        GemmResidualLaunch g{};
        g.K = F;
        g.a16 = ffn16;
        g.lda = F;
        g.a_inv = ffn_inv;
        g.w16 = ly.down16.f16;
        g.w_inv = ly.down16.inv;
        g.out16 = xn16;
        g.out = kOutCopy;
        g.res.T = T;
        g.res.hidden = hidden;
        g.res.w_post = ly.post_ff;
        g.res.layer_scalar = 1.0f;
        g.res.apply_scalar = 0;
        g.res.eps = eps;
        g.res.xn_inv_out = xn_inv;
        g.res.err = err_d;
        Profiler::Scope sd(&prof, kProfGemm, st);
        if (launch_gemm_residual(g, st) != cudaSuccess) {
          *msg = "fused down projection launch failed";
          return SVL_INTERNAL;
        }
      }
    } else if (split) {
      SVL_GS(xn, H, x3, ly.wgu, ffn, F, T, 2 * F_pad, H, kEpiGeglu, 1.0f, nullptr, 0, F);
      SVL_GS(ffn, F, x3, ly.wdown, tmp, H, T, H, F, kEpiStore, 1.0f, nullptr, 0, 0);
    } else {
      SVL_G(xn, H, ly.wgu, H, ffn, F, T, 2 * F_pad, H, kEpiGeglu, 1.0f, nullptr, 0, 1, F, st);
      SVL_G(ffn, F, ly.wdown, F, tmp, H, T, H, F, kEpiStore, 1.0f, nullptr, 0, 0, 0, st);
    }
    if (!down_fused) {
      Profiler::Scope s9(&prof, kProfNorm, st);
      launch_residual_norm(hidden, tmp, T, H, ly.post_ff, 1.0f, 0, nullptr, xn, kResRoundedCopy | exact, eps, err_d, st, xn16,
                           xn_inv, gemm_f16 && !(ple_fused && ple_stats) ? &gated_bound : nullptr);
    }
    // per-layer-input block (text.rs:474-513): one fused kernel (both GEMMs,
    // the gate, the residual step and the next pre-norm) at the manifest
    // widths, else two GEMMs and the residual kernel
    const float* w_next = l + 1 < L ? layers[l + 1].in_ln : final_norm;
    if (ple_fused && ple_stats) {
      PleBlockParams pb{};
      pb.T = T;
      pb.xn16 = xn16;
      pb.xn_inv = xn_inv;
      pb.w_gate16 = ly.pg16.f16;
      pb.w_gate_inv = ly.pg16.inv;
      pb.w_proj16 = ly.pp16.f16;
      pb.w_proj_inv = ly.pp16.inv;
      pb.per_layer16 = (const uint16_t*)per_layer + (size_t)l * P;
      pb.ld_pl = L * P;
      pb.pss = pss + (size_t)l * (P / 128);
      pb.pgi = pgi + (size_t)l * (P / 128);
      pb.pss_stride = L * P / 128;
      pb.ple_norm = ple_norm;
      pb.hidden = hidden;
      pb.w_post = ly.post_ple;
      pb.layer_scalar = ly.layer_scalar;
      pb.w_next = w_next;
      pb.eps = eps;
      pb.xn16_out = xn16;
      pb.xn_inv_out = xn_inv;
      pb.err = err_d;
      Profiler::Scope sp(&prof, kProfGemm, st);
      if (launch_ple_block(pb, st) != cudaSuccess) {
        *msg = "fused per-layer-input block launch failed";
        return SVL_INTERNAL;
      }
    } else if (gemm_f16) {
      if ((st_code = gemm16(xn16, H, xn_inv, ly.pg16, H, (float*)gated16, P, T, P, H, kEpiPleGate, 1.0f,
                            per_layer + (size_t)l * P, L * P, 0, 0, st, gated_inv, ple_stats ? pinv + l : nullptr, L,
                            ple_stats ? ple_norm : nullptr)) != SVL_OK ||
          (st_code = gemm16(gated16, P, gated_inv, ly.pp16, P, tmp, H, T, H, P, kEpiStore, 1.0f, nullptr, 0, 0, 0,
                            st)) != SVL_OK) {
        *msg = "GEMM launch failed";
        return st_code;
      }
    } else if (split) {
      SVL_GS(xn, H, x3, ly.wpg, gated, P, T, P, H, kEpiPleGate, 1.0f, per_layer + (size_t)l * P, L * P, 0);
      SVL_GS(gated, P, x3, ly.wpp, tmp, H, T, H, P, kEpiStore, 1.0f, nullptr, 0, 0);
    } else {
      SVL_G(xn, H, ly.wpg, H, gated, P, T, P, H, kEpiPleGate, 1.0f, per_layer + (size_t)l * P, L * P, 1, 0, st);
      SVL_G(gated, P, ly.wpp, P, tmp, H, T, H, P, kEpiStore, 1.0f, nullptr, 0, 0, 0, st);
    }
    if (!(ple_fused && ple_stats)) {
      Profiler::Scope s10(&prof, kProfNorm, st);
      launch_residual_norm(hidden, tmp, T, H, ly.post_ple, ly.layer_scalar, 1, w_next, xn, kResNormNext | exact, eps, err_d,
                           st, xn16, xn_inv);
    }
    if (d_hidden)
      cudaMemcpyAsync(d_hidden + (size_t)(l + 1) * T * H, hidden, (size_t)T * H * 4, cudaMemcpyDeviceToDevice, st);
  }
  // final (text.rs:520-531): xn = rmsnorm(hidden, norm) from the last residual step
  if (split)
    SVL_GS(xn, H, x3, wemb, projected, E, T, E, H, kEpiStore, 1.0f, nullptr, 0, 0);
  else
    SVL_GX(emb16, wemb, projected, E, T, E, H, kEpiStore, 1.0f, nullptr, 0, 0, 0);
  {
    Profiler::Scope s11(&prof, kProfOther, st);
    float* mean = (float*)workspace(tag + "pool_mean", (size_t)batch * E * 4);
    if (!mean) {
      *msg = "out of device memory for activations";
      return SVL_LIMIT_EXCEEDED;
    }
    launch_pool_normalize(projected, E, d_cu, (int)batch, dim, mean, d_pooled, d_normalized, d_out, err_d, st);
  }
#undef SVL_G
#undef SVL_GS
#undef SVL_GX
  if (cudaGetLastError() != cudaSuccess) {
    *msg = "kernel launch failed";
    return SVL_INTERNAL;
  }
  return SVL_OK;
}

// FP16 attention schedules of one group: one per (head dim, window), each
// appended 16-byte aligned to `words` (AttnSched::word = offset in words).
int Model::attention_schedules(const uint64_t* cu, uint32_t batch, std::vector<AttnSched>* scheds,
                               std::vector<uint32_t>* words, std::string* msg) {
  const int NH = (int)cfg.num_attention_heads;
  std::vector<uint32_t> one;
  for (const LayerDev& ly : layers) {
    const int window = ly.full ? -1 : (int)cfg.sliding_window;
    if (!attn_f16 || !attention_f16_supported(ly.hd, NH, ly.kvh)) continue;
    bool have = false;
    for (const AttnSched& sc : *scheds) have |= sc.hd == ly.hd && sc.window == window;
    if (have) continue;
    const int pairs = attention_f16_schedule(cu, (int)batch, NH, ly.hd, window, &one);
    if (pairs < 0) {
      *msg = "attention schedule failed";
      return SVL_INTERNAL;
    }
    scheds->push_back({ly.hd, window, pairs, words->size()});
    words->insert(words->end(), one.begin(), one.end());
    words->resize((words->size() + 3) / 4 * 4, 0u);
  }
  return SVL_OK;
}

// Relative device work of one sequence of L tokens: the projections' FLOPs
// (linear in L) plus attention's FLOPs over the attended (query, key) pairs
// (a sliding layer's keys clipped to the window radius), the latter weighted
// by 1.4 -- the encoder GEMMs run at ~1.4x attention's FLOP rate on B200.
double Model::sequence_cost(uint64_t L) const {
  const double H = (double)cfg.hidden_size, F = (double)cfg.intermediate_size,
               P = (double)cfg.hidden_size_per_layer_input, E = (double)cfg.embedding_dim,
               NH = (double)cfg.num_attention_heads;
  const double n = (double)L;
  // attended pairs of a sliding layer (keys within radius w of the query):
  // sum over q of min(q + w, n - 1) - max(q - w, 0) + 1, in closed form
  const double w = (double)cfg.sliding_window;
  const double m = n - w > 0.0 ? n - w : 0.0, t = n - 1.0 - w > 0.0 ? n - 1.0 - w : 0.0;
  const double sliding_pairs = m * (w + 1.0) + m * (m - 1.0) / 2.0 + (n - m) * n - t * (t + 1.0) / 2.0;
  double lin = H * (double)layers.size() * P + H * E;  // PLE projection, output projection (per token)
  double att = 0.0;
  for (const LayerDev& ly : layers) {
    lin += H * ly.ld_qkv + (double)ly.qd * H + 2.0 * H * F + F * H + 2.0 * H * P;
    att += 4.0 * NH * ly.hd * (ly.full ? n * n : sliding_pairs);
  }
  return 2.0 * lin * n + 1.4 * att;
}

// text.rs:182-538 for a packed batch.  Batches of at least kSplitTokens run
// as two halves (split at the sequence boundary closest to the middle token)
// on two streams, so each half's kernels fill the other's last, partly empty
// wave of CTAs (a 512-wide projection of 19,339 rows is 152 tiles for 74 CTA
// pairs).  Hidden-state capture, soft tokens and the profiling pass keep one
// stream.
int Model::forward(const uint32_t* d_ids, const uint64_t* cu, uint32_t batch, const uint64_t* d_cu,
                   const FeatureRows* features, uint32_t dim, float* d_out, float* d_pooled, float* d_normalized,
                   float* d_projected, float* d_hidden, cudaStream_t st, std::string* msg) {
  constexpr uint64_t kSplitTokens = 8192;
  const uint64_t T = cu[batch];
  uint32_t k = 0;
  if (!prof.enabled && !features && !d_hidden && batch >= 2 && T >= kSplitTokens && stream2) {
    // split at the sequence boundary that best balances the two halves' work:
    // the streams join at the end, and while one runs alone its one-CTA-per-SM
    // row-fused kernels leave half the GPU idle
    std::vector<double> pre(batch + 1, 0.0);
    for (uint32_t i = 0; i < batch; ++i) pre[i + 1] = pre[i] + sequence_cost(cu[i + 1] - cu[i]);
    double best = -1.0;
    for (uint32_t i = 1; i < batch; ++i) {
      const double d = std::fabs(2.0 * pre[i] - pre[batch]);
      if (best < 0.0 || d < best) {
        best = d;
        k = i;
      }
    }
  }
  // one upload: [group-1 offsets (as 32-bit word pairs)][group 0 schedules][group 1 schedules]
  std::vector<uint64_t> cu1;
  if (k) {
    cu1.resize(batch - k + 1);
    for (uint32_t i = 0; i <= batch - k; ++i) cu1[i] = cu[k + i] - cu[k];
  }
  std::vector<uint32_t> words(cu1.size() * 2);
  if (!cu1.empty()) std::memcpy(words.data(), cu1.data(), cu1.size() * 8);
  words.resize((words.size() + 3) / 4 * 4, 0u);
  std::vector<AttnSched> s0, s1;  // word offsets are into the whole upload
  int rc = attention_schedules(cu, k ? k : batch, &s0, &words, msg);
  if (rc == SVL_OK && k) rc = attention_schedules(cu1.data(), batch - k, &s1, &words, msg);
  if (rc != SVL_OK) return rc;
  uint32_t* d_words = nullptr;
  if (!words.empty()) {
    d_words = (uint32_t*)workspace("forward_words", words.size() * 4);
    if (!d_words || !upload_pinned(words.data(), words.size() * 4, d_words, st)) {
      *msg = "schedule upload failed";
      return SVL_INTERNAL;
    }
  }
  if (!k)
    return forward_part("", d_ids, cu, batch, d_cu, features, dim, d_out, d_pooled, d_normalized, d_projected,
                        d_hidden, s0, d_words, st, msg);
  const uint32_t E = (uint32_t)cfg.embedding_dim;
  if (cudaEventRecord(fork_ev, st) != cudaSuccess || cudaStreamWaitEvent(stream2, fork_ev, 0) != cudaSuccess) {
    *msg = "stream fork failed";
    return SVL_INTERNAL;
  }
  rc = forward_part("", d_ids, cu, k, d_cu, nullptr, dim, d_out, d_pooled, d_normalized, d_projected, nullptr, s0,
                    d_words, st, msg);
  int rc1 = forward_part("#1", d_ids + cu[k], cu1.data(), batch - k, (const uint64_t*)d_words, nullptr, dim,
                         d_out ? d_out + (size_t)k * dim : nullptr, d_pooled ? d_pooled + (size_t)k * E : nullptr,
                         d_normalized ? d_normalized + (size_t)k * E : nullptr,
                         d_projected ? d_projected + cu[k] * E : nullptr, nullptr, s1, d_words, stream2, msg);
  // join even after a failed launch, so the caller's stream orders after both halves
  cudaEventRecord(join_ev, stream2);
  cudaStreamWaitEvent(st, join_ev, 0);
  return rc != SVL_OK ? rc : rc1;
}

}  // namespace svl
