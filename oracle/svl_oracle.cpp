// svl_oracle.cpp -- CPU restatement of the reference's scalar FP32 text encoder
// and exact f64 vector rank.
//
// TEST INFRASTRUCTURE ONLY: the parity checker for libsvl_gpu.so and the timed
// CPU baseline.  Never linked into the product library.  Parity is pinned by
// tests/test_oracle_golden.py against the reference's own tiny_text golden
// fixture (fixtures/model/tiny_text/golden.json) and its kernel known-answer
// tests (src/tensor/kernels.rs:1150-1580, src/index/vector.rs:139-205).
//
// Build: oracle/Makefile (g++ -O3 -ffp-contract=off).  Contraction must stay
// off: Rust evaluates `sum += a * b` as a rounded multiply then a rounded add.
//
// Vectorisation note: orc_linear computes OUT_BLOCK output columns side by
// side.  Each column's sum is still the reference's sequential
// `sum += input[k] * weight[c][k]` for k = 0..in_features, so the result is
// bit-identical to kernels.rs:666-677; only independent columns share SIMD
// lanes.

#include "svl_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <thread>
#include <vector>

namespace {

constexpr size_t kMaxTensorElements = size_t(1) << 30;   // src/tensor/owned.rs:16-23
constexpr size_t kMaxActivationElements = size_t(1) << 28; // src/model/text.rs:34
constexpr size_t kMaxTextTokens = 8192;                    // src/model/config.rs:27
constexpr size_t kMaxEmbeddingDimension = 8192;            // src/storage/model.rs:35

void set_err(char* err, size_t len, const std::string& msg) {
  if (err && len) {
    size_t n = std::min(len - 1, msg.size());
    std::memcpy(err, msg.data(), n);
    err[n] = 0;
  }
}

bool all_finite(const float* v, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (!std::isfinite(v[i])) return false;
  return true;
}

}  // namespace

extern "C" {

// kernels.rs:655-685 linear_into_scalar: out[r,c] = sum_k in[r,k] * W[c,k],
// sequential f32 sum over k, then a non-finite check.
int orc_linear(const float* input, const float* weight, size_t rows, size_t in_features,
               size_t out_features, float* output) {
  if (rows * out_features > kMaxTensorElements) return SVL_LIMIT_EXCEEDED;
  constexpr size_t OUT_BLOCK = 16;
  for (size_t r = 0; r < rows; ++r) {
    const float* in_row = input + r * in_features;
    float* out_row = output + r * out_features;
    size_t c = 0;
    for (; c + OUT_BLOCK <= out_features; c += OUT_BLOCK) {
      float sum[OUT_BLOCK];
      for (size_t j = 0; j < OUT_BLOCK; ++j) sum[j] = 0.0f;
      const float* w0 = weight + c * in_features;
      for (size_t k = 0; k < in_features; ++k) {
        const float x = in_row[k];
        for (size_t j = 0; j < OUT_BLOCK; ++j) sum[j] += x * w0[j * in_features + k];
      }
      for (size_t j = 0; j < OUT_BLOCK; ++j) out_row[c + j] = sum[j];
    }
    for (; c < out_features; ++c) {
      const float* w = weight + c * in_features;
      float sum = 0.0f;
      for (size_t k = 0; k < in_features; ++k) sum += in_row[k] * w[k];
      out_row[c] = sum;
    }
  }
  if (!all_finite(output, rows * out_features)) return SVL_INTERNAL;
  return SVL_OK;
}

// A linear weight [out, in] re-laid as column blocks of 16: block b holds
// W[16b + j][k] at packed[(b * in + k) * 16 + j].  The packed product below
// computes every output column with the same sequential sum over k as
// kernels.rs:666-677, four input rows at a time; only the memory layout
// differs, so results are bit-identical to orc_linear.
struct PackedLinear {
  size_t in = 0, out = 0;
  std::vector<float> blocks;  // ceil(out / 16) * in * 16
};

static void pack_linear(const float* w, size_t out, size_t in, PackedLinear* p) {
  p->in = in;
  p->out = out;
  const size_t nb = (out + 15) / 16;
  p->blocks.assign(nb * in * 16, 0.0f);
  for (size_t c = 0; c < out; ++c)
    for (size_t k = 0; k < in; ++k) p->blocks[((c / 16) * in + k) * 16 + (c % 16)] = w[c * in + k];
}

typedef float v8f __attribute__((vector_size(32)));

static int linear_packed(const float* input, const PackedLinear& p, size_t rows, float* output) {
  const size_t in = p.in, out = p.out, nb = (out + 15) / 16;
  size_t r = 0;
  for (; r + 4 <= rows; r += 4) {
    const float* x0 = input + r * in;
    for (size_t b = 0; b < nb; ++b) {
      // lane j of acc[i][h] is output column 16b + 8h + j of row r + i; each
      // lane performs the rounded multiply then the rounded add, in k order
      v8f acc[4][2];
      for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = v8f{};
      const float* wb = p.blocks.data() + b * in * 16;
      for (size_t k = 0; k < in; ++k) {
        v8f w0, w1;
        std::memcpy(&w0, wb + k * 16, 32);
        std::memcpy(&w1, wb + k * 16 + 8, 32);
        for (int i = 0; i < 4; ++i) {
          const float x = x0[i * in + k];
          const v8f xv = {x, x, x, x, x, x, x, x};
          acc[i][0] += xv * w0;
          acc[i][1] += xv * w1;
        }
      }
      const size_t ncol = std::min<size_t>(16, out - b * 16);
      for (int i = 0; i < 4; ++i)
        for (size_t j = 0; j < ncol; ++j) output[(r + i) * out + b * 16 + j] = acc[i][j / 8][j % 8];
    }
  }
  for (; r < rows; ++r) {
    const float* x = input + r * in;
    for (size_t b = 0; b < nb; ++b) {
      float acc[16];
      for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
      const float* wb = p.blocks.data() + b * in * 16;
      for (size_t k = 0; k < in; ++k)
        for (int j = 0; j < 16; ++j) acc[j] += x[k] * wb[k * 16 + j];
      const size_t ncol = std::min<size_t>(16, out - b * 16);
      for (size_t j = 0; j < ncol; ++j) output[r * out + b * 16 + j] = acc[j];
    }
  }
  if (!all_finite(output, rows * out)) return SVL_INTERNAL;
  return SVL_OK;
}

// kernels.rs:234-260 matmul_into_scalar: row-major A[m,k] * B[k,n], output
// accumulated in (row, inner, column) order.
int orc_matmul(const float* left, const float* right, size_t m, size_t k, size_t n,
               float* output) {
  if (m * n > kMaxTensorElements) return SVL_LIMIT_EXCEEDED;
  std::fill(output, output + m * n, 0.0f);
  for (size_t row = 0; row < m; ++row) {
    float* out_row = output + row * n;
    for (size_t inner = 0; inner < k; ++inner) {
      const float lv = left[row * k + inner];
      const float* right_row = right + inner * n;
      for (size_t c = 0; c < n; ++c) out_row[c] += lv * right_row[c];
    }
  }
  if (!all_finite(output, m * n)) return SVL_INTERNAL;
  return SVL_OK;
}

// kernels.rs:743-776 (weighted) and 825-857 (unscaled): per row, sequential
// f32 sum of squares, inverse = 1 / sqrt(sum / width + eps), out = v * inv * w.
int orc_rms_norm_rows(const float* input, const float* weight, size_t rows, size_t width,
                      float epsilon, float* output) {
  if (width == 0) return SVL_INTERNAL;
  if (!std::isfinite(epsilon) || epsilon < 0.0f) return SVL_INTERNAL;
  if (rows * width > kMaxTensorElements) return SVL_LIMIT_EXCEEDED;
  for (size_t r = 0; r < rows; ++r) {
    const float* in_row = input + r * width;
    float* out_row = output + r * width;
    float sum = 0.0f;
    for (size_t i = 0; i < width; ++i) {
      if (!std::isfinite(in_row[i])) return SVL_INTERNAL;
      sum += in_row[i] * in_row[i];
    }
    if (!std::isfinite(sum)) return SVL_INTERNAL;
    const float inverse = 1.0f / std::sqrt(sum / (float)width + epsilon);
    if (weight) {
      for (size_t i = 0; i < width; ++i) out_row[i] = in_row[i] * inverse * weight[i];
    } else {
      for (size_t i = 0; i < width; ++i) out_row[i] = in_row[i] * inverse;
    }
  }
  if (!all_finite(output, rows * width)) return SVL_INTERNAL;
  return SVL_OK;
}

// kernels.rs:380-383
float orc_gelu_tanh_value(float value) {
  const float cubic = value * value * value;
  return 0.5f * value * (1.0f + std::tanh(0.7978846f * (value + 0.044715f * cubic)));
}

// kernels.rs:391-400
int orc_geglu(const float* gate, const float* up, size_t n, float* output) {
  if (n > kMaxTensorElements) return SVL_LIMIT_EXCEEDED;
  for (size_t i = 0; i < n; ++i) output[i] = orc_gelu_tanh_value(gate[i]) * up[i];
  return SVL_OK;
}

// kernels.rs:267-321
int orc_softmax(const float* values, size_t n, float* output) {
  if (n == 0) return SVL_INTERNAL;
  float maximum = -INFINITY;
  for (size_t i = 0; i < n; ++i) {
    if (std::isnan(values[i])) return SVL_INTERNAL;
    if (values[i] > maximum) maximum = values[i];
  }
  if (maximum == -INFINITY) return SVL_INTERNAL;
  if (maximum == INFINITY) {
    size_t count = 0;
    for (size_t i = 0; i < n; ++i) count += values[i] == INFINITY;
    const float p = 1.0f / (float)count;
    for (size_t i = 0; i < n; ++i) output[i] = values[i] == INFINITY ? p : 0.0f;
    return SVL_OK;
  }
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    const float e = std::exp(values[i] - maximum);
    sum += e;
    output[i] = e;
  }
  if (sum == 0.0f || !std::isfinite(sum)) return SVL_INTERNAL;
  for (size_t i = 0; i < n; ++i) output[i] /= sum;
  return SVL_OK;
}

// kernels.rs:424-444
int orc_l2_normalize(const float* input, size_t n, float* output) {
  if (n == 0) return SVL_INTERNAL;
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    if (!std::isfinite(input[i])) return SVL_INTERNAL;
    sum += input[i] * input[i];
  }
  if (!std::isfinite(sum) || sum <= 0.0f) return SVL_INTERNAL;
  const float inverse = 1.0f / std::sqrt(sum);
  for (size_t i = 0; i < n; ++i) output[i] = input[i] * inverse;
  return SVL_OK;
}

// kernels.rs:892-909
int orc_mean_pool(const float* values, size_t rows, size_t width, float* output) {
  if (rows == 0) return SVL_INTERNAL;
  std::fill(output, output + width, 0.0f);
  for (size_t r = 0; r < rows; ++r)
    for (size_t c = 0; c < width; ++c) output[c] += values[r * width + c];
  const float inverse = 1.0f / (float)rows;
  for (size_t c = 0; c < width; ++c) {
    output[c] *= inverse;
    if (!std::isfinite(output[c])) return SVL_INTERNAL;
  }
  return SVL_OK;
}

// kernels.rs:916-927
int orc_truncate_and_normalize(const float* values, size_t n, size_t dimension, float* output) {
  if (dimension == 0 || dimension > n) return SVL_INTERNAL;
  return orc_l2_normalize(values, dimension, output);
}

// kernels.rs:991-1010: inv[p] = 1 / base.powf(2p / head_dim), all in f32.
int orc_rope_inv_freq(size_t head_dim, float base, float* output) {
  if (head_dim == 0 || head_dim % 2) return SVL_INTERNAL;
  if (!std::isfinite(base) || base <= 1.0f) return SVL_INTERNAL;
  for (size_t p = 0; p < head_dim / 2; ++p) {
    const float exponent = (float)(2 * p) / (float)head_dim;
    output[p] = 1.0f / std::pow(base, exponent);
  }
  return SVL_OK;
}

// kernels.rs:936-988: angle = (position as f32) * inv[p]; rotate-half pairs
// (p, p + half).  sin_cos in Rust is (sin, cos) of the same f32 angle.
int orc_rope_with_inv_freq(float* values, size_t seq_len, size_t num_heads, size_t head_dim,
                           const float* inv_freq, size_t inv_len, size_t position_offset) {
  if (head_dim == 0 || head_dim % 2) return SVL_INTERNAL;
  if (inv_len != head_dim / 2) return SVL_INTERNAL;
  const size_t half = head_dim / 2;
  for (size_t pos = 0; pos < seq_len; ++pos) {
    const size_t absolute = position_offset + pos;
    for (size_t h = 0; h < num_heads; ++h) {
      float* v = values + (pos * num_heads + h) * head_dim;
      for (size_t p = 0; p < half; ++p) {
        const float angle = (float)absolute * inv_freq[p];
        const float s = std::sin(angle);
        const float c = std::cos(angle);
        const float first = v[p];
        const float second = v[p + half];
        v[p] = first * c - second * s;
        v[p + half] = first * s + second * c;
      }
    }
  }
  if (!all_finite(values, seq_len * num_heads * head_dim)) return SVL_INTERNAL;
  return SVL_OK;
}

// kernels.rs:1037-1135
int orc_bidirectional_attention(const float* query, const float* key, const float* value,
                                size_t seq_len, size_t num_heads, size_t num_kv_heads,
                                size_t head_dim, int64_t sliding_window, float scale,
                                float* output) {
  if (head_dim == 0 || num_heads == 0 || num_kv_heads == 0) return SVL_INTERNAL;
  if (num_heads % num_kv_heads) return SVL_INTERNAL;
  if (!std::isfinite(scale)) return SVL_INTERNAL;
  const size_t groups = num_heads / num_kv_heads;
  std::fill(output, output + seq_len * num_heads * head_dim, 0.0f);
  std::vector<float> scores(seq_len), probs(seq_len);
  for (size_t pos = 0; pos < seq_len; ++pos) {
    size_t start = 0, end = seq_len - 1;
    if (sliding_window >= 0) {
      const size_t w = (size_t)sliding_window;
      start = pos >= w ? pos - w : 0;
      end = std::min(pos + w, seq_len - 1);
    }
    const size_t width = end - start + 1;
    for (size_t h = 0; h < num_heads; ++h) {
      const size_t kv = h / groups;
      const float* q = query + (pos * num_heads + h) * head_dim;
      for (size_t col = 0; col < width; ++col) {
        const float* k = key + ((start + col) * num_kv_heads + kv) * head_dim;
        float dot = 0.0f;
        for (size_t i = 0; i < head_dim; ++i) dot += q[i] * k[i];
        const float score = dot * scale;
        if (!std::isfinite(score)) return SVL_INTERNAL;
        scores[col] = score;
      }
      int st = orc_softmax(scores.data(), width, probs.data());
      if (st) return st;
      float* out = output + (pos * num_heads + h) * head_dim;
      for (size_t col = 0; col < width; ++col) {
        const float p = probs[col];
        if (p == 0.0f) continue;
        const float* v = value + ((start + col) * num_kv_heads + kv) * head_dim;
        for (size_t i = 0; i < head_dim; ++i) out[i] += p * v[i];
      }
    }
  }
  if (!all_finite(output, seq_len * num_heads * head_dim)) return SVL_INTERNAL;
  return SVL_OK;
}

}  // extern "C"

// ----------------------------------------------------------------- model --

struct OrcLayer {
  const float *input_layernorm, *post_attention_layernorm, *pre_feedforward_layernorm,
      *post_feedforward_layernorm;
  float layer_scalar;
  const float *gate_proj, *up_proj, *down_proj, *per_layer_input_gate, *per_layer_projection,
      *post_per_layer_input_norm, *q_proj, *k_proj, *v_proj, *o_proj, *q_norm, *k_norm;
  PackedLinear pq, pk, pv, po, pgate, pup, pdown, ppg, ppp;
};

struct orc_model {
  svl_text_config cfg;
  std::vector<svl_layer_config> layer_cfg;
  std::map<std::string, std::vector<float>> owned;  // FP32 copies (BF16 widened)
  const float *embed_tokens, *embedding_projection, *norm, *ple_projection, *ple_norm;
  std::vector<OrcLayer> layers;
  std::vector<float> full_inv, sliding_inv;
  PackedLinear p_ple, p_emb;
};

namespace {

float bf16_to_f32(uint16_t b) {  // src/binary/bf16.rs:40: bits << 16
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

}  // namespace

extern "C" int orc_model_create(const svl_text_config* config, const svl_tensor_view* tensors,
                                size_t n_tensors, orc_model** out, char* err, size_t err_len) {
  auto m = new orc_model();
  m->cfg = *config;
  m->layer_cfg.assign(config->layers, config->layers + config->num_hidden_layers);
  m->cfg.layers = m->layer_cfg.data();
  std::map<std::string, const svl_tensor_view*> by_name;
  for (size_t i = 0; i < n_tensors; ++i) by_name[tensors[i].name] = &tensors[i];
  auto get = [&](const std::string& name, size_t expected) -> const float* {
    auto it = by_name.find(name);
    if (it == by_name.end()) return nullptr;
    const svl_tensor_view* t = it->second;
    size_t numel = 1;
    for (uint32_t d = 0; d < t->ndim; ++d) numel *= t->shape[d];
    if (numel != expected) return nullptr;
    std::vector<float>& dst = m->owned[name];
    dst.resize(numel);
    if (t->dtype == SVL_DTYPE_BF16) {
      const uint16_t* src = (const uint16_t*)t->data;
      for (size_t i = 0; i < numel; ++i) dst[i] = bf16_to_f32(src[i]);
    } else {
      std::memcpy(dst.data(), t->data, numel * 4);
    }
    return dst.data();
  };
  const size_t H = config->hidden_size, P = config->hidden_size_per_layer_input,
               F = config->intermediate_size, L = config->num_hidden_layers,
               NH = config->num_attention_heads;
  bool ok = true;
  auto need = [&](const float* p, const std::string& name) {
    if (!p) {
      ok = false;
      set_err(err, err_len, "text weight " + name + " is missing or has the wrong shape");
    }
    return p;
  };
  m->embed_tokens = need(get("language_model.embed_tokens.weight", (size_t)config->vocab_size * H),
                         "language_model.embed_tokens.weight");
  m->embedding_projection =
      need(get("language_model.embedding_projection.weight", config->embedding_dim * H),
           "embedding_projection");
  m->norm = need(get("language_model.norm.weight", H), "norm");
  m->ple_projection =
      need(get("language_model.ple.per_layer_model_projection.weight", L * P * H), "ple proj");
  m->ple_norm = need(get("language_model.ple.per_layer_projection_norm.weight", P), "ple norm");
  for (size_t l = 0; ok && l < L; ++l) {
    const std::string pre = "language_model.layers." + std::to_string(l) + ".";
    const size_t hd = config->layers[l].head_dim, kvh = config->layers[l].num_key_value_heads;
    OrcLayer ly;
    ly.input_layernorm = need(get(pre + "input_layernorm.weight", H), pre + "input_layernorm");
    ly.post_attention_layernorm = need(get(pre + "post_attention_layernorm.weight", H), pre);
    ly.pre_feedforward_layernorm = need(get(pre + "pre_feedforward_layernorm.weight", H), pre);
    ly.post_feedforward_layernorm = need(get(pre + "post_feedforward_layernorm.weight", H), pre);
    const float* scalar = need(get(pre + "layer_scalar", 1), pre + "layer_scalar");
    ly.layer_scalar = scalar ? scalar[0] : 0.0f;
    ly.gate_proj = need(get(pre + "mlp.gate_proj.weight", F * H), pre);
    ly.up_proj = need(get(pre + "mlp.up_proj.weight", F * H), pre);
    ly.down_proj = need(get(pre + "mlp.down_proj.weight", H * F), pre);
    ly.per_layer_input_gate = need(get(pre + "ple_block.per_layer_input_gate.weight", P * H), pre);
    ly.per_layer_projection = need(get(pre + "ple_block.per_layer_projection.weight", H * P), pre);
    ly.post_per_layer_input_norm =
        need(get(pre + "ple_block.post_per_layer_input_norm.weight", H), pre);
    ly.q_proj = need(get(pre + "self_attn.q_proj.weight", NH * hd * H), pre + "q_proj");
    ly.k_proj = need(get(pre + "self_attn.k_proj.weight", kvh * hd * H), pre + "k_proj");
    ly.v_proj = need(get(pre + "self_attn.v_proj.weight", kvh * hd * H), pre + "v_proj");
    ly.o_proj = need(get(pre + "self_attn.o_proj.weight", H * NH * hd), pre + "o_proj");
    ly.q_norm = need(get(pre + "self_attn.q_norm.weight", hd), pre);
    ly.k_norm = need(get(pre + "self_attn.k_norm.weight", hd), pre);
    if (ok) {
      pack_linear(ly.q_proj, NH * hd, H, &ly.pq);
      pack_linear(ly.k_proj, kvh * hd, H, &ly.pk);
      pack_linear(ly.v_proj, kvh * hd, H, &ly.pv);
      pack_linear(ly.o_proj, H, NH * hd, &ly.po);
      pack_linear(ly.gate_proj, F, H, &ly.pgate);
      pack_linear(ly.up_proj, F, H, &ly.pup);
      pack_linear(ly.down_proj, H, F, &ly.pdown);
      pack_linear(ly.per_layer_input_gate, P, H, &ly.ppg);
      pack_linear(ly.per_layer_projection, H, P, &ly.ppp);
    }
    m->layers.push_back(std::move(ly));
  }
  if (ok) {
    pack_linear(m->ple_projection, L * P, H, &m->p_ple);
    pack_linear(m->embedding_projection, config->embedding_dim, H, &m->p_emb);
  }
  if (!ok) {
    delete m;
    return SVL_CORRUPT;
  }
  // config.rs:366-373: inverse frequencies per layer type from its head_dim.
  size_t full_hd = 0, sliding_hd = 0;
  for (size_t l = 0; l < L; ++l) {
    if (config->layers[l].layer_type == SVL_LAYER_FULL && !full_hd) full_hd = config->layers[l].head_dim;
    if (config->layers[l].layer_type == SVL_LAYER_SLIDING && !sliding_hd)
      sliding_hd = config->layers[l].head_dim;
  }
  if (full_hd) {
    m->full_inv.resize(full_hd / 2);
    orc_rope_inv_freq(full_hd, config->full_rope_theta, m->full_inv.data());
  }
  if (sliding_hd) {
    m->sliding_inv.resize(sliding_hd / 2);
    orc_rope_inv_freq(sliding_hd, config->sliding_rope_theta, m->sliding_inv.data());
  }
  *out = m;
  return SVL_OK;
}

extern "C" void orc_model_destroy(orc_model* model) { delete model; }

// text.rs:182-538, operation by operation.
extern "C" int orc_forward(const orc_model* m, const uint32_t* ids, size_t seq,
                           const float* features, size_t feature_start, size_t feature_count,
                           float* projected_out, float* pooled_out, float* normalized_out,
                           float* hidden_states, char* err, size_t err_len) {
  const svl_text_config& c = m->cfg;
  if (seq == 0) {
    set_err(err, err_len, "cannot embed an empty token sequence");
    return SVL_CORRUPT;
  }
  if (seq > kMaxTextTokens || seq > c.max_position_embeddings) {
    set_err(err, err_len, "sequence above the context");
    return SVL_LIMIT_EXCEEDED;
  }
  const size_t H = c.hidden_size, P = c.hidden_size_per_layer_input, L = c.num_hidden_layers,
               E = c.embedding_dim, F = c.intermediate_size, NH = c.num_attention_heads;
  const float eps = c.rms_norm_eps;
  if (seq * F > kMaxActivationElements || seq * L * P > kMaxActivationElements) {
    set_err(err, err_len, "activation cap");
    return SVL_LIMIT_EXCEEDED;
  }
  std::vector<float> hidden(seq * H);
  for (size_t r = 0; r < seq; ++r) {
    if (ids[r] >= c.vocab_size) {
      set_err(err, err_len, "token id " + std::to_string(ids[r]) + " is outside the vocabulary");
      return SVL_CORRUPT;
    }
    const float* src = m->embed_tokens + (size_t)ids[r] * H;
    for (size_t i = 0; i < H; ++i) hidden[r * H + i] = src[i] * c.embedding_scale;
  }
  if (features) {  // text.rs:226-275
    if (feature_count == 0 || feature_start + feature_count > seq) return SVL_CORRUPT;
    if (c.pad_token_id < 0) return SVL_UNSUPPORTED;
    const float* pad = m->embed_tokens + (size_t)c.pad_token_id * H;
    for (size_t r = feature_start; r < feature_start + feature_count; ++r)
      for (size_t i = 0; i < H; ++i) hidden[r * H + i] = pad[i] * c.embedding_scale;
    for (size_t o = 0; o < feature_count; ++o)
      std::memcpy(&hidden[(feature_start + o) * H], features + o * H, H * 4);
    if (!all_finite(hidden.data(), hidden.size())) return SVL_INTERNAL;
  }
  size_t captured = 0;
  auto capture = [&]() {
    if (hidden_states) std::memcpy(hidden_states + captured * seq * H, hidden.data(), seq * H * 4);
    ++captured;
  };
  capture();

  int st;
#define ORC_TRY(expr)                                           \
  do {                                                          \
    st = (expr);                                                \
    if (st) {                                                   \
      set_err(err, err_len, "oracle step failed: " #expr);      \
      return st;                                                \
    }                                                           \
  } while (0)

  // PLE (text.rs:282-306)
  std::vector<float> per_layer(seq * L * P);
  ORC_TRY(linear_packed(hidden.data(), m->p_ple, seq, per_layer.data()));
  for (auto& v : per_layer) v *= c.ple_scale;
  ORC_TRY(orc_rms_norm_rows(per_layer.data(), m->ple_norm, seq * L, P, eps, per_layer.data()));

  std::vector<float> residual, normalized(seq * H), tmp(seq * H);
  for (size_t l = 0; l < L; ++l) {
    const OrcLayer& ly = m->layers[l];
    const size_t hd = c.layers[l].head_dim, kvh = c.layers[l].num_key_value_heads;
    const bool full = c.layers[l].layer_type == SVL_LAYER_FULL;
    const size_t qd = NH * hd, kvd = kvh * hd;
    // attention block (text.rs:345-433)
    residual = hidden;
    ORC_TRY(orc_rms_norm_rows(hidden.data(), ly.input_layernorm, seq, H, eps, normalized.data()));
    std::vector<float> q(seq * qd), k(seq * kvd), v(seq * kvd), attn(seq * qd);
    ORC_TRY(linear_packed(normalized.data(), ly.pq, seq, q.data()));
    ORC_TRY(linear_packed(normalized.data(), ly.pk, seq, k.data()));
    ORC_TRY(linear_packed(normalized.data(), ly.pv, seq, v.data()));
    ORC_TRY(orc_rms_norm_rows(q.data(), ly.q_norm, seq * NH, hd, eps, q.data()));
    ORC_TRY(orc_rms_norm_rows(k.data(), ly.k_norm, seq * kvh, hd, eps, k.data()));
    ORC_TRY(orc_rms_norm_rows(v.data(), nullptr, seq * kvh, hd, eps, v.data()));
    const std::vector<float>& inv = full ? m->full_inv : m->sliding_inv;
    ORC_TRY(orc_rope_with_inv_freq(q.data(), seq, NH, hd, inv.data(), inv.size(), 0));
    ORC_TRY(orc_rope_with_inv_freq(k.data(), seq, kvh, hd, inv.data(), inv.size(), 0));
    ORC_TRY(orc_bidirectional_attention(q.data(), k.data(), v.data(), seq, NH, kvh, hd,
                                        full ? -1 : (int64_t)c.sliding_window, 1.0f,
                                        attn.data()));
    ORC_TRY(linear_packed(attn.data(), ly.po, seq, tmp.data()));
    ORC_TRY(orc_rms_norm_rows(tmp.data(), ly.post_attention_layernorm, seq, H, eps, tmp.data()));
    for (size_t i = 0; i < seq * H; ++i) hidden[i] = residual[i] + tmp[i];
    // feed-forward block (text.rs:435-472)
    residual = hidden;
    ORC_TRY(orc_rms_norm_rows(hidden.data(), ly.pre_feedforward_layernorm, seq, H, eps,
                              normalized.data()));
    std::vector<float> gate(seq * F), up(seq * F);
    ORC_TRY(linear_packed(normalized.data(), ly.pgate, seq, gate.data()));
    ORC_TRY(linear_packed(normalized.data(), ly.pup, seq, up.data()));
    ORC_TRY(orc_geglu(gate.data(), up.data(), seq * F, gate.data()));
    ORC_TRY(linear_packed(gate.data(), ly.pdown, seq, tmp.data()));
    ORC_TRY(orc_rms_norm_rows(tmp.data(), ly.post_feedforward_layernorm, seq, H, eps, tmp.data()));
    for (size_t i = 0; i < seq * H; ++i) hidden[i] = residual[i] + tmp[i];
    // per-layer-input block (text.rs:474-513)
    residual = hidden;
    std::vector<float> pg(seq * P), gated(seq * P);
    ORC_TRY(linear_packed(hidden.data(), ly.ppg, seq, pg.data()));
    for (size_t r = 0; r < seq; ++r)
      for (size_t i = 0; i < P; ++i)
        gated[r * P + i] = orc_gelu_tanh_value(pg[r * P + i]) * per_layer[r * L * P + l * P + i];
    ORC_TRY(linear_packed(gated.data(), ly.ppp, seq, tmp.data()));
    ORC_TRY(orc_rms_norm_rows(tmp.data(), ly.post_per_layer_input_norm, seq, H, eps, tmp.data()));
    for (size_t i = 0; i < seq * H; ++i) hidden[i] = residual[i] + tmp[i];
    for (auto& x : hidden) x *= ly.layer_scalar;
    capture();
  }
  // final (text.rs:520-531)
  ORC_TRY(orc_rms_norm_rows(hidden.data(), m->norm, seq, H, eps, hidden.data()));
  std::vector<float> projected(seq * E), pooled(E), norm(E);
  ORC_TRY(linear_packed(hidden.data(), m->p_emb, seq, projected.data()));
  ORC_TRY(orc_mean_pool(projected.data(), seq, E, pooled.data()));
  ORC_TRY(orc_l2_normalize(pooled.data(), E, norm.data()));
#undef ORC_TRY
  if (projected_out) std::memcpy(projected_out, projected.data(), seq * E * 4);
  if (pooled_out) std::memcpy(pooled_out, pooled.data(), E * 4);
  if (normalized_out) std::memcpy(normalized_out, norm.data(), E * 4);
  return SVL_OK;
}

extern "C" int orc_embed_many(const orc_model* m, const uint32_t* ids, const uint64_t* cu,
                              size_t batch, size_t dimension, float* out, int n_threads) {
  const size_t E = m->cfg.embedding_dim;
  if (dimension == 0 || dimension > E) return SVL_INTERNAL;
  if (n_threads < 1) n_threads = 1;
  std::vector<int> status(batch, 0);
  auto work = [&](int t) {
    std::vector<float> normalized(E);
    for (size_t b = (size_t)t; b < batch; b += (size_t)n_threads) {
      int st = orc_forward(m, ids + cu[b], cu[b + 1] - cu[b], nullptr, 0, 0, nullptr, nullptr,
                           normalized.data(), nullptr, nullptr, 0);
      if (!st) st = orc_truncate_and_normalize(normalized.data(), E, dimension, out + b * dimension);
      status[b] = st;
    }
  };
  std::vector<std::thread> pool;
  for (int t = 0; t < n_threads; ++t) pool.emplace_back(work, t);
  for (auto& th : pool) th.join();
  for (int s : status)
    if (s) return s;
  return SVL_OK;
}

// ---------------------------------------------------------------- search --

// storage/model.rs:546-581: f64 sum of squares, value = (v / norm) as f32.
extern "C" int orc_normalize_embedding(float* values, size_t n) {
  if (n == 0) return SVL_USAGE;
  if (n > kMaxEmbeddingDimension) return SVL_LIMIT_EXCEEDED;
  double sum = 0.0;
  for (size_t i = 0; i < n; ++i) {
    if (!std::isfinite(values[i])) return SVL_USAGE;
    sum += (double)values[i] * (double)values[i];
  }
  if (!std::isfinite(sum) || sum <= 0.0) return SVL_USAGE;
  const double norm = std::sqrt(sum);
  for (size_t i = 0; i < n; ++i) {
    const float x = (float)((double)values[i] / norm);
    if (!std::isfinite(x)) return SVL_USAGE;
    values[i] = x;
  }
  return SVL_OK;
}

namespace {

int validate_query(const float* query, size_t dim, double* norm_out) {  // vector.rs:23-46
  if (dim == 0) return SVL_USAGE;
  if (dim > kMaxEmbeddingDimension) return SVL_LIMIT_EXCEEDED;
  double sum = 0.0;
  for (size_t i = 0; i < dim; ++i) {
    if (!std::isfinite(query[i])) return SVL_USAGE;
    sum += (double)query[i] * (double)query[i];
  }
  if (!std::isfinite(sum) || sum <= 0.0) return SVL_USAGE;
  *norm_out = std::sqrt(sum);
  return SVL_OK;
}

// vector.rs:72-86 for one row.
int score_row(const float* query, double qnorm, const float* row, size_t dim, double* out) {
  double dot = 0.0, vsum = 0.0;
  for (size_t i = 0; i < dim; ++i) {
    const double q = query[i], v = row[i];
    dot += q * v;
    vsum += v * v;
  }
  if (!std::isfinite(vsum) || vsum <= 0.0) return SVL_INTERNAL;
  *out = dot / (qnorm * std::sqrt(vsum));
  return SVL_OK;
}

// vector.rs:90-95: score descending (f64::total_cmp), then chunk id ascending.
// total_cmp orders by the IEEE total order; scores here are finite, so the
// plain comparison agrees except for -0.0 < +0.0, which total_cmp separates.
bool total_gt(double a, double b) {
  int64_t ia, ib;
  std::memcpy(&ia, &a, 8);
  std::memcpy(&ib, &b, 8);
  ia ^= (int64_t)((uint64_t)(ia >> 63) >> 1);
  ib ^= (int64_t)((uint64_t)(ib >> 63) >> 1);
  return ia > ib;
}

}  // namespace

extern "C" int orc_vector_rank(const float* query, size_t dim, const float* corpus,
                               size_t n_rows, const uint64_t* chunk_ids, const uint8_t* row_mask,
                               uint64_t* out_rows, double* out_scores, size_t* out_count,
                               int n_threads) {
  double qnorm;
  int st = validate_query(query, dim, &qnorm);
  if (st) return st;
  std::vector<std::pair<double, uint64_t>> scored;
  scored.reserve(n_rows);
  for (size_t r = 0; r < n_rows; ++r) {
    if (row_mask && !row_mask[r]) continue;
    double s;
    st = score_row(query, qnorm, corpus + r * dim, dim, &s);
    if (st) return st;
    scored.emplace_back(s, (uint64_t)r);
  }
  (void)n_threads;
  std::sort(scored.begin(), scored.end(), [&](const auto& a, const auto& b) {
    if (total_gt(a.first, b.first)) return true;
    if (total_gt(b.first, a.first)) return false;
    return chunk_ids[a.second] < chunk_ids[b.second];
  });
  for (size_t i = 0; i < scored.size(); ++i) {
    out_rows[i] = scored[i].second;
    out_scores[i] = scored[i].first;
  }
  *out_count = scored.size();
  return SVL_OK;
}

// The first k entries of the full ranking, computed with a bounded selection
// so a 10M-row corpus does not need a 10M-entry sort per query.  Entries are
// identical to orc_vector_rank's first k (same scores, same total order).
extern "C" int orc_vector_topk(const float* queries, size_t n_queries, size_t dim,
                               const float* corpus, size_t n_rows, const uint64_t* chunk_ids,
                               size_t k, uint64_t* out_rows, double* out_scores, int n_threads) {
  if (n_threads < 1) n_threads = 1;
  std::vector<int> status(n_queries, 0);
  auto better = [&](const std::pair<double, uint64_t>& a, const std::pair<double, uint64_t>& b) {
    if (total_gt(a.first, b.first)) return true;
    if (total_gt(b.first, a.first)) return false;
    return chunk_ids[a.second] < chunk_ids[b.second];
  };
  auto work = [&](int t) {
    for (size_t qi = (size_t)t; qi < n_queries; qi += (size_t)n_threads) {
      const float* q = queries + qi * dim;
      double qnorm;
      int st = validate_query(q, dim, &qnorm);
      if (st) {
        status[qi] = st;
        continue;
      }
      std::vector<std::pair<double, uint64_t>> heap;  // min-heap by `better`
      heap.reserve(k + 1);
      for (size_t r = 0; r < n_rows && !st; ++r) {
        double s;
        st = score_row(q, qnorm, corpus + r * dim, dim, &s);
        if (st) break;
        std::pair<double, uint64_t> e(s, (uint64_t)r);
        if (heap.size() < k) {
          heap.push_back(e);
          std::push_heap(heap.begin(), heap.end(), better);
        } else if (k && better(e, heap.front())) {
          std::pop_heap(heap.begin(), heap.end(), better);
          heap.back() = e;
          std::push_heap(heap.begin(), heap.end(), better);
        }
      }
      status[qi] = st;
      std::sort(heap.begin(), heap.end(), better);
      for (size_t i = 0; i < k; ++i) {
        out_rows[qi * k + i] = i < heap.size() ? heap[i].second : ~(uint64_t)0;
        out_scores[qi * k + i] = i < heap.size() ? heap[i].first : -INFINITY;
      }
    }
  };
  std::vector<std::thread> pool;
  for (int t = 0; t < n_threads; ++t) pool.emplace_back(work, t);
  for (auto& th : pool) th.join();
  for (int s : status)
    if (s) return s;
  return SVL_OK;
}
