/*
 * svl_oracle.h -- CPU restatement of Seldon Vault Lite's scalar FP32 text
 * encoder and exact f64 vector rank.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * sm_100a kernels in libsvl_gpu.so.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg load it; no product code path calls it.
 *
 * Every function follows the reference's scalar path operation by operation
 * (same loop nesting, same sequential f32 accumulation, same libm calls) so
 * that, built with -ffp-contract=off, its results equal the Rust reference on
 * x86-64 Linux up to glibc-vs-Rust-std libm differences (Rust std forwards
 * expf/tanhf/sinf/cosf/powf to the platform libm, so on glibc they coincide).
 *
 * Citations are to the reference crate (src/...:line).
 */
#ifndef SVL_ORACLE_H
#define SVL_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/svl_gpu.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Element kernels (src/tensor/kernels.rs). All return an svl_status. */
int orc_linear(const float* input, const float* weight, size_t rows, size_t in_features,
               size_t out_features, float* output);
int orc_matmul(const float* left, const float* right, size_t m, size_t k, size_t n, float* output);
int orc_rms_norm_rows(const float* input, const float* weight /* NULL = unscaled */, size_t rows,
                      size_t width, float epsilon, float* output);
float orc_gelu_tanh_value(float value);
int orc_geglu(const float* gate, const float* up, size_t n, float* output);
int orc_softmax(const float* values, size_t n, float* output);
int orc_l2_normalize(const float* input, size_t n, float* output);
int orc_mean_pool(const float* values, size_t rows, size_t width, float* output);
int orc_truncate_and_normalize(const float* values, size_t n, size_t dimension, float* output);
int orc_rope_inv_freq(size_t head_dim, float base, float* output);
int orc_rope_with_inv_freq(float* values, size_t seq_len, size_t num_heads, size_t head_dim,
                           const float* inv_freq, size_t inv_len, size_t position_offset);
int orc_bidirectional_attention(const float* query, const float* key, const float* value,
                                size_t seq_len, size_t num_heads, size_t num_kv_heads,
                                size_t head_dim, int64_t sliding_window /* <0 = full */,
                                float scale, float* output);

/* Whole encoder (src/model/text.rs:182-538). */
typedef struct orc_model orc_model;
int orc_model_create(const svl_text_config* config, const svl_tensor_view* tensors,
                     size_t n_tensors, orc_model** out, char* err, size_t err_len);
void orc_model_destroy(orc_model* model);
/* features may be NULL (plain forward).  hidden_states, when non-NULL, receives
 * (num_hidden_layers + 1) x seq x hidden floats; projected seq x embedding_dim;
 * pooled / normalized embedding_dim floats each. */
int orc_forward(const orc_model* model, const uint32_t* ids, size_t seq, const float* features,
                size_t feature_start, size_t feature_count, float* projected, float* pooled,
                float* normalized, float* hidden_states, char* err, size_t err_len);

/* Exact cosine rank (src/index/vector.rs:17-97) over a dense corpus.
 * row_mask (nullable) excludes rows whose byte is 0 (the Filters::matches
 * test).  Writes all surviving rows sorted by (score desc, chunk id asc);
 * *out_count receives their number. */
int orc_vector_rank(const float* query, size_t dim, const float* corpus, size_t n_rows,
                    const uint64_t* chunk_ids, const uint8_t* row_mask, uint64_t* out_rows,
                    double* out_scores, size_t* out_count, int n_threads);
/* Top-k of the same ranking for many queries (the first k entries of
 * orc_vector_rank per query), parallel over queries. */
int orc_vector_topk(const float* queries, size_t n_queries, size_t dim, const float* corpus,
                    size_t n_rows, const uint64_t* chunk_ids, size_t k, uint64_t* out_rows,
                    double* out_scores, int n_threads);
/* Chunk::new embedding normalisation (src/storage/model.rs:546-581), in place. */
int orc_normalize_embedding(float* values, size_t n);

/* CPU baseline: forward + embed of several sequences, one per thread. */
int orc_embed_many(const orc_model* model, const uint32_t* ids, const uint64_t* cu_seqlens,
                   size_t batch, size_t dimension, float* out, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
