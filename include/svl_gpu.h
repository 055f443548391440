/*
 * svl_gpu.h -- C ABI of the B200 (sm_100a) text-embedding and exact-search
 * library (libsvl_gpu.so).
 *
 * The library replaces the bodies of these reference (Seldon Vault Lite,
 * Rust) entry points; each declaration below names the one it stands behind:
 *
 *   TextModel::new / from_files        src/model/text.rs:104-126, weights.rs:125-241
 *   TextModel::forward                 src/model/text.rs:150
 *   TextModel::forward_with_features   src/model/text.rs:167
 *   TextModel::embed_ids               src/model/text.rs:546
 *   ForwardOutput::embedding           src/model/text.rs:72 (truncate_and_normalize)
 *   vector::rank                       src/index/vector.rs:17-97
 *   Index::search (vector mode)        src/index/mod.rs:325-388
 *   Chunk::new normalisation           src/storage/model.rs:325, 546-581
 *
 * Conventions (mirroring the reference):
 *   - every call returns an svl_status; the enumerators map one to one onto
 *     the reference's Error variants (src/error.rs:24-36).  A human-readable
 *     message is written to `err` (NUL-terminated, truncated to err_len) when
 *     err is non-NULL.  No call aborts the process.
 *   - inputs are borrowed; outputs are caller-owned buffers of the stated
 *     size; the library never retains caller pointers after returning.
 *   - plain pointers and sizes only: no C++ or PyTorch types cross the ABI.
 *   - an svl_model / svl_index is bound to one CUDA device.  Calls on one
 *     handle are serialised by an internal mutex, so a handle may be shared
 *     between threads (TextModel is Send + Sync in the reference).
 *   - *_device entry points take device pointers and an optional cudaStream_t
 *     (passed as void*; NULL = the handle's own stream) and return once the
 *     work is queued; the host-pointer entry points copy in, run and copy out
 *     synchronously.
 */
#ifndef SVL_GPU_H
#define SVL_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SVL_ABI_VERSION 1u

/* src/error.rs:24-36 */
typedef enum svl_status {
  SVL_OK = 0,
  SVL_USAGE = 1,           /* Error::Usage         */
  SVL_IO = 2,              /* Error::Io            */
  SVL_CORRUPT = 3,         /* Error::Corrupt       */
  SVL_LIMIT_EXCEEDED = 4,  /* Error::LimitExceeded */
  SVL_UNSUPPORTED = 5,     /* Error::Unsupported   */
  SVL_INTERNAL = 6         /* Error::Internal      */
} svl_status;

/* src/model/config.rs:55-70 */
typedef enum svl_layer_type { SVL_LAYER_SLIDING = 0, SVL_LAYER_FULL = 1 } svl_layer_type;

typedef struct svl_layer_config {
  uint32_t layer_type;           /* svl_layer_type */
  uint32_t head_dim;
  uint32_t num_key_value_heads;
} svl_layer_config;

/* Validated text configuration (TextConfig, src/model/config.rs:76-97).  The
 * host side parses config.json (config.rs:112-269) and fills this struct;
 * embedding_scale = sqrt(hidden_size) and ple_scale = 1 / embedding_scale are
 * the f32 values config.rs:241-242 computes. */
typedef struct svl_text_config {
  uint32_t vocab_size;
  uint32_t hidden_size;
  uint32_t intermediate_size;
  uint32_t num_hidden_layers;
  uint32_t num_attention_heads;
  uint32_t hidden_size_per_layer_input;
  uint32_t embedding_dim;
  uint32_t max_position_embeddings;
  uint32_t sliding_window;       /* inclusive two-sided radius */
  int64_t pad_token_id;          /* -1 when the config declares none */
  float rms_norm_eps;
  float embedding_scale;
  float ple_scale;
  float full_rope_theta;
  float sliding_rope_theta;
  const svl_layer_config* layers; /* num_hidden_layers entries */
} svl_text_config;

typedef enum svl_dtype { SVL_DTYPE_F32 = 0, SVL_DTYPE_BF16 = 1 } svl_dtype;

/* One named weight tensor in host memory (a Safetensors entry,
 * src/binary/safetensors.rs:69-123).  BF16 data is widened to FP32 exactly
 * (src/binary/bf16.rs:40) while it is uploaded. */
typedef struct svl_tensor_view {
  const char* name;              /* e.g. "language_model.layers.0.mlp.up_proj.weight" */
  const void* data;
  uint32_t dtype;                /* svl_dtype */
  uint32_t ndim;
  uint64_t shape[4];
} svl_tensor_view;

/* Soft-token override of a row range of one sequence
 * (TextModel::forward_with_features, src/model/text.rs:167, 226-275). */
typedef struct svl_feature_span {
  uint32_t sequence;             /* index into the batch */
  uint32_t start;                /* first row within the sequence */
  uint32_t count;                /* rows replaced (>= 1) */
  uint32_t reserved;
  uint64_t feature_offset;       /* first float of this span in `features` */
} svl_feature_span;

typedef struct svl_model svl_model;
typedef struct svl_index svl_index;

/* ---------------------------------------------------------------- model -- */

/* Library ABI version (SVL_ABI_VERSION). */
uint32_t svl_abi_version(void);

/* Number of visible CUDA devices, or a negative value on error. */
int svl_device_count(void);

/* TextModel::new (text.rs:117) over TextWeights::decode (weights.rs:125-189):
 * checks the tensor inventory against the configuration (missing, extra
 * "language_model." tensor, shape mismatch -> SVL_CORRUPT; non-finite weight
 * -> SVL_CORRUPT), uploads the weights to `device` in FP32 and builds the
 * fused device layouts.  Weights are copied; `tensors` may be freed after. */
int svl_model_create(const svl_text_config* config, const svl_tensor_view* tensors,
                     size_t n_tensors, int device, svl_model** out, char* err, size_t err_len);
void svl_model_destroy(svl_model* model);

/* Arithmetic of the encoder's tensor-core products (no counterpart in the
 * reference, whose scalar path is FP32 throughout):
 *   SVL_PRECISION_FAST  (default) every projection and attention product on
 *       11-bit-significand operands (FP16 with power-of-two scales, or TF32)
 *       accumulated in FP32: the fastest path.
 *   SVL_PRECISION_SPLIT each operand x is split into hi = TF32(x) and
 *       lo = TF32(x - hi) and every projection accumulates hi*hi + hi*lo +
 *       lo*hi in one TF32 product over three times the reduction width
 *       (~22-bit products); attention runs in FP32 on the CUDA cores.  For
 *       trained weights whose activations amplify rounding, at several times
 *       the cost of the default.
 * svl_model_create takes SVL_PRECISION_SPLIT when the environment variable
 * SVL_PRECISION is "split" at creation, else SVL_PRECISION_FAST. */
typedef enum svl_precision { SVL_PRECISION_FAST = 0, SVL_PRECISION_SPLIT = 1 } svl_precision;

typedef struct svl_model_options {
  uint32_t precision;            /* svl_precision */
  uint32_t reserved[7];          /* zero */
} svl_model_options;

/* svl_model_create with explicit options (NULL = defaults, environment
 * ignored).  An unknown precision or non-zero reserved word -> SVL_USAGE. */
int svl_model_create_ex(const svl_text_config* config, const svl_tensor_view* tensors,
                        size_t n_tensors, int device, const svl_model_options* options,
                        svl_model** out, char* err, size_t err_len);

/* The model's svl_precision. */
int svl_model_precision(const svl_model* model, uint32_t* out);

/* TextModel::parameters (text.rs:139). */
int svl_model_parameters(const svl_model* model, uint64_t* out);

/* TextModel::forward / forward_with_features over a packed batch of
 * sequences (text.rs:150, 167, 182-538).  Host pointers.
 *   ids        : cu_seqlens[batch] token ids, sequence b = ids[cu_seqlens[b] .. cu_seqlens[b+1])
 *   cu_seqlens : batch + 1 offsets, cu_seqlens[0] = 0
 *   features / spans : optional soft-token rows (n_spans may be 0)
 *   normalized : batch x embedding_dim   (ForwardOutput::normalized)
 *   pooled     : batch x embedding_dim or NULL (ForwardOutput::pooled)
 *   projected  : T x embedding_dim or NULL     (ForwardOutput::projected)
 *   hidden_states : (num_hidden_layers + 1) x T x hidden_size or NULL
 *               (ForwardOutput::hidden_states, capture_hidden = true)
 * Errors follow text.rs:188-218: empty sequence / id >= vocab -> SVL_CORRUPT,
 * sequence > 8192 or > max_position_embeddings -> SVL_LIMIT_EXCEEDED,
 * non-finite activation -> SVL_INTERNAL. */
int svl_forward_batch(svl_model* model, const uint32_t* ids, const uint64_t* cu_seqlens,
                      uint32_t batch, const float* features, const svl_feature_span* spans,
                      uint32_t n_spans, float* normalized, float* pooled, float* projected,
                      float* hidden_states, char* err, size_t err_len);

/* TextModel::embed_ids (text.rs:546-554) for a batch: forward, then
 * truncate_and_normalize to `dimension` (kernels.rs:916-927).  Host pointers;
 * out is batch x dimension.  dimension outside 1..=embedding_dim ->
 * SVL_INTERNAL before any work, as in the reference. */
int svl_embed_batch(svl_model* model, const uint32_t* ids, const uint64_t* cu_seqlens,
                    uint32_t batch, uint32_t dimension, float* out, char* err, size_t err_len);

/* Same as svl_embed_batch with ids and out in device memory of the model's
 * device (cu_seqlens stays on the host: it drives the tile schedule).  ids
 * are validated on the device; an out-of-vocabulary id is reported by the
 * next call to svl_model_check (SVL_CORRUPT) because this call does not
 * synchronise. */
int svl_embed_batch_device(svl_model* model, const uint32_t* d_ids, const uint64_t* cu_seqlens,
                           uint32_t batch, uint32_t dimension, float* d_out, void* stream,
                           char* err, size_t err_len);

/* Synchronises the model's stream and reports a deferred device-side error
 * (out-of-vocabulary id, non-finite activation) raised by *_device calls. */
int svl_model_check(svl_model* model, char* err, size_t err_len);

/* ---------------------------------------------------------------- index -- */

/* A device-resident, append-only store of unit-norm embedding rows with their
 * chunk ids (the in-memory Index view, src/index/mod.rs:271-308).
 * `capacity` rows of `dim` floats are reserved in HBM up front. */
int svl_index_create(int device, uint32_t dim, uint64_t capacity, svl_index** out, char* err,
                     size_t err_len);
void svl_index_destroy(svl_index* index);
uint64_t svl_index_len(const svl_index* index);
uint32_t svl_index_dim(const svl_index* index);

/* Appends n host rows; each row is L2-normalised in f64 exactly as
 * Chunk::new does (src/storage/model.rs:546-581: zero or non-finite norm ->
 * SVL_USAGE).  chunk_ids are the rows' ChunkId values (tie-break key). */
int svl_index_append(svl_index* index, const float* rows, const uint64_t* chunk_ids, uint64_t n,
                     char* err, size_t err_len);
/* Device-pointer variant (rows and chunk_ids in device memory). */
int svl_index_append_device(svl_index* index, const float* d_rows, const uint64_t* d_chunk_ids,
                            uint64_t n, void* stream, char* err, size_t err_len);

/* Document ingest into the device index (Store::put_document's chunk
 * embedding, src/storage/store.rs:524, then Chunk::new's normalisation and
 * the index append): embeds `batch` packed sequences (host ids and cu_seqlens
 * as for svl_embed_batch) at the index's dimension (Matryoshka truncation and
 * L2 normalisation, text.rs:546-554) and appends the embeddings with
 * `chunk_ids` (host, one per sequence) without copying them to the host.  The
 * model and the index must live on the same GPU and the index dimension must
 * be 1..=embedding_dim (else SVL_USAGE); a batch that does not fit the
 * index's remaining capacity is rejected before any work
 * (SVL_LIMIT_EXCEEDED).  Model errors (bad ids, non-finite activations) are
 * reported before anything is appended.  Synchronous, like svl_embed_batch. */
int svl_ingest_batch(svl_model* model, svl_index* index, const uint32_t* ids, const uint64_t* cu_seqlens,
                     uint32_t batch, const uint64_t* chunk_ids, char* err, size_t err_len);

/* Exact cosine top-k for a batch of queries: for each query the first k
 * entries of vector::rank (src/index/vector.rs:17-97), i.e. rows sorted by
 * f64 score = dot / (|q| |v|) descending, ties by ascending chunk id, and the
 * slice Index::search takes (offset + limit = k, src/index/mod.rs:349-359).
 *   queries   : n_queries x dim (host)
 *   row_mask  : NULL, or svl_index_len bytes; rows whose byte is 0 are
 *               filtered out (Filters::matches, src/index/mod.rs:63-72)
 *   out_rows / out_chunk_ids / out_scores : n_queries x k (entries past
 *               out_counts[q] are unspecified); out_chunk_ids may be NULL
 *   out_counts: n_queries, min(k, rows surviving the filter)
 * Query validation follows vector.rs:23-55 (empty, non-finite, zero norm,
 * dimension mismatch -> SVL_USAGE; dim > 8192 -> SVL_LIMIT_EXCEEDED). */
int svl_index_search(svl_index* index, const float* queries, uint32_t n_queries, uint32_t dim,
                     const uint8_t* row_mask, uint32_t k, uint64_t* out_rows,
                     uint64_t* out_chunk_ids, double* out_scores, uint32_t* out_counts,
                     char* err, size_t err_len);

/* Device-pointer variant: queries, outputs and row_mask in device memory;
 * returns once queued on `stream`.  Queries are not validated on the host;
 * an invalid query is reported by svl_index_check. */
int svl_index_search_device(svl_index* index, const float* d_queries, uint32_t n_queries,
                            const uint8_t* d_row_mask, uint32_t k, uint64_t* d_out_rows,
                            uint64_t* d_out_chunk_ids, double* d_out_scores,
                            uint32_t* d_out_counts, void* stream, char* err, size_t err_len);

/* Synchronises the index's stream and reports deferred device-side errors. */
int svl_index_check(svl_index* index, char* err, size_t err_len);

/* Merges per-shard top-k lists (gathered from every GPU of a row-sharded
 * index) into the global top-k, in device memory on `device`:
 *   d_scores / d_chunk_ids / d_rows : n_shards x n_queries x k (shard-major,
 *       as an all-gather lays them out); d_counts n_shards x n_queries
 *   outputs n_queries x k plus d_out_shard (which shard each hit came from)
 * Order: score descending, chunk id ascending (vector.rs:90-95). */
int svl_merge_topk_device(int device, const double* d_scores, const uint64_t* d_chunk_ids,
                          const uint64_t* d_rows, const uint32_t* d_counts, uint32_t n_shards,
                          uint32_t n_queries, uint32_t k, double* d_out_scores,
                          uint64_t* d_out_chunk_ids, uint64_t* d_out_rows,
                          uint32_t* d_out_shard, uint32_t* d_out_counts, void* stream,
                          char* err, size_t err_len);

/* ------------------------------------------------------------ multi-GPU --
 * One process per GPU over an NCCL communicator (NVLink / NVSwitch).  The
 * reference is single-process, so these have no counterpart there: they are
 * how the row-sharded index of this build reaches vector::rank
 * (src/index/vector.rs:17-97) over several GPUs.  NCCL is opened at run time
 * (libnccl.so.2; the copy already loaded in the process when there is one):
 * without it these calls return SVL_UNSUPPORTED.  Every rank must make the
 * same calls in the same order with the same sizes. */

/* 128 bytes (an ncclUniqueId) for svl_nccl_comm_create, made on one rank and
 * handed to the others by the host. */
int svl_nccl_unique_id(void* id_out, char* err, size_t err_len);

/* Joins rank `rank` of `n_ranks` (1..64) on `device`; *comm_out is the
 * communicator (an ncclComm_t) the calls below take.  Blocks until every
 * rank has joined. */
int svl_nccl_comm_create(int device, int n_ranks, int rank, const void* id, void** comm_out, char* err,
                         size_t err_len);

/* Destroys (abort = 0) or aborts (abort = 1: after an error that left other
 * ranks waiting) a communicator from svl_nccl_comm_create. */
int svl_nccl_comm_destroy(void* comm, int abort);

/* Query stage of ingest-then-query: every rank passes n_local x dim floats
 * (the same n_local on every rank); d_all (n_ranks * n_local x dim, rank
 * major) receives every rank's rows on every rank.  Queued on `stream`. */
int svl_allgather_rows(void* comm, const float* d_local, uint64_t n_local, uint32_t dim, float* d_all,
                       void* stream, char* err, size_t err_len);

#define SVL_SHARDED_MAX_K 4096u

/* Exact top-k over a corpus row-sharded across the communicator's ranks:
 * every rank passes its shard (an svl_index whose rows start at global row
 * `row_offset`) and the SAME n_queries x dim queries (device memory).  Each
 * rank searches its shard (svl_index_search's exact path, near-ties
 * included), the per-shard lists are exchanged in one all-gather, and every
 * rank receives the global answer in reference order (score descending, chunk
 * id ascending; vector.rs:90-95):
 *   d_out_rows      n_queries x k global rows (row_offset + local row)
 *   d_out_chunk_ids n_queries x k (may be NULL); d_out_scores n_queries x k
 *   d_out_counts    n_queries: min(k, total rows)
 * k is 1..SVL_SHARDED_MAX_K.  The call synchronises `stream` once (between
 * the shard search and the exchange) and returns with the exchange and the
 * merge queued.  A rank whose own search fails still takes part in the
 * exchange and returns the error; the other ranks skip its list and report
 * SVL_INTERNAL ("another rank's shard search failed") at svl_index_check.
 * If the exchange buffers cannot be allocated the call returns
 * SVL_LIMIT_EXCEEDED without taking part: abort the communicator on every
 * rank. */
int svl_sharded_search(void* comm, svl_index* shard, uint64_t row_offset, const float* d_queries,
                       uint32_t n_queries, uint32_t k, uint64_t* d_out_rows, uint64_t* d_out_chunk_ids,
                       double* d_out_scores, uint32_t* d_out_counts, void* stream, char* err,
                       size_t err_len);

/* Exact cosine top-k like svl_index_search_device, for callers that cannot
 * allocate device memory: no counterpart in the reference.  Some hosts cannot
 * let a library call cudaMalloc -- device memory is carved up up front by a
 * pool this library must not bypass, a serving loop runs under a fixed memory
 * budget, or the calling thread may not take the driver's allocation lock.
 * This entry point allocates nothing: its scratch is one static device array
 * of about 2.6 MiB that every GPU loading the library holds until the process
 * exits.
 *   d_rows     : n_rows x dim unit-norm rows (as svl_index_append stores them),
 *                16-byte aligned, on the current device; d_chunk_ids n_rows
 *   d_queries  : n_queries x dim, 16-byte aligned; d_row_mask NULL or n_rows
 *                bytes (0 = filtered); a misaligned pointer is SVL_USAGE
 *   outputs    : as svl_index_search_device (n_queries x k, counts n_queries);
 *                d_out_chunk_ids may be NULL
 * Limits: 1..128 queries, dim a multiple of 4 up to 1024, k 1..32; larger
 * requests are rejected with SVL_LIMIT_EXCEEDED.  Synchronous: returns after
 * `stream` has finished the search; a query with too many near-ties for the
 * candidate screen returns SVL_UNSUPPORTED (svl_index_search answers it).
 * The first call on each device looks up the scratch address and sets kernel
 * attributes, so make it before any stream capture.  Every call on a device
 * shares the one scratch array: calls that overlap on the GPU (other threads
 * or streams) race and must be serialised by the caller. */
int svl_search_noalloc(const float* d_rows, const uint64_t* d_chunk_ids, uint64_t n_rows, uint32_t dim,
                       const float* d_queries, uint32_t n_queries, const uint8_t* d_row_mask, uint32_t k,
                       uint64_t* d_out_rows, uint64_t* d_out_chunk_ids, double* d_out_scores,
                       uint32_t* d_out_counts, void* stream, char* err, size_t err_len);

#ifdef __cplusplus
}
#endif
#endif /* SVL_GPU_H */
