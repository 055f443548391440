/* svl_tokenizer.h -- C ABI of the frozen-model BPE tokenizer (host code in
 * libsvl_gpu.so), the text front end of the embedding path.
 *
 * Replaces src/model/tokenizer.rs (Tokenizer::from_json_str :98-103,
 * from_json :110-385, encode :392-434, decode :441-466 and the accessors
 * :469-516) and keeps its error variants as svl_status values:
 *   an inconsistent document          -> SVL_CORRUPT
 *   a pipeline other than the model's -> SVL_UNSUPPORTED
 *   a cap (file, vocabulary, merges, added tokens, input, tokens) exceeded
 *                                     -> SVL_LIMIT_EXCEEDED
 * The tokenizer is immutable once created: concurrent calls on one handle
 * are safe.  No call touches a GPU.
 */
#ifndef SVL_TOKENIZER_H
#define SVL_TOKENIZER_H

#include <stddef.h>
#include <stdint.h>

#include "svl_gpu.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct svl_tokenizer svl_tokenizer;

/* Caps of tokenizer.rs:25-43. */
#define SVL_TOKENIZER_MAX_FILE_BYTES (64u * 1024u * 1024u)
#define SVL_TOKENIZER_MAX_INPUT_BYTES (1024u * 1024u)
#define SVL_TOKENIZER_MAX_TOKENS 262144u

typedef struct svl_tokenizer_info {
  uint64_t vocab_size;   /* Tokenizer::vocab_size   */
  uint32_t max_token_id; /* Tokenizer::max_token_id */
  uint32_t bos_id;       /* Tokenizer::bos_id       */
  uint32_t eos_id;       /* Tokenizer::eos_id       */
  uint32_t unk_id;       /* Tokenizer::unk_id       */
  uint32_t pad_id;       /* Tokenizer::pad_id (valid when has_pad) */
  uint32_t has_pad;
} svl_tokenizer_info;

/* Tokenizer::from_json_str: `json` holds json_len bytes of a tokenizer.json
 * document (UTF-8; not NUL-terminated).  The document must describe the
 * model's pipeline (BPE with byte fallback and fuse_unk, Replace(' ' -> U+2581)
 * normaliser, Split(' ', MergedWithPrevious) pre-tokeniser, <bos> A <eos>
 * template, Replace / ByteFallback / Fuse decoder). */
int svl_tokenizer_create(const char* json, size_t json_len, svl_tokenizer** out, char* err, size_t err_len);

void svl_tokenizer_destroy(svl_tokenizer* tokenizer);

/* Tokenizer::encode: `text` is text_len bytes of UTF-8 (invalid UTF-8 ->
 * SVL_USAGE).  Added tokens are matched in the raw text, longest first;
 * add_special != 0 adds <bos> ... <eos>.  *n_ids receives the token count;
 * `ids` takes up to `capacity` of them (capacity >= text_len + 2 always
 * suffices; a smaller buffer that cannot hold the result -> SVL_USAGE, with
 * *n_ids set to the count needed). */
int svl_tokenizer_encode(const svl_tokenizer* tokenizer, const char* text, size_t text_len, int add_special,
                         uint32_t* ids, size_t capacity, size_t* n_ids, char* err, size_t err_len);

/* Tokenizer::encode over n texts in one call, on up to `threads` host
 * threads (0: one per hardware thread).  Text i is bytes[offsets[i] ..
 * offsets[i + 1]) (offsets has n + 1 entries).  The ids come out packed as
 * svl_embed_batch takes them: ids[cu_seqlens[i] .. cu_seqlens[i + 1]) are
 * text i's (cu_seqlens has n + 1 entries); `capacity` (ids) of offsets[n] +
 * 2 n always suffices.  The result does not depend on the thread count.  On
 * an error (per text as for svl_tokenizer_encode, or SVL_USAGE for a buffer
 * too small) *failed receives the lowest failing text index (n when the
 * error is not a text's). */
int svl_tokenizer_encode_batch(const svl_tokenizer* tokenizer, const char* bytes, const uint64_t* offsets, uint64_t n,
                               int add_special, uint32_t threads, uint32_t* ids, uint64_t capacity,
                               uint64_t* cu_seqlens, uint64_t* failed, char* err, size_t err_len);

/* Tokenizer::decode: UTF-8 text of the ids (byte-fallback tokens reassembled,
 * U+2581 -> ' '; special tokens skipped when skip_special != 0).  An unknown
 * id or a result that is not valid UTF-8 -> SVL_CORRUPT.  *out_len receives
 * the byte length; `out` may be NULL to ask for it, else it must hold
 * out_len bytes (a smaller capacity -> SVL_USAGE).  No NUL is appended. */
int svl_tokenizer_decode(const svl_tokenizer* tokenizer, const uint32_t* ids, size_t n_ids, int skip_special,
                         char* out, size_t capacity, size_t* out_len, char* err, size_t err_len);

/* Tokenizer::token_id: 1 and *id when `token` (token_len bytes) is in the
 * vocabulary, else 0. */
int svl_tokenizer_token_id(const svl_tokenizer* tokenizer, const char* token, size_t token_len, uint32_t* id);

/* Tokenizer::token: 1 with *token / *token_len pointing at the handle's own
 * copy (valid until svl_tokenizer_destroy) when `id` is in the vocabulary,
 * else 0. */
int svl_tokenizer_token(const svl_tokenizer* tokenizer, uint32_t id, const char** token, size_t* token_len);

/* Tokenizer::is_special_id. */
int svl_tokenizer_is_special(const svl_tokenizer* tokenizer, uint32_t id);

int svl_tokenizer_get_info(const svl_tokenizer* tokenizer, svl_tokenizer_info* info);

#ifdef __cplusplus
}
#endif

#endif /* SVL_TOKENIZER_H */
