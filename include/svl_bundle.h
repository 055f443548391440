/* svl_bundle.h -- C ABI of the `.svlm` model bundle reader / writer (host
 * code in libsvl_gpu.so), the weight-ingress front end of the embedding path.
 *
 * Replaces src/bundle/mod.rs (Bundle::parse :179-375, Bundle::build :382-441,
 * Bundle::section / data :453-466, Bundle::verify :470-482) with the same
 * format (docs/formats.md "Model bundle"): little-endian fixed header
 * [magic "SVLMDL01" | version u16 = 1 | header length u32 | section count u32 |
 * total length u64 | header CRC-32 u32], then per section [path length u16 |
 * role u8 | flags u8 = 0 | offset u64 | length u64 | SHA-256 | path], the
 * section bytes in path order, and a 32-byte catalog digest = SHA-256(header ||
 * section digests in order).  Errors keep the reference's variants:
 *   a corrupt or truncated bundle, a bad path          -> SVL_CORRUPT
 *   another format version, non-zero section flags     -> SVL_UNSUPPORTED
 *   a cap (8 GiB, 1 MiB header, 1,024 sections, 4,096-byte path)
 *                                                      -> SVL_LIMIT_EXCEEDED
 *   a duplicate path given to svl_bundle_build         -> SVL_USAGE
 * No call touches a GPU.
 */
#ifndef SVL_BUNDLE_H
#define SVL_BUNDLE_H

#include <stddef.h>
#include <stdint.h>

#include "svl_gpu.h"

#ifdef __cplusplus
extern "C" {
#endif

/* src/bundle/mod.rs:49-58 */
typedef enum svl_section_role {
  SVL_ROLE_MANIFEST = 0,
  SVL_ROLE_CONFIG = 1,
  SVL_ROLE_TOKENIZER = 2,
  SVL_ROLE_PROCESSOR = 3,
  SVL_ROLE_WEIGHTS = 4,
  SVL_ROLE_OTHER = 5
} svl_section_role;

typedef struct svl_bundle svl_bundle;

/* One section of a parsed bundle; `path` and `data` point into the bytes
 * given to svl_bundle_parse (not NUL-terminated). */
typedef struct svl_bundle_section {
  const char* path;
  uint64_t path_len;
  uint32_t role; /* svl_section_role */
  uint32_t reserved;
  uint64_t offset;
  uint64_t length;
  uint8_t sha256[32];
  const uint8_t* data;
} svl_bundle_section;

/* One input of svl_bundle_build (mod.rs:106-114). */
typedef struct svl_bundle_input {
  const char* path;
  uint64_t path_len;
  uint32_t role; /* svl_section_role */
  uint32_t reserved;
  const uint8_t* data;
  uint64_t length;
} svl_bundle_input;

/* Bundle::parse: checks the structure, the header CRC-32 and the catalog
 * digest (not the section digests: svl_bundle_verify).  The handle borrows
 * `bytes`, which must outlive it. */
int svl_bundle_parse(const uint8_t* bytes, uint64_t len, svl_bundle** out, char* err, size_t err_len);

void svl_bundle_destroy(svl_bundle* bundle);

/* Bundle::verify: the SHA-256 of every section against the header. */
int svl_bundle_verify(const svl_bundle* bundle, char* err, size_t err_len);

uint64_t svl_bundle_header_len(const svl_bundle* bundle);
uint64_t svl_bundle_section_count(const svl_bundle* bundle);

/* Section `index` (sorted path order): SVL_OK, or SVL_USAGE past the end. */
int svl_bundle_section_at(const svl_bundle* bundle, uint64_t index, svl_bundle_section* out);

/* Bundle::section: 1 and *index when a section has exactly this path, else 0. */
int svl_bundle_find(const svl_bundle* bundle, const char* path, uint64_t path_len, uint64_t* index);

/* Bundle::build: the deterministic bundle of `n` inputs (sorted by path).
 * *out_len receives the bundle length; `out` may be NULL to ask for it, else
 * it must hold out_len bytes (a smaller capacity -> SVL_USAGE). */
int svl_bundle_build(const svl_bundle_input* sections, uint64_t n, uint8_t* out, uint64_t capacity,
                     uint64_t* out_len, char* err, size_t err_len);

/* SHA-256 (FIPS 180-4) and CRC-32 (IEEE: polynomial 0xEDB88320, initial and
 * final XOR 0xFFFFFFFF) as the bundle uses them (src/binary/sha256.rs,
 * src/binary/crc32.rs). */
void svl_sha256(const uint8_t* data, uint64_t len, uint8_t digest[32]);
uint32_t svl_crc32(const uint8_t* data, uint64_t len);

#ifdef __cplusplus
}
#endif

#endif /* SVL_BUNDLE_H */
