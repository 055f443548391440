// bundle.cpp -- the `.svlm` model bundle behind include/svl_bundle.h (host
// code; src/bundle/mod.rs, docs/formats.md "Model bundle").
//
// parse() walks the header in the reference's order of checks (fixed header,
// caps, declared length, header CRC-32, then each section entry: path bytes,
// path rules, strict path order, contiguous offsets, end inside the data
// area; then the table end, the data-area coverage and the catalog digest),
// so a damaged bundle is rejected with the same error variant.  build()
// writes the same deterministic bytes as Bundle::build (sections sorted by
// path bytes, offsets contiguous from the end of the header).  SHA-256
// follows FIPS 180-4 and CRC-32 the IEEE polynomial; both are written here
// from their published definitions (SHA-256 also on the x86 SHA extensions
// when the CPU has them: ~1 GB/s instead of ~0.16 GB/s, which is what
// verifying a bundle's weights section costs).

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <memory>
#include <new>
#include <string>
#include <vector>

#if defined(__x86_64__)
#include <cpuid.h>
#include <immintrin.h>
#endif

#include "../../include/svl_bundle.h"

namespace {

constexpr uint8_t kMagic[8] = {'S', 'V', 'L', 'M', 'D', 'L', '0', '1'};
constexpr uint16_t kVersion = 1;
constexpr uint64_t kMaxBundle = 1ull << 33;  // 8 GiB
constexpr uint64_t kMaxHeader = 1ull << 20;  // 1 MiB
constexpr uint64_t kMaxSections = 1024;
constexpr uint64_t kMaxPath = 4096;
constexpr uint64_t kFixed = 30, kEntry = 52, kTrailer = 32, kCrcAt = 26;

struct Status {
  int code = SVL_OK;
  std::string msg;
  bool ok() const { return code == SVL_OK; }
};
Status corrupt(std::string m) { return Status{SVL_CORRUPT, std::move(m)}; }
Status limit(std::string m) { return Status{SVL_LIMIT_EXCEEDED, std::move(m)}; }

void put_err(char* err, size_t err_len, const std::string& msg) {
  if (!err || err_len == 0) return;
  const size_t n = std::min(msg.size(), err_len - 1);
  std::memcpy(err, msg.data(), n);
  err[n] = '\0';
}

// ---------------------------------------------------------------- SHA-256 --
// FIPS 180-4 section 6.2: 64 rounds over 512-bit blocks, the K table being the
// first 32 bits of the fractional parts of the cube roots of the first 64
// primes, the initial H the same for the square roots of the first 8.
constexpr uint32_t kK[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

#if defined(__x86_64__)
// The same compression function on the x86 SHA extensions (SHA-NI): the
// state lives as (A, B, E, F) and (C, D, G, H) lane pairs, sha256rnds2 runs
// two rounds from the low two W + K words, sha256msg1 / msg2 extend the
// message schedule four words at a time.  Selected at run time when CPUID
// reports SHA, SSSE3 and SSE4.1; the scalar block function is the fallback.
__attribute__((target("sha,sse4.1,ssse3"))) void sha256_blocks_ni(uint32_t h[8], const uint8_t* p, uint64_t blocks) {
  const __m128i bswap = _mm_set_epi64x(0x0c0d0e0f08090a0bULL, 0x0405060700010203ULL);
  // lane contents listed from the high lane to the low one
  __m128i t = _mm_loadu_si128((const __m128i*)&h[0]);        // D C B A
  __m128i s1 = _mm_loadu_si128((const __m128i*)&h[4]);       // H G F E
  t = _mm_shuffle_epi32(t, 0xB1);                            // C D A B
  s1 = _mm_shuffle_epi32(s1, 0x1B);                          // E F G H
  __m128i s0 = _mm_alignr_epi8(t, s1, 8);                    // A B E F
  s1 = _mm_blend_epi16(s1, t, 0xF0);                         // C D G H
  for (; blocks; --blocks, p += 64) {
    const __m128i a0 = s0, c0 = s1;
    __m128i w[4];
    for (int g = 0; g < 16; ++g) {
      if (g < 4) {
        w[g] = _mm_shuffle_epi8(_mm_loadu_si128((const __m128i*)(p + 16 * g)), bswap);
      } else {
        // W[t..t+3] from W[t-16..], W[t-12..], W[t-8..] and W[t-4..]
        __m128i x = _mm_sha256msg1_epu32(w[g & 3], w[(g + 1) & 3]);
        x = _mm_add_epi32(x, _mm_alignr_epi8(w[(g + 3) & 3], w[(g + 2) & 3], 4));
        w[g & 3] = _mm_sha256msg2_epu32(x, w[(g + 3) & 3]);
      }
      const __m128i k = _mm_add_epi32(w[g & 3], _mm_loadu_si128((const __m128i*)&kK[4 * g]));
      s1 = _mm_sha256rnds2_epu32(s1, s0, k);
      s0 = _mm_sha256rnds2_epu32(s0, s1, _mm_shuffle_epi32(k, 0x0E));
    }
    s0 = _mm_add_epi32(s0, a0);
    s1 = _mm_add_epi32(s1, c0);
  }
  t = _mm_shuffle_epi32(s0, 0x1B);                           // F E B A
  s1 = _mm_shuffle_epi32(s1, 0xB1);                          // D C H G
  s0 = _mm_blend_epi16(t, s1, 0xF0);                         // D C B A
  s1 = _mm_alignr_epi8(s1, t, 8);                            // H G F E
  _mm_storeu_si128((__m128i*)&h[0], s0);
  _mm_storeu_si128((__m128i*)&h[4], s1);
}

bool cpu_has_sha_ni() {
  unsigned a, b, c, d;
  if (!__get_cpuid(1, &a, &b, &c, &d)) return false;
  const bool ssse3 = c & (1u << 9), sse41 = c & (1u << 19);
  if (!__get_cpuid_count(7, 0, &a, &b, &c, &d)) return false;
  return ssse3 && sse41 && (b & (1u << 29));
}
const bool kShaNi = cpu_has_sha_ni();
#endif

class Sha256 {
 public:
  void update(const uint8_t* p, uint64_t n) {
    total_ += n;
    if (fill_) {
      const uint64_t take = std::min<uint64_t>(n, 64 - fill_);
      std::memcpy(buf_ + fill_, p, take);
      fill_ += (uint32_t)take;
      p += take;
      n -= take;
      if (fill_ == 64) {
        blocks(buf_, 1);
        fill_ = 0;
      }
    }
    if (n >= 64) {
      blocks(p, n / 64);
      p += n / 64 * 64;
      n %= 64;
    }
    if (n) {
      std::memcpy(buf_, p, n);
      fill_ = (uint32_t)n;
    }
  }
  void finish(uint8_t out[32]) {
    const uint64_t bits = total_ * 8;
    uint8_t pad[72] = {0x80};
    const uint64_t pad_len = (fill_ < 56 ? 56 - fill_ : 120 - fill_);
    for (int i = 0; i < 8; ++i) pad[pad_len + i] = (uint8_t)(bits >> (56 - 8 * i));
    update(pad, pad_len + 8);
    for (int i = 0; i < 8; ++i)
      for (int j = 0; j < 4; ++j) out[4 * i + j] = (uint8_t)(h_[i] >> (24 - 8 * j));
  }

 private:
  uint32_t h_[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  uint8_t buf_[64];
  uint32_t fill_ = 0;
  uint64_t total_ = 0;

  void blocks(const uint8_t* p, uint64_t count) {
#if defined(__x86_64__)
    if (kShaNi) {
      sha256_blocks_ni(h_, p, count);
      return;
    }
#endif
    for (uint64_t i = 0; i < count; ++i) block(p + 64 * i);
  }

  void block(const uint8_t* p) {
    uint32_t w[64];
    for (int t = 0; t < 16; ++t)
      w[t] = (uint32_t)p[4 * t] << 24 | (uint32_t)p[4 * t + 1] << 16 | (uint32_t)p[4 * t + 2] << 8 | p[4 * t + 3];
    for (int t = 16; t < 64; ++t) {
      const uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
      const uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
      w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
    for (int t = 0; t < 64; ++t) {
      const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + kK[t] + w[t];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      h = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h_[0] += a;
    h_[1] += b;
    h_[2] += c;
    h_[3] += d;
    h_[4] += e;
    h_[5] += f;
    h_[6] += g;
    h_[7] += h;
  }
};

// ----------------------------------------------------------------- CRC-32 --
struct CrcTable {
  uint32_t t[256];
  CrcTable() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
      t[i] = c;
    }
  }
};
const CrcTable kCrc;

uint32_t crc_update(uint32_t crc, const uint8_t* p, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i) crc = kCrc.t[(crc ^ p[i]) & 0xFF] ^ (crc >> 8);
  return crc;
}

// CRC-32 of a header, every byte but the CRC field (mod.rs:674-679)
uint32_t header_crc(const uint8_t* h, uint64_t len) {
  uint32_t c = crc_update(0xFFFFFFFFu, h, kCrcAt);
  c = crc_update(c, h + kCrcAt + 4, len - kCrcAt - 4);
  return c ^ 0xFFFFFFFFu;
}

uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | p[1] << 8); }
uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}
uint64_t rd64(const uint8_t* p) { return (uint64_t)rd32(p) | (uint64_t)rd32(p + 4) << 32; }
void wr(std::vector<uint8_t>* o, uint64_t v, int bytes) {
  for (int i = 0; i < bytes; ++i) o->push_back((uint8_t)(v >> (8 * i)));
}

bool utf8_ok(const uint8_t* s, uint64_t n) {
  uint64_t i = 0;
  while (i < n) {
    const uint8_t c = s[i];
    if (c < 0x80) {
      ++i;
      continue;
    }
    int len;
    uint32_t min;
    if (c >= 0xC2 && c <= 0xDF) {
      len = 2;
      min = 0x80;
    } else if (c >= 0xE0 && c <= 0xEF) {
      len = 3;
      min = 0x800;
    } else if (c >= 0xF0 && c <= 0xF4) {
      len = 4;
      min = 0x10000;
    } else {
      return false;
    }
    if (i + len > n) return false;
    uint32_t cp = c & (len == 2 ? 0x1F : len == 3 ? 0x0F : 0x07);
    for (int k = 1; k < len; ++k) {
      if ((s[i + k] & 0xC0) != 0x80) return false;
      cp = cp << 6 | (s[i + k] & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    i += len;
  }
  return true;
}

// mod.rs:692-719: relative, normalised, no empty / "." / ".." component
Status validate_path(const std::string& path) {
  if (path.empty()) return corrupt("bundle path is empty");
  if (path.size() > kMaxPath)
    return limit("bundle path is " + std::to_string(path.size()) + " bytes, above the 4096-byte cap");
  if (path[0] == '/' || path.find('\\') != std::string::npos || path.find('\0') != std::string::npos)
    return corrupt("bundle path " + path + " is absolute or contains a forbidden character");
  size_t start = 0;
  for (;;) {
    const size_t slash = path.find('/', start);
    const std::string comp = path.substr(start, slash == std::string::npos ? std::string::npos : slash - start);
    if (comp.empty() || comp == "." || comp == "..")
      return corrupt("bundle path " + path + " contains an empty, current, or parent component");
    if (slash == std::string::npos) break;
    start = slash + 1;
  }
  return Status{};
}

}  // namespace

struct svl_bundle {
  const uint8_t* bytes = nullptr;
  uint64_t len = 0, header_len = 0;
  std::vector<svl_bundle_section> sections;

  // mod.rs:179-375
  Status parse(const uint8_t* b, uint64_t n) {
    bytes = b;
    len = n;
    if (n < kFixed + kTrailer) return corrupt("bundle is shorter than its fixed header");
    if (std::memcmp(b, kMagic, 8) != 0) return corrupt("bundle magic does not match SVLMDL01");
    const uint16_t version = rd16(b + 8);
    if (version != kVersion)
      return Status{SVL_UNSUPPORTED, "bundle format version " + std::to_string(version) + " is not supported"};
    const uint64_t hlen = rd32(b + 10), count = rd32(b + 14), total = rd64(b + 18);
    if (hlen < kFixed) return corrupt("bundle header length is below the fixed header");
    if (hlen > kMaxHeader)
      return limit("bundle header is " + std::to_string(hlen) + " bytes, above the 1048576-byte cap");
    if (count > kMaxSections)
      return limit("bundle has " + std::to_string(count) + " sections, above the 1024-section cap");
    if (total != n) return corrupt("bundle declares " + std::to_string(total) + " bytes but has " + std::to_string(n));
    if (total > kMaxBundle)
      return limit("bundle is " + std::to_string(total) + " bytes, above the 8589934592-byte cap");
    if (hlen + kTrailer > n) return corrupt("bundle header overlaps the catalog digest");
    if (rd32(b + kCrcAt) != header_crc(b, hlen)) return corrupt("bundle header CRC-32 mismatch");
    const uint64_t data_end = total - kTrailer;
    uint64_t cursor = kFixed, expected = hlen;
    std::string prev;
    bool have_prev = false;
    sections.reserve(count);
    for (uint64_t s = 0; s < count; ++s) {
      if (cursor + kEntry > hlen) return corrupt("bundle section table is truncated");
      const uint8_t* e = b + cursor;
      const uint64_t path_len = rd16(e);
      const uint8_t role = e[2], flags = e[3];
      if (role > SVL_ROLE_OTHER) return corrupt("unknown bundle section role " + std::to_string(role));
      if (flags != 0)
        return Status{SVL_UNSUPPORTED, "bundle section flags " + std::to_string(flags) + " are not supported"};
      const uint64_t offset = rd64(e + 4), length = rd64(e + 12);
      svl_bundle_section sec{};
      std::memcpy(sec.sha256, e + 20, 32);
      cursor += kEntry;
      if (cursor + path_len > hlen) return corrupt("bundle path is truncated");
      if (!utf8_ok(b + cursor, path_len)) return corrupt("bundle path is not valid UTF-8");
      const std::string path((const char*)b + cursor, path_len);
      Status st = validate_path(path);
      if (!st.ok()) return st;
      sec.path = (const char*)b + cursor;
      sec.path_len = path_len;
      cursor += path_len;
      if (have_prev && path <= prev) return corrupt("bundle section paths are not strictly sorted");
      prev = path;
      have_prev = true;
      if (offset != expected)
        return corrupt("bundle section " + path + " starts at " + std::to_string(offset) + ", expected " +
                       std::to_string(expected));
      if (length > UINT64_MAX - offset) return limit("bundle section end overflow");
      const uint64_t end = offset + length;
      if (end > data_end)
        return corrupt("bundle section " + path + " ends at " + std::to_string(end) + ", beyond the data area " +
                       std::to_string(data_end));
      expected = end;
      sec.role = role;
      sec.offset = offset;
      sec.length = length;
      sec.data = b + offset;
      sections.push_back(sec);
    }
    if (cursor != hlen) return corrupt("bundle section table does not end at the declared header length");
    if (expected != data_end) return corrupt("bundle sections do not cover the declared data area");
    Sha256 h;
    h.update(b, hlen);
    for (const auto& sec : sections) h.update(sec.sha256, 32);
    uint8_t digest[32];
    h.finish(digest);
    if (std::memcmp(digest, b + n - kTrailer, 32) != 0) return corrupt("bundle catalog digest mismatch");
    header_len = hlen;
    return Status{};
  }
};

namespace {

// mod.rs:382-441 and encode_header :599-672.  Validates the inputs and sizes
// the bundle; with `out` (capacity >= the size) also writes it: header, the
// sections in path order, the catalog digest.
Status build(const svl_bundle_input* in, uint64_t n, uint8_t* out, uint64_t capacity, uint64_t* total_len) {
  if (n > kMaxSections) return limit("bundle has " + std::to_string(n) + " sections, above the 1024-section cap");
  std::vector<const svl_bundle_input*> order(n);
  for (uint64_t i = 0; i < n; ++i) order[i] = &in[i];
  auto path_of = [](const svl_bundle_input* s) { return std::string(s->path ? s->path : "", s->path_len); };
  std::stable_sort(order.begin(), order.end(),
                   [&](const svl_bundle_input* a, const svl_bundle_input* b) { return path_of(a) < path_of(b); });
  for (uint64_t i = 1; i < n; ++i)
    if (path_of(order[i - 1]) == path_of(order[i]))
      return Status{SVL_USAGE, "duplicate bundle section path " + path_of(order[i])};
  uint64_t hlen = kFixed, data_len = 0;
  for (const svl_bundle_input* s : order) {
    const std::string path = path_of(s);
    Status st = validate_path(path);
    if (!st.ok()) return st;
    if (s->role > SVL_ROLE_OTHER) return Status{SVL_USAGE, "unknown bundle section role " + std::to_string(s->role)};
    if (!utf8_ok((const uint8_t*)path.data(), path.size())) return corrupt("bundle path is not valid UTF-8");
    hlen += kEntry + path.size();
    if (s->length > kMaxBundle) return limit("bundle section length is above the 8589934592-byte cap");
    data_len += s->length;
  }
  if (hlen > kMaxHeader)
    return limit("bundle header is " + std::to_string(hlen) + " bytes, above the 1048576-byte cap");
  const uint64_t total = hlen + data_len + kTrailer;
  if (total > kMaxBundle)
    return limit("bundle would be " + std::to_string(total) + " bytes, above the 8589934592-byte cap");
  *total_len = total;
  if (!out) return Status{};
  if (total > capacity)
    return Status{SVL_USAGE, "output buffer holds " + std::to_string(capacity) + " bytes, " + std::to_string(total) +
                                 " are needed"};
  std::vector<uint8_t> h;
  h.reserve(hlen);
  h.insert(h.end(), kMagic, kMagic + 8);
  wr(&h, kVersion, 2);
  wr(&h, hlen, 4);
  wr(&h, n, 4);
  wr(&h, total, 8);
  wr(&h, 0, 4);  // CRC, filled below
  std::vector<uint8_t> digests;
  uint64_t offset = hlen;
  for (const svl_bundle_input* s : order) {
    uint8_t d[32];
    svl_sha256(s->data, s->length, d);
    digests.insert(digests.end(), d, d + 32);
    wr(&h, s->path_len, 2);
    h.push_back((uint8_t)s->role);
    h.push_back(0);
    wr(&h, offset, 8);
    wr(&h, s->length, 8);
    h.insert(h.end(), d, d + 32);
    h.insert(h.end(), s->path, s->path + s->path_len);
    if (s->length) std::memcpy(out + offset, s->data, s->length);
    offset += s->length;
  }
  const uint32_t crc = header_crc(h.data(), hlen);
  for (int i = 0; i < 4; ++i) h[kCrcAt + i] = (uint8_t)(crc >> (8 * i));
  std::memcpy(out, h.data(), hlen);
  Sha256 cat;
  cat.update(h.data(), hlen);
  cat.update(digests.data(), digests.size());
  cat.finish(out + offset);
  return Status{};
}

}  // namespace

extern "C" {

void svl_sha256(const uint8_t* data, uint64_t len, uint8_t digest[32]) {
  Sha256 h;
  if (len) h.update(data, len);
  h.finish(digest);
}

uint32_t svl_crc32(const uint8_t* data, uint64_t len) { return crc_update(0xFFFFFFFFu, data, len) ^ 0xFFFFFFFFu; }

int svl_bundle_parse(const uint8_t* bytes, uint64_t len, svl_bundle** out, char* err, size_t err_len) {
  if (!out || (!bytes && len)) {
    put_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  *out = nullptr;
  try {
    std::unique_ptr<svl_bundle> b(new svl_bundle());
    Status st = b->parse(bytes, len);
    if (!st.ok()) {
      put_err(err, err_len, st.msg);
      return st.code;
    }
    *out = b.release();
    return SVL_OK;
  } catch (const std::bad_alloc&) {
    put_err(err, err_len, "out of host memory");
    return SVL_LIMIT_EXCEEDED;
  }
}

void svl_bundle_destroy(svl_bundle* bundle) { delete bundle; }

int svl_bundle_verify(const svl_bundle* bundle, char* err, size_t err_len) {
  if (!bundle) {
    put_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  for (const auto& sec : bundle->sections) {
    uint8_t d[32];
    svl_sha256(sec.data, sec.length, d);
    if (std::memcmp(d, sec.sha256, 32) != 0) {
      put_err(err, err_len, "bundle section " + std::string(sec.path, sec.path_len) + " SHA-256 mismatch");
      return SVL_CORRUPT;
    }
  }
  return SVL_OK;
}

uint64_t svl_bundle_header_len(const svl_bundle* bundle) { return bundle ? bundle->header_len : 0; }

uint64_t svl_bundle_section_count(const svl_bundle* bundle) { return bundle ? bundle->sections.size() : 0; }

int svl_bundle_section_at(const svl_bundle* bundle, uint64_t index, svl_bundle_section* out) {
  if (!bundle || !out || index >= bundle->sections.size()) return SVL_USAGE;
  *out = bundle->sections[index];
  return SVL_OK;
}

int svl_bundle_find(const svl_bundle* bundle, const char* path, uint64_t path_len, uint64_t* index) {
  if (!bundle || (!path && path_len)) return 0;
  const std::string want(path ? path : "", path_len);
  size_t lo = 0, hi = bundle->sections.size();
  while (lo < hi) {  // sections are strictly sorted by path bytes
    const size_t mid = (lo + hi) / 2;
    const auto& s = bundle->sections[mid];
    const std::string p(s.path, s.path_len);
    if (p == want) {
      if (index) *index = mid;
      return 1;
    }
    if (p < want)
      lo = mid + 1;
    else
      hi = mid;
  }
  return 0;
}

int svl_bundle_build(const svl_bundle_input* sections, uint64_t n, uint8_t* out, uint64_t capacity,
                     uint64_t* out_len, char* err, size_t err_len) {
  if (!out_len || (!sections && n)) {
    put_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  *out_len = 0;
  for (uint64_t i = 0; i < n; ++i)
    if ((!sections[i].path && sections[i].path_len) || (!sections[i].data && sections[i].length)) {
      put_err(err, err_len, "null section data");
      return SVL_USAGE;
    }
  try {
    Status st = build(sections, n, out, capacity, out_len);
    if (!st.ok()) {
      put_err(err, err_len, st.msg);
      return st.code;
    }
    return SVL_OK;
  } catch (const std::bad_alloc&) {
    put_err(err, err_len, "out of host memory");
    return SVL_LIMIT_EXCEEDED;
  }
}

}  // extern "C"
