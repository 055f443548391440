// tokenizer.cpp -- the frozen-model BPE tokenizer behind include/svl_tokenizer.h
// (host code; src/model/tokenizer.rs).
//
// Pipeline (tokenizer.rs:1-14, docs/tokenizer.md): added tokens matched in the
// raw text, longest first; every other character normalised (' ' -> U+2581)
// and looked up as a one-character token, or split into <0xXX> byte tokens;
// BPE merges by rank; <bos> / <eos> around the result on request.
//
// The merge loop gives exactly the reference's result (tokenizer.rs:520-560:
// repeatedly take the adjacent pair of lowest rank and merge all of its
// non-overlapping occurrences left to right) in O(n log n) instead of a full
// rescan per round: a min-heap holds (rank, left position) of every adjacent
// pair; a round pops every entry of the lowest live rank, which are exactly
// that pair's current occurrences (a rank names one pair), and merges them in
// position order, skipping any whose left symbol the previous merge of the
// round consumed.  A merge only creates pairs that contain the merged token,
// never the round's own pair, so the new pairs wait for later rounds, as in
// the reference.
//
// The JSON reader follows the reference's strict parser (src/json/mod.rs:
// duplicate keys, trailing commas, leading zeros, control characters, lone
// surrogates, non-finite numbers and trailing content are errors) with the
// tokenizer's limits (tokenizer.rs:563-572).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <memory>
#include <new>
#include <queue>
#include <string>
#include <system_error>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <utility>
#include <vector>

#include "../../include/svl_tokenizer.h"

namespace {

// ---------------------------------------------------------------- errors --
struct Status {
  int code = SVL_OK;
  std::string msg;
  bool ok() const { return code == SVL_OK; }
};

Status fail(int code, std::string msg) { return Status{code, std::move(msg)}; }
Status corrupt(std::string msg) { return fail(SVL_CORRUPT, std::move(msg)); }
Status unsupported(std::string msg) { return fail(SVL_UNSUPPORTED, std::move(msg)); }
Status limit(std::string msg) { return fail(SVL_LIMIT_EXCEEDED, std::move(msg)); }

void put_err(char* err, size_t err_len, const std::string& msg) {
  if (!err || err_len == 0) return;
  const size_t n = std::min(msg.size(), err_len - 1);
  std::memcpy(err, msg.data(), n);
  err[n] = '\0';
}

// ------------------------------------------------------------------ UTF-8 --
// Decodes one scalar value at s[i] (valid UTF-8 assumed checked), returns its
// byte length.
int utf8_next(const unsigned char* s, size_t i, uint32_t* cp) {
  const unsigned char c = s[i];
  if (c < 0x80) {
    *cp = c;
    return 1;
  }
  if (c < 0xE0) {
    *cp = ((uint32_t)(c & 0x1F) << 6) | (s[i + 1] & 0x3F);
    return 2;
  }
  if (c < 0xF0) {
    *cp = ((uint32_t)(c & 0x0F) << 12) | ((uint32_t)(s[i + 1] & 0x3F) << 6) | (s[i + 2] & 0x3F);
    return 3;
  }
  *cp = ((uint32_t)(c & 0x07) << 18) | ((uint32_t)(s[i + 1] & 0x3F) << 12) | ((uint32_t)(s[i + 2] & 0x3F) << 6) |
        (s[i + 3] & 0x3F);
  return 4;
}

// Strict UTF-8 check (no overlongs, no surrogates, nothing above U+10FFFF).
bool utf8_valid(const unsigned char* s, size_t n) {
  size_t i = 0;
  while (i < n) {
    const unsigned char c = s[i];
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
    for (int k = 1; k < len; ++k)
      if ((s[i + k] & 0xC0) != 0x80) return false;
    uint32_t cp;
    utf8_next(s, i, &cp);
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    i += len;
  }
  return true;
}

void utf8_append(std::string* out, uint32_t cp) {
  if (cp < 0x80) {
    out->push_back((char)cp);
  } else if (cp < 0x800) {
    out->push_back((char)(0xC0 | (cp >> 6)));
    out->push_back((char)(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    out->push_back((char)(0xE0 | (cp >> 12)));
    out->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    out->push_back((char)(0x80 | (cp & 0x3F)));
  } else {
    out->push_back((char)(0xF0 | (cp >> 18)));
    out->push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
    out->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    out->push_back((char)(0x80 | (cp & 0x3F)));
  }
}

// ------------------------------------------------------------------- JSON --
struct Json {
  enum Kind { kNull, kBool, kUnsigned, kSigned, kFloat, kString, kArray, kObject } kind = kNull;
  bool b = false;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  std::vector<Json> items;                             // array elements / object values
  std::vector<std::string> keys;                       // object keys, document order
  const Json* get(const char* key) const {
    if (kind != kObject) return nullptr;
    for (size_t k = 0; k < keys.size(); ++k)
      if (keys[k] == key) return &items[k];
    return nullptr;
  }
};

struct JsonLimits {
  size_t max_input_bytes = SVL_TOKENIZER_MAX_FILE_BYTES;
  size_t max_depth = 64;
  size_t max_string_bytes = 1024 * 1024;
  size_t max_container_entries = 600000;
  size_t max_total_values = 3000000;
};

class JsonReader {
 public:
  JsonReader(const char* p, size_t n, const JsonLimits& lim) : in_((const unsigned char*)p), n_(n), lim_(lim) {}

  Status parse(Json* out) {
    if (n_ > lim_.max_input_bytes)
      return limit("JSON input is " + std::to_string(n_) + " bytes, above the " +
                   std::to_string(lim_.max_input_bytes) + "-byte cap");
    ws();
    Status st = value(0, out);
    if (!st.ok()) return st;
    ws();
    if (pos_ != n_) return err("trailing content after the top-level value");
    return Status{};
  }

 private:
  const unsigned char* in_;
  size_t n_, pos_ = 0, values_ = 0;
  const JsonLimits& lim_;

  Status err(const std::string& m) const { return corrupt("JSON at byte " + std::to_string(pos_) + ": " + m); }
  void ws() {
    while (pos_ < n_ && (in_[pos_] == ' ' || in_[pos_] == '\t' || in_[pos_] == '\n' || in_[pos_] == '\r')) ++pos_;
  }
  bool literal(const char* lit) {
    const size_t l = std::strlen(lit);
    if (pos_ + l > n_ || std::memcmp(in_ + pos_, lit, l) != 0) return false;
    pos_ += l;
    return true;
  }

  Status value(size_t depth, Json* out) {
    if (depth > lim_.max_depth)
      return limit("JSON nesting exceeds the depth cap of " + std::to_string(lim_.max_depth));
    if (++values_ > lim_.max_total_values)
      return limit("JSON document exceeds the " + std::to_string(lim_.max_total_values) + "-value cap");
    ws();
    if (pos_ >= n_) return err("unexpected end of input");
    const unsigned char c = in_[pos_];
    if (c == '{') return object(depth, out);
    if (c == '[') return array(depth, out);
    if (c == '"') {
      out->kind = Json::kString;
      return string(&out->s);
    }
    if (c == 't' || c == 'f' || c == 'n') {
      if (literal("true")) {
        out->kind = Json::kBool;
        out->b = true;
      } else if (literal("false")) {
        out->kind = Json::kBool;
        out->b = false;
      } else if (literal("null")) {
        out->kind = Json::kNull;
      } else {
        return err("invalid literal");
      }
      return Status{};
    }
    if (c == '-' || (c >= '0' && c <= '9')) return number(out);
    return err("unexpected character");
  }

  Status array(size_t depth, Json* out) {
    out->kind = Json::kArray;
    ++pos_;  // [
    ws();
    if (pos_ < n_ && in_[pos_] == ']') {
      ++pos_;
      return Status{};
    }
    for (;;) {
      if (out->items.size() >= lim_.max_container_entries)
        return limit("JSON container exceeds the " + std::to_string(lim_.max_container_entries) + "-entry cap");
      out->items.emplace_back();
      Status st = value(depth + 1, &out->items.back());
      if (!st.ok()) return st;
      ws();
      if (pos_ >= n_) return err("unexpected end of input");
      if (in_[pos_] == ',') {
        ++pos_;
        ws();
        if (pos_ < n_ && in_[pos_] == ']') return err("trailing comma in array");
        continue;
      }
      if (in_[pos_] == ']') {
        ++pos_;
        return Status{};
      }
      return err("expected ',' or ']' in array");
    }
  }

  Status object(size_t depth, Json* out) {
    out->kind = Json::kObject;
    ++pos_;  // {
    ws();
    if (pos_ < n_ && in_[pos_] == '}') {
      ++pos_;
      return Status{};
    }
    std::unordered_set<std::string> seen;
    for (;;) {
      if (out->items.size() >= lim_.max_container_entries)
        return limit("JSON container exceeds the " + std::to_string(lim_.max_container_entries) + "-entry cap");
      ws();
      if (pos_ >= n_ || in_[pos_] != '"') return err("expected a string key");
      std::string key;
      Status st = string(&key);
      if (!st.ok()) return st;
      if (!seen.insert(key).second) return err("duplicate object key");
      ws();
      if (pos_ >= n_ || in_[pos_] != ':') return err("expected ':' after an object key");
      ++pos_;
      out->keys.push_back(std::move(key));
      out->items.emplace_back();
      st = value(depth + 1, &out->items.back());
      if (!st.ok()) return st;
      ws();
      if (pos_ >= n_) return err("unexpected end of input");
      if (in_[pos_] == ',') {
        ++pos_;
        ws();
        if (pos_ < n_ && in_[pos_] == '}') return err("trailing comma in object");
        continue;
      }
      if (in_[pos_] == '}') {
        ++pos_;
        return Status{};
      }
      return err("expected ',' or '}' in object");
    }
  }

  static int hex(unsigned char c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
  }
  bool hex4(uint32_t* v) {
    if (pos_ + 4 > n_) return false;
    uint32_t r = 0;
    for (int k = 0; k < 4; ++k) {
      const int h = hex(in_[pos_ + k]);
      if (h < 0) return false;
      r = r * 16 + (uint32_t)h;
    }
    pos_ += 4;
    *v = r;
    return true;
  }

  Status string(std::string* out) {
    ++pos_;  // opening quote
    for (;;) {
      if (pos_ >= n_) return err("unterminated string");
      const unsigned char c = in_[pos_];
      if (c == '"') {
        ++pos_;
        break;
      }
      if (c < 0x20) return err("unescaped control character in string");
      if (c == '\\') {
        ++pos_;
        if (pos_ >= n_) return err("unterminated escape");
        const unsigned char e = in_[pos_++];
        switch (e) {
          case '"': out->push_back('"'); break;
          case '\\': out->push_back('\\'); break;
          case '/': out->push_back('/'); break;
          case 'b': out->push_back('\b'); break;
          case 'f': out->push_back('\f'); break;
          case 'n': out->push_back('\n'); break;
          case 'r': out->push_back('\r'); break;
          case 't': out->push_back('\t'); break;
          case 'u': {
            uint32_t cp;
            if (!hex4(&cp)) return err("invalid \\u escape");
            if (cp >= 0xD800 && cp <= 0xDBFF) {
              if (pos_ >= n_ || in_[pos_] != '\\') return err("high surrogate is not followed by an escape");
              if (pos_ + 1 >= n_ || in_[pos_ + 1] != 'u') return err("high surrogate is not followed by a \\u escape");
              pos_ += 2;
              uint32_t lo;
              if (!hex4(&lo)) return err("invalid \\u escape");
              if (lo < 0xDC00 || lo > 0xDFFF) return err("high surrogate is not followed by a low surrogate");
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            } else if (cp >= 0xDC00 && cp <= 0xDFFF) {
              return err("lone low surrogate");
            }
            utf8_append(out, cp);
            break;
          }
          default:
            return err("invalid escape");
        }
      } else {
        out->push_back((char)c);  // raw UTF-8 (the whole input was checked)
        ++pos_;
      }
      if (out->size() > lim_.max_string_bytes)
        return limit("JSON string exceeds the " + std::to_string(lim_.max_string_bytes) + "-byte cap");
    }
    return Status{};
  }

  Status number(Json* out) {
    const size_t start = pos_;
    const bool neg = in_[pos_] == '-';
    if (neg) ++pos_;
    if (pos_ >= n_ || !(in_[pos_] >= '0' && in_[pos_] <= '9')) return err("invalid number");
    if (in_[pos_] == '0') {
      ++pos_;
      if (pos_ < n_ && in_[pos_] >= '0' && in_[pos_] <= '9') return err("leading zero in number");
    } else {
      while (pos_ < n_ && in_[pos_] >= '0' && in_[pos_] <= '9') ++pos_;
    }
    bool integer = true;
    if (pos_ < n_ && in_[pos_] == '.') {
      integer = false;
      ++pos_;
      if (pos_ >= n_ || !(in_[pos_] >= '0' && in_[pos_] <= '9')) return err("invalid fraction");
      while (pos_ < n_ && in_[pos_] >= '0' && in_[pos_] <= '9') ++pos_;
    }
    if (pos_ < n_ && (in_[pos_] == 'e' || in_[pos_] == 'E')) {
      integer = false;
      ++pos_;
      if (pos_ < n_ && (in_[pos_] == '+' || in_[pos_] == '-')) ++pos_;
      if (pos_ >= n_ || !(in_[pos_] >= '0' && in_[pos_] <= '9')) return err("invalid exponent");
      while (pos_ < n_ && in_[pos_] >= '0' && in_[pos_] <= '9') ++pos_;
    }
    const std::string text((const char*)in_ + start, pos_ - start);
    if (integer) {
      // exact when it fits u64 (non-negative) or i64 (negative), else a double
      const char* digits = text.c_str() + (neg ? 1 : 0);
      unsigned __int128 v = 0;
      bool fits = true;
      for (const char* d = digits; *d; ++d) {
        v = v * 10 + (unsigned)(*d - '0');
        if (v > (unsigned __int128)UINT64_MAX) {
          fits = false;
          break;
        }
      }
      if (fits && !neg) {
        out->kind = Json::kUnsigned;
        out->u = (uint64_t)v;
        return Status{};
      }
      if (fits && neg && v <= (unsigned __int128)INT64_MAX + 1) {
        out->kind = Json::kSigned;
        out->i = v == (unsigned __int128)INT64_MAX + 1 ? INT64_MIN : -(int64_t)v;
        return Status{};
      }
    }
    const double d = std::strtod(text.c_str(), nullptr);
    if (!std::isfinite(d)) return err("number is not finite");
    out->kind = Json::kFloat;
    out->f = d;
    return Status{};
  }
};

// typed accessors (tokenizer.rs:1000-1046): wrong type -> Corrupt
Status need_object(const Json* v, const std::string& ctx) {
  return v->kind == Json::kObject ? Status{} : corrupt("tokenizer " + ctx + " must be a JSON object");
}
Status need_array(const Json* v, const std::string& ctx) {
  return v->kind == Json::kArray ? Status{} : corrupt("tokenizer " + ctx + " must be a JSON array");
}
Status need_string(const Json* v, const std::string& ctx, const std::string** s) {
  if (v->kind != Json::kString) return corrupt("tokenizer " + ctx + " must be a string");
  *s = &v->s;
  return Status{};
}
Status need_bool(const Json* v, const std::string& ctx, bool* b) {
  if (v->kind != Json::kBool) return corrupt("tokenizer " + ctx + " must be a boolean");
  *b = v->b;
  return Status{};
}
Status need_unsigned(const Json* v, const std::string& ctx, uint64_t* u) {
  if (v->kind == Json::kUnsigned) {
    *u = v->u;
    return Status{};
  }
  return corrupt("tokenizer " + ctx + " must be an unsigned integer");
}
Status need_null(const Json* v, const std::string& ctx) {
  return v->kind == Json::kNull ? Status{} : unsupported("tokenizer " + ctx + " is not null");
}
// A required member; a missing one -> Corrupt(`missing`).
Status member(const Json* obj, const char* key, const std::string& missing, const Json** out) {
  *out = obj->get(key);
  return *out ? Status{} : corrupt(missing);
}

#define SVL_TRY(expr)           \
  do {                          \
    Status st_ = (expr);        \
    if (!st_.ok()) return st_;  \
  } while (0)

// The value of a {"String": s} pattern member.
Status pattern_string(const Json* obj, const char* owner, const std::string** s) {
  const Json* pat;
  SVL_TRY(member(obj, "pattern", std::string(owner) + " is missing pattern", &pat));
  SVL_TRY(need_object(pat, std::string(owner) + ".pattern"));
  const Json* str;
  SVL_TRY(member(pat, "String", std::string(owner) + " pattern is missing String", &str));
  return need_string(str, std::string(owner) + ".pattern.String", s);
}

Status type_of(const Json* obj, const std::string& owner, const std::string** t) {
  const Json* v;
  SVL_TRY(member(obj, "type", owner + " is missing type", &v));
  return need_string(v, owner + ".type", t);
}

const char* kMarker = "\xE2\x96\x81";  // U+2581, the SentencePiece space marker
constexpr uint32_t kMarkerCp = 0x2581;

// ------------------------------------------------------------- tokenizer --
struct AddedToken {
  std::string text;
  uint32_t id;
};

struct Merge {
  uint32_t rank, merged;
};

inline uint64_t pair_key(uint32_t l, uint32_t r) { return ((uint64_t)l << 32) | r; }

}  // namespace

struct svl_tokenizer {
  std::unordered_map<std::string, uint32_t> vocab;
  std::unordered_map<uint32_t, std::string> id_to_token;
  std::unordered_map<uint32_t, uint32_t> char_ids;  // scalar value -> id of its one-character token
  uint32_t byte_ids[256] = {};
  std::unordered_map<uint64_t, Merge> merges;
  std::vector<std::pair<uint32_t, uint32_t>> rank_pair;  // rank -> (left, right)
  std::vector<AddedToken> added;                         // longest first, then by id
  std::vector<uint32_t> added_by_byte[256];              // indices into `added` by first byte, same order
  std::unordered_set<uint32_t> special;
  uint32_t unk_id = 0, bos_id = 0, eos_id = 0, pad_id = 0, max_token_id = 0;
  bool has_pad = false;

  Status load(const Json& root);
  Status encode(const unsigned char* text, size_t n, bool add_special, std::vector<uint32_t>* ids) const;
  Status decode(const uint32_t* ids, size_t n, bool skip_special, std::string* out) const;

 private:
  Status encode_segment(std::vector<uint32_t>* symbols, std::vector<uint32_t>* ids) const;
  void merge_symbols(std::vector<uint32_t>* symbols) const;
};

namespace {

Status token_limit(size_t count) {
  if (count > SVL_TOKENIZER_MAX_TOKENS)
    return limit("tokenization exceeds the " + std::to_string(SVL_TOKENIZER_MAX_TOKENS) + "-token cap");
  return Status{};
}

// tokenizer.rs:575-620
Status validate_normalizer(const Json* v) {
  SVL_TRY(need_object(v, "normalizer"));
  const std::string* t;
  SVL_TRY(type_of(v, "normalizer", &t));
  if (*t != "Replace") return unsupported("tokenizer normalizer is not a Replace normalizer");
  const std::string* s;
  SVL_TRY(pattern_string(v, "normalizer", &s));
  if (*s != " ") return unsupported("tokenizer normalizer does not replace a space");
  const Json* c;
  SVL_TRY(member(v, "content", "normalizer is missing content", &c));
  const std::string* cs;
  SVL_TRY(need_string(c, "normalizer.content", &cs));
  if (*cs != kMarker) return unsupported("tokenizer normalizer does not use the expected space marker");
  return Status{};
}

// tokenizer.rs:623-676
Status validate_pre_tokenizer(const Json* v) {
  SVL_TRY(need_object(v, "pre_tokenizer"));
  const std::string* t;
  SVL_TRY(type_of(v, "pre_tokenizer", &t));
  if (*t != "Split") return unsupported("tokenizer pre_tokenizer is not a Split pre-tokenizer");
  const std::string* s;
  SVL_TRY(pattern_string(v, "pre_tokenizer", &s));
  if (*s != " ") return unsupported("tokenizer pre_tokenizer does not split on a space");
  const Json* b;
  SVL_TRY(member(v, "behavior", "pre_tokenizer is missing behavior", &b));
  const std::string* bs;
  SVL_TRY(need_string(b, "pre_tokenizer.behavior", &bs));
  if (*bs != "MergedWithPrevious") return unsupported("tokenizer pre_tokenizer does not use MergedWithPrevious");
  const Json* inv;
  SVL_TRY(member(v, "invert", "pre_tokenizer is missing invert", &inv));
  bool invert;
  SVL_TRY(need_bool(inv, "pre_tokenizer.invert", &invert));
  if (invert) return unsupported("tokenizer pre_tokenizer is inverted");
  return Status{};
}

// The special-token name of one TemplateProcessing part (tokenizer.rs:977-990).
Status special_part(const Json* v, const std::string& ctx, const std::string** name) {
  SVL_TRY(need_object(v, ctx));
  const Json* sp;
  SVL_TRY(member(v, "SpecialToken", ctx + " is missing SpecialToken", &sp));
  SVL_TRY(need_object(sp, ctx));
  const Json* id;
  SVL_TRY(member(sp, "id", ctx + " is missing id", &id));
  return need_string(id, ctx, name);
}

// tokenizer.rs:679-735
Status validate_post_processor(const Json* v, const std::unordered_map<std::string, uint32_t>& vocab, uint32_t* bos,
                               uint32_t* eos) {
  SVL_TRY(need_object(v, "post_processor"));
  const std::string* t;
  SVL_TRY(type_of(v, "post_processor", &t));
  if (*t != "TemplateProcessing") return unsupported("tokenizer post_processor is not TemplateProcessing");
  const Json* single;
  SVL_TRY(member(v, "single", "post_processor is missing single", &single));
  SVL_TRY(need_array(single, "post_processor.single"));
  if (single->items.size() != 3) return unsupported("tokenizer post_processor single template must have three parts");
  const std::string* first;
  SVL_TRY(special_part(&single->items[0], "post_processor.single[0]", &first));
  if (*first != "<bos>") return unsupported("tokenizer post_processor does not prepend <bos>");
  SVL_TRY(need_object(&single->items[1], "post_processor.single[1]"));
  if (!single->items[1].get("Sequence")) return unsupported("tokenizer post_processor middle part is not a Sequence");
  const std::string* third;
  SVL_TRY(special_part(&single->items[2], "post_processor.single[2]", &third));
  if (*third != "<eos>") return unsupported("tokenizer post_processor does not append <eos>");
  auto b = vocab.find("<bos>");
  if (b == vocab.end()) return corrupt("tokenizer vocabulary is missing <bos>");
  auto e = vocab.find("<eos>");
  if (e == vocab.end()) return corrupt("tokenizer vocabulary is missing <eos>");
  *bos = b->second;
  *eos = e->second;
  return Status{};
}

// tokenizer.rs:738-835
Status validate_decoder(const Json* v) {
  SVL_TRY(need_object(v, "decoder"));
  const std::string* t;
  SVL_TRY(type_of(v, "decoder", &t));
  if (*t != "Sequence") return unsupported("tokenizer decoder is not a Sequence decoder");
  const Json* ds;
  SVL_TRY(member(v, "decoders", "decoder is missing decoders", &ds));
  SVL_TRY(need_array(ds, "decoder.decoders"));
  if (ds->items.size() != 3) return unsupported("tokenizer decoder chain must have three stages");
  const Json* rep = &ds->items[0];
  SVL_TRY(need_object(rep, "decoder.decoders[0]"));
  const std::string* rt;
  SVL_TRY(type_of(rep, "decoder stage", &rt));
  if (*rt != "Replace") return unsupported("tokenizer decoder first stage is not Replace");
  const std::string* s;
  SVL_TRY(pattern_string(rep, "decoder Replace", &s));
  if (*s != kMarker) return unsupported("tokenizer decoder does not replace the space marker");
  const Json* c;
  SVL_TRY(member(rep, "content", "decoder Replace is missing content", &c));
  const std::string* cs;
  SVL_TRY(need_string(c, "decoder.decoders[0].content", &cs));
  if (*cs != " ") return unsupported("tokenizer decoder does not replace the marker with a space");
  const Json* bf = &ds->items[1];
  SVL_TRY(need_object(bf, "decoder.decoders[1]"));
  const std::string* bt;
  SVL_TRY(type_of(bf, "decoder stage", &bt));
  if (*bt != "ByteFallback") return unsupported("tokenizer decoder second stage is not ByteFallback");
  const Json* fu = &ds->items[2];
  SVL_TRY(need_object(fu, "decoder.decoders[2]"));
  const std::string* ft;
  SVL_TRY(type_of(fu, "decoder stage", &ft));
  if (*ft != "Fuse") return unsupported("tokenizer decoder third stage is not Fuse");
  return Status{};
}

// <0xXX> -> the byte (tokenizer.rs:993-998: two characters read as a
// base-16 u8, which admits a leading '+')
bool byte_token(const std::string& t, uint8_t* b) {
  if (t.size() != 6 || t.compare(0, 3, "<0x") != 0 || t[5] != '>') return false;
  auto hv = [](char c) -> int {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
  };
  const int h = hv(t[3]), l = hv(t[4]);
  if (t[3] == '+' && l >= 0) {
    *b = (uint8_t)l;
    return true;
  }
  if (h < 0 || l < 0) return false;
  *b = (uint8_t)(h * 16 + l);
  return true;
}

}  // namespace

// tokenizer.rs:110-385, in the reference's order of checks
Status svl_tokenizer::load(const Json& root) {
  if (root.kind != Json::kObject) return corrupt("tokenizer is missing model");
  const Json* model;
  SVL_TRY(member(&root, "model", "tokenizer is missing model", &model));
  SVL_TRY(need_object(model, "model"));
  const std::string* mtype;
  SVL_TRY(type_of(model, "tokenizer model", &mtype));
  if (*mtype != "BPE") return unsupported("tokenizer model " + *mtype + "; only BPE is implemented");
  const Json* v;
  bool flag;
  SVL_TRY(member(model, "byte_fallback", "tokenizer model is missing byte_fallback", &v));
  SVL_TRY(need_bool(v, "model.byte_fallback", &flag));
  if (!flag) return unsupported("tokenizer without byte fallback is not supported");
  SVL_TRY(member(model, "fuse_unk", "tokenizer model is missing fuse_unk", &v));
  SVL_TRY(need_bool(v, "model.fuse_unk", &flag));
  if (!flag) return unsupported("tokenizer with fuse_unk disabled is not supported");
  SVL_TRY(member(model, "ignore_merges", "tokenizer model is missing ignore_merges", &v));
  SVL_TRY(need_bool(v, "model.ignore_merges", &flag));
  if (flag) return unsupported("tokenizer with ignore_merges enabled is not supported");
  SVL_TRY(member(model, "continuing_subword_prefix", "tokenizer model is missing continuing_subword_prefix", &v));
  SVL_TRY(need_null(v, "model.continuing_subword_prefix"));
  SVL_TRY(member(model, "end_of_word_suffix", "tokenizer model is missing end_of_word_suffix", &v));
  SVL_TRY(need_null(v, "model.end_of_word_suffix"));
  SVL_TRY(member(model, "dropout", "tokenizer model is missing dropout", &v));
  SVL_TRY(need_null(v, "model.dropout"));

  const Json* vocab_v;
  SVL_TRY(member(model, "vocab", "tokenizer model is missing vocab", &vocab_v));
  SVL_TRY(need_object(vocab_v, "model.vocab"));
  if (vocab_v->items.size() > 1000000)
    return limit("tokenizer vocabulary has " + std::to_string(vocab_v->items.size()) +
                 " entries, above the 1000000-entry cap");
  vocab.reserve(vocab_v->items.size() * 2);
  id_to_token.reserve(vocab_v->items.size() * 2);
  for (size_t k = 0; k < vocab_v->items.size(); ++k) {
    uint64_t id;
    SVL_TRY(need_unsigned(&vocab_v->items[k], "model.vocab id", &id));
    if (id > UINT32_MAX) return limit("tokenizer vocabulary id does not fit u32");
    if (!vocab.emplace(vocab_v->keys[k], (uint32_t)id).second) return corrupt("duplicate tokenizer vocabulary token");
    if (!id_to_token.emplace((uint32_t)id, vocab_v->keys[k]).second)
      return corrupt("duplicate tokenizer vocabulary id");
  }
  for (const auto& kv : vocab) {
    const unsigned char* p = (const unsigned char*)kv.first.data();
    if (kv.first.empty()) continue;
    uint32_t cp;
    const int len = utf8_next(p, 0, &cp);
    if ((size_t)len == kv.first.size()) char_ids[cp] = kv.second;
  }
  if (!char_ids.count(kMarkerCp)) return corrupt("tokenizer vocabulary is missing the space marker token");
  for (int b = 0; b < 256; ++b) {
    char name[8];
    std::snprintf(name, sizeof name, "<0x%02X>", b);
    auto it = vocab.find(name);
    if (it == vocab.end()) return corrupt(std::string("tokenizer vocabulary is missing byte token ") + name);
    byte_ids[b] = it->second;
  }

  const Json* merges_v;
  SVL_TRY(member(model, "merges", "tokenizer model is missing merges", &merges_v));
  SVL_TRY(need_array(merges_v, "model.merges"));
  if (merges_v->items.size() > 1000000)
    return limit("tokenizer has " + std::to_string(merges_v->items.size()) + " merges, above the 1000000-merge cap");
  merges.reserve(merges_v->items.size() * 2);
  rank_pair.reserve(merges_v->items.size());
  for (size_t rank = 0; rank < merges_v->items.size(); ++rank) {
    const Json* pair = &merges_v->items[rank];
    SVL_TRY(need_array(pair, "model.merges entry"));
    if (pair->items.size() != 2) return corrupt("tokenizer merge must contain exactly two strings");
    const std::string *l, *r;
    SVL_TRY(need_string(&pair->items[0], "merge left", &l));
    SVL_TRY(need_string(&pair->items[1], "merge right", &r));
    auto li = vocab.find(*l);
    if (li == vocab.end()) return corrupt("merge left \"" + *l + "\" is not in the vocabulary");
    auto ri = vocab.find(*r);
    if (ri == vocab.end()) return corrupt("merge right \"" + *r + "\" is not in the vocabulary");
    auto mi = vocab.find(*l + *r);
    if (mi == vocab.end()) return corrupt("merge result \"" + *l + *r + "\" is not in the vocabulary");
    if (!merges.emplace(pair_key(li->second, ri->second), Merge{(uint32_t)rank, mi->second}).second)
      return corrupt("duplicate tokenizer merge pair");
    rank_pair.emplace_back(li->second, ri->second);
  }

  const Json* unk_v;
  SVL_TRY(member(model, "unk_token", "tokenizer model is missing unk_token", &unk_v));
  const std::string* unk;
  SVL_TRY(need_string(unk_v, "model.unk_token", &unk));
  auto ui = vocab.find(*unk);
  if (ui == vocab.end()) return corrupt("unknown token \"" + *unk + "\" is not in the vocabulary");
  unk_id = ui->second;

  const Json* added_v;
  SVL_TRY(member(&root, "added_tokens", "tokenizer is missing added_tokens", &added_v));
  SVL_TRY(need_array(added_v, "added_tokens"));
  if (added_v->items.size() > 10000)
    return limit("tokenizer has " + std::to_string(added_v->items.size()) +
                 " added tokens, above the 10000-token cap");
  std::unordered_set<uint32_t> seen;
  for (const Json& d : added_v->items) {
    SVL_TRY(need_object(&d, "added token"));
    const Json* c;
    SVL_TRY(member(&d, "content", "added token is missing content", &c));
    const std::string* text;
    SVL_TRY(need_string(c, "added token content", &text));
    if (text->empty()) return corrupt("added token content must not be empty");
    const Json* idv;
    SVL_TRY(member(&d, "id", "added token is missing id", &idv));
    uint64_t id;
    SVL_TRY(need_unsigned(idv, "added token id", &id));
    if (id > UINT32_MAX) return limit("added token id does not fit u32");
    if (!seen.insert((uint32_t)id).second) return corrupt("duplicate added token id");
    if (!id_to_token.count((uint32_t)id))
      return corrupt("added token \"" + *text + "\" has id " + std::to_string(id) + " outside the vocabulary");
    const Json* sv;
    SVL_TRY(member(&d, "special", "added token is missing special", &sv));
    bool is_special;
    SVL_TRY(need_bool(sv, "added token special", &is_special));
    if (is_special) special.insert((uint32_t)id);
    added.push_back(AddedToken{*text, (uint32_t)id});
  }
  std::sort(added.begin(), added.end(), [](const AddedToken& a, const AddedToken& b) {
    return a.text.size() != b.text.size() ? a.text.size() > b.text.size() : a.id < b.id;
  });
  for (size_t k = 0; k < added.size(); ++k) added_by_byte[(unsigned char)added[k].text[0]].push_back((uint32_t)k);

  const Json* part;
  SVL_TRY(member(&root, "normalizer", "tokenizer is missing normalizer", &part));
  SVL_TRY(validate_normalizer(part));
  SVL_TRY(member(&root, "pre_tokenizer", "tokenizer is missing pre_tokenizer", &part));
  SVL_TRY(validate_pre_tokenizer(part));
  SVL_TRY(member(&root, "post_processor", "tokenizer is missing post_processor", &part));
  SVL_TRY(validate_post_processor(part, vocab, &bos_id, &eos_id));
  SVL_TRY(member(&root, "decoder", "tokenizer is missing decoder", &part));
  SVL_TRY(validate_decoder(part));

  auto pi = vocab.find("<pad>");
  has_pad = pi != vocab.end();
  pad_id = has_pad ? pi->second : 0;
  max_token_id = 0;
  for (const auto& kv : id_to_token) max_token_id = std::max(max_token_id, kv.first);
  return Status{};
}

// BPE over one normalised segment (see the file comment for the rounds).
void svl_tokenizer::merge_symbols(std::vector<uint32_t>* symbols) const {
  std::vector<uint32_t>& sym = *symbols;
  const int n = (int)sym.size();
  if (n < 2) return;
  std::vector<int> next(n), prev(n);
  std::vector<char> alive(n, 1);
  for (int i = 0; i < n; ++i) {
    next[i] = i + 1 < n ? i + 1 : -1;
    prev[i] = i - 1;
  }
  // (rank << 32 | left position), smallest first
  std::priority_queue<uint64_t, std::vector<uint64_t>, std::greater<uint64_t>> heap;
  auto push_pair = [&](int left) {
    if (left < 0 || next[left] < 0) return;
    auto it = merges.find(pair_key(sym[left], sym[next[left]]));
    if (it != merges.end()) heap.push(((uint64_t)it->second.rank << 32) | (uint32_t)left);
  };
  auto live_rank = [&](uint64_t e, uint32_t* rank) {
    const int left = (int)(uint32_t)e;
    if (!alive[left] || next[left] < 0) return false;
    auto it = merges.find(pair_key(sym[left], sym[next[left]]));
    if (it == merges.end() || it->second.rank != (uint32_t)(e >> 32)) return false;
    *rank = it->second.rank;
    return true;
  };
  for (int i = 0; i + 1 < n; ++i) push_pair(i);
  std::vector<int> occ, changed;
  for (;;) {
    uint32_t rank = 0;
    while (!heap.empty() && !live_rank(heap.top(), &rank)) heap.pop();
    if (heap.empty()) break;
    occ.clear();
    while (!heap.empty() && (uint32_t)(heap.top() >> 32) == rank) {
      occ.push_back((int)(uint32_t)heap.top());
      heap.pop();
    }
    std::sort(occ.begin(), occ.end());
    occ.erase(std::unique(occ.begin(), occ.end()), occ.end());
    const uint32_t L = rank_pair[rank].first, R = rank_pair[rank].second;
    const uint32_t M = merges.find(pair_key(L, R))->second.merged;
    changed.clear();
    for (int left : occ) {
      if (!alive[left]) continue;  // the right symbol of this round's previous merge
      const int right = next[left];
      if (right < 0 || sym[left] != L || sym[right] != R) continue;
      sym[left] = M;
      alive[right] = 0;
      next[left] = next[right];
      if (next[right] >= 0) prev[next[right]] = left;
      changed.push_back(left);
    }
    for (int left : changed) {
      if (!alive[left]) continue;
      push_pair(prev[left]);
      push_pair(left);
    }
  }
  size_t w = 0;
  for (int i = 0; i >= 0 && i < n; i = next[i]) sym[w++] = sym[i];
  sym.resize(w);
}

// tokenizer.rs:520-546
Status svl_tokenizer::encode_segment(std::vector<uint32_t>* symbols, std::vector<uint32_t>* ids) const {
  if (symbols->size() > SVL_TOKENIZER_MAX_TOKENS) return token_limit(symbols->size());
  merge_symbols(symbols);
  ids->insert(ids->end(), symbols->begin(), symbols->end());
  symbols->clear();
  return token_limit(ids->size());
}

// tokenizer.rs:392-434 (text already checked to be UTF-8)
Status svl_tokenizer::encode(const unsigned char* text, size_t n, bool add_special, std::vector<uint32_t>* ids) const {
  if (n > SVL_TOKENIZER_MAX_INPUT_BYTES)
    return limit("tokenizer input is " + std::to_string(n) + " bytes, above the " +
                 std::to_string(SVL_TOKENIZER_MAX_INPUT_BYTES) + "-byte cap");
  ids->clear();
  if (add_special) ids->push_back(bos_id);
  std::vector<uint32_t> symbols;
  size_t i = 0;
  while (i < n) {
    // the first added token, in (longest, lowest id) order, that starts here
    // (tokenizer.rs:503-507); only those beginning with this byte can match
    const AddedToken* hit = nullptr;
    for (uint32_t k : added_by_byte[text[i]]) {
      const AddedToken& a = added[k];
      if (a.text.size() <= n - i && std::memcmp(text + i, a.text.data(), a.text.size()) == 0) {
        hit = &a;
        break;
      }
    }
    if (hit) {
      if (!symbols.empty()) SVL_TRY(encode_segment(&symbols, ids));
      ids->push_back(hit->id);
      SVL_TRY(token_limit(ids->size()));
      i += hit->text.size();
      continue;
    }
    uint32_t cp;
    const int len = utf8_next(text, i, &cp);
    const uint32_t norm = cp == ' ' ? kMarkerCp : cp;
    auto it = char_ids.find(norm);
    if (it != char_ids.end()) {
      symbols.push_back(it->second);
    } else {
      std::string bytes;
      utf8_append(&bytes, norm);
      for (unsigned char b : bytes) symbols.push_back(byte_ids[b]);
    }
    i += len;
  }
  if (!symbols.empty()) SVL_TRY(encode_segment(&symbols, ids));
  if (add_special) ids->push_back(eos_id);
  return token_limit(ids->size());
}

// tokenizer.rs:441-466
Status svl_tokenizer::decode(const uint32_t* ids, size_t n, bool skip_special, std::string* out) const {
  out->clear();
  for (size_t k = 0; k < n; ++k) {
    auto it = id_to_token.find(ids[k]);
    if (it == id_to_token.end()) return corrupt("cannot decode unknown token id " + std::to_string(ids[k]));
    if (skip_special && special.count(ids[k])) continue;
    uint8_t b;
    if (byte_token(it->second, &b)) {
      out->push_back((char)b);
      continue;
    }
    const std::string& t = it->second;
    for (size_t j = 0; j < t.size();) {
      if (j + 3 <= t.size() && std::memcmp(t.data() + j, kMarker, 3) == 0) {
        out->push_back(' ');
        j += 3;
      } else {
        out->push_back(t[j]);
        ++j;
      }
    }
  }
  if (!utf8_valid((const unsigned char*)out->data(), out->size()))
    return corrupt("decoded token sequence is not valid UTF-8");
  return Status{};
}

// ----------------------------------------------------------------- C ABI --
extern "C" {

int svl_tokenizer_create(const char* json, size_t json_len, svl_tokenizer** out, char* err, size_t err_len) {
  if (!out || (!json && json_len)) {
    put_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  *out = nullptr;
  const JsonLimits lim;
  if (json_len > lim.max_input_bytes) {
    put_err(err, err_len, "JSON input is " + std::to_string(json_len) + " bytes, above the " +
                              std::to_string(lim.max_input_bytes) + "-byte cap");
    return SVL_LIMIT_EXCEEDED;
  }
  if (!utf8_valid((const unsigned char*)json, json_len)) {
    put_err(err, err_len, "tokenizer file is not valid UTF-8");
    return SVL_CORRUPT;
  }
  try {
    Json root;
    Status st = JsonReader(json, json_len, lim).parse(&root);
    std::unique_ptr<svl_tokenizer> t(new svl_tokenizer());
    if (st.ok()) st = t->load(root);
    if (!st.ok()) {
      put_err(err, err_len, st.msg);
      return st.code;
    }
    *out = t.release();
    return SVL_OK;
  } catch (const std::bad_alloc&) {
    put_err(err, err_len, "out of host memory");
    return SVL_LIMIT_EXCEEDED;
  }
}

void svl_tokenizer_destroy(svl_tokenizer* tokenizer) { delete tokenizer; }

int svl_tokenizer_encode(const svl_tokenizer* tokenizer, const char* text, size_t text_len, int add_special,
                         uint32_t* ids, size_t capacity, size_t* n_ids, char* err, size_t err_len) {
  if (!tokenizer || !n_ids || (!text && text_len) || (!ids && capacity)) {
    put_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  *n_ids = 0;
  if (text_len > SVL_TOKENIZER_MAX_INPUT_BYTES) {
    put_err(err, err_len, "tokenizer input is " + std::to_string(text_len) + " bytes, above the " +
                              std::to_string(SVL_TOKENIZER_MAX_INPUT_BYTES) + "-byte cap");
    return SVL_LIMIT_EXCEEDED;
  }
  if (!utf8_valid((const unsigned char*)text, text_len)) {
    put_err(err, err_len, "tokenizer input is not valid UTF-8");
    return SVL_USAGE;
  }
  try {
    std::vector<uint32_t> v;
    Status st = tokenizer->encode((const unsigned char*)text, text_len, add_special != 0, &v);
    if (!st.ok()) {
      put_err(err, err_len, st.msg);
      return st.code;
    }
    *n_ids = v.size();
    if (v.size() > capacity) {
      put_err(err, err_len, "id buffer holds " + std::to_string(capacity) + " ids, " + std::to_string(v.size()) +
                                " are needed");
      return SVL_USAGE;
    }
    if (!v.empty()) std::memcpy(ids, v.data(), v.size() * sizeof(uint32_t));
    return SVL_OK;
  } catch (const std::bad_alloc&) {
    put_err(err, err_len, "out of host memory");
    return SVL_LIMIT_EXCEEDED;
  }
}

int svl_tokenizer_encode_batch(const svl_tokenizer* tokenizer, const char* bytes, const uint64_t* offsets, uint64_t n,
                               int add_special, uint32_t threads, uint32_t* ids, uint64_t capacity,
                               uint64_t* cu_seqlens, uint64_t* failed, char* err, size_t err_len) {
  if (failed) *failed = n;
  if (!tokenizer || !offsets || !cu_seqlens || (!bytes && offsets[n]) || (!ids && capacity)) {
    put_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  for (uint64_t i = 0; i < n; ++i)
    if (offsets[i + 1] < offsets[i]) {
      put_err(err, err_len, "text offsets must not decrease");
      return SVL_USAGE;
    }
  try {
    // texts are dealt in contiguous ranges of roughly equal byte counts
    uint32_t nt = threads ? threads : std::max(1u, std::thread::hardware_concurrency());
    nt = (uint32_t)std::min<uint64_t>(nt, std::max<uint64_t>(n, 1));
    std::vector<uint64_t> lo(nt + 1, n);
    lo[0] = 0;
    const uint64_t total = offsets[n] - offsets[0];
    uint64_t i = 0;
    for (uint32_t w = 1; w < nt; ++w) {
      const uint64_t target = offsets[0] + total * w / nt;
      while (i < n && offsets[i] < target) ++i;
      lo[w] = std::max<uint64_t>(i, lo[w - 1]);
    }
    std::vector<std::vector<uint32_t>> part(nt);
    std::vector<std::vector<uint64_t>> lens(nt);
    std::vector<Status> status(nt);
    std::vector<uint64_t> bad(nt, n);
    // tokenises range w; i is the text in progress (read by the handler below)
    auto run_range = [&](uint32_t w, uint64_t& i) {
      std::vector<uint32_t> one;
      for (; i < lo[w + 1]; ++i) {
        const unsigned char* t = (const unsigned char*)bytes + offsets[i];
        const uint64_t len = offsets[i + 1] - offsets[i];
        Status st;
        if (len > SVL_TOKENIZER_MAX_INPUT_BYTES)
          st = limit("tokenizer input is " + std::to_string(len) + " bytes, above the " +
                     std::to_string(SVL_TOKENIZER_MAX_INPUT_BYTES) + "-byte cap");
        else if (!utf8_valid(t, len))
          st = fail(SVL_USAGE, "tokenizer input is not valid UTF-8");
        else
          st = tokenizer->encode(t, len, add_special != 0, &one);
        if (!st.ok()) {
          status[w] = st;
          bad[w] = i;
          return;
        }
        part[w].insert(part[w].end(), one.begin(), one.end());
        lens[w].push_back(one.size());
      }
    };
    // a worker that runs out of memory records it here (no allocation in the
    // handler) instead of letting the exception escape its thread
    std::vector<char> oom(nt, 0);
    auto work = [&](uint32_t w) {
      uint64_t i = lo[w];
      try {
        run_range(w, i);
      } catch (...) {
        oom[w] = 1;
        bad[w] = i;
      }
    };
    std::vector<std::thread> pool;
    pool.reserve(nt);
    uint32_t started = 1;
    try {
      for (; started < nt; ++started) pool.emplace_back(work, started);
    } catch (const std::system_error&) {
      // fewer host threads than asked: the calling thread runs the ranges not started
    }
    for (uint32_t w = started; w < nt; ++w) work(w);
    work(0);
    for (auto& th : pool) th.join();
    for (uint32_t w = 0; w < nt; ++w) {  // ranges are in text order: the first failing range has the lowest index
      if (oom[w]) {
        if (failed) *failed = bad[w];
        put_err(err, err_len, "out of host memory");
        return SVL_LIMIT_EXCEEDED;
      }
      if (!status[w].ok()) {
        if (failed) *failed = bad[w];
        put_err(err, err_len, "text " + std::to_string(bad[w]) + ": " + status[w].msg);
        return status[w].code;
      }
    }
    uint64_t count = 0;
    for (const auto& p : part) count += p.size();
    if (count > capacity) {
      put_err(err, err_len, "id buffer holds " + std::to_string(capacity) + " ids, " + std::to_string(count) +
                                " are needed");
      return SVL_USAGE;
    }
    uint64_t at = 0, k = 0;
    cu_seqlens[0] = 0;
    for (uint32_t w = 0; w < nt; ++w) {
      if (!part[w].empty()) std::memcpy(ids + at, part[w].data(), part[w].size() * sizeof(uint32_t));
      for (uint64_t len : lens[w]) {
        cu_seqlens[k + 1] = cu_seqlens[k] + len;
        ++k;
      }
      at += part[w].size();
    }
    return SVL_OK;
  } catch (const std::bad_alloc&) {
    put_err(err, err_len, "out of host memory");
    return SVL_LIMIT_EXCEEDED;
  } catch (const std::system_error&) {
    put_err(err, err_len, "could not start a host thread");
    return SVL_INTERNAL;
  }
}

int svl_tokenizer_decode(const svl_tokenizer* tokenizer, const uint32_t* ids, size_t n_ids, int skip_special,
                         char* out, size_t capacity, size_t* out_len, char* err, size_t err_len) {
  if (!tokenizer || !out_len || (!ids && n_ids)) {
    put_err(err, err_len, "null argument");
    return SVL_USAGE;
  }
  *out_len = 0;
  try {
    std::string s;
    Status st = tokenizer->decode(ids, n_ids, skip_special != 0, &s);
    if (!st.ok()) {
      put_err(err, err_len, st.msg);
      return st.code;
    }
    *out_len = s.size();
    if (!out) return SVL_OK;
    if (s.size() > capacity) {
      put_err(err, err_len, "output buffer holds " + std::to_string(capacity) + " bytes, " +
                                std::to_string(s.size()) + " are needed");
      return SVL_USAGE;
    }
    if (!s.empty()) std::memcpy(out, s.data(), s.size());
    return SVL_OK;
  } catch (const std::bad_alloc&) {
    put_err(err, err_len, "out of host memory");
    return SVL_LIMIT_EXCEEDED;
  }
}

int svl_tokenizer_token_id(const svl_tokenizer* tokenizer, const char* token, size_t token_len, uint32_t* id) {
  if (!tokenizer || (!token && token_len)) return 0;
  auto it = tokenizer->vocab.find(std::string(token ? token : "", token_len));
  if (it == tokenizer->vocab.end()) return 0;
  if (id) *id = it->second;
  return 1;
}

int svl_tokenizer_token(const svl_tokenizer* tokenizer, uint32_t id, const char** token, size_t* token_len) {
  if (!tokenizer) return 0;
  auto it = tokenizer->id_to_token.find(id);
  if (it == tokenizer->id_to_token.end()) return 0;
  if (token) *token = it->second.data();
  if (token_len) *token_len = it->second.size();
  return 1;
}

int svl_tokenizer_is_special(const svl_tokenizer* tokenizer, uint32_t id) {
  return tokenizer && tokenizer->special.count(id) ? 1 : 0;
}

int svl_tokenizer_get_info(const svl_tokenizer* tokenizer, svl_tokenizer_info* info) {
  if (!tokenizer || !info) return SVL_USAGE;
  info->vocab_size = tokenizer->vocab.size();
  info->max_token_id = tokenizer->max_token_id;
  info->bos_id = tokenizer->bos_id;
  info->eos_id = tokenizer->eos_id;
  info->unk_id = tokenizer->unk_id;
  info->pad_id = tokenizer->pad_id;
  info->has_pad = tokenizer->has_pad ? 1u : 0u;
  return SVL_OK;
}

}  // extern "C"
