// pw_checkpoint.cpp -- checkpoint ingestion: safetensors and PWEXPRT1 files
// mapped read-only, validated fail-closed, and uploaded into HBM expert banks.
//
// Restates, as C++ behind the C ABI:
//  * MappedSafetensors::open / tensor (src/lib.rs:784-976): the 8-byte
//    little-endian header length (non-zero, at most 256 MiB, a multiple of 8,
//    inside the file), a strict JSON header with unique keys everywhere, known
//    dtypes, non-empty shapes without zero dimensions, byte counts that match
//    shape x dtype, payload ranges inside the file that do not overlap, at
//    least one tensor;
//  * the PWEXPRT1 expert container (docs/EXPERT_CONTAINER.md,
//    repack_expert_container / verify_expert_container src/lib.rs:7190-7347):
//    magic, u64 header length, JSON header (schema 1, 64-byte alignment),
//    tensors at aligned, increasing, in-range payload offsets, each with a
//    SHA-256 that must match, and no trailing bytes; creation refuses to
//    overwrite and publishes through a verified temporary file and a hard link;
//  * the checkpoint's naming of a routed expert's projections,
//    model.layers.{L}.mlp.experts.{e}.{gate,up,down}_proj.weight with the
//    block scales under the same name + "_scale_inv" (src/text_endpoint.rs:3067).
//
// The JSON reader and SHA-256 are written here from their specifications
// (RFC 8259, FIPS 180-4); no third-party library is involved.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cinttypes>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include <cuda_runtime.h>

#include "pw_cuda.h"
#include "pw_internal.h"

namespace {

constexpr uint64_t kMaxHeaderBytes = 256ull * 1024 * 1024;
constexpr uint64_t kContainerAlignment = 64;
const char kContainerMagic[9] = "PWEXPRT1";

// ------------------------------------------------------------------ errors
struct Error {
  int code = PW_OK;
  std::string text;
};

bool set_err(Error &e, int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  e.code = code;
  e.text = buf;
  return false;
}

void copy_err(const Error &e, char *err, size_t err_len) {
  if (err && err_len) {
    const size_t n = std::min(err_len - 1, e.text.size());
    memcpy(err, e.text.data(), n);
    err[n] = '\0';
  }
}

// ------------------------------------------------------------------- JSON
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  std::string text;  // number literal or string value
  std::vector<Json> items;
  std::vector<std::pair<std::string, Json>> members;

  const Json *get(const char *key) const {
    for (const auto &m : members)
      if (m.first == key) return &m.second;
    return nullptr;
  }
  // A non-negative integer literal without fraction or exponent that fits u64.
  bool as_u64(uint64_t &v) const {
    if (kind != Number || text.empty() || text[0] == '-') return false;
    v = 0;
    for (char c : text) {
      if (c < '0' || c > '9') return false;
      const uint64_t d = (uint64_t)(c - '0');
      if (v > (UINT64_MAX - d) / 10u) return false;
      v = v * 10u + d;
    }
    return true;
  }
};

// Strict RFC 8259 reader: one value, only whitespace after it, valid UTF-8,
// duplicate object keys rejected at every depth (the reference's UniqueJson).
class JsonReader {
 public:
  JsonReader(const char *p, size_t n) : p_(p), end_(p + n) {}
  bool read(Json &out, std::string &err) {
    if (!value(out, 0)) {
      err = err_.empty() ? "malformed JSON" : err_;
      return false;
    }
    ws();
    if (p_ != end_) {
      err = "trailing data after the JSON value";
      return false;
    }
    return true;
  }

 private:
  const char *p_, *end_;
  std::string err_;

  bool fail(const char *what) {
    if (err_.empty()) err_ = what;
    return false;
  }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char *s) {
    const size_t n = strlen(s);
    if ((size_t)(end_ - p_) < n || memcmp(p_, s, n) != 0) return fail("invalid literal");
    p_ += n;
    return true;
  }
  bool value(Json &v, int depth) {
    if (depth > 128) return fail("JSON nested too deeply");
    ws();
    if (p_ >= end_) return fail("unexpected end of JSON");
    switch (*p_) {
      case '{': return object(v, depth);
      case '[': return array(v, depth);
      case '"': v.kind = Json::String; return string(v.text);
      case 't': v.kind = Json::Bool; v.b = true; return lit("true");
      case 'f': v.kind = Json::Bool; v.b = false; return lit("false");
      case 'n': v.kind = Json::Null; return lit("null");
      default: return number(v);
    }
  }
  bool object(Json &v, int depth) {
    v.kind = Json::Object;
    ++p_;
    ws();
    if (p_ < end_ && *p_ == '}') {
      ++p_;
      return true;
    }
    for (;;) {
      ws();
      if (p_ >= end_ || *p_ != '"') return fail("expected an object key");
      std::string key;
      if (!string(key)) return false;
      for (const auto &m : v.members)
        if (m.first == key) return fail("duplicate JSON object key");
      ws();
      if (p_ >= end_ || *p_ != ':') return fail("expected ':'");
      ++p_;
      Json item;
      if (!value(item, depth + 1)) return false;
      v.members.emplace_back(std::move(key), std::move(item));
      ws();
      if (p_ < end_ && *p_ == ',') {
        ++p_;
        continue;
      }
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      return fail("expected ',' or '}'");
    }
  }
  bool array(Json &v, int depth) {
    v.kind = Json::Array;
    ++p_;
    ws();
    if (p_ < end_ && *p_ == ']') {
      ++p_;
      return true;
    }
    for (;;) {
      Json item;
      if (!value(item, depth + 1)) return false;
      v.items.push_back(std::move(item));
      ws();
      if (p_ < end_ && *p_ == ',') {
        ++p_;
        continue;
      }
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      return fail("expected ',' or ']'");
    }
  }
  static void put_utf8(std::string &s, uint32_t cp) {
    if (cp < 0x80) {
      s += (char)cp;
    } else if (cp < 0x800) {
      s += (char)(0xC0 | (cp >> 6));
      s += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      s += (char)(0xE0 | (cp >> 12));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    } else {
      s += (char)(0xF0 | (cp >> 18));
      s += (char)(0x80 | ((cp >> 12) & 0x3F));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    }
  }
  bool hex4(uint32_t &cp) {
    if (end_ - p_ < 4) return fail("short \\u escape");
    cp = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      cp <<= 4;
      if (c >= '0' && c <= '9') cp |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') cp |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') cp |= (uint32_t)(c - 'A' + 10);
      else return fail("bad \\u escape");
    }
    return true;
  }
  // One UTF-8 sequence starting at p_ (first byte >= 0x80), validated.
  bool utf8(std::string &s) {
    const unsigned char c = (unsigned char)*p_;
    int n = 0;
    uint32_t cp = 0, min = 0;
    if ((c & 0xE0) == 0xC0) n = 1, cp = c & 0x1F, min = 0x80;
    else if ((c & 0xF0) == 0xE0) n = 2, cp = c & 0x0F, min = 0x800;
    else if ((c & 0xF8) == 0xF0) n = 3, cp = c & 0x07, min = 0x10000;
    else return fail("invalid UTF-8");
    if (end_ - p_ < n + 1) return fail("truncated UTF-8");
    for (int i = 1; i <= n; ++i) {
      const unsigned char d = (unsigned char)p_[i];
      if ((d & 0xC0) != 0x80) return fail("invalid UTF-8");
      cp = (cp << 6) | (d & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return fail("invalid UTF-8");
    s.append(p_, (size_t)n + 1);
    p_ += n + 1;
    return true;
  }
  bool string(std::string &s) {
    ++p_;
    s.clear();
    while (p_ < end_) {
      const unsigned char c = (unsigned char)*p_;
      if (c == '"') {
        ++p_;
        return true;
      }
      if (c < 0x20) return fail("control character in a JSON string");
      if (c == '\\') {
        if (++p_ >= end_) return fail("unterminated escape");
        const char e = *p_++;
        switch (e) {
          case '"': s += '"'; break;
          case '\\': s += '\\'; break;
          case '/': s += '/'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'n': s += '\n'; break;
          case 'r': s += '\r'; break;
          case 't': s += '\t'; break;
          case 'u': {
            uint32_t cp;
            if (!hex4(cp)) return false;
            if (cp >= 0xD800 && cp <= 0xDBFF) {
              uint32_t lo;
              if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return fail("unpaired surrogate");
              p_ += 2;
              if (!hex4(lo)) return false;
              if (lo < 0xDC00 || lo > 0xDFFF) return fail("unpaired surrogate");
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            } else if (cp >= 0xDC00 && cp <= 0xDFFF) {
              return fail("unpaired surrogate");
            }
            put_utf8(s, cp);
            break;
          }
          default: return fail("bad escape");
        }
        continue;
      }
      if (c >= 0x80) {
        if (!utf8(s)) return false;
        continue;
      }
      s += (char)c;
      ++p_;
    }
    return fail("unterminated string");
  }
  bool number(Json &v) {
    const char *s = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    if (p_ >= end_) return fail("bad number");
    if (*p_ == '0') {
      ++p_;
    } else if (*p_ >= '1' && *p_ <= '9') {
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    } else {
      return fail("unexpected character");
    }
    if (p_ < end_ && *p_ == '.') {
      ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return fail("bad number");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      ++p_;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return fail("bad number");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    v.kind = Json::Number;
    v.text.assign(s, (size_t)(p_ - s));
    return true;
  }
};

std::string json_quote(const std::string &s) {
  std::string o = "\"";
  for (unsigned char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if (c < 0x20) {
          char b[8];
          snprintf(b, sizeof b, "\\u%04x", c);
          o += b;
        } else {
          o += (char)c;
        }
    }
  }
  return o + "\"";
}

// ---------------------------------------------------------------- SHA-256
// FIPS 180-4.
class Sha256 {
 public:
  Sha256() { reset(); }
  void reset() {
    static const uint32_t init[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                     0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    memcpy(h_, init, sizeof h_);
    len_ = 0;
    fill_ = 0;
  }
  void update(const void *data, size_t n) {
    const unsigned char *p = static_cast<const unsigned char *>(data);
    len_ += n;
    if (fill_) {
      const size_t take = std::min(n, (size_t)64 - fill_);
      memcpy(buf_ + fill_, p, take);
      fill_ += take;
      p += take;
      n -= take;
      if (fill_ == 64) {
        block(buf_);
        fill_ = 0;
      }
    }
    while (n >= 64) {
      block(p);
      p += 64;
      n -= 64;
    }
    if (n) {
      memcpy(buf_, p, n);
      fill_ = n;
    }
  }
  std::string hex() {
    const uint64_t bits = len_ * 8u;
    const unsigned char one = 0x80, zero = 0;
    update(&one, 1);
    while (fill_ != 56) update(&zero, 1);
    unsigned char lenb[8];
    for (int i = 0; i < 8; ++i) lenb[i] = (unsigned char)(bits >> (56 - 8 * i));
    update(lenb, 8);
    char out[65];
    for (int i = 0; i < 8; ++i) snprintf(out + 8 * i, 9, "%08x", h_[i]);
    return std::string(out, 64);
  }

 private:
  uint32_t h_[8];
  uint64_t len_;
  unsigned char buf_[64];
  size_t fill_;
  static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
  void block(const unsigned char *p) {
    static const uint32_t k[64] = {
        0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
        0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
        0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
        0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
        0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
        0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
        0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
        0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = ((uint32_t)p[4 * i] << 24) | ((uint32_t)p[4 * i + 1] << 16) | ((uint32_t)p[4 * i + 2] << 8) | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[i] + w[i];
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
    h_[0] += a, h_[1] += b, h_[2] += c, h_[3] += d, h_[4] += e, h_[5] += f, h_[6] += g, h_[7] += h;
  }
};

std::string sha256_hex(const void *data, size_t n) {
  Sha256 s;
  s.update(data, n);
  return s.hex();
}

// ------------------------------------------------------------ mapped file
struct Mapping {
  const unsigned char *base = nullptr;
  size_t bytes = 0;
  ~Mapping() {
    if (base && bytes) munmap(const_cast<unsigned char *>(base), bytes);
  }
};

bool map_file(const char *path, Mapping &m, Error &e) {
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return set_err(e, PW_ERR_IO, "%s: %s", path, strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0) {
    const int er = errno;
    close(fd);
    return set_err(e, PW_ERR_IO, "%s: %s", path, strerror(er));
  }
  m.bytes = (size_t)st.st_size;
  if (m.bytes == 0) {
    close(fd);
    return set_err(e, PW_ERR_FORMAT, "%s: empty file", path);
  }
  void *p = mmap(nullptr, m.bytes, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);  // the mapping keeps its own reference
  if (p == MAP_FAILED) {
    m.bytes = 0;
    return set_err(e, PW_ERR_IO, "%s: mmap: %s", path, strerror(errno));
  }
  m.base = static_cast<const unsigned char *>(p);
  return true;
}

uint64_t le64(const unsigned char *p) {
  uint64_t v = 0;
  for (int i = 7; i >= 0; --i) v = (v << 8) | p[i];
  return v;
}

uint64_t dtype_bytes(const std::string &d) {
  if (d == "BOOL" || d == "U8" || d == "I8" || d == "F8_E4M3" || d == "F8_E4M3FN" || d == "F8_E5M2") return 1;
  if (d == "U16" || d == "I16" || d == "F16" || d == "BF16") return 2;
  if (d == "U32" || d == "I32" || d == "F32") return 4;
  if (d == "U64" || d == "I64" || d == "F64") return 8;
  return 0;
}

bool u64_array(const Json *v, std::vector<uint64_t> &out) {
  if (!v || v->kind != Json::Array) return false;
  out.clear();
  for (const Json &it : v->items) {
    uint64_t x;
    if (!it.as_u64(x)) return false;
    out.push_back(x);
  }
  return true;
}

}  // namespace

// One tensor of an opened file: metadata plus its bytes in the mapping.
struct PwTensorRec {
  std::string name, dtype;
  std::vector<uint64_t> shape;
  uint64_t begin = 0, end = 0;  // source data offsets (safetensors) or payload range
  const unsigned char *data = nullptr;
  uint64_t bytes = 0;
  std::string sha256;           // containers only
};

struct pw_tensor_file {
  std::string path;
  bool container = false;
  Mapping map;
  std::vector<PwTensorRec> tensors;  // sorted by name
  std::map<std::string, size_t> index;
  // container header fields
  std::string source_file, source_sha256;
  uint64_t source_file_bytes = 0;
};

namespace {

// Shape x dtype gives the byte count, or an error.
bool tensor_bytes(const std::string &name, const std::string &dtype, const std::vector<uint64_t> &shape,
                  uint64_t &bytes, Error &e) {
  const uint64_t eb = dtype_bytes(dtype);
  if (!eb) return set_err(e, PW_ERR_FORMAT, "%s: unknown dtype %s", name.c_str(), dtype.c_str());
  if (shape.empty()) return set_err(e, PW_ERR_FORMAT, "%s: empty or zero tensor shape", name.c_str());
  uint64_t n = 1;
  for (uint64_t d : shape) {
    if (d == 0) return set_err(e, PW_ERR_FORMAT, "%s: empty or zero tensor shape", name.c_str());
    if (n > UINT64_MAX / d) return set_err(e, PW_ERR_FORMAT, "%s: shape overflow", name.c_str());
    n *= d;
  }
  if (n > UINT64_MAX / eb) return set_err(e, PW_ERR_FORMAT, "%s: tensor byte overflow", name.c_str());
  bytes = n * eb;
  return true;
}

void finish_index(pw_tensor_file &f) {
  std::sort(f.tensors.begin(), f.tensors.end(),
            [](const PwTensorRec &a, const PwTensorRec &b) { return a.name < b.name; });
  for (size_t i = 0; i < f.tensors.size(); ++i) f.index[f.tensors[i].name] = i;
}

// MappedSafetensors::open (src/lib.rs:784-905).
bool open_safetensors(const char *path, pw_tensor_file &f, Error &e) {
  f.path = path;
  if (!map_file(path, f.map, e)) return false;
  const uint64_t file_bytes = f.map.bytes;
  if (file_bytes < 16) return set_err(e, PW_ERR_FORMAT, "safetensors file is too short");
  const uint64_t header_bytes = le64(f.map.base);
  if (header_bytes == 0 || header_bytes > kMaxHeaderBytes || header_bytes % 8u != 0 || 8u + header_bytes > file_bytes)
    return set_err(e, PW_ERR_FORMAT, "invalid safetensors header length %" PRIu64, header_bytes);
  const uint64_t payload_start = 8u + header_bytes;
  Json header;
  std::string jerr;
  if (!JsonReader(reinterpret_cast<const char *>(f.map.base + 8), header_bytes).read(header, jerr))
    return set_err(e, PW_ERR_FORMAT, "malformed safetensors header: %s", jerr.c_str());
  if (header.kind != Json::Object) return set_err(e, PW_ERR_FORMAT, "safetensors header must be an object");
  const uint64_t payload_bytes = file_bytes - payload_start;
  for (const auto &m : header.members) {
    const std::string &name = m.first;
    if (name == "__metadata__") {
      if (m.second.kind != Json::Object) return set_err(e, PW_ERR_FORMAT, "__metadata__ must be an object");
      continue;
    }
    if (m.second.kind != Json::Object) return set_err(e, PW_ERR_FORMAT, "%s must be an object", name.c_str());
    const Json *dt = m.second.get("dtype");
    if (!dt || dt->kind != Json::String) return set_err(e, PW_ERR_FORMAT, "%s: missing dtype", name.c_str());
    PwTensorRec t;
    t.name = name;
    t.dtype = dt->text;
    if (!dtype_bytes(t.dtype)) return set_err(e, PW_ERR_FORMAT, "%s: unknown dtype %s", name.c_str(), t.dtype.c_str());
    if (!u64_array(m.second.get("shape"), t.shape)) return set_err(e, PW_ERR_FORMAT, "%s: missing shape", name.c_str());
    uint64_t expected = 0;
    if (!tensor_bytes(name, t.dtype, t.shape, expected, e)) return false;
    std::vector<uint64_t> offs;
    if (!u64_array(m.second.get("data_offsets"), offs) || offs.size() != 2)
      return set_err(e, PW_ERR_FORMAT, "%s: missing offsets", name.c_str());
    if (offs[1] < offs[0]) return set_err(e, PW_ERR_FORMAT, "%s: tensor offsets reversed", name.c_str());
    t.begin = offs[0];
    t.end = offs[1];
    t.bytes = t.end - t.begin;
    if (t.bytes != expected)
      return set_err(e, PW_ERR_FORMAT, "%s: shape/dtype requires %" PRIu64 " bytes, got %" PRIu64, name.c_str(),
                     expected, t.bytes);
    if (t.end > payload_bytes) return set_err(e, PW_ERR_FORMAT, "%s: tensor payload exceeds file", name.c_str());
    t.data = f.map.base + payload_start + t.begin;
    f.tensors.push_back(std::move(t));
  }
  if (f.tensors.empty()) return set_err(e, PW_ERR_FORMAT, "safetensors file contains no tensors");
  std::vector<const PwTensorRec *> by_range;
  for (const auto &t : f.tensors) by_range.push_back(&t);
  std::sort(by_range.begin(), by_range.end(), [](const PwTensorRec *a, const PwTensorRec *b) {
    return a->begin != b->begin ? a->begin < b->begin : a->end < b->end;
  });
  uint64_t prev_end = 0;
  for (const PwTensorRec *t : by_range) {
    if (t->begin < prev_end) return set_err(e, PW_ERR_FORMAT, "%s: overlapping tensor payload", t->name.c_str());
    prev_end = t->end;
  }
  finish_index(f);
  return true;
}

bool align_up(uint64_t v, uint64_t a, uint64_t &out) {
  if (a == 0 || (a & (a - 1)) != 0) return false;
  if (v > UINT64_MAX - (a - 1)) return false;
  out = (v + a - 1) & ~(a - 1);
  return true;
}

// verify_expert_container (src/lib.rs:7282-7345), keeping the mapping.
bool open_container(const char *path, pw_tensor_file &f, Error &e) {
  f.path = path;
  f.container = true;
  if (!map_file(path, f.map, e)) return false;
  const uint64_t file_bytes = f.map.bytes;
  if (file_bytes < 16 || memcmp(f.map.base, kContainerMagic, 8) != 0)
    return set_err(e, PW_ERR_FORMAT, "unknown expert-container magic");
  const uint64_t header_length = le64(f.map.base + 8);
  if (header_length == 0 || header_length > kMaxHeaderBytes || 16u + header_length > file_bytes)
    return set_err(e, PW_ERR_FORMAT, "invalid expert-container header length");
  Json h;
  std::string jerr;
  if (!JsonReader(reinterpret_cast<const char *>(f.map.base + 16), header_length).read(h, jerr))
    return set_err(e, PW_ERR_FORMAT, "malformed expert-container header: %s", jerr.c_str());
  uint64_t schema = 0, alignment = 0;
  const Json *sv = h.get("schema_version"), *al = h.get("payload_alignment"), *sf = h.get("source_file"),
             *sb = h.get("source_file_bytes"), *ss = h.get("source_sha256"), *ts = h.get("tensors");
  if (h.kind != Json::Object || !sv || !sv->as_u64(schema) || !al || !al->as_u64(alignment) || !sf ||
      sf->kind != Json::String || !sb || !sb->as_u64(f.source_file_bytes) || !ss || ss->kind != Json::String || !ts ||
      ts->kind != Json::Array)
    return set_err(e, PW_ERR_FORMAT, "malformed expert-container header: missing or mistyped fields");
  if (schema != 1 || alignment != kContainerAlignment)
    return set_err(e, PW_ERR_FORMAT, "unknown expert-container schema");
  f.source_file = sf->text;
  f.source_sha256 = ss->text;
  uint64_t payload_start = 0;
  if (!align_up(16u + header_length, alignment, payload_start))
    return set_err(e, PW_ERR_FORMAT, "expert-container header overflow");
  uint64_t prev_end = 0;
  std::map<std::string, int> names;
  for (const Json &j : ts->items) {
    PwTensorRec t;
    const Json *nm = j.get("name"), *dt = j.get("dtype"), *po = j.get("payload_offset"), *db = j.get("data_bytes"),
               *hs = j.get("sha256");
    std::vector<uint64_t> src;
    uint64_t off = 0;
    if (j.kind != Json::Object || !nm || nm->kind != Json::String || !dt || dt->kind != Json::String || !po ||
        !po->as_u64(off) || !db || !db->as_u64(t.bytes) || !hs || hs->kind != Json::String ||
        !u64_array(j.get("shape"), t.shape) || !u64_array(j.get("source_data_offsets"), src) || src.size() != 2)
      return set_err(e, PW_ERR_FORMAT, "malformed expert-container tensor record");
    t.name = nm->text;
    t.dtype = dt->text;
    t.sha256 = hs->text;
    if (!names.emplace(t.name, 0).second) return set_err(e, PW_ERR_FORMAT, "duplicate tensor in expert container");
    if (off % alignment != 0 || off < prev_end)
      return set_err(e, PW_ERR_FORMAT, "invalid or overlapping expert payload offsets");
    if (off > UINT64_MAX - t.bytes) return set_err(e, PW_ERR_FORMAT, "expert payload overflow");
    const uint64_t end = off + t.bytes;
    if (payload_start > UINT64_MAX - end || payload_start + end > file_bytes)
      return set_err(e, PW_ERR_FORMAT, "expert payload exceeds container");
    // the payload must still be a tensor of its declared dtype and shape
    uint64_t expected = 0;
    if (!tensor_bytes(t.name, t.dtype, t.shape, expected, e)) return false;
    if (expected != t.bytes) return set_err(e, PW_ERR_FORMAT, "%s: shape/dtype disagree with data_bytes", t.name.c_str());
    t.begin = off;
    t.end = end;
    t.data = f.map.base + payload_start + off;
    if (sha256_hex(t.data, t.bytes) != t.sha256)
      return set_err(e, PW_ERR_FORMAT, "tensor hash mismatch: %s", t.name.c_str());
    prev_end = end;
    f.tensors.push_back(std::move(t));
  }
  if (payload_start + prev_end != file_bytes)
    return set_err(e, PW_ERR_FORMAT, "unexpected trailing or missing expert-container bytes");
  finish_index(f);
  return true;
}

void fill_view(const PwTensorRec &t, pw_tensor_view *v) {
  memset(v, 0, sizeof *v);
  v->name = t.name.c_str();
  v->dtype = t.dtype.c_str();
  v->rank = (uint32_t)t.shape.size();
  for (size_t i = 0; i < t.shape.size() && i < 8; ++i) v->shape[i] = t.shape[i];
  v->data = t.data;
  v->bytes = t.bytes;
}

// The one tensor called `name` across `files`; two files holding it is an error.
const PwTensorRec *find_in(const pw_tensor_file *const *files, uint32_t n, const std::string &name, Error &e) {
  const PwTensorRec *hit = nullptr;
  for (uint32_t i = 0; i < n; ++i) {
    if (!files[i]) continue;
    auto it = files[i]->index.find(name);
    if (it == files[i]->index.end()) continue;
    if (hit) {
      set_err(e, PW_ERR_FORMAT, "tensor %s is present in more than one file", name.c_str());
      return nullptr;
    }
    hit = &files[i]->tensors[it->second];
  }
  if (!hit) set_err(e, PW_ERR_FORMAT, "tensor is absent: %s", name.c_str());
  return hit;
}

bool write_all(int fd, const void *p, size_t n) {
  const char *c = static_cast<const char *>(p);
  while (n) {
    const ssize_t w = write(fd, c, n);
    if (w < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    c += w;
    n -= (size_t)w;
  }
  return true;
}

}  // namespace

extern "C" {

int pw_safetensors_open(const char *path, pw_tensor_file **out, char *err, size_t err_len) {
  Error e;
  if (!path || !out) {
    set_err(e, PW_ERR_ARGUMENT, "null argument");
    copy_err(e, err, err_len);
    return e.code;
  }
  *out = nullptr;
  std::unique_ptr<pw_tensor_file> f(new (std::nothrow) pw_tensor_file);
  if (!f) return PW_ERR_ARGUMENT;
  if (!open_safetensors(path, *f, e)) {
    copy_err(e, err, err_len);
    return e.code;
  }
  *out = f.release();
  copy_err(e, err, err_len);
  return PW_OK;
}

int pw_container_open(const char *path, pw_tensor_file **out, char *err, size_t err_len) {
  Error e;
  if (!path || !out) {
    set_err(e, PW_ERR_ARGUMENT, "null argument");
    copy_err(e, err, err_len);
    return e.code;
  }
  *out = nullptr;
  std::unique_ptr<pw_tensor_file> f(new (std::nothrow) pw_tensor_file);
  if (!f) return PW_ERR_ARGUMENT;
  if (!open_container(path, *f, e)) {
    copy_err(e, err, err_len);
    return e.code;
  }
  *out = f.release();
  copy_err(e, err, err_len);
  return PW_OK;
}

void pw_tensor_file_close(pw_tensor_file *f) { delete f; }

int pw_tensor_file_count(const pw_tensor_file *f, uint32_t *n) {
  if (!f || !n) return PW_ERR_ARGUMENT;
  *n = (uint32_t)f->tensors.size();
  return PW_OK;
}

int pw_tensor_file_at(const pw_tensor_file *f, uint32_t i, pw_tensor_view *out) {
  if (!f || !out || i >= f->tensors.size()) return PW_ERR_ARGUMENT;
  fill_view(f->tensors[i], out);
  return PW_OK;
}

int pw_tensor_file_find(const pw_tensor_file *f, const char *name, pw_tensor_view *out) {
  if (!f || !name || !out) return PW_ERR_ARGUMENT;
  auto it = f->index.find(name);
  if (it == f->index.end()) return PW_ERR_FORMAT;
  fill_view(f->tensors[it->second], out);
  return PW_OK;
}

int pw_container_repack(const char *source, const char *output, const char *const *names, uint32_t n_names,
                        char *err, size_t err_len) {
  Error e;
  auto done = [&](int code) {
    copy_err(e, err, err_len);
    return code;
  };
  if (!source || !output || (!names && n_names)) {
    set_err(e, PW_ERR_ARGUMENT, "null argument");
    return done(e.code);
  }
  if (n_names == 0) {
    set_err(e, PW_ERR_ARGUMENT, "at least one tensor is required");
    return done(e.code);
  }
  if (access(output, F_OK) == 0) {
    set_err(e, PW_ERR_IO, "refusing to overwrite %s", output);
    return done(e.code);
  }
  std::vector<std::string> sorted;
  for (uint32_t i = 0; i < n_names; ++i) {
    if (!names[i]) {
      set_err(e, PW_ERR_ARGUMENT, "null tensor name");
      return done(e.code);
    }
    sorted.emplace_back(names[i]);
  }
  std::sort(sorted.begin(), sorted.end());
  for (size_t i = 1; i < sorted.size(); ++i)
    if (sorted[i] == sorted[i - 1]) {
      set_err(e, PW_ERR_ARGUMENT, "duplicate tensor name");
      return done(e.code);
    }
  pw_tensor_file src;
  if (!open_safetensors(source, src, e)) return done(e.code);
  const std::string source_sha = sha256_hex(src.map.base, src.map.bytes);
  // payload layout: each tensor at the next 64-byte boundary
  struct Item {
    const PwTensorRec *t;
    uint64_t off;
    std::string sha;
  };
  std::vector<Item> items;
  uint64_t cursor = 0;
  for (const std::string &nm : sorted) {
    auto it = src.index.find(nm);
    if (it == src.index.end()) {
      set_err(e, PW_ERR_FORMAT, "tensor is absent: %s", nm.c_str());
      return done(e.code);
    }
    const PwTensorRec &t = src.tensors[it->second];
    uint64_t off = 0;
    align_up(cursor, kContainerAlignment, off);
    items.push_back({&t, off, sha256_hex(t.data, t.bytes)});
    cursor = off + t.bytes;
  }
  const char *base = strrchr(source, '/');
  std::string h = "{\"schema_version\":1,\"source_file\":" + json_quote(base ? base + 1 : source) +
                  ",\"source_file_bytes\":" + std::to_string(src.map.bytes) + ",\"source_sha256\":\"" + source_sha +
                  "\",\"payload_alignment\":" + std::to_string(kContainerAlignment) + ",\"tensors\":[";
  for (size_t i = 0; i < items.size(); ++i) {
    const PwTensorRec &t = *items[i].t;
    if (i) h += ",";
    h += "{\"name\":" + json_quote(t.name) + ",\"dtype\":" + json_quote(t.dtype) + ",\"shape\":[";
    for (size_t d = 0; d < t.shape.size(); ++d) h += (d ? "," : "") + std::to_string(t.shape[d]);
    h += "],\"source_data_offsets\":[" + std::to_string(t.begin) + "," + std::to_string(t.end) +
         "],\"payload_offset\":" + std::to_string(items[i].off) + ",\"data_bytes\":" + std::to_string(t.bytes) +
         ",\"sha256\":\"" + items[i].sha + "\"}";
  }
  h += "]}";
  uint64_t payload_start = 0;
  align_up(16u + h.size(), kContainerAlignment, payload_start);
  // write a same-directory temporary file, verify it, publish with a hard link
  const std::string out_s(output);
  const size_t slash = out_s.rfind('/');
  const std::string dir = slash == std::string::npos ? std::string() : out_s.substr(0, slash + 1);
  const std::string leaf = slash == std::string::npos ? out_s : out_s.substr(slash + 1);
  const std::string tmp = dir + "." + leaf + ".tmp." + std::to_string((long)getpid());
  const int fd = open(tmp.c_str(), O_WRONLY | O_CREAT | O_EXCL | O_CLOEXEC, 0644);
  if (fd < 0) {
    set_err(e, PW_ERR_IO, "%s: %s", tmp.c_str(), strerror(errno));
    return done(e.code);
  }
  unsigned char hdr[16];
  memcpy(hdr, kContainerMagic, 8);
  for (int i = 0; i < 8; ++i) hdr[8 + i] = (unsigned char)((uint64_t)h.size() >> (8 * i));
  bool ok = write_all(fd, hdr, 16) && write_all(fd, h.data(), h.size());
  uint64_t pos = 16u + h.size();
  static const char zeros[64] = {0};
  while (ok && pos < payload_start) {
    const size_t k = (size_t)std::min<uint64_t>(64, payload_start - pos);
    ok = write_all(fd, zeros, k);
    pos += k;
  }
  uint64_t ppos = 0;
  for (const Item &it : items) {
    while (ok && ppos < it.off) {
      const size_t k = (size_t)std::min<uint64_t>(64, it.off - ppos);
      ok = write_all(fd, zeros, k);
      ppos += k;
    }
    ok = ok && write_all(fd, it.t->data, it.t->bytes);
    ppos += it.t->bytes;
  }
  ok = ok && fsync(fd) == 0;
  close(fd);
  if (!ok) {
    set_err(e, PW_ERR_IO, "%s: write failed", tmp.c_str());
    unlink(tmp.c_str());
    return done(e.code);
  }
  {
    pw_tensor_file check;
    if (!open_container(tmp.c_str(), check, e)) {
      unlink(tmp.c_str());
      return done(e.code);
    }
  }
  const int lr = link(tmp.c_str(), output);
  const int le = errno;
  unlink(tmp.c_str());
  if (lr != 0) {
    set_err(e, PW_ERR_IO, "%s: %s", output, strerror(le));
    return done(e.code);
  }
  return done(PW_OK);
}

int pw_tensor_upload(pw_runtime *rt, const pw_tensor_file *const *files, uint32_t n_files, const char *name,
                     const char *dtype, const uint64_t *shape, uint32_t rank, void **device_ptr, char *err,
                     size_t err_len) {
  Error e;
  auto done = [&](int code) {
    copy_err(e, err, err_len);
    return code;
  };
  if (!rt || !files || !name || !device_ptr) {
    set_err(e, PW_ERR_ARGUMENT, "null argument");
    return done(e.code);
  }
  *device_ptr = nullptr;
  const PwTensorRec *t = find_in(files, n_files, name, e);
  if (!t) return done(e.code);
  if (dtype && t->dtype != dtype) {
    set_err(e, PW_ERR_SHAPE, "%s: dtype %s, expected %s", name, t->dtype.c_str(), dtype);
    return done(e.code);
  }
  if (shape) {
    bool same = t->shape.size() == rank;
    for (uint32_t i = 0; same && i < rank; ++i) same = t->shape[i] == shape[i];
    if (!same) {
      set_err(e, PW_ERR_SHAPE, "%s: shape mismatch", name);
      return done(e.code);
    }
  }
  int dev = 0;
  if (pw::runtime_device(rt, &dev) != PW_OK || cudaSetDevice(dev) != cudaSuccess) {
    set_err(e, PW_ERR_CUDA, "cannot select the runtime's device");
    return done(e.code);
  }
  void *p = nullptr;
  cudaError_t ce = cudaMalloc(&p, (size_t)t->bytes);
  if (ce == cudaSuccess) ce = cudaMemcpy(p, t->data, (size_t)t->bytes, cudaMemcpyHostToDevice);
  if (ce != cudaSuccess) {
    if (p) cudaFree(p);
    set_err(e, PW_ERR_CUDA, "%s: upload: %s", name, cudaGetErrorString(ce));
    return done(e.code);
  }
  *device_ptr = p;
  return done(PW_OK);
}

int pw_device_free(pw_runtime *rt, void *device_ptr) {
  if (!rt) return PW_ERR_ARGUMENT;
  if (!device_ptr) return PW_OK;
  int dev = 0;
  if (pw::runtime_device(rt, &dev) != PW_OK || cudaSetDevice(dev) != cudaSuccess) return PW_ERR_CUDA;
  return cudaFree(device_ptr) == cudaSuccess ? PW_OK : PW_ERR_CUDA;
}

int pw_bank_load(pw_runtime *rt, const pw_tensor_file *const *files, uint32_t n_files, uint32_t layer,
                 uint32_t first_expert, uint32_t n_experts, pw_expert_bank **out, char *err, size_t err_len) {
  Error e;
  auto done = [&](int code) {
    copy_err(e, err, err_len);
    return code;
  };
  if (!rt || !files || !out) {
    set_err(e, PW_ERR_ARGUMENT, "null argument");
    return done(e.code);
  }
  *out = nullptr;
  if (n_experts == 0) {
    set_err(e, PW_ERR_ARGUMENT, "a bank needs at least one expert");
    return done(e.code);
  }
  static const char *kProj[3] = {"gate_proj", "up_proj", "down_proj"};
  struct Src {
    const PwTensorRec *w, *s;
  };
  std::vector<Src> srcs((size_t)n_experts * 3);
  uint64_t H = 0, I = 0, total = 0;
  auto room = [](uint64_t b) { return (b + 255u) & ~uint64_t(255); };
  for (uint32_t k = 0; k < n_experts; ++k) {
    for (int p = 0; p < 3; ++p) {
      char nm[256];
      snprintf(nm, sizeof nm, "model.layers.%u.mlp.experts.%u.%s.weight", layer, first_expert + k, kProj[p]);
      const PwTensorRec *w = find_in(files, n_files, nm, e);
      if (!w) return done(e.code);
      const PwTensorRec *s = find_in(files, n_files, std::string(nm) + "_scale_inv", e);
      if (!s) return done(e.code);
      // validate_fp8_views (src/lib.rs:1217): F8_E4M3 rank 2, F32 [rows/128, cols/128]
      if (w->dtype != "F8_E4M3" || w->shape.size() != 2 || s->dtype != "F32" || s->shape.size() != 2) {
        set_err(e, PW_ERR_SHAPE, "%s: expected an F8_E4M3 matrix with an F32 scale grid", nm);
        return done(e.code);
      }
      const uint64_t rows = w->shape[0], cols = w->shape[1];
      if (k == 0 && p == 0) {
        I = rows;
        H = cols;
      }
      const uint64_t want_r = p < 2 ? I : H, want_c = p < 2 ? H : I;
      if (rows != want_r || cols != want_c || rows % 128u || cols % 128u || s->shape[0] != rows / 128u ||
          s->shape[1] != cols / 128u) {
        set_err(e, PW_ERR_SHAPE, "%s: shape [%" PRIu64 ", %" PRIu64 "] or its scale grid does not match the bank", nm,
                rows, cols);
        return done(e.code);
      }
      srcs[(size_t)k * 3 + p] = {w, s};
      total += room(w->bytes) + room(s->bytes);
    }
  }
  int dev = 0;
  if (pw::runtime_device(rt, &dev) != PW_OK || cudaSetDevice(dev) != cudaSuccess) {
    set_err(e, PW_ERR_CUDA, "cannot select the runtime's device");
    return done(e.code);
  }
  unsigned char *block = nullptr;
  cudaError_t ce = cudaMalloc(reinterpret_cast<void **>(&block), (size_t)total);
  if (ce != cudaSuccess) {
    set_err(e, PW_ERR_CUDA, "bank allocation of %" PRIu64 " bytes: %s", total, cudaGetErrorString(ce));
    return done(e.code);
  }
  std::vector<pw_expert_weights> ew(n_experts);
  uint64_t off = 0;
  for (uint32_t k = 0; k < n_experts && ce == cudaSuccess; ++k) {
    pw_fp8_tensor *dst[3] = {&ew[k].gate, &ew[k].up, &ew[k].down};
    for (int p = 0; p < 3 && ce == cudaSuccess; ++p) {
      const Src &sr = srcs[(size_t)k * 3 + p];
      unsigned char *wd = block + off;
      off += room(sr.w->bytes);
      unsigned char *sd = block + off;
      off += room(sr.s->bytes);
      ce = cudaMemcpy(wd, sr.w->data, (size_t)sr.w->bytes, cudaMemcpyHostToDevice);
      if (ce == cudaSuccess) ce = cudaMemcpy(sd, sr.s->data, (size_t)sr.s->bytes, cudaMemcpyHostToDevice);
      dst[p]->weight = wd;
      dst[p]->scale = reinterpret_cast<const float *>(sd);
      dst[p]->rows = (uint32_t)sr.w->shape[0];
      dst[p]->cols = (uint32_t)sr.w->shape[1];
      dst[p]->scale_rows = (uint32_t)sr.s->shape[0];
      dst[p]->scale_cols = (uint32_t)sr.s->shape[1];
    }
  }
  if (ce != cudaSuccess) {
    cudaFree(block);
    set_err(e, PW_ERR_CUDA, "bank upload: %s", cudaGetErrorString(ce));
    return done(e.code);
  }
  // pw_bank_create validates every weight byte and scale on the device (fail-closed)
  pw_expert_bank *bank = nullptr;
  const int s = pw_bank_create(rt, ew.data(), n_experts, &bank);
  if (s != PW_OK) {
    cudaFree(block);
    set_err(e, s, "%s", pw_last_error(rt));
    return done(s);
  }
  pw::bank_adopt_memory(bank, block);
  *out = bank;
  return done(PW_OK);
}

}  // extern "C"
