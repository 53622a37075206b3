// flat_format.cpp -- `.gaje.flat` v2 reader, validator, quantisers and writer.
//
// Reader: src/io/header/flat.rs:14-148 (header, ArchitectureDescriptor),
//         src/io/flat_reader.rs:33-251 (metadata + directory JSON, tensor
//         lookup), src/io/config.rs:137-145 (ModelConfig fields).
// Quantisers: src/compute/quantize/python.rs:152-303.
// Writer: scripts/export_gaje_flat.py:184-483.
//
// The reference panics (unwrap) or reads out of bounds on several malformed
// inputs; this reader turns every one of them into a status code instead.
#include "flat_format.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace gaje {

// ------------------------------------------------------------------ errors
namespace {
thread_local std::string g_err;
}
int set_error(int status, const std::string& msg) {
  g_err = msg;
  return status;
}
void clear_error() { g_err.clear(); }

// ------------------------------------------------------------------- f16
uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) {  // inf / nan (quiet the payload like the half crate)
    if (ax == 0x7F800000u) return uint16_t(sign | 0x7C00u);
    return uint16_t(sign | 0x7E00u | ((ax >> 13) & 0x3FFu));
  }
  if (ax >= 0x477FF000u) return uint16_t(sign | 0x7C00u);  // >= 65520 rounds to inf
  if (ax < 0x38800000u) {  // result is subnormal (or zero): round(|f| * 2^24)
    float a;
    memcpy(&a, &ax, 4);
    float scaled = a * 16777216.0f;  // exact: power-of-two scaling
    uint32_t m = uint32_t(nearbyintf(scaled));  // default rounding: nearest even
    return uint16_t(sign | m);
  }
  uint32_t t = ax - 0x38000000u + 0x0FFFu + ((ax >> 13) & 1u);
  return uint16_t(sign | (t >> 13));
}

float f16_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, out;
  if (e == 0) {
    if (m == 0) {
      out = sign;
    } else {  // subnormal: m * 2^-24 is exact in f32
      float v = float(m) * 5.9604644775390625e-08f;
      memcpy(&out, &v, 4);
      out |= sign;
    }
  } else if (e == 31) {
    out = sign | 0x7F800000u | (m << 13);
  } else {
    out = sign | ((e + 112u) << 23) | (m << 13);
  }
  float r;
  memcpy(&r, &out, 4);
  return r;
}

// ---------------------------------------------------------- python repr
std::string py_float_repr(double v) {
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v > 0 ? "Infinity" : "-Infinity";
  if (v == 0.0) return std::signbit(v) ? "-0.0" : "0.0";
  char buf[64];
  int prec = 1;
  for (; prec <= 17; ++prec) {
    snprintf(buf, sizeof buf, "%.*e", prec - 1, v);
    if (strtod(buf, nullptr) == v) break;
  }
  // buf = [-]d.ddde[+-]XX ; split digits and exponent
  std::string s(buf);
  bool neg = s[0] == '-';
  if (neg) s = s.substr(1);
  size_t epos = s.find('e');
  int exp10 = atoi(s.c_str() + epos + 1);
  std::string digits;
  for (size_t i = 0; i < epos; ++i)
    if (s[i] != '.') digits += s[i];
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  std::string out;
  if (exp10 >= -5 && exp10 < 16) {  // float_repr_style 'r': fixed notation
    if (exp10 < 0) {
      out = "0." + std::string(size_t(-exp10 - 1), '0') + digits;
    } else if (size_t(exp10) + 1 >= digits.size()) {
      out = digits + std::string(size_t(exp10) + 1 - digits.size(), '0') + ".0";
    } else {
      out = digits.substr(0, size_t(exp10) + 1) + "." + digits.substr(size_t(exp10) + 1);
    }
    // Python uses scientific notation below 1e-4
    if (exp10 < -4) out.clear();
  }
  if (out.empty()) {
    out = digits.substr(0, 1);
    if (digits.size() > 1) out += "." + digits.substr(1);
    char eb[16];
    snprintf(eb, sizeof eb, "e%c%02d", exp10 < 0 ? '-' : '+', exp10 < 0 ? -exp10 : exp10);
    out += eb;
  }
  return neg ? "-" + out : out;
}

// ------------------------------------------------------------ JSON reader
// A small DOM parser; the metadata can embed a multi-megabyte tokenizer
// string, which is skipped without copying when the caller does not ask for it.
namespace {

struct Json {
  enum T { Null, Bool, Num, Str, Arr, Obj } t = Null;
  bool b = false;
  std::string text;  // number literal or string value
  std::vector<Json> items;
  std::vector<std::string> keys;
  const Json* at(const char* k) const {
    for (size_t i = 0; i < keys.size(); ++i)
      if (keys[i] == k) return &items[i];
    return nullptr;
  }
};

class JsonReader {
 public:
  JsonReader(const char* s, size_t n) : p_(s), end_(s + n) {}
  bool document(Json& out) {
    if (!value(out, 0)) return false;
    skip_ws();
    return p_ == end_ || fail("trailing characters after the JSON value");
  }
  const std::string& error() const { return err_; }

 private:
  bool fail(const char* m) {
    if (err_.empty()) err_ = m;
    return false;
  }
  void skip_ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  static int hex(char c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
  }
  static void utf8(std::string& o, uint32_t cp) {
    if (cp < 0x80) {
      o += char(cp);
    } else if (cp < 0x800) {
      o += char(0xC0 | (cp >> 6));
      o += char(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += char(0xE0 | (cp >> 12));
      o += char(0x80 | ((cp >> 6) & 0x3F));
      o += char(0x80 | (cp & 0x3F));
    } else {
      o += char(0xF0 | (cp >> 18));
      o += char(0x80 | ((cp >> 12) & 0x3F));
      o += char(0x80 | ((cp >> 6) & 0x3F));
      o += char(0x80 | (cp & 0x3F));
    }
  }
  bool u4(uint32_t& cp) {
    if (end_ - p_ < 4) return fail("truncated \\u escape");
    cp = 0;
    for (int i = 0; i < 4; ++i) {
      int h = hex(p_[i]);
      if (h < 0) return fail("bad \\u escape");
      cp = cp * 16 + uint32_t(h);
    }
    p_ += 4;
    return true;
  }
  bool string(std::string& o) {
    ++p_;  // opening quote
    for (;;) {
      const char* run = p_;
      while (p_ < end_ && *p_ != '"' && *p_ != '\\') {
        if (static_cast<unsigned char>(*p_) < 0x20) return fail("control character in string");
        ++p_;
      }
      o.append(run, p_);
      if (p_ >= end_) return fail("unterminated string");
      if (*p_ == '"') {
        ++p_;
        return true;
      }
      ++p_;  // backslash
      if (p_ >= end_) return fail("unterminated escape");
      char c = *p_++;
      switch (c) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t cp;
          if (!u4(cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
            p_ += 2;
            uint32_t lo;
            if (!u4(lo)) return false;
            if (lo >= 0xDC00 && lo < 0xE000) cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            else { utf8(o, cp); cp = lo; }
          }
          utf8(o, cp);
          break;
        }
        default: return fail("bad escape");
      }
    }
  }
  bool value(Json& v, int depth) {
    if (depth > 128) return fail("JSON nested too deeply");
    skip_ws();
    if (p_ >= end_) return fail("unexpected end of JSON");
    char c = *p_;
    if (c == '{') {
      v.t = Json::Obj;
      ++p_;
      skip_ws();
      if (p_ < end_ && *p_ == '}') { ++p_; return true; }
      for (;;) {
        skip_ws();
        if (p_ >= end_ || *p_ != '"') return fail("expected an object key");
        std::string k;
        if (!string(k)) return false;
        skip_ws();
        if (p_ >= end_ || *p_ != ':') return fail("expected ':'");
        ++p_;
        v.keys.push_back(std::move(k));
        v.items.emplace_back();
        if (!value(v.items.back(), depth + 1)) return false;
        skip_ws();
        if (p_ < end_ && *p_ == ',') { ++p_; continue; }
        if (p_ < end_ && *p_ == '}') { ++p_; return true; }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.t = Json::Arr;
      ++p_;
      skip_ws();
      if (p_ < end_ && *p_ == ']') { ++p_; return true; }
      for (;;) {
        v.items.emplace_back();
        if (!value(v.items.back(), depth + 1)) return false;
        skip_ws();
        if (p_ < end_ && *p_ == ',') { ++p_; continue; }
        if (p_ < end_ && *p_ == ']') { ++p_; return true; }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.t = Json::Str;
      return string(v.text);
    }
    auto lit = [&](const char* w) {
      size_t n = strlen(w);
      if (size_t(end_ - p_) >= n && memcmp(p_, w, n) == 0) { p_ += n; return true; }
      return false;
    };
    if (lit("true")) { v.t = Json::Bool; v.b = true; return true; }
    if (lit("false")) { v.t = Json::Bool; v.b = false; return true; }
    if (lit("null")) { v.t = Json::Null; return true; }
    const char* s = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                         *p_ == '+' || *p_ == '-'))
      ++p_;
    if (p_ == s) return fail("unexpected character in JSON");
    v.t = Json::Num;
    v.text.assign(s, p_);
    char* ep = nullptr;
    strtod(v.text.c_str(), &ep);
    if (*ep != '\0') return fail("malformed number");
    return true;
  }

  const char* p_;
  const char* end_;
  std::string err_;
};

// serde's usize: a non-negative integer literal.
bool as_u64(const Json* j, uint64_t& out) {
  if (!j || j->t != Json::Num || j->text.empty() || j->text[0] == '-' ||
      j->text.find_first_of(".eE") != std::string::npos)
    return false;
  errno = 0;
  char* ep = nullptr;
  unsigned long long v = strtoull(j->text.c_str(), &ep, 10);
  if (errno || *ep) return false;
  out = v;
  return true;
}

bool as_f32(const Json* j, float& out) {
  if (!j || j->t != Json::Num) return false;
  out = float(strtod(j->text.c_str(), nullptr));  // serde: f64 then `as f32`
  return true;
}

}  // namespace

// ----------------------------------------------------------------- reader
FlatFile::~FlatFile() {
  if (data_) munmap(const_cast<uint8_t*>(data_), size_);
}

const uint8_t* FlatFile::blob(uint64_t off, uint64_t len) const {
  uint64_t s = hdr.weights_offset + off;
  if (s < hdr.weights_offset || s + len < s || s + len > size_) return nullptr;
  return data_ + s;
}

int decode_header(const uint8_t* p, size_t len, gaje_flat_header& h, std::string& err) {
  if (len < 4096) {
    err = "header buffer is shorter than 4096 bytes";
    return GAJE_ERR_IO;
  }
  if (memcmp(p, "GAJE", 4) != 0) {
    err = "invalid magic (expected \"GAJE\")";
    return GAJE_ERR_IO;
  }
  // Little-endian packed layout "<4sIIIQQQQIIIIIIII" (export_gaje_flat.py:450-471).
  auto u32 = [&](size_t o) { uint32_t v; memcpy(&v, p + o, 4); return v; };
  auto u64 = [&](size_t o) { uint64_t v; memcpy(&v, p + o, 8); return v; };
  h.version = u32(4);
  h.flags = u32(8);
  h.num_tensors = u32(12);
  h.meta_len = u64(16);
  h.dir_len = u64(24);
  h.weights_offset = u64(32);
  h.weights_len = u64(40);
  h.group_size = u32(48);
  h.quant_format = u32(52);
  h.arch_family = u32(56);
  h.arch_n_embd = u32(60);
  h.arch_n_head = u32(64);
  h.arch_n_head_kv = u32(68);
  h.arch_n_blocks = u32(72);
  h.arch_qk_permute = u32(76);
  return GAJE_OK;
}

int FlatFile::open(const char* path, std::string& err) {
  if (!path) { err = "path is NULL"; return GAJE_ERR_INVALID; }
  int fd = ::open(path, O_RDONLY);
  if (fd < 0) {
    err = std::string("cannot open ") + path + ": " + strerror(errno);
    return GAJE_ERR_IO;
  }
  struct stat st;
  if (fstat(fd, &st) != 0) { ::close(fd); err = "fstat failed"; return GAJE_ERR_IO; }
  size_ = size_t(st.st_size);
  if (size_ < 4096) {
    ::close(fd);
    err = "file is shorter than the 4096-byte FlatHeaderV2";
    return GAJE_ERR_IO;
  }
  void* m = mmap(nullptr, size_, PROT_READ, MAP_SHARED, fd, 0);
  ::close(fd);
  if (m == MAP_FAILED) { err = "mmap failed"; return GAJE_ERR_IO; }
  data_ = static_cast<const uint8_t*>(m);
  madvise(m, size_, MADV_SEQUENTIAL);
  if (int s = decode_header(data_, size_, hdr, err)) return s;
  info.header = hdr;
  if (hdr.meta_len > size_ || hdr.dir_len > size_ || 4096 + hdr.meta_len + hdr.dir_len > size_) {
    err = "metadata/directory extend past the end of the file";
    return GAJE_ERR_IO;
  }
  const char* meta = reinterpret_cast<const char*>(data_) + 4096;
  const char* dirp = meta + hdr.meta_len;
  Json mj, dj;
  {
    JsonReader r(meta, hdr.meta_len);
    if (!r.document(mj)) { err = "metadata JSON: " + r.error(); return GAJE_ERR_IO; }
  }
  {
    JsonReader r(dirp, hdr.dir_len);
    if (!r.document(dj)) { err = "directory JSON: " + r.error(); return GAJE_ERR_IO; }
  }
  // ModelConfig (config.rs:137-145): config, n_embd, n_head, n_head_kv,
  // n_blocks and eps are required; vocab_size is optional; unknown keys ignored.
  const Json* cfg = mj.t == Json::Obj ? mj.at("config") : nullptr;
  uint64_t n_embd, n_head, n_head_kv, n_blocks;
  float eps;
  if (!cfg || cfg->t != Json::Obj || !as_u64(mj.at("n_embd"), n_embd) ||
      !as_u64(mj.at("n_head"), n_head) || !as_u64(mj.at("n_head_kv"), n_head_kv) ||
      !as_u64(mj.at("n_blocks"), n_blocks) || !as_f32(mj.at("eps"), eps)) {
    err = "metadata JSON lacks a required ModelConfig field (config, n_embd, n_head, "
          "n_head_kv, n_blocks, eps)";
    return GAJE_ERR_IO;
  }
  // ArchConfig defaults (config.rs:92-129).
  float rope_base = 10000.0f;
  std::string rope_style = "split";
  bool use_gnorm = false;
  if (const Json* j = cfg->at("rope_base")) {
    if (!as_f32(j, rope_base)) { err = "config.rope_base is not a number"; return GAJE_ERR_IO; }
  }
  if (const Json* j = cfg->at("rope_style")) {
    if (j->t != Json::Str) { err = "config.rope_style is not a string"; return GAJE_ERR_IO; }
    rope_style = j->text;
  }
  if (const Json* j = cfg->at("use_genomic_norm")) {
    if (j->t != Json::Bool) { err = "config.use_genomic_norm is not a bool"; return GAJE_ERR_IO; }
    use_gnorm = j->b;
  }
  // Header descriptor override (flat_reader.rs:127-139, flat.rs:82-148):
  // every family forces "split" RoPE; the base is per family.
  if (hdr.arch_family != 0) {
    n_embd = hdr.arch_n_embd;
    n_head = hdr.arch_n_head;
    n_head_kv = hdr.arch_n_head_kv;
    n_blocks = hdr.arch_n_blocks;
    switch (hdr.arch_family) {
      case 2: rope_base = 100000.0f; break;
      case 3: case 4: rope_base = 1000000.0f; break;
      default: rope_base = 10000.0f; break;
    }
    rope_style = "split";
  }
  info.n_embd = uint32_t(n_embd);
  info.n_head = uint32_t(n_head);
  info.n_head_kv = uint32_t(n_head_kv);
  info.n_blocks = uint32_t(n_blocks);
  info.eps = eps;
  info.rope_base = rope_base;
  info.rope_split = rope_style == "split" ? 1 : 0;
  info.use_genomic_norm = use_gnorm ? 1 : 0;
  if (n_head == 0 || n_head_kv == 0 || n_embd == 0 || n_embd % n_head != 0 ||
      n_head % n_head_kv != 0 || (n_embd / n_head) % 2 != 0 || n_embd > (1u << 20) ||
      n_blocks > 4096) {
    err = "unsupported attention geometry (n_embd % n_head, n_head % n_head_kv and an even "
          "head_dim are required)";
    return GAJE_ERR_SHAPE;
  }
  info.head_dim = uint32_t(n_embd / n_head);

  if (dj.t != Json::Arr) { err = "directory JSON is not an array"; return GAJE_ERR_IO; }
  for (const Json& e : dj.items) {
    FlatEntry fe;
    const Json* nm = e.t == Json::Obj ? e.at("name") : nullptr;
    if (!nm || nm->t != Json::Str || !as_u64(e.at("bit_depth"), fe.bit_depth) ||
        !as_u64(e.at("out_features"), fe.out) || !as_u64(e.at("in_features"), fe.in) ||
        !as_u64(e.at("dna_off"), fe.dna_off) || !as_u64(e.at("dna_len"), fe.dna_len) ||
        !as_u64(e.at("c_off"), fe.c_off) || !as_u64(e.at("c_len"), fe.c_len) ||
        !as_u64(e.at("anc_off"), fe.anc_off) || !as_u64(e.at("anc_len"), fe.anc_len) ||
        !as_u64(e.at("bias_off"), fe.bias_off) || !as_u64(e.at("bias_len"), fe.bias_len)) {
      err = "directory entry lacks a FlatTensorEntry field";
      return GAJE_ERR_IO;
    }
    fe.name = nm->text;
    dir[fe.name] = fe;  // later duplicates win, as HashMap::insert does
  }
  info.n_entries = uint32_t(dir.size());
  return resolve(err);
}

namespace {
uint64_t data_bytes(int bits, uint64_t out, uint64_t in) {
  switch (bits) {
    case 4: return out * (in / 32) * 20;
    case 8: return out * (in / 32) * 34;
    case 32: return out * in * 4;
    default: return 0;
  }
}
}  // namespace

// Tensor lookup of load_genomic (flat_reader.rs:143-227) plus the shape checks
// the reference leaves to slice panics.
int FlatFile::resolve(std::string& err) {
  auto find = [&](const std::string& n) -> const FlatEntry* {
    auto it = dir.find(n);
    return it == dir.end() ? nullptr : &it->second;
  };
  auto need = [&](const std::string& n, const FlatEntry*& out) -> int {
    out = find(n);
    if (!out) { err = "Flat tensor entry '" + n + "' not found"; return GAJE_ERR_NOT_FOUND; }
    return GAJE_OK;
  };
  auto check_entry = [&](const FlatEntry* e, bool matrix) -> int {
    if (e->anc_len != 0) {
      err = "tensor '" + e->name + "' carries sparse anchors, which this engine does not implement";
      return GAJE_ERR_UNSUPPORTED;
    }
    if (matrix) {
      int bits = int(e->bit_depth);
      if (bits == 4 && e->c_len != 0) {  // Genomic4Bit: nibbles + 16-centroid tables (init.rs:29-38, 109-124)
        const uint64_t nb = e->in / 32;
        if (e->in % 32 != 0) {
          err = "tensor '" + e->name + "': in_features is not a multiple of 32";
          return GAJE_ERR_SHAPE;
        }
        if (e->dna_len != e->out * e->in / 2) {
          err = "tensor '" + e->name + "': dna_len does not match out_features x in_features / 2";
          return GAJE_ERR_SHAPE;
        }
        if (e->c_len != 64 && e->c_len != nb * 64 && e->c_len != e->out * nb * 64) {
          err = "unsupported centroid count for " + e->name;
          return GAJE_ERR_SHAPE;
        }
        if (e->bias_len % 4 != 0 || e->bias_len > e->out * 4) {
          err = "tensor '" + e->name + "': bias_len is not a multiple of 4 up to out_features";
          return GAJE_ERR_SHAPE;
        }
      } else if (bits != 4 && bits != 8 && bits != 32) {
        err = "tensor '" + e->name + "' has unsupported bit_depth " + std::to_string(bits);
        return GAJE_ERR_UNSUPPORTED;
      }
      if ((bits == 4 || bits == 8) && e->in % 32 != 0) {
        err = "tensor '" + e->name + "': in_features is not a multiple of 32";
        return GAJE_ERR_SHAPE;
      }
      if (!(bits == 4 && e->c_len != 0) && e->dna_len != data_bytes(bits, e->out, e->in)) {
        err = "tensor '" + e->name + "': dna_len does not match out_features x in_features";
        return GAJE_ERR_SHAPE;
      }
      if (e->bias_len % 4 != 0 || e->bias_len > e->out * 4) {
        err = "tensor '" + e->name + "': bias_len is not a multiple of 4 up to out_features";
        return GAJE_ERR_SHAPE;
      }
    }
    if (!blob(e->dna_off, e->dna_len) || !blob(e->bias_off, e->bias_len) ||
        !blob(e->c_off, e->c_len)) {
      err = "tensor '" + e->name + "' extends past the end of the file";
      return GAJE_ERR_IO;
    }
    return GAJE_OK;
  };
  auto matrix = [&](std::vector<std::string> names, MatrixRef& m) -> int {
    m = MatrixRef();
    for (auto& n : names) {
      const FlatEntry* e;
      if (int s = need(n, e)) return s;
      if (int s = check_entry(e, true)) return s;
      const bool lut = e->bit_depth == 4 && e->c_len != 0;
      if (!m.parts.empty() && (int(e->bit_depth) != m.bit_depth || e->in != m.in || lut || m.lut)) {
        err = "unfused tensors '" + names[0] + "' and '" + n + "' differ in format or in_features";
        if (lut || m.lut) err = "unfused q/k/v or gate/up tensors must not be Genomic4Bit tables ('" + n + "')";
        return GAJE_ERR_UNSUPPORTED;
      }
      m.parts.push_back(e);
      m.lut = lut;
      m.bit_depth = int(e->bit_depth);
      m.in = e->in;
      m.out += e->out;
      m.has_bias |= e->bias_len != 0;
    }
    return GAJE_OK;
  };
  const uint64_t d = info.n_embd, qd = uint64_t(info.n_head) * info.head_dim,
                 kvd = uint64_t(info.n_head_kv) * info.head_dim;
  if (int s = need("token_embd", token_embd)) return s;
  if (int s = check_entry(token_embd, true)) return s;
  if (int s = need("output_norm", output_norm)) return s;
  if (int s = check_entry(output_norm, false)) return s;
  if (int s = need("lm_head", lm_head)) return s;
  if (int s = check_entry(lm_head, true)) return s;
  if (token_embd->in != d || lm_head->in != d || output_norm->dna_len != d * 4 ||
      token_embd->out == 0 || lm_head->out == 0) {
    err = "token_embd/lm_head/output_norm shapes do not match n_embd";
    return GAJE_ERR_SHAPE;
  }
  if (token_embd->bit_depth == 4 || lm_head->bit_depth == 4) {
    err = "Q4_0 embeddings or lm_head are not implemented (f32 and Q8_0 are)";
    return GAJE_ERR_UNSUPPORTED;
  }
  info.vocab_size = uint32_t(lm_head->out);
  info.embd_bit_depth = int(token_embd->bit_depth);
  info.lm_head_bit_depth = int(lm_head->bit_depth);
  blocks.assign(info.n_blocks, BlockRefs());
  info.fused_qkv = info.fused_gate_up = 1;
  for (uint32_t i = 0; i < info.n_blocks; ++i) {
    std::string p = "blk." + std::to_string(i) + ".";
    BlockRefs& b = blocks[i];
    if (int s = need(p + "attn_norm", b.attn_norm)) return s;
    if (int s = need(p + "ffn_norm", b.ffn_norm)) return s;
    if (int s = check_entry(b.attn_norm, false)) return s;
    if (int s = check_entry(b.ffn_norm, false)) return s;
    if (b.attn_norm->dna_len != d * 4 || b.ffn_norm->dna_len != d * 4) {
      err = "block " + std::to_string(i) + ": norm length does not match n_embd";
      return GAJE_ERR_SHAPE;
    }
    bool fq = find(p + "attn_qkv") != nullptr, fg = find(p + "ffn_gate_up") != nullptr;
    if (!fq) info.fused_qkv = 0;
    if (!fg) info.fused_gate_up = 0;
    int s = fq ? matrix({p + "attn_qkv"}, b.qkv)
               : matrix({p + "attn_q", p + "attn_k", p + "attn_v"}, b.qkv);
    if (s) return s;
    if ((s = matrix({p + "attn_output"}, b.wo))) return s;
    s = fg ? matrix({p + "ffn_gate_up"}, b.gate_up) : matrix({p + "ffn_gate", p + "ffn_up"}, b.gate_up);
    if (s) return s;
    if ((s = matrix({p + "ffn_down"}, b.down))) return s;
    if (b.qkv.out != qd + 2 * kvd || b.qkv.in != d || b.wo.out != d || b.wo.in != qd ||
        b.gate_up.in != d || b.gate_up.out % 2 != 0 || b.down.out != d ||
        b.down.in != b.gate_up.out / 2) {
      err = "block " + std::to_string(i) + ": projection shapes do not match the config";
      return GAJE_ERR_SHAPE;
    }
    for (const MatrixRef* m : {&b.qkv, &b.wo, &b.gate_up, &b.down}) {
      if (m->bit_depth != 4) {
        err = "block " + std::to_string(i) +
              ": only Q4_0 body tensors are implemented (found bit_depth " +
              std::to_string(m->bit_depth) + ")";
        return GAJE_ERR_UNSUPPORTED;
      }
    }
    if (!fg) {
      // gate and up must split the concatenation exactly in half
      if (b.gate_up.parts[0]->out * 2 != b.gate_up.out) {
        err = "block " + std::to_string(i) + ": ffn_gate and ffn_up differ in out_features";
        return GAJE_ERR_SHAPE;
      }
    }
    if (i == 0) info.ffn_dim = uint32_t(b.gate_up.out / 2);
    else if (b.gate_up.out / 2 != info.ffn_dim) {
      err = "blocks differ in ffn width";
      return GAJE_ERR_SHAPE;
    }
  }
  info.body_bit_depth = 4;
  return GAJE_OK;
}

// --------------------------------------------------------------- quantise
namespace {
inline float rust_clamp(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

void q4_block(const float* b, uint8_t* out) {
  float mn = 3.40282347e+38f, mx = -3.40282347e+38f;
  for (int i = 0; i < 32; ++i) {
    if (b[i] < mn) mn = b[i];
    if (b[i] > mx) mx = b[i];
  }
  volatile float range = mx - mn;  // keep (max-min)/15 as two roundings
  float scale = range / 15.0f;
  float inv = scale > 1e-7f ? 1.0f / scale : 0.0f;
  for (int k = 0; k < 16; ++k) {
    uint8_t q[2] = {0, 0};
    if (scale > 1e-7f) {
      for (int t = 0; t < 2; ++t) {
        volatile float diff = b[2 * k + t] - mn;
        float r = roundf(diff * inv);  // f32::round: half away from zero
        r = rust_clamp(r, 0.0f, 15.0f);
        q[t] = (r != r) ? 0 : uint8_t(r);
      }
    }
    out[4 + k] = uint8_t(q[0] | (q[1] << 4));
  }
  uint16_t hs = f32_to_f16(scale), hm = f32_to_f16(mn);
  memcpy(out, &hs, 2);
  memcpy(out + 2, &hm, 2);
}

void q8_block(const float* b, uint8_t* out) {
  float max_abs = 0.0f;
  for (int i = 0; i < 32; ++i) {
    float a = fabsf(b[i]);
    if (a > max_abs) max_abs = a;
  }
  float scale = max_abs / 127.0f;
  float inv = scale > 1e-7f ? 1.0f / scale : 0.0f;
  for (int k = 0; k < 32; ++k) {
    int8_t q = 0;
    if (scale > 1e-7f) {
      volatile float prod = b[k] * inv;
      float r = roundf(prod);
      r = rust_clamp(r, -128.0f, 127.0f);
      q = (r != r) ? 0 : int8_t(r);
    }
    out[2 + k] = uint8_t(q);
  }
  uint16_t hs = f32_to_f16(scale);
  memcpy(out, &hs, 2);
}
}  // namespace

}  // namespace gaje

using namespace gaje;

extern "C" {

const char* gaje_cuda_last_error(void) { return g_err.c_str(); }

int gaje_quantize_q4_0(const float* w, size_t n, uint8_t* out) {
  if (!w || !out) return set_error(GAJE_ERR_INVALID, "NULL pointer");
  if (n % 32) return set_error(GAJE_ERR_INVALID, "Weights length must be divisible by 32");
  const long long nb = (long long)(n / 32);
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < nb; ++i) q4_block(w + i * 32, out + i * 20);
  return GAJE_OK;
}

int gaje_quantize_q8_0(const float* w, size_t n, uint8_t* out) {
  if (!w || !out) return set_error(GAJE_ERR_INVALID, "NULL pointer");
  if (n % 32) return set_error(GAJE_ERR_INVALID, "Weights length must be divisible by 32");
  const long long nb = (long long)(n / 32);
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < nb; ++i) q8_block(w + i * 32, out + i * 34);
  return GAJE_OK;
}

int gaje_flat_header_decode(const uint8_t* bytes, size_t len, gaje_flat_header* out) {
  if (!bytes || !out) return set_error(GAJE_ERR_INVALID, "NULL argument");
  std::string err;
  if (int s = decode_header(bytes, len, *out, err)) return set_error(s, err);
  clear_error();
  return GAJE_OK;
}

int gaje_flat_inspect(const char* path, gaje_flat_info* info) {
  if (!info) return set_error(GAJE_ERR_INVALID, "info is NULL");
  FlatFile f;
  std::string err;
  int s = f.open(path, err);
  if (s) return set_error(s, err);
  *info = f.info;
  clear_error();
  return GAJE_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ writer
struct gaje_flat_writer {
  std::string path;
  // Blobs are held in memory (a list of chunks) until close(): the file is
  // then written once, header + metadata + directory + blobs, with no
  // temporary file (the directory, and so weights_offset, is only known at
  // the end).
  std::vector<std::vector<uint8_t>> chunks;
  uint64_t blob_len = 0;
  std::vector<FlatEntry> dir;
  gaje_flat_meta meta{};
  std::string name, tokenizer_id, tokenizer;
  std::string err;
};

namespace {

// json.dumps string escaping with ensure_ascii=True.
std::string json_str(const std::string& s) {
  std::string o = "\"";
  size_t i = 0;
  while (i < s.size()) {
    unsigned char c = (unsigned char)s[i];
    uint32_t cp;
    size_t len = 1;
    if (c < 0x80) cp = c;
    else if ((c >> 5) == 6 && i + 1 < s.size()) { cp = ((c & 0x1F) << 6) | (s[i + 1] & 0x3F); len = 2; }
    else if ((c >> 4) == 14 && i + 2 < s.size()) { cp = ((c & 0x0F) << 12) | ((s[i + 1] & 0x3F) << 6) | (s[i + 2] & 0x3F); len = 3; }
    else if ((c >> 3) == 30 && i + 3 < s.size()) { cp = ((c & 0x07) << 18) | ((s[i + 1] & 0x3F) << 12) | ((s[i + 2] & 0x3F) << 6) | (s[i + 3] & 0x3F); len = 4; }
    else cp = 0xFFFD;
    i += len;
    char buf[16];
    switch (cp) {
      case '"': o += "\\\""; continue;
      case '\\': o += "\\\\"; continue;
      case '\n': o += "\\n"; continue;
      case '\r': o += "\\r"; continue;
      case '\t': o += "\\t"; continue;
      case '\b': o += "\\b"; continue;
      case '\f': o += "\\f"; continue;
      default: break;
    }
    if (cp >= 0x20 && cp < 0x7F) {
      o += char(cp);
    } else if (cp < 0x10000) {
      snprintf(buf, sizeof buf, "\\u%04x", cp);
      o += buf;
    } else {
      uint32_t v = cp - 0x10000;
      snprintf(buf, sizeof buf, "\\u%04x\\u%04x", 0xD800 + (v >> 10), 0xDC00 + (v & 0x3FF));
      o += buf;
    }
  }
  return o + "\"";
}

bool blob_put(gaje_flat_writer* w, const void* p, uint64_t n, uint64_t& off, uint64_t& len) {
  off = w->blob_len;
  len = n;
  const uint64_t pad = (64 - ((w->blob_len + n) % 64)) % 64;
  if (n + pad == 0) return true;
  std::vector<uint8_t> c(size_t(n + pad), 0);
  if (n) memcpy(c.data(), p, size_t(n));
  w->chunks.push_back(std::move(c));
  w->blob_len += n + pad;
  return true;
}

}  // namespace

extern "C" {

gaje_flat_writer* gaje_flat_writer_open(const char* path, const gaje_flat_meta* meta) {
  if (!path || !meta) { set_error(GAJE_ERR_INVALID, "NULL argument"); return nullptr; }
  auto* w = new gaje_flat_writer();
  w->path = path;
  w->meta = *meta;
  w->name = meta->name ? meta->name : "gaje";
  w->tokenizer_id = meta->tokenizer_id ? meta->tokenizer_id : "";
  w->tokenizer = meta->tokenizer ? meta->tokenizer : "";
  return w;
}

int gaje_flat_writer_add_linear(gaje_flat_writer* w, const char* name, int bit_depth,
                                size_t out_features, size_t in_features, const float* weights,
                                const float* bias) {
  if (!w || !name || !weights) return set_error(GAJE_ERR_INVALID, "NULL argument");
  size_t n = out_features * in_features;
  std::vector<uint8_t> dna;
  const void* src = weights;
  uint64_t bytes = 0;
  if (bit_depth == 4 || bit_depth == 8) {
    if (in_features % 32) return set_error(GAJE_ERR_SHAPE, "in_features must be a multiple of 32");
    dna.resize(n / 32 * (bit_depth == 4 ? 20 : 34));
    int s = bit_depth == 4 ? gaje_quantize_q4_0(weights, n, dna.data())
                           : gaje_quantize_q8_0(weights, n, dna.data());
    if (s) return s;
    src = dna.data();
    bytes = dna.size();
  } else if (bit_depth == 32) {
    bytes = uint64_t(n) * 4;
  } else {
    return set_error(GAJE_ERR_UNSUPPORTED, "bit_depth must be 4, 8 or 32");
  }
  FlatEntry e;
  e.name = name;
  e.bit_depth = uint64_t(bit_depth);
  e.out = out_features;
  e.in = in_features;
  bool ok = blob_put(w, src, bytes, e.dna_off, e.dna_len) &&
            blob_put(w, nullptr, 0, e.c_off, e.c_len) &&
            blob_put(w, nullptr, 0, e.anc_off, e.anc_len);
  if (ok && bias) ok = blob_put(w, bias, uint64_t(out_features) * 4, e.bias_off, e.bias_len);
  if (!ok) return set_error(GAJE_ERR_IO, "write failed");
  w->dir.push_back(e);
  return GAJE_OK;
}

int gaje_flat_writer_add_norm(gaje_flat_writer* w, const char* name, const float* v, size_t n) {
  if (!w || !name || !v) return set_error(GAJE_ERR_INVALID, "NULL argument");
  FlatEntry e;
  e.name = name;
  e.bit_depth = 32;
  e.out = w->meta.n_embd;  // the exporter records n_embd here
  e.in = 1;
  if (!blob_put(w, v, uint64_t(n) * 4, e.dna_off, e.dna_len)) return set_error(GAJE_ERR_IO, "write failed");
  w->dir.push_back(e);
  return GAJE_OK;
}

int gaje_flat_writer_close(gaje_flat_writer* w) {
  if (!w) return set_error(GAJE_ERR_INVALID, "writer is NULL");
  std::unique_ptr<gaje_flat_writer> guard(w);
  const gaje_flat_meta& m = w->meta;
  // Metadata dict in the exporter's key order (export_gaje_flat.py:184-200).
  std::string meta = "{\"config\": {\"name\": " + json_str(w->name) +
                     ", \"version\": \"0.9.8\", \"tokenizer_id\": " + json_str(w->tokenizer_id) +
                     ", \"rope_base\": " + py_float_repr(m.rope_base) + ", \"ffn_act\": " +
                     (m.arch_family == 5 ? "\"geglu\"" : "\"swiglu\"") +
                     ", \"use_genomic_norm\": false}, \"n_embd\": " + std::to_string(m.n_embd) +
                     ", \"n_head\": " + std::to_string(m.n_head) +
                     ", \"n_head_kv\": " + std::to_string(m.n_head_kv) +
                     ", \"n_blocks\": " + std::to_string(m.n_blocks) +
                     ", \"vocab_size\": " + std::to_string(m.vocab_size) +
                     ", \"eps\": " + py_float_repr(double(m.eps)) +
                     ", \"tokenizer\": " + json_str(w->tokenizer) + "}";
  std::string dir = "[";
  for (size_t i = 0; i < w->dir.size(); ++i) {
    const FlatEntry& e = w->dir[i];
    if (i) dir += ", ";
    dir += "{\"name\": " + json_str(e.name) + ", \"bit_depth\": " + std::to_string(e.bit_depth) +
           ", \"out_features\": " + std::to_string(e.out) + ", \"in_features\": " +
           std::to_string(e.in) + ", \"dna_off\": " + std::to_string(e.dna_off) +
           ", \"dna_len\": " + std::to_string(e.dna_len) + ", \"c_off\": " +
           std::to_string(e.c_off) + ", \"c_len\": " + std::to_string(e.c_len) +
           ", \"anc_off\": " + std::to_string(e.anc_off) + ", \"anc_len\": " +
           std::to_string(e.anc_len) + ", \"bias_off\": " + std::to_string(e.bias_off) +
           ", \"bias_len\": " + std::to_string(e.bias_len) + "}";
  }
  dir += "]";
  uint64_t woff = 4096 + meta.size() + dir.size();
  if (woff % 4096) woff = (woff / 4096 + 1) * 4096;
  uint8_t hdr[4096] = {0};
  auto p32 = [&](size_t o, uint32_t v) { memcpy(hdr + o, &v, 4); };
  auto p64 = [&](size_t o, uint64_t v) { memcpy(hdr + o, &v, 8); };
  memcpy(hdr, "GAJE", 4);
  p32(4, 0x000908u);  // FlatHeaderV2 version
  p32(8, 0x3u);       // bit 0 fused qkv, bit 1 fused gate_up
  p32(12, uint32_t(w->dir.size()));
  p64(16, meta.size());
  p64(24, dir.size());
  p64(32, woff);
  p64(40, w->blob_len);
  p32(48, 32);  // group_size
  p32(52, 1);   // quant_format: the exporter always records Q4_0
  p32(56, m.arch_family);
  p32(60, m.n_embd);
  p32(64, m.n_head);
  p32(68, m.n_head_kv);
  p32(72, m.n_blocks);
  p32(76, m.qk_permute ? 1u : 0u);
  FILE* f = fopen(w->path.c_str(), "wb");
  if (!f) return set_error(GAJE_ERR_IO, "cannot create " + w->path);
  bool ok = fwrite(hdr, 1, 4096, f) == 4096 && fwrite(meta.data(), 1, meta.size(), f) == meta.size() &&
            fwrite(dir.data(), 1, dir.size(), f) == dir.size();
  std::vector<char> zeros(size_t(woff - 4096 - meta.size() - dir.size()), 0);
  ok = ok && (zeros.empty() || fwrite(zeros.data(), 1, zeros.size(), f) == zeros.size());
  for (size_t i = 0; ok && i < w->chunks.size(); ++i) {
    ok = fwrite(w->chunks[i].data(), 1, w->chunks[i].size(), f) == w->chunks[i].size();
    std::vector<uint8_t>().swap(w->chunks[i]);
  }
  ok = (fclose(f) == 0) && ok;
  if (!ok) return set_error(GAJE_ERR_IO, "write failed for " + w->path);
  clear_error();
  return GAJE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- synthetic
namespace {

inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t name_key(uint64_t seed, const std::string& name) {
  uint64_t h = 0xCBF29CE484222325ull;  // FNV-1a
  for (char c : name) h = (h ^ uint8_t(c)) * 0x100000001B3ull;
  return mix64(seed ^ h);
}

// Counter-based N(0, std): element pair p draws two splitmix64 values and
// applies Box-Muller in double precision, so any thread count gives the same
// tensor.
void fill_normal(std::vector<float>& v, uint64_t key, float std) {
  const long long pairs = (long long)((v.size() + 1) / 2);
#pragma omp parallel for schedule(static)
  for (long long p = 0; p < pairs; ++p) {
    uint64_t a = mix64(key + 0x9E3779B97F4A7C15ull * uint64_t(2 * p + 1));
    uint64_t b = mix64(key + 0x9E3779B97F4A7C15ull * uint64_t(2 * p + 2));
    double u1 = double((a >> 11) + 1) * (1.0 / 9007199254740992.0);  // (0, 1]
    double u2 = double(b >> 11) * (1.0 / 9007199254740992.0);
    double r = sqrt(-2.0 * log(u1));
    double z0 = r * cos(6.283185307179586 * u2), z1 = r * sin(6.283185307179586 * u2);
    v[size_t(2 * p)] = float(double(std) * z0);
    if (size_t(2 * p + 1) < v.size()) v[size_t(2 * p + 1)] = float(double(std) * z1);
  }
}

}  // namespace

extern "C" int gaje_flat_write_synthetic(const char* path, const gaje_synth_spec* sp) {
  if (!path || !sp) return set_error(GAJE_ERR_INVALID, "NULL argument");
  const gaje_synth_spec& s = *sp;
  if (!s.n_embd || !s.n_head || !s.n_head_kv || s.n_embd % s.n_head || s.n_head % s.n_head_kv ||
      s.n_embd % 32 || s.ffn_dim % 32 || !s.vocab_size)
    return set_error(GAJE_ERR_SHAPE, "inconsistent synthetic spec");
  const float std_ = s.std > 0 ? s.std : 0.02f;
  const uint32_t hd = s.n_embd / s.n_head;
  const size_t d = s.n_embd, qd = size_t(s.n_head) * hd, kvd = size_t(s.n_head_kv) * hd,
               ff = s.ffn_dim, V = s.vocab_size;
  gaje_flat_meta m{};
  std::string nm = "synthetic-family" + std::to_string(s.arch_family);
  m.name = nm.c_str();
  m.tokenizer_id = "";
  m.tokenizer = "";
  m.arch_family = s.arch_family;
  m.qk_permute = (s.arch_family == 1 || s.arch_family == 2) ? 1 : 0;
  m.n_embd = s.n_embd;
  m.n_head = s.n_head;
  m.n_head_kv = s.n_head_kv;
  m.n_blocks = s.n_blocks;
  m.vocab_size = s.vocab_size;
  m.eps = s.eps;
  m.rope_base = s.rope_base;
  gaje_flat_writer* w = gaje_flat_writer_open(path, &m);
  if (!w) return GAJE_ERR_IO;
  const int eb = s.embd_bit_depth ? s.embd_bit_depth : 32;
  int st = GAJE_OK;
  std::vector<float> buf, bias;
  auto fail = [&](int code) {
    delete w;
    return code;
  };
  {
    buf.assign(V * d, 0.0f);
    fill_normal(buf, name_key(s.seed, "token_embd"), std_);
    // tied: the same matrix is written as token_embd and as lm_head
    if ((st = gaje_flat_writer_add_linear(w, "token_embd", eb, V, d, buf.data(), nullptr))) return fail(st);
    std::vector<float> ones(d, 1.0f);
    if ((st = gaje_flat_writer_add_norm(w, "output_norm", ones.data(), d))) return fail(st);
    if ((st = gaje_flat_writer_add_linear(w, "lm_head", eb, V, d, buf.data(), nullptr))) return fail(st);
  }
  std::vector<float> ones(d, 1.0f);
  for (uint32_t i = 0; i < s.n_blocks; ++i) {
    std::string p = "blk." + std::to_string(i) + ".";
    if ((st = gaje_flat_writer_add_norm(w, (p + "attn_norm").c_str(), ones.data(), d))) return fail(st);
    if ((st = gaje_flat_writer_add_norm(w, (p + "ffn_norm").c_str(), ones.data(), d))) return fail(st);
    const size_t qkv = qd + 2 * kvd;
    buf.assign(qkv * d, 0.0f);
    fill_normal(buf, name_key(s.seed, p + "attn_qkv"), std_);
    const float* bp = nullptr;
    if (s.qkv_bias) {
      bias.assign(qkv, 0.0f);
      fill_normal(bias, name_key(s.seed, p + "attn_qkv.bias"), std_);
      bp = bias.data();
    }
    if ((st = gaje_flat_writer_add_linear(w, (p + "attn_qkv").c_str(), 4, qkv, d, buf.data(), bp))) return fail(st);
    buf.assign(d * qd, 0.0f);
    fill_normal(buf, name_key(s.seed, p + "attn_output"), std_);
    if ((st = gaje_flat_writer_add_linear(w, (p + "attn_output").c_str(), 4, d, qd, buf.data(), nullptr))) return fail(st);
    buf.assign(2 * ff * d, 0.0f);
    fill_normal(buf, name_key(s.seed, p + "ffn_gate_up"), std_);
    if ((st = gaje_flat_writer_add_linear(w, (p + "ffn_gate_up").c_str(), 4, 2 * ff, d, buf.data(), nullptr))) return fail(st);
    buf.assign(d * ff, 0.0f);
    fill_normal(buf, name_key(s.seed, p + "ffn_down"), std_);
    if ((st = gaje_flat_writer_add_linear(w, (p + "ffn_down").c_str(), 4, d, ff, buf.data(), nullptr))) return fail(st);
  }
  return gaje_flat_writer_close(w);
}
