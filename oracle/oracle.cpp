// oracle.cpp -- CPU restatement of the GAJE reference decode path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA engine, not
// part of it: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
// --impl reference legs may load liboracle.so.  Nothing in the shipped library
// links or calls it.
//
// It restates, in C++ with the same AVX2/FMA intrinsic sequences, the Rust
// reference's CPU engine for `.gaje.flat` v2 models (paths are relative to the
// reference project root):
//   header / reader  src/io/header/flat.rs:14-148, src/io/flat_reader.rs:9-251,
//                    src/io/config.rs:137-145
//   blocks           src/io/header/blocks.rs:9-50
//   linear           src/nn/linear/init.rs:12-161, src/nn/linear/forward.rs:11-132,195-285
//   kernels          src/compute/kernels/genomic.rs:149-448 (Q4_0, Q8_0, 4-bit LUT),
//                    src/compute/kernels/dot.rs:23-67, norm.rs:17-87,
//                    activation.rs:35-51, lut.rs:45-61
//   attention        src/nn/attention.rs:45-128
//   block / model    src/nn/block/forward.rs:10-157, src/nn/llm/forward.rs:7-63,215-330
//   quantiser        src/compute/quantize/python.rs:152-303
//
// Build flags matter: -O3 -mavx2 -mfma -mf16c -ffp-contract=off.  Rust never
// contracts a*b+c, so every scalar expression here must stay uncontracted.
// OpenMP over output rows / heads stands in for rayon; every row or head is
// reduced by one thread, so results are deterministic.
//
// Parity status: header layout, Q4_0 block round trip, Q4_0 linear forward and
// the split-RoPE formula are pinned by the reference's own unit tests (restated
// in tests/test_oracle_kat.py).  Whole-model forward is pinned only by this
// restatement: the Rust crate cannot be built in this container (no rustc, no
// vendored crates), so no reference-produced logits exist.

#include <immintrin.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ---------------------------------------------------------------- f16 helpers
// half::f16::to_f32 is exact; F16C's vcvtph2ps is exact too.
inline float h2f(uint16_t h) { return _cvtsh_ss(h); }
// half::f16::from_f32 rounds to nearest, ties to even (imm 0 = RNE).
inline uint16_t f2h(float f) { return _cvtss_sh(f, 0); }

#pragma pack(push, 1)
struct Q4Block {  // blocks.rs:9-14, 20 bytes
  uint16_t scale;
  uint16_t min;
  uint8_t qs[16];
};
struct Q8Block {  // blocks.rs:37-41, 34 bytes
  uint16_t scale;
  int8_t qs[32];
};
#pragma pack(pop)
static_assert(sizeof(Q4Block) == 20, "Q4Block");
static_assert(sizeof(Q8Block) == 34, "Q8Block");

// ------------------------------------------------------------------ kernels
// The 128-bit horizontal sum used by dot.rs:57-63 and norm.rs:62-68:
// ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)).
inline float hsum_dot_order(__m256 acc) {
  __m128 hi = _mm256_extractf128_ps(acc, 1);
  __m128 lo = _mm256_castps256_ps128(acc);
  __m128 sum128 = _mm_add_ps(lo, hi);
  __m128 shuf = _mm_movehdup_ps(sum128);
  __m128 sums = _mm_add_ps(sum128, shuf);
  __m128 shuf2 = _mm_movehl_ps(sums, sums);
  __m128 result = _mm_add_ss(sums, shuf2);
  return _mm_cvtss_f32(result);
}

// The horizontal sum used by genomic.rs:322-329 (Q4_0) and :436-443 (Q8_0):
// ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)).
inline float hsum_q_order(__m256 acc) {
  __m128 vlow = _mm256_castps256_ps128(acc);
  __m128 vhigh = _mm256_extractf128_ps(acc, 1);
  __m128 v128 = _mm_add_ps(vlow, vhigh);
  __m128 hi = _mm_movehl_ps(v128, v128);
  __m128 sum = _mm_add_ps(v128, hi);
  __m128 shuf = _mm_shuffle_ps(sum, sum, 1);
  __m128 final_sum = _mm_add_ss(sum, shuf);
  return _mm_cvtss_f32(final_sum);
}

// dot.rs:23-67 (x86_64, AVX2+FMA arm)
float dot_f32(const float* a, const float* b, size_t n) {
  __m256 acc = _mm256_setzero_ps();
  size_t i = 0;
  while (i + 8 <= n) {
    __m256 va = _mm256_loadu_ps(a + i);
    __m256 vb = _mm256_loadu_ps(b + i);
    acc = _mm256_fmadd_ps(va, vb, acc);
    i += 8;
  }
  float sum = hsum_dot_order(acc);
  while (i < n) {
    sum += a[i] * b[i];
    i += 1;
  }
  return sum;
}

// genomic.rs:267-336 genomic_dot_product_q4_0_avx2
float q4_0_dot_avx2(const Q4Block* blocks, const float* input, size_t n_blocks) {
  __m256 acc = _mm256_setzero_ps();
  const __m128i mask_low = _mm_set1_epi8(0x0F);
  for (size_t j = 0; j < n_blocks; ++j) {
    const Q4Block& block = blocks[j];
    float scale = h2f(block.scale);
    float mn = h2f(block.min);
    __m256 v_scale = _mm256_set1_ps(scale);
    __m256 v_min = _mm256_set1_ps(mn);
    size_t off = j * 32;
    __m128i v_qs = _mm_loadu_si128(reinterpret_cast<const __m128i*>(block.qs));
    __m128i low_nibbles = _mm_and_si128(v_qs, mask_low);
    __m128i high_nibbles = _mm_and_si128(_mm_srli_epi16(v_qs, 4), mask_low);
    __m128i il_lo = _mm_unpacklo_epi8(low_nibbles, high_nibbles);
    __m128i il_hi = _mm_unpackhi_epi8(low_nibbles, high_nibbles);

    __m256 q0 = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(il_lo));
    __m256 d0 = _mm256_fmadd_ps(q0, v_scale, v_min);
    acc = _mm256_fmadd_ps(d0, _mm256_loadu_ps(input + off), acc);

    __m256 q1 = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(_mm_srli_si128(il_lo, 8)));
    __m256 d1 = _mm256_fmadd_ps(q1, v_scale, v_min);
    acc = _mm256_fmadd_ps(d1, _mm256_loadu_ps(input + off + 8), acc);

    __m256 q2 = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(il_hi));
    __m256 d2 = _mm256_fmadd_ps(q2, v_scale, v_min);
    acc = _mm256_fmadd_ps(d2, _mm256_loadu_ps(input + off + 16), acc);

    __m256 q3 = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(_mm_srli_si128(il_hi, 8)));
    __m256 d3 = _mm256_fmadd_ps(q3, v_scale, v_min);
    acc = _mm256_fmadd_ps(d3, _mm256_loadu_ps(input + off + 24), acc);
  }
  float total = hsum_q_order(acc);
  return std::fabs(total) < 1e-6f ? 0.0f : total;
}

// genomic.rs:228-260, the scalar fallback (factored sum; only used off-AVX2).
float q4_0_dot_scalar(const Q4Block* blocks, const float* input, size_t n_blocks) {
  float total = 0.0f;
  for (size_t j = 0; j < n_blocks; ++j) {
    const Q4Block& b = blocks[j];
    float scale = h2f(b.scale), mn = h2f(b.min);
    size_t off = j * 32;
    float sum_q_in = 0.0f, sum_in = 0.0f;
    for (int k = 0; k < 16; ++k) {
      uint8_t byte = b.qs[k];
      float q0 = float(byte & 0x0F), q1 = float(byte >> 4);
      float x0 = input[off + k * 2], x1 = input[off + k * 2 + 1];
      float p0 = q0 * x0, p1 = q1 * x1;
      sum_q_in += p0 + p1;
      sum_in += x0 + x1;
    }
    float a = sum_q_in * scale, c = sum_in * mn;
    total += a + c;
  }
  return std::fabs(total) < 1e-6f ? 0.0f : total;
}

// genomic.rs:381-448 genomic_dot_product_q8_0_avx2
float q8_0_dot_avx2(const Q8Block* blocks, const float* input, size_t n_blocks) {
  __m256 acc = _mm256_setzero_ps();
  for (size_t j = 0; j < n_blocks; ++j) {
    const Q8Block& block = blocks[j];
    __m256 v_scale = _mm256_set1_ps(h2f(block.scale));
    size_t off = j * 32;
    __m256i v_qs = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(block.qs));
    __m128i lo_128 = _mm256_castsi256_si128(v_qs);
    __m128i hi_128 = _mm256_extracti128_si256(v_qs, 1);
    __m128i lo_lo_16 = _mm_cvtepi8_epi16(lo_128);
    __m128i lo_hi_16 = _mm_cvtepi8_epi16(_mm_srli_si128(lo_128, 8));
    __m256 q_0 = _mm256_cvtepi32_ps(_mm256_cvtepi16_epi32(lo_lo_16));
    __m256 q_1 = _mm256_cvtepi32_ps(_mm256_cvtepi16_epi32(lo_hi_16));
    __m128i hi_lo_16 = _mm_cvtepi8_epi16(hi_128);
    __m128i hi_hi_16 = _mm_cvtepi8_epi16(_mm_srli_si128(hi_128, 8));
    __m256 q_2 = _mm256_cvtepi32_ps(_mm256_cvtepi16_epi32(hi_lo_16));
    __m256 q_3 = _mm256_cvtepi32_ps(_mm256_cvtepi16_epi32(hi_hi_16));
    __m256 x_0 = _mm256_loadu_ps(input + off);
    __m256 x_1 = _mm256_loadu_ps(input + off + 8);
    __m256 x_2 = _mm256_loadu_ps(input + off + 16);
    __m256 x_3 = _mm256_loadu_ps(input + off + 24);
    __m256 dq_0 = _mm256_mul_ps(q_0, v_scale);
    __m256 dq_1 = _mm256_mul_ps(q_1, v_scale);
    __m256 dq_2 = _mm256_mul_ps(q_2, v_scale);
    __m256 dq_3 = _mm256_mul_ps(q_3, v_scale);
    acc = _mm256_fmadd_ps(dq_0, x_0, acc);
    acc = _mm256_fmadd_ps(dq_1, x_1, acc);
    acc = _mm256_fmadd_ps(dq_2, x_2, acc);
    acc = _mm256_fmadd_ps(dq_3, x_3, acc);
  }
  float total = hsum_q_order(acc);
  return std::fabs(total) < 1e-6f ? 0.0f : total;
}

// genomic.rs:149-204 genomic_dot_product_4bit: 16 f32 centroids per block,
// HIGH nibble first, four interleaved scalar accumulators.
float lut4_dot(const uint8_t* w, const float* input, const float* centroids,
               size_t stride, size_t n_blocks) {
  size_t block_size = stride * 2;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  for (size_t j = 0; j < n_blocks; ++j) {
    const float* in = input + j * block_size;
    const uint8_t* wb = w + j * stride;
    const float* c = centroids + j * 16;
    size_t k = 0;
    while (k + 4 <= stride) {
      uint8_t b0 = wb[k], b1 = wb[k + 1], b2 = wb[k + 2], b3 = wb[k + 3];
      const float* ip = in + k * 2;
      float t;
      t = c[b0 >> 4] * ip[0]; s0 += t;
      t = c[b0 & 15] * ip[1]; s1 += t;
      t = c[b1 >> 4] * ip[2]; s2 += t;
      t = c[b1 & 15] * ip[3]; s3 += t;
      t = c[b2 >> 4] * ip[4]; s0 += t;
      t = c[b2 & 15] * ip[5]; s1 += t;
      t = c[b3 >> 4] * ip[6]; s2 += t;
      t = c[b3 & 15] * ip[7]; s3 += t;
      k += 4;
    }
    while (k < stride) {
      uint8_t byte = wb[k];
      float t;
      t = c[byte >> 4] * in[k * 2]; s0 += t;
      t = c[byte & 15] * in[k * 2 + 1]; s1 += t;
      k += 1;
    }
  }
  float total = s0 + s1;
  total = total + s2;
  total = total + s3;
  return std::fabs(total) < 1e-6f ? 0.0f : total;
}

// norm.rs:54-87 (AVX2 arm)
void rms_norm(const float* x, const float* w, float eps, size_t n, float* out) {
  __m256 acc = _mm256_setzero_ps();
  size_t i = 0;
  while (i + 8 <= n) {
    __m256 vx = _mm256_loadu_ps(x + i);
    acc = _mm256_fmadd_ps(vx, vx, acc);
    i += 8;
  }
  float sum_sq = hsum_dot_order(acc);
  while (i < n) {
    float t = x[i] * x[i];
    sum_sq += t;
    i += 1;
  }
  float mean = sum_sq / float(n);
  float inv_rms = 1.0f / std::sqrt(mean + eps);
  __m256 inv_v = _mm256_set1_ps(inv_rms);
  i = 0;
  while (i + 8 <= n) {
    __m256 vx = _mm256_loadu_ps(x + i);
    __m256 vw = _mm256_loadu_ps(w + i);
    _mm256_storeu_ps(out + i, _mm256_mul_ps(_mm256_mul_ps(vx, inv_v), vw));
    i += 8;
  }
  while (i < n) {
    float t = x[i] * inv_rms;
    out[i] = t * w[i];
    i += 1;
  }
}

// Rust f32::clamp: NaN passes through.
inline float rust_clamp(float v, float lo, float hi) {
  if (v < lo) return lo;
  if (v > hi) return hi;
  return v;
}

// activation.rs:35-51 swiglu_balanced
void swiglu_balanced(const float* gate, const float* up, float* out, size_t n) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; ++i) {
    float g = gate[i], u = up[i];
    float gs = rust_clamp(g, -64.0f, 64.0f);
    float sig;
    if (gs >= 0.0f) {
      float e = std::exp(-gs);
      float d = 1.0f + e;
      sig = 1.0f / d;
    } else {
      float ex = std::exp(gs);
      float d = 1.0f + ex;
      sig = ex / d;
    }
    float silu = g * sig;
    out[i] = silu * u;
  }
}

// lut.rs:45-61 lateral_inhibition_kwta: k-th largest by a full descending
// sort; everything strictly below it becomes -1e9.
void kwta(float* scores, size_t n, size_t k) {
  if (n <= k) return;
  std::vector<float> s(scores, scores + n);
  std::nth_element(s.begin(), s.begin() + (k - 1), s.end(), std::greater<float>());
  float thr = s[k - 1];
  for (size_t i = 0; i < n; ++i)
    if (scores[i] < thr) scores[i] = -1e9f;
}

// attention.rs:62-84, the RoPE closure.  powf/sinf/cosf are glibc's, as Rust
// std lowers f32::powf / sin / cos to libm calls on Linux.
void rope_apply(float* vec, size_t heads, size_t head_dim, size_t pos, float base,
                bool split) {
  size_t half = head_dim / 2;
  for (size_t h = 0; h < heads; ++h) {
    size_t hs = h * head_dim;
    for (size_t i = 0; i < half; ++i) {
      float e = (2.0f * float(i)) / float(head_dim);
      float freq = 1.0f / powf(base, e);
      float theta = float(pos) * freq;
      float sn = sinf(theta), cs = cosf(theta);
      size_t a = split ? hs + i : hs + 2 * i;
      size_t b = split ? hs + i + half : hs + 2 * i + 1;
      float v0 = vec[a], v1 = vec[b];
      float p0 = v0 * cs, p1 = v1 * sn;
      float p2 = v0 * sn, p3 = v1 * cs;
      vec[a] = p0 - p1;
      vec[b] = p2 + p3;
    }
  }
}

// quantize/python.rs:152-232 quantize_q4_0_native, one 32-element block.
Q4Block quantize_q4_block(const float* b) {
  float mn = 3.40282347e+38f, mx = -3.40282347e+38f;
  for (int i = 0; i < 32; ++i) {
    if (b[i] < mn) mn = b[i];
    if (b[i] > mx) mx = b[i];
  }
  float scale = (mx - mn) / 15.0f;
  float inv = scale > 1e-7f ? 1.0f / scale : 0.0f;
  Q4Block out;
  for (int k = 0; k < 16; ++k) {
    uint8_t q[2] = {0, 0};
    for (int t = 0; t < 2; ++t) {
      if (scale > 1e-7f) {
        float d = b[k * 2 + t] - mn;
        float r = roundf(d * inv);  // Rust f32::round: half away from zero
        r = rust_clamp(r, 0.0f, 15.0f);
        q[t] = (r != r) ? 0 : uint8_t(r);  // `as u8` saturates, NaN -> 0
      }
    }
    out.qs[k] = uint8_t(q[0] | (q[1] << 4));
  }
  out.scale = f2h(scale);
  out.min = f2h(mn);
  return out;
}

// quantize/python.rs:235-303 quantize_q8_0_native, one block.
Q8Block quantize_q8_block(const float* b) {
  float max_abs = 0.0f;
  for (int i = 0; i < 32; ++i) {
    float a = std::fabs(b[i]);
    if (a > max_abs) max_abs = a;
  }
  float scale = max_abs / 127.0f;
  float inv = scale > 1e-7f ? 1.0f / scale : 0.0f;
  Q8Block out;
  for (int k = 0; k < 32; ++k) {
    if (scale > 1e-7f) {
      float r = roundf(b[k] * inv);
      r = rust_clamp(r, -128.0f, 127.0f);
      out.qs[k] = (r != r) ? 0 : int8_t(r);
    } else {
      out.qs[k] = 0;
    }
  }
  out.scale = f2h(scale);
  return out;
}

// --------------------------------------------------------------- mini JSON
// Just enough JSON for the flat metadata (serde ModelConfig) and directory.
struct JVal {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  double num = 0;
  std::string raw_num, str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char* p;
  const char* e;
  std::string err;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool fail(const char* m) {
    if (err.empty()) err = m;
    return false;
  }
  bool parse_str(std::string& out) {
    if (p >= e || *p != '"') return fail("expected string");
    ++p;
    while (p < e && *p != '"') {
      if (*p == '\\') {
        ++p;
        if (p >= e) return fail("bad escape");
        char c = *p++;
        switch (c) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (e - p < 4) return fail("bad \\u");
            unsigned cp = 0;
            for (int i = 0; i < 4; ++i) {
              char h = p[i];
              cp <<= 4;
              if (h >= '0' && h <= '9') cp |= h - '0';
              else if (h >= 'a' && h <= 'f') cp |= h - 'a' + 10;
              else if (h >= 'A' && h <= 'F') cp |= h - 'A' + 10;
              else return fail("bad \\u");
            }
            p += 4;
            // UTF-8 encode (surrogate pairs are kept as two code points; the
            // names this reader looks up are ASCII).
            if (cp < 0x80) out += char(cp);
            else if (cp < 0x800) { out += char(0xC0 | (cp >> 6)); out += char(0x80 | (cp & 63)); }
            else { out += char(0xE0 | (cp >> 12)); out += char(0x80 | ((cp >> 6) & 63)); out += char(0x80 | (cp & 63)); }
            break;
          }
          default: out += c;
        }
      } else {
        out += *p++;
      }
    }
    if (p >= e) return fail("unterminated string");
    ++p;
    return true;
  }
  bool parse(JVal& v, int depth = 0) {
    if (depth > 64) return fail("too deep");
    ws();
    if (p >= e) return fail("unexpected end");
    char c = *p;
    if (c == '{') {
      v.kind = JVal::OBJ;
      ++p;
      ws();
      if (p < e && *p == '}') { ++p; return true; }
      for (;;) {
        ws();
        std::string k;
        if (!parse_str(k)) return false;
        ws();
        if (p >= e || *p != ':') return fail("expected ':'");
        ++p;
        JVal child;
        if (!parse(child, depth + 1)) return false;
        v.obj.emplace_back(std::move(k), std::move(child));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == '}') { ++p; return true; }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = JVal::ARR;
      ++p;
      ws();
      if (p < e && *p == ']') { ++p; return true; }
      for (;;) {
        JVal child;
        if (!parse(child, depth + 1)) return false;
        v.arr.push_back(std::move(child));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == ']') { ++p; return true; }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') { v.kind = JVal::STR; return parse_str(v.str); }
    if (e - p >= 4 && !strncmp(p, "true", 4)) { v.kind = JVal::BOOL; v.b = true; p += 4; return true; }
    if (e - p >= 5 && !strncmp(p, "false", 5)) { v.kind = JVal::BOOL; v.b = false; p += 5; return true; }
    if (e - p >= 4 && !strncmp(p, "null", 4)) { v.kind = JVal::NUL; p += 4; return true; }
    const char* s = p;
    while (p < e && (isdigit((unsigned char)*p) || *p == '-' || *p == '+' || *p == '.' || *p == 'e' || *p == 'E')) ++p;
    if (p == s) return fail("unexpected character");
    v.kind = JVal::NUM;
    v.raw_num.assign(s, p);
    v.num = strtod(v.raw_num.c_str(), nullptr);
    return true;
  }
};

bool json_parse(const char* data, size_t len, JVal& out, std::string& err) {
  JParser jp{data, data + len, {}};
  if (!jp.parse(out)) { err = jp.err; return false; }
  jp.ws();
  if (jp.p != jp.e) { err = "trailing characters"; return false; }
  return true;
}

bool j_usize(const JVal* v, size_t& out) {
  if (!v || v->kind != JVal::NUM) return false;
  if (v->num < 0 || v->raw_num.find_first_of(".eE") != std::string::npos) return false;
  out = size_t(strtoull(v->raw_num.c_str(), nullptr, 10));
  return true;
}

// ------------------------------------------------------------------- model
enum class WKind { F32, Q4_0, Q8_0, LUT4 };

struct Linear {  // GenomicLinear restricted to the arms a flat load produces
  WKind kind = WKind::F32;
  size_t out = 0, in = 0, block_size = 32, stride = 32;
  std::vector<uint8_t> dna;       // raw bytes (Q4/Q8 blocks, nibbles, or f32)
  std::vector<float> centroids;   // LUT4 only, expanded as init.rs:109-124
  std::vector<float> bias;

  const float* f32() const { return reinterpret_cast<const float*>(dna.data()); }
  const Q4Block* q4() const { return reinterpret_cast<const Q4Block*>(dna.data()); }
  const Q8Block* q8() const { return reinterpret_cast<const Q8Block*>(dna.data()); }
  size_t n_items() const {
    switch (kind) {
      case WKind::F32: return dna.size() / 4;
      case WKind::Q4_0: return dna.size() / sizeof(Q4Block);
      case WKind::Q8_0: return dna.size() / sizeof(Q8Block);
      default: return dna.size();
    }
  }

  // linear/forward.rs:11-117 compute_single_row
  float row(size_t i, const float* input, size_t input_len) const {
    size_t nb = in / block_size;
    float sum = 0.0f;
    switch (kind) {
      case WKind::F32: {
        const float* r = f32() + i * in;
        if (in == input_len) {
          sum = dot_f32(input, r, in);
        } else {
          size_t m = std::min(in, input_len);
          for (size_t k = 0; k < m; ++k) { float t = input[k] * r[k]; sum += t; }
        }
        break;
      }
      case WKind::Q4_0:
        if ((i + 1) * nb <= n_items()) sum = q4_0_dot_avx2(q4() + i * nb, input, nb);
        break;
      case WKind::Q8_0:
        if ((i + 1) * nb <= n_items()) sum = q8_0_dot_avx2(q8() + i * nb, input, nb);
        break;
      case WKind::LUT4: {
        size_t off = i * nb * stride;
        if (off + nb * stride <= dna.size()) {
          size_t c0 = i * nb * 16;
          if (centroids.size() >= c0 + nb * 16)
            sum = lut4_dot(dna.data() + off, input, centroids.data() + c0, stride, nb);
        }
        break;
      }
    }
    if (i < bias.size()) sum += bias[i];
    return sum;
  }

  void forward(const float* input, size_t input_len, float* y) const {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < out; ++i) y[i] = row(i, input, input_len);
  }

  // linear/forward.rs:195-285 get_row_core
  std::vector<float> get_row(size_t idx) const {
    std::vector<float> res(in, 0.0f);
    if (out == 0 || in == 0) return res;
    size_t r = idx % out;
    size_t nb = in / block_size;
    switch (kind) {
      case WKind::F32:
        if ((r + 1) * in <= n_items()) memcpy(res.data(), f32() + r * in, in * 4);
        break;
      case WKind::Q4_0:
        if ((r + 1) * nb <= n_items())
          for (size_t b = 0; b < nb; ++b) {
            const Q4Block& blk = q4()[r * nb + b];
            float sc = h2f(blk.scale), mn = h2f(blk.min);
            for (size_t k = 0; k < 32; ++k) {
              uint8_t q = (k % 2 == 0) ? (blk.qs[k / 2] & 0x0F) : (blk.qs[k / 2] >> 4);
              float t = float(q) * sc;  // blocks.rs:29, unfused
              res[b * block_size + k] = t + mn;
            }
          }
        break;
      case WKind::Q8_0:
        if ((r + 1) * nb <= n_items())
          for (size_t b = 0; b < nb; ++b) {
            const Q8Block& blk = q8()[r * nb + b];
            float sc = h2f(blk.scale);
            for (size_t k = 0; k < 32; ++k) res[b * block_size + k] = float(blk.qs[k]) * sc;
          }
        break;
      case WKind::LUT4: {
        size_t off = r * nb * stride;
        if (off + nb * stride <= dna.size())
          for (size_t b = 0; b < nb; ++b) {
            const float* c = centroids.data() + (r * nb + b) * 16;
            for (size_t k = 0; k < stride; ++k) {
              uint8_t byte = dna[off + b * stride + k];
              res[b * block_size + k * 2] = c[byte >> 4];
              res[b * block_size + k * 2 + 1] = c[byte & 15];
            }
          }
        break;
      }
    }
    return res;
  }
};

struct Block {
  std::vector<float> attn_norm, ffn_norm;
  Linear qkv, wo, gate_up, down;
  std::vector<std::vector<float>> k_cache, v_cache;  // attention.rs:14-15
  float k_wta_ratio = 0.0f;                          // block/init.rs:42
};

struct Model {
  size_t n_embd = 0, n_head = 0, n_head_kv = 0, n_blocks = 0, head_dim = 0;
  float eps = 1e-6f, rope_base = 10000.0f;
  bool rope_split = true, use_genomic_norm = false;
  float h_scale = 1.0f;
  Linear embd, lm_head;
  std::vector<float> output_norm;
  std::vector<Block> blocks;
  float k_wta_ratio = 0.5f;  // flat_reader.rs:234
};

// attention.rs:45-128 forward_attention_core
void attention(Block& blk, const Model& m, std::vector<float>& q, std::vector<float>& k,
               std::vector<float>& v, size_t pos, float* out) {
  size_t nh = m.n_head, nkv = m.n_head_kv, hd = m.head_dim;
  size_t groups = nh / nkv;
  float scale = 1.0f / std::sqrt(float(hd));
  rope_apply(q.data(), nh, hd, pos, m.rope_base, m.rope_split);
  rope_apply(k.data(), nkv, hd, pos, m.rope_base, m.rope_split);
  blk.k_cache.push_back(k);
  blk.v_cache.push_back(v);
  size_t T = blk.k_cache.size();
#pragma omp parallel for schedule(static)
  for (size_t h = 0; h < nh; ++h) {
    size_t kvo = (h / groups) * hd;
    const float* qh = q.data() + h * hd;
    std::vector<float> scores(T);
    float mx = -INFINITY;
    for (size_t t = 0; t < T; ++t) {
      float s = dot_f32(qh, blk.k_cache[t].data() + kvo, hd) * scale;
      scores[t] = s;
      if (s > mx) mx = s;
    }
    float sum_e = 0.0f;
    for (size_t t = 0; t < T; ++t) {
      float d = scores[t] - mx;
      scores[t] = std::exp(d);
      sum_e += scores[t];
    }
    float inv_s = 1.0f / (sum_e + 1e-12f);
    float* o = out + h * hd;
    for (size_t i = 0; i < hd; ++i) o[i] = 0.0f;
    for (size_t t = 0; t < T; ++t) {
      float w = scores[t] * inv_s;
      const float* vh = blk.v_cache[t].data() + kvo;
      for (size_t i = 0; i < hd; ++i) {
        float p = w * vh[i];
        o[i] += p;
      }
    }
  }
}

bool has_nan(const float* v, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (v[i] != v[i]) return true;
  return false;
}

// block/forward.rs:10-157 forward_core (topology is None for flat loads)
bool block_forward(Block& b, const Model& m, std::vector<float>& x, size_t pos,
                   std::string& err) {
  size_t d = x.size();
  if (has_nan(x.data(), d)) { err = "Input x is NaN"; return false; }
  std::vector<float> xn(d);
  if (!b.attn_norm.empty()) {
    rms_norm(x.data(), b.attn_norm.data(), m.eps, d, xn.data());
    if (has_nan(xn.data(), d)) { err = "NaN after attn rms_norm"; return false; }
  } else {
    xn = x;
  }
  size_t qd = m.n_head * m.head_dim, kvd = m.n_head_kv * m.head_dim;
  std::vector<float> qkv(b.qkv.out);
  b.qkv.forward(xn.data(), d, qkv.data());
  std::vector<float> q(qkv.begin(), qkv.begin() + qd);
  std::vector<float> k(qkv.begin() + qd, qkv.begin() + qd + kvd);
  std::vector<float> v(qkv.begin() + qd + kvd, qkv.begin() + qd + 2 * kvd);
  std::vector<float> att(qd);
  attention(b, m, q, k, v, pos, att.data());
  std::vector<float> proj(b.wo.out);
  b.wo.forward(att.data(), qd, proj.data());
  for (size_t i = 0; i < d && i < proj.size(); ++i) x[i] += proj[i];
  std::vector<float> xf(d);
  rms_norm(x.data(), b.ffn_norm.data(), m.eps, d, xf.data());
  std::vector<float> gu(b.gate_up.out);
  b.gate_up.forward(xf.data(), d, gu.data());
  size_t ff = gu.size() / 2;
  if (has_nan(gu.data() + ff, ff)) { err = "NaN in up"; return false; }
  std::vector<float> act(ff);
  swiglu_balanced(gu.data(), gu.data() + ff, act.data(), ff);
  if (has_nan(act.data(), ff)) { err = "NaN in ffn_out"; return false; }
  if (m.use_genomic_norm) {
    // block/forward.rs:115-123.  The reference sums with a rayon reduction
    // (order not reproducible); this restatement sums sequentially.
    float ss = 0.0f;
    for (size_t i = 0; i < ff; ++i) { float t = act[i] * act[i]; ss += t; }
    float rms = std::sqrt(ss / float(ff) + m.eps);
    if (rms > m.h_scale) {
      float s = m.h_scale / rms;
      for (size_t i = 0; i < ff; ++i) act[i] *= s;
    }
  }
  std::vector<float> pf(b.down.out);
  b.down.forward(act.data(), ff, pf.data());
  if (has_nan(pf.data(), pf.size())) { err = "NaN in projected_ffn"; return false; }
  for (size_t i = 0; i < d && i < pf.size(); ++i) x[i] += pf[i];
  if (has_nan(x.data(), d)) { err = "NaN after projected_ffn addition"; return false; }
  if (b.k_wta_ratio > 0.0f && b.k_wta_ratio < 1.0f) {
    float kf = float(d) * b.k_wta_ratio;
    size_t kk = std::max<size_t>(1, size_t(kf));
    kwta(x.data(), d, kk);
  }
  return true;
}

// llm/forward.rs:7-63 forward_core
bool model_forward(Model& m, size_t token, bool clear, std::vector<float>& logits,
                   std::string& err) {
  if (clear)
    for (auto& b : m.blocks) { b.k_cache.clear(); b.v_cache.clear(); }
  size_t pos = m.blocks.empty() ? 0 : m.blocks[0].k_cache.size();
  std::vector<float> h = m.embd.get_row(token);
  for (auto& b : m.blocks)
    if (!block_forward(b, m, h, pos, err)) return false;
  std::vector<float> hn(h.size());
  rms_norm(h.data(), m.output_norm.data(), m.eps, h.size(), hn.data());
  if (m.lm_head.out == 0) { err = "LM Head out_features is 0!"; return false; }
  logits.assign(m.lm_head.out, 0.0f);
  m.lm_head.forward(hn.data(), hn.size(), logits.data());
  if (m.k_wta_ratio > 0.0f && m.k_wta_ratio < 1.0f) {
    float kf = float(logits.size()) * m.k_wta_ratio;
    size_t kk = std::max<size_t>(1, size_t(kf));
    kwta(logits.data(), logits.size(), kk);
  }
  return true;
}

// ----------------------------------------------------------------- loader
struct Entry {
  std::string name;
  size_t bit_depth = 0, out = 0, in = 0, dna_off = 0, dna_len = 0, c_off = 0, c_len = 0,
         anc_off = 0, anc_len = 0, bias_off = 0, bias_len = 0;
};

struct Mapped {
  void* base = nullptr;
  size_t size = 0;
  ~Mapped() { if (base && base != MAP_FAILED) munmap(base, size); }
};

bool rd_u32(const uint8_t* p, size_t off, uint32_t& v) { memcpy(&v, p + off, 4); return true; }

bool load_model(const char* path, Model& m, std::string& err) {
  int fd = open(path, O_RDONLY);
  if (fd < 0) { err = std::string("cannot open ") + path; return false; }
  struct stat st;
  fstat(fd, &st);
  Mapped mp;
  mp.size = size_t(st.st_size);
  if (mp.size < 4096) { close(fd); err = "file shorter than the 4096-byte header"; return false; }
  mp.base = mmap(nullptr, mp.size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (mp.base == MAP_FAILED) { err = "mmap failed"; return false; }
  const uint8_t* f = static_cast<const uint8_t*>(mp.base);
  // header/flat.rs:47-60: only the magic is validated.
  if (memcmp(f, "GAJE", 4) != 0) { err = "invalid magic"; return false; }
  uint64_t meta_len, dir_len, weights_offset;
  memcpy(&meta_len, f + 16, 8);
  memcpy(&dir_len, f + 24, 8);
  memcpy(&weights_offset, f + 32, 8);
  uint32_t arch_family, a_embd, a_head, a_head_kv, a_blocks;
  rd_u32(f, 56, arch_family);
  rd_u32(f, 60, a_embd);
  rd_u32(f, 64, a_head);
  rd_u32(f, 68, a_head_kv);
  rd_u32(f, 72, a_blocks);
  if (4096 + meta_len + dir_len > mp.size) { err = "metadata/directory past end of file"; return false; }
  JVal meta, dir;
  if (!json_parse(reinterpret_cast<const char*>(f) + 4096, meta_len, meta, err)) { err = "metadata JSON: " + err; return false; }
  if (!json_parse(reinterpret_cast<const char*>(f) + 4096 + meta_len, dir_len, dir, err)) { err = "directory JSON: " + err; return false; }
  // config.rs:137-145 ModelConfig (required: config, n_embd, n_head, n_head_kv, n_blocks, eps)
  const JVal* cfg = meta.get("config");
  const JVal* eps = meta.get("eps");
  if (meta.kind != JVal::OBJ || !cfg || cfg->kind != JVal::OBJ || !eps || eps->kind != JVal::NUM ||
      !j_usize(meta.get("n_embd"), m.n_embd) || !j_usize(meta.get("n_head"), m.n_head) ||
      !j_usize(meta.get("n_head_kv"), m.n_head_kv) || !j_usize(meta.get("n_blocks"), m.n_blocks)) {
    err = "metadata JSON is missing a required ModelConfig field";
    return false;
  }
  m.eps = float(eps->num);
  if (const JVal* rb = cfg->get("rope_base")) if (rb->kind == JVal::NUM) m.rope_base = float(rb->num);
  std::string rope_style = "split";
  if (const JVal* rs = cfg->get("rope_style")) if (rs->kind == JVal::STR) rope_style = rs->str;
  if (const JVal* g = cfg->get("use_genomic_norm")) if (g->kind == JVal::BOOL) m.use_genomic_norm = g->b;
  // flat_reader.rs:127-139 header descriptor override (flat.rs:82-148)
  if (arch_family != 0) {
    m.n_embd = a_embd; m.n_head = a_head; m.n_head_kv = a_head_kv; m.n_blocks = a_blocks;
    switch (arch_family) {
      case 2: m.rope_base = 100000.0f; break;
      case 3: case 4: m.rope_base = 1000000.0f; break;
      default: m.rope_base = 10000.0f; break;
    }
    rope_style = "split";
  }
  m.rope_split = (rope_style == "split");
  if (m.n_head == 0 || m.n_head_kv == 0) { err = "n_head and n_head_kv must be non-zero"; return false; }
  m.head_dim = m.n_embd / m.n_head;

  std::map<std::string, Entry> dmap;
  if (dir.kind != JVal::ARR) { err = "directory JSON is not an array"; return false; }
  for (const JVal& ev : dir.arr) {
    Entry e;
    const JVal* nm = ev.get("name");
    if (!nm || nm->kind != JVal::STR ||
        !j_usize(ev.get("bit_depth"), e.bit_depth) || !j_usize(ev.get("out_features"), e.out) ||
        !j_usize(ev.get("in_features"), e.in) || !j_usize(ev.get("dna_off"), e.dna_off) ||
        !j_usize(ev.get("dna_len"), e.dna_len) || !j_usize(ev.get("c_off"), e.c_off) ||
        !j_usize(ev.get("c_len"), e.c_len) || !j_usize(ev.get("anc_off"), e.anc_off) ||
        !j_usize(ev.get("anc_len"), e.anc_len) || !j_usize(ev.get("bias_off"), e.bias_off) ||
        !j_usize(ev.get("bias_len"), e.bias_len)) {
      err = "directory entry is missing a field";
      return false;
    }
    e.name = nm->str;
    dmap[e.name] = e;
  }
  auto slice = [&](size_t off, size_t len, std::vector<uint8_t>& out) -> bool {
    out.clear();
    if (len == 0) return true;
    size_t s = size_t(weights_offset) + off;
    if (s + len > mp.size) { err = "tensor data past end of file"; return false; }
    out.assign(f + s, f + s + len);
    return true;
  };
  auto fslice = [&](size_t off, size_t len, std::vector<float>& out) -> bool {
    std::vector<uint8_t> b;
    if (!slice(off, len, b)) return false;
    out.resize(b.size() / 4);
    if (!out.empty()) memcpy(out.data(), b.data(), out.size() * 4);
    return true;
  };
  // flat_reader.rs:92-122 get_linear + init.rs:12-161 GenomicLinear::new
  auto linear = [&](const std::string& name, Linear& L) -> bool {
    auto it = dmap.find(name);
    if (it == dmap.end()) { err = "Flat tensor entry '" + name + "' not found"; return false; }
    const Entry& e = it->second;
    if (!slice(e.dna_off, e.dna_len, L.dna)) return false;
    std::vector<float> cents;
    if (!fslice(e.c_off, e.c_len, cents)) return false;
    if (!fslice(e.bias_off, e.bias_len, L.bias)) return false;
    if (e.anc_len != 0) { err = "sparse anchors are not supported (" + name + ")"; return false; }
    L.out = e.out; L.in = e.in; L.block_size = 32;
    size_t nb = L.in / 32;
    switch (e.bit_depth) {
      case 4:
        L.stride = 16;
        if (cents.empty()) { L.kind = WKind::Q4_0; }
        else {
          L.kind = WKind::LUT4;
          if (cents.size() == 16) {
            L.centroids.reserve(L.out * nb * 16);
            for (size_t i = 0; i < L.out * nb; ++i) L.centroids.insert(L.centroids.end(), cents.begin(), cents.end());
          } else if (cents.size() == nb * 16) {
            for (size_t i = 0; i < L.out; ++i) L.centroids.insert(L.centroids.end(), cents.begin(), cents.end());
          } else if (cents.size() == L.out * nb * 16) {
            L.centroids = cents;
          } else { err = "unsupported centroid count for " + name; return false; }
        }
        break;
      case 8: L.kind = WKind::Q8_0; L.stride = 32; break;
      case 32: L.kind = WKind::F32; L.stride = 32; break;
      default: err = "unsupported bit_depth for " + name; return false;
    }
    return true;
  };
  auto norm = [&](const std::string& name, std::vector<float>& out) -> bool {
    auto it = dmap.find(name);
    if (it == dmap.end()) { err = "Flat tensor entry '" + name + "' not found"; return false; }
    return fslice(it->second.dna_off, it->second.dna_len, out);
  };
  if (!linear("token_embd", m.embd)) return false;
  if (!norm("output_norm", m.output_norm)) return false;
  if (!linear("lm_head", m.lm_head)) return false;
  m.blocks.resize(m.n_blocks);
  for (size_t i = 0; i < m.n_blocks; ++i) {
    std::string p = "blk." + std::to_string(i) + ".";
    Block& b = m.blocks[i];
    if (!norm(p + "attn_norm", b.attn_norm) || !norm(p + "ffn_norm", b.ffn_norm)) return false;
    if (dmap.count(p + "attn_qkv")) {
      if (!linear(p + "attn_qkv", b.qkv)) return false;
    } else {
      // forward_fused_3 (linear/forward.rs:134-166) yields the concatenation.
      Linear lq, lk, lv;
      if (!linear(p + "attn_q", lq) || !linear(p + "attn_k", lk) || !linear(p + "attn_v", lv)) return false;
      if (lq.kind != lk.kind || lq.kind != lv.kind || lq.kind == WKind::LUT4) { err = "unfused q/k/v must share one format"; return false; }
      b.qkv = lq;
      b.qkv.out = lq.out + lk.out + lv.out;
      b.qkv.dna.insert(b.qkv.dna.end(), lk.dna.begin(), lk.dna.end());
      b.qkv.dna.insert(b.qkv.dna.end(), lv.dna.begin(), lv.dna.end());
      std::vector<float> bias;
      auto addb = [&](const Linear& L) { for (size_t r = 0; r < L.out; ++r) bias.push_back(r < L.bias.size() ? L.bias[r] : 0.0f); };
      addb(lq); addb(lk); addb(lv);
      b.qkv.bias = (lq.bias.empty() && lk.bias.empty() && lv.bias.empty()) ? std::vector<float>() : bias;
    }
    if (!linear(p + "attn_output", b.wo)) return false;
    if (dmap.count(p + "ffn_gate_up")) {
      if (!linear(p + "ffn_gate_up", b.gate_up)) return false;
    } else {
      Linear lg, lu;
      if (!linear(p + "ffn_gate", lg) || !linear(p + "ffn_up", lu)) return false;
      if (lg.kind != lu.kind || lg.kind == WKind::LUT4) { err = "unfused gate/up must share one format"; return false; }
      b.gate_up = lg;
      b.gate_up.out = lg.out + lu.out;
      b.gate_up.dna.insert(b.gate_up.dna.end(), lu.dna.begin(), lu.dna.end());
      b.gate_up.bias.clear();
    }
    if (!linear(p + "ffn_down", b.down)) return false;
  }
  return true;
}

// rand 0.8 `gen::<f32>()` from a u32: (x >> 8) * 2^-24.  The reference draws
// from the unseeded thread_rng; this restatement and the CUDA engine share one
// seeded splitmix64 stream instead so that sampled streams can be compared.
struct Rng {
  uint64_t s;
  uint64_t next() {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  float uniform() { return float(uint32_t(next() >> 32) >> 8) * (1.0f / 16777216.0f); }
};

}  // namespace

// ============================================================== C interface
extern "C" {

struct or_model {
  Model m;
  std::string err;
};

// genomize_4bit_core (src/compute/quantize/genomize.rs:286-382) without
// anchors: per block of 32, min / max by strict comparison from f32::MAX /
// f32::MIN, step = (max - min) / 15, c[j] = min + j * step (two roundings),
// each value to the first nearest centroid by |v - c[j]| < best; byte k
// holds element 2k in its HIGH nibble.  nibbles[n/2], centroids[n/32 * 16].
void or_genomize_4bit(const float* w, size_t n, uint8_t* nibbles, float* centroids) {
  const long long nb = (long long)(n / 32);
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < nb; ++i) {
    const float* b = w + i * 32;
    float mn = 3.40282347e+38f, mx = -3.40282347e+38f;
    for (int k = 0; k < 32; ++k) {
      if (b[k] < mn) mn = b[k];
      if (b[k] > mx) mx = b[k];
    }
    volatile float range = mx - mn;
    const float step = range / 15.0f;
    float c[16];
    for (int j = 0; j < 16; ++j) {
      volatile float t = float(j) * step;
      c[j] = mn + t;
      centroids[i * 16 + j] = c[j];
    }
    for (int k = 0; k < 16; ++k) {
      uint8_t byte = 0;
      for (int s2 = 0; s2 < 2; ++s2) {
        const float v = b[2 * k + s2];
        int best = 0;
        float md = 3.40282347e+38f;
        for (int j = 0; j < 16; ++j) {
          volatile float diff = v - c[j];
          const float dist = std::fabs(diff);
          if (dist < md) {
            md = dist;
            best = j;
          }
        }
        byte |= s2 == 0 ? uint8_t(best << 4) : uint8_t(best);
      }
      nibbles[i * 16 + k] = byte;
    }
  }
}

// sample_top_p_core (src/compute/sampling.rs:14-55) with the uniform r in
// [0, 1) passed in (the reference draws it from thread_rng): probabilities
// exp((l - max) / T) summed in index order, normalised, stably sorted by
// descending probability, cut after the first prefix whose running sum
// exceeds top_p, then the first kept token whose running sum reaches
// r * (sum of the kept probabilities); the largest-probability token when
// none does.  Also returns the kept count through *kept.
size_t or_sample_top_p(const float* logits, size_t n, float temperature, float top_p, float r, size_t* kept) {
  if (kept) *kept = 0;
  if (n == 0) return 0;
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, logits[i]);
  std::vector<std::pair<size_t, float>> probs(n);
  float sum_exp = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    volatile float z = (logits[i] - mx) / temperature;
    probs[i] = {i, std::exp(float(z))};
  }
  for (size_t i = 0; i < n; ++i) sum_exp += probs[i].second;
  if (!(sum_exp > 0.0f)) return 0;
  for (auto& p : probs) p.second /= sum_exp;
  std::stable_sort(probs.begin(), probs.end(),
                   [](const std::pair<size_t, float>& a, const std::pair<size_t, float>& b) { return a.second > b.second; });
  float cum = 0.0f;
  size_t cutoff = n;
  for (size_t i = 0; i < n; ++i) {
    cum += probs[i].second;
    if (cum > top_p) {
      cutoff = i + 1;
      break;
    }
  }
  if (kept) *kept = cutoff;
  float final_sum = 0.0f;
  for (size_t i = 0; i < cutoff; ++i) final_sum += probs[i].second;
  const float target = r * final_sum;
  float cur = 0.0f;
  for (size_t i = 0; i < cutoff; ++i) {
    cur += probs[i].second;
    if (target <= cur) return probs[i].first;
  }
  return probs[0].first;
}

// The synthetic weights of the benchmark and test models, restated from the
// product's description of its generator so that the CPU arm can write the
// same `.gaje.flat` file without loading the product: key = splitmix64
// finaliser of (seed ^ FNV-1a(name)); element pair p takes the finalised
// key + golden * (2p+1) and key + golden * (2p+2), u1 = ((a >> 11) + 1) / 2^53,
// u2 = (b >> 11) / 2^53, and Box-Muller in double: std * r cos(2 pi u2),
// std * r sin(2 pi u2) with r = sqrt(-2 ln u1), each rounded to f32.
static uint64_t syn_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
void or_fill_normal(float* v, size_t n, uint64_t seed, const char* name, float std_) {
  uint64_t h = 0xCBF29CE484222325ull;
  for (const char* c = name; *c; ++c) h = (h ^ uint8_t(*c)) * 0x100000001B3ull;
  const uint64_t key = syn_mix(seed ^ h);
  const long long pairs = (long long)((n + 1) / 2);
#pragma omp parallel for schedule(static)
  for (long long p = 0; p < pairs; ++p) {
    const uint64_t a = syn_mix(key + 0x9E3779B97F4A7C15ull * uint64_t(2 * p + 1));
    const uint64_t b = syn_mix(key + 0x9E3779B97F4A7C15ull * uint64_t(2 * p + 2));
    const double u1 = double((a >> 11) + 1) * (1.0 / 9007199254740992.0);
    const double u2 = double(b >> 11) * (1.0 / 9007199254740992.0);
    const double r = sqrt(-2.0 * log(u1));
    v[size_t(2 * p)] = float(double(std_) * (r * cos(6.283185307179586 * u2)));
    if (size_t(2 * p + 1) < n) v[size_t(2 * p + 1)] = float(double(std_) * (r * sin(6.283185307179586 * u2)));
  }
}

void or_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#endif
}

int or_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

int or_quantize_q4_0(const float* w, size_t n, uint8_t* out) {
  if (n % 32) return -1;
  size_t nb = n / 32;
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < nb; ++i) {
    Q4Block b = quantize_q4_block(w + i * 32);
    memcpy(out + i * 20, &b, 20);
  }
  return 0;
}

int or_quantize_q8_0(const float* w, size_t n, uint8_t* out) {
  if (n % 32) return -1;
  size_t nb = n / 32;
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < nb; ++i) {
    Q8Block b = quantize_q8_block(w + i * 32);
    memcpy(out + i * 34, &b, 34);
  }
  return 0;
}

// blocks.rs:18-31 (unfused) and the AVX2 kernel's fused fma(q, scale, min).
void or_q4_0_dequant(const uint8_t* blocks, size_t n_blocks, int fused, float* out) {
  const Q4Block* b = reinterpret_cast<const Q4Block*>(blocks);
  for (size_t j = 0; j < n_blocks; ++j) {
    float sc = h2f(b[j].scale), mn = h2f(b[j].min);
    for (int k = 0; k < 32; ++k) {
      uint8_t q = (k % 2 == 0) ? (b[j].qs[k / 2] & 0x0F) : (b[j].qs[k / 2] >> 4);
      if (fused) {
        out[j * 32 + k] = fmaf(float(q), sc, mn);
      } else {
        float t = float(q) * sc;
        out[j * 32 + k] = t + mn;
      }
    }
  }
}

float or_q4_0_dot_avx2(const uint8_t* blocks, const float* x, size_t nb) {
  return q4_0_dot_avx2(reinterpret_cast<const Q4Block*>(blocks), x, nb);
}
float or_q4_0_dot_scalar(const uint8_t* blocks, const float* x, size_t nb) {
  return q4_0_dot_scalar(reinterpret_cast<const Q4Block*>(blocks), x, nb);
}
float or_q8_0_dot_avx2(const uint8_t* blocks, const float* x, size_t nb) {
  return q8_0_dot_avx2(reinterpret_cast<const Q8Block*>(blocks), x, nb);
}
float or_lut4_dot(const uint8_t* w, const float* x, const float* c, size_t stride, size_t nb) {
  return lut4_dot(w, x, c, stride, nb);
}
float or_dot_f32(const float* a, const float* b, size_t n) { return dot_f32(a, b, n); }
void or_rms_norm(const float* x, const float* w, float eps, size_t n, float* out) {
  rms_norm(x, w, eps, n, out);
}
void or_swiglu_balanced(const float* g, const float* u, float* out, size_t n) {
  swiglu_balanced(g, u, out, n);
}
void or_kwta(float* s, size_t n, size_t k) { kwta(s, n, k); }
void or_rope(float* v, size_t heads, size_t hd, size_t pos, float base, int split) {
  rope_apply(v, heads, hd, pos, base, split != 0);
}

// Q4_0 GEMV over raw 20-byte blocks (rows x (K/32)), with flush and bias,
// as compute_single_row does for a GenomicQ4_0 database.
void or_q4_0_gemv(const uint8_t* blocks, const float* x, const float* bias, size_t N,
                  size_t K, float* y) {
  const Q4Block* b = reinterpret_cast<const Q4Block*>(blocks);
  size_t nb = K / 32;
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < N; ++i) {
    float s = q4_0_dot_avx2(b + i * nb, x, nb);
    if (bias) s += bias[i];
    y[i] = s;
  }
}

void or_f32_gemv(const float* W, const float* x, size_t N, size_t K, float* y) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < N; ++i) y[i] = dot_f32(x, W + i * K, K);
}

or_model* or_load(const char* path, char* err, size_t errlen) {
  auto* h = new or_model();
  std::string e;
  if (!load_model(path, h->m, e)) {
    if (err && errlen) snprintf(err, errlen, "%s", e.c_str());
    delete h;
    return nullptr;
  }
  return h;
}

void or_free(or_model* h) { delete h; }

size_t or_info(or_model* h, size_t which) {
  const Model& m = h->m;
  switch (which) {
    case 0: return m.embd.out;
    case 1: return m.n_embd;
    case 2: return m.n_head;
    case 3: return m.n_head_kv;
    case 4: return m.n_blocks;
    case 5: return m.head_dim;
    case 6: return m.blocks.empty() ? 0 : m.blocks[0].gate_up.out / 2;
    case 7: return m.blocks.empty() ? 0 : m.blocks[0].k_cache.size();
    default: return 0;
  }
}

float or_info_f(or_model* h, size_t which) {
  switch (which) {
    case 0: return h->m.eps;
    case 1: return h->m.rope_base;
    case 2: return h->m.k_wta_ratio;
    default: return 0.0f;
  }
}

const char* or_last_error(or_model* h) { return h->err.c_str(); }

void or_set_k_wta_ratio(or_model* h, float r) {  // llm/python.rs:53-59
  h->m.k_wta_ratio = r;
  for (auto& b : h->m.blocks) b.k_wta_ratio = r;
}

void or_clear_cache(or_model* h) {
  for (auto& b : h->m.blocks) { b.k_cache.clear(); b.v_cache.clear(); }
}

int or_forward(or_model* h, size_t token, int clear, float* logits_out) {
  std::vector<float> logits;
  h->err.clear();
  if (!model_forward(h->m, token, clear != 0, logits, h->err)) return -1;
  if (logits_out) memcpy(logits_out, logits.data(), logits.size() * 4);
  return 0;
}

// Hidden state probe: runs a forward and returns h_norm (the lm_head input).
int or_forward_hidden(or_model* h, size_t token, int clear, float* hnorm_out) {
  Model& m = h->m;
  h->err.clear();
  if (clear) or_clear_cache(h);
  size_t pos = m.blocks.empty() ? 0 : m.blocks[0].k_cache.size();
  std::vector<float> x = m.embd.get_row(token);
  for (auto& b : m.blocks)
    if (!block_forward(b, m, x, pos, h->err)) return -1;
  rms_norm(x.data(), m.output_norm.data(), m.eps, x.size(), hnorm_out);
  return 0;
}

// Runs one named linear of the loaded model (op-level parity on real tensors).
int or_linear(or_model* h, int layer, int which, const float* x, size_t xlen, float* y) {
  Model& m = h->m;
  const Linear* L = nullptr;
  if (layer < 0) L = (which == 0) ? &m.lm_head : &m.embd;
  else if (size_t(layer) < m.blocks.size()) {
    Block& b = m.blocks[layer];
    L = which == 0 ? &b.qkv : which == 1 ? &b.wo : which == 2 ? &b.gate_up : &b.down;
  }
  if (!L) return -1;
  L->forward(x, xlen, y);
  return 0;
}

int or_get_row(or_model* h, int layer, int which, size_t idx, float* out) {
  Model& m = h->m;
  const Linear* L = nullptr;
  if (layer < 0) L = (which == 0) ? &m.lm_head : &m.embd;
  else if (size_t(layer) < m.blocks.size()) {
    Block& b = m.blocks[layer];
    L = which == 0 ? &b.qkv : which == 1 ? &b.wo : which == 2 ? &b.gate_up : &b.down;
  }
  if (!L) return -1;
  std::vector<float> r = L->get_row(idx);
  memcpy(out, r.data(), r.size() * 4);
  return 0;
}

// llm/forward.rs:215-330 generate_native_core.  Sampling uses the seeded
// splitmix64 stream described above (the reference is unseeded).
int or_generate(or_model* h, const size_t* prompt, size_t n_prompt, size_t max_new,
                float temperature, float rep_penalty, const size_t* eos, size_t n_eos,
                uint64_t seed, size_t* out, size_t* n_out) {
  Model& m = h->m;
  h->err.clear();
  *n_out = 0;
  if (n_prompt == 0) { h->err = "Prompt tokens cannot be empty"; return -1; }
  or_clear_cache(h);
  std::vector<float> last;
  for (size_t i = 0; i < n_prompt; ++i)
    if (!model_forward(m, prompt[i], false, last, h->err)) return -1;
  std::vector<size_t> gen;
  std::set<size_t> eos_set(eos, eos + n_eos);
  Rng rng{seed};
  for (size_t step = 0; step < max_new; ++step) {
    if (last.empty()) break;
    std::vector<float> lg = last;
    if (rep_penalty > 1.0f) {
      std::set<size_t> seen(gen.begin(), gen.end());
      for (size_t e : eos_set) seen.erase(e);
      for (size_t t : seen)
        if (t < lg.size()) {
          if (lg[t] < 0.0f) lg[t] *= rep_penalty;
          else lg[t] /= rep_penalty;
        }
    }
    size_t next = 0;
    if (temperature <= 1e-5f) {
      float mv = -INFINITY;
      for (size_t i = 0; i < lg.size(); ++i)
        if (lg[i] > mv) { mv = lg[i]; next = i; }
    } else {
      float ml = -INFINITY;
      for (float v : lg) if (v > ml) ml = v;
      std::vector<float> probs(lg.size());
      float sum = 0.0f;
      for (size_t i = 0; i < lg.size(); ++i) {
        float d = (lg[i] - ml) / temperature;
        probs[i] = std::exp(d);
        sum += probs[i];
      }
      float r = rng.uniform() * sum;
      float cum = 0.0f;
      for (size_t i = 0; i < probs.size(); ++i) {
        cum += probs[i];
        if (r <= cum) { next = i; break; }
      }
    }
    gen.push_back(next);
    if (eos_set.count(next)) break;
    bool repeated = false;
    for (size_t w = 2; w <= 48; ++w) {
      if (gen.size() >= w * 3) {
        size_t L = gen.size();
        if (std::equal(gen.begin() + (L - w), gen.end(), gen.begin() + (L - 2 * w)) &&
            std::equal(gen.begin() + (L - w), gen.end(), gen.begin() + (L - 3 * w))) {
          repeated = true;
          break;
        }
      }
    }
    if (repeated) break;
    if (!model_forward(m, next, false, last, h->err)) return -1;
  }
  for (size_t i = 0; i < gen.size(); ++i) out[i] = gen[i];
  *n_out = gen.size();
  return 0;
}

}  // extern "C"
