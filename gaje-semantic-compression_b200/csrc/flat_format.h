// flat_format.h -- host-side `.gaje.flat` v2 support for the B200 engine:
// header/metadata/directory parsing, shape validation, Q4_0/Q8_0 quantisers
// and the file writer.  No CUDA in here.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "../../include/gaje_cuda.h"

namespace gaje {

// One FlatTensorEntry (src/io/flat_reader.rs:9-22).
struct FlatEntry {
  std::string name;
  uint64_t bit_depth = 0, out = 0, in = 0, dna_off = 0, dna_len = 0, c_off = 0, c_len = 0,
           anc_off = 0, anc_len = 0, bias_off = 0, bias_len = 0;
};

// How one engine matrix is stored.  Unfused q/k/v or gate/up tensors are
// listed in order; their rows concatenate (forward_fused_3/_2 in
// src/nn/linear/forward.rs:134-193 produce exactly that concatenation).
struct MatrixRef {
  std::vector<const FlatEntry*> parts;
  uint64_t out = 0, in = 0;
  int bit_depth = 0;  // 4 (Q4_0, or Genomic4Bit with lut), 8 (Q8_0), 32 (f32)
  bool lut = false;   // Genomic4Bit: nibbles (high nibble first) + 16-centroid tables
  bool has_bias = false;
};

struct BlockRefs {
  const FlatEntry* attn_norm = nullptr;
  const FlatEntry* ffn_norm = nullptr;
  MatrixRef qkv, wo, gate_up, down;
};

class FlatFile {
 public:
  FlatFile() = default;
  FlatFile(const FlatFile&) = delete;
  FlatFile& operator=(const FlatFile&) = delete;
  ~FlatFile();

  // GajeFlatFileReader::open + load_genomic's config/tensor resolution.
  // Returns a gaje_status; err gets the message.
  int open(const char* path, std::string& err);

  // Bytes of a blob at a weights-relative offset; nullptr when out of range.
  const uint8_t* blob(uint64_t off, uint64_t len) const;

  gaje_flat_header hdr{};
  gaje_flat_info info{};
  std::map<std::string, FlatEntry> dir;
  const FlatEntry* token_embd = nullptr;
  const FlatEntry* lm_head = nullptr;
  const FlatEntry* output_norm = nullptr;
  std::vector<BlockRefs> blocks;

 private:
  int resolve(std::string& err);
  const uint8_t* data_ = nullptr;
  size_t size_ = 0;
};

// FlatHeaderV2::from_bytes: decode the fixed fields, validate the magic.
int decode_header(const uint8_t* p, size_t len, gaje_flat_header& h, std::string& err);

// f16 <-> f32 (round to nearest even), the conversions of the `half` crate.
uint16_t f32_to_f16(float f);
float f16_to_f32(uint16_t h);

// Python's repr() of a float (shortest round trip), as json.dumps emits it.
std::string py_float_repr(double v);

// Records the thread-local message behind gaje_cuda_last_error(); returns status.
int set_error(int status, const std::string& msg);
void clear_error();

}  // namespace gaje
