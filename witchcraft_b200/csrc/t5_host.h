// Host-side pieces of the backend that need no GPU: GGUF parsing, config.json
// parsing and the relative-position bucket thresholds.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "attention.h"

namespace wc {

enum GgmlType : uint32_t { kGgmlF32 = 0, kGgmlF16 = 1, kGgmlQ4K = 12 };

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;  // GGUF order: innermost first
  uint32_t type = 0;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  // rows x cols view of a rank-1/2 tensor (cols = innermost)
  uint64_t cols() const { return dims.empty() ? 0 : dims[0]; }
  uint64_t rows() const { return dims.size() < 2 ? 1 : dims[1]; }
};

// Parses GGUF v2/v3 (header, metadata, tensor infos, aligned data section).
// Returns false with a message in *err when the buffer is malformed or
// truncated or holds a tensor type other than F32, F16 or Q4_K.
bool gguf_parse(const uint8_t* buf, size_t len, std::unordered_map<std::string, GgufTensor>* out, std::string* err);

struct T5Config {
  int vocab_size = 0, d_model = 0, d_kv = 0, d_ff = 0, num_layers = 0, num_heads = 0;
  int num_buckets = 32, max_distance = 128;
  float eps = 1e-6f;
  bool gated_gelu = false;
};

// Upper bound of |d*sc*q - dmin*m| over nblocks Q4_K super-blocks (the
// largest magnitude a dequantised weight can take).
double q4k_max_abs_bound(const uint8_t* blocks, size_t nblocks);

// Parses the fields of config.json the reference's Config reads
// (src/quantized_t5.rs:90-115).  Returns false with *err on a missing field.
bool config_parse(const char* json, T5Config* cfg, std::string* err);

// The reference's bucket of (query i, key j) (src/quantized_t5.rs:447-483),
// evaluated with the same f32 formula: ln(d / max_exact) / ln(max_distance /
// max_exact) * (half - max_exact), truncated.
int t5_bucket_reference(int i, int j, int num_buckets, int max_distance);

// Threshold form of the bucket function for distances below max_len.
BucketThresholds t5_bucket_thresholds(int num_buckets, int max_distance, int max_len);

// Bucket from thresholds (the arithmetic the attention kernel performs).
int t5_bucket_from_thresholds(const BucketThresholds& bt, int delta);

}  // namespace wc
