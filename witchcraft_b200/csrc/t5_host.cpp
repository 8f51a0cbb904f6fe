// GGUF / config.json parsing and the relative-position bucket thresholds.
// Replaces candle's VarBuilder::from_gguf_buffer (src/quantized_t5.rs:740)
// and the serde Config (src/quantized_t5.rs:90-115) for this backend.
#include "t5_host.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <climits>

namespace wc {

namespace {

struct Reader {
  const uint8_t* p;
  size_t len, pos = 0;
  bool ok = true;
  bool need(size_t n) {
    if (!ok || len - pos < n || pos > len) ok = false;
    return ok;
  }
  template <class T>
  T get() {
    T v{};
    if (need(sizeof(T))) {
      memcpy(&v, p + pos, sizeof(T));
      pos += sizeof(T);
    }
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > (1u << 20) || !need(n)) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(p + pos), n);
    pos += n;
    return s;
  }
};

// Size in bytes of one scalar of GGUF metadata type t (0 for string/array).
size_t kv_scalar_size(uint32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;            // u8 i8 bool
    case 2: case 3: return 2;                    // u16 i16
    case 4: case 5: case 6: return 4;            // u32 i32 f32
    case 10: case 11: case 12: return 8;         // u64 i64 f64
    default: return 0;
  }
}

bool skip_value(Reader& r, uint32_t t, uint64_t* as_uint) {
  if (t == 8) {
    r.str();
    return r.ok;
  }
  if (t == 9) {
    const uint32_t et = r.get<uint32_t>();
    const uint64_t n = r.get<uint64_t>();
    if (!r.ok || et == 9) return false;
    for (uint64_t i = 0; i < n && r.ok; ++i) skip_value(r, et, nullptr);
    return r.ok;
  }
  const size_t sz = kv_scalar_size(t);
  if (sz == 0 || !r.need(sz)) return false;
  if (as_uint) {
    uint64_t v = 0;
    memcpy(&v, r.p + r.pos, sz);
    *as_uint = v;
  }
  r.pos += sz;
  return true;
}

}  // namespace

bool gguf_parse(const uint8_t* buf, size_t len, std::unordered_map<std::string, GgufTensor>* out, std::string* err) {
  if (!buf || len < 24) {
    *err = "GGUF buffer is empty or shorter than its header";
    return false;
  }
  Reader r{buf, len};
  if (memcmp(buf, "GGUF", 4) != 0) {
    *err = "not a GGUF file (bad magic)";
    return false;
  }
  r.pos = 4;
  const uint32_t version = r.get<uint32_t>();
  if (version < 2 || version > 3) {
    *err = "unsupported GGUF version " + std::to_string(version);
    return false;
  }
  const uint64_t n_tensors = r.get<uint64_t>();
  const uint64_t n_kv = r.get<uint64_t>();
  if (n_tensors > (1u << 20) || n_kv > (1u << 20)) {
    *err = "GGUF header counts are implausible";
    return false;
  }
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < n_kv; ++i) {
    const std::string key = r.str();
    const uint32_t t = r.get<uint32_t>();
    uint64_t v = 0;
    if (!r.ok || !skip_value(r, t, &v)) {
      *err = "truncated GGUF metadata";
      return false;
    }
    if (key == "general.alignment" && (t == 4 || t == 10)) alignment = v;
  }
  if (alignment == 0 || (alignment & (alignment - 1)) != 0) {
    *err = "GGUF alignment is not a power of two";
    return false;
  }
  std::vector<std::pair<GgufTensor, uint64_t>> infos;
  for (uint64_t i = 0; i < n_tensors; ++i) {
    GgufTensor t;
    t.name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    if (!r.ok || nd == 0 || nd > 4) {
      *err = "bad GGUF tensor info";
      return false;
    }
    uint64_t nel = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      const uint64_t dim = r.get<uint64_t>();
      if (dim == 0 || dim > (1ull << 32)) r.ok = false;
      t.dims.push_back(dim);
      nel *= dim;
    }
    t.type = r.get<uint32_t>();
    const uint64_t off = r.get<uint64_t>();
    if (!r.ok) {
      *err = "truncated GGUF tensor info";
      return false;
    }
    if (t.type == kGgmlF32) {
      t.nbytes = nel * 4;
    } else if (t.type == kGgmlF16) {
      t.nbytes = nel * 2;
    } else if (t.type == kGgmlQ4K) {
      if (t.dims[0] % 256 != 0) {
        *err = "Q4_K tensor " + t.name + " has an inner dimension not divisible by 256";
        return false;
      }
      t.nbytes = nel / 256 * 144;
    } else {
      *err = "tensor " + t.name + " has unsupported GGML type " + std::to_string(t.type);
      return false;
    }
    infos.emplace_back(std::move(t), off);
  }
  const uint64_t data0 = (r.pos + alignment - 1) / alignment * alignment;
  for (auto& it : infos) {
    const uint64_t start = data0 + it.second;
    if (start < data0 || start > len || it.first.nbytes > len - start) {
      *err = "GGUF tensor " + it.first.name + " lies past the end of the buffer (truncated file?)";
      return false;
    }
    it.first.data = buf + start;
    (*out)[it.first.name] = std::move(it.first);
  }
  return true;
}

namespace {

double half_bits_to_double(uint16_t h) {
  const int e = (h >> 10) & 0x1f, m = h & 0x3ff;
  double v;
  if (e == 0)
    v = ldexp(static_cast<double>(m), -24);
  else if (e == 31)
    v = m ? NAN : INFINITY;
  else
    v = ldexp(static_cast<double>(m | 0x400), e - 25);
  return (h & 0x8000) ? -v : v;
}

}  // namespace

double q4k_max_abs_bound(const uint8_t* blocks, size_t nblocks) {
  double mx = 0.0;
  for (size_t b = 0; b < nblocks; ++b) {
    const uint8_t* p = blocks + b * 144;
    const double d = fabs(half_bits_to_double(static_cast<uint16_t>(p[0] | (p[1] << 8))));
    const double dm = fabs(half_bits_to_double(static_cast<uint16_t>(p[2] | (p[3] << 8))));
    const double v = d * 63.0 * 15.0 + dm * 63.0;
    if (!(v <= mx)) mx = v;  // also propagates NaN
  }
  return mx;
}

namespace {

const char* find_key(const char* json, const char* key) {
  const std::string pat = std::string("\"") + key + "\"";
  const char* p = strstr(json, pat.c_str());
  if (!p) return nullptr;
  p += pat.size();
  while (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r') ++p;
  if (*p != ':') return nullptr;
  ++p;
  while (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r') ++p;
  return p;
}

bool get_num(const char* json, const char* key, double* v) {
  const char* p = find_key(json, key);
  if (!p) return false;
  char* end = nullptr;
  *v = strtod(p, &end);
  return end != p;
}

}  // namespace

bool config_parse(const char* json, T5Config* cfg, std::string* err) {
  if (!json) {
    *err = "config.json text is NULL";
    return false;
  }
  struct {
    const char* key;
    int* dst;
    bool required;
  } ints[] = {
      {"vocab_size", &cfg->vocab_size, true},
      {"d_model", &cfg->d_model, true},
      {"d_kv", &cfg->d_kv, true},
      {"d_ff", &cfg->d_ff, true},
      {"num_layers", &cfg->num_layers, true},
      {"num_heads", &cfg->num_heads, true},
      {"relative_attention_num_buckets", &cfg->num_buckets, true},
      {"relative_attention_max_distance", &cfg->max_distance, false},  // serde default 128
  };
  for (auto& f : ints) {
    double v;
    if (!get_num(json, f.key, &v)) {
      if (f.required) {
        *err = std::string("config.json: missing or non-numeric field ") + f.key;
        return false;
      }
      continue;
    }
    *f.dst = static_cast<int>(v);
  }
  double eps;
  if (!get_num(json, "layer_norm_epsilon", &eps)) {
    *err = "config.json: missing field layer_norm_epsilon";
    return false;
  }
  cfg->eps = static_cast<float>(eps);
  // feed_forward_proj: "gated-gelu" -> gated NewGelu (tanh GELU), as candle's
  // deserialize_feed_forward_proj_activation maps it; default (absent) is relu.
  const char* p = find_key(json, "feed_forward_proj");
  cfg->gated_gelu = false;
  if (p && *p == '"') {
    const char* e = strchr(p + 1, '"');
    if (!e) {
      *err = "config.json: unterminated feed_forward_proj";
      return false;
    }
    const std::string s(p + 1, e);
    cfg->gated_gelu = (s == "gated-gelu" || s == "gated-gelu_new" || s == "gated-gelu_pytorch_tanh");
  }
  return true;
}

int t5_bucket_reference(int i, int j, int num_buckets, int max_distance) {
  const int nb = num_buckets / 2;
  const int max_exact = nb / 2;
  const int d = i < j ? j - i : i - j;
  int v;
  if (d < max_exact) {
    v = d;
  } else {
    // Rust f32::log(x, base) == ln(x) / ln(base), all in f32
    const float b = (logf(static_cast<float>(d) / static_cast<float>(max_exact)) /
                     logf(static_cast<float>(max_distance) / static_cast<float>(max_exact))) *
                    static_cast<float>(nb - max_exact);
    const uint32_t bi = b > 0.f ? static_cast<uint32_t>(b) : 0u;  // Rust `as u32` saturates
    v = max_exact + static_cast<int>(bi);
    if (v > nb - 1) v = nb - 1;
  }
  return i < j ? v + nb : v;
}

BucketThresholds t5_bucket_thresholds(int num_buckets, int max_distance, int max_len) {
  BucketThresholds bt{};
  bt.half = num_buckets / 2;
  for (int v = 0; v < 32; ++v) bt.thr[v] = INT_MAX;
  bt.thr[0] = 0;
  int prev = 0;
  for (int d = 0; d < max_len; ++d) {
    const int f = t5_bucket_reference(d, 0, num_buckets, max_distance);  // query after key: no offset
    for (int v = prev + 1; v <= f && v < 32; ++v) bt.thr[v] = d;
    if (f > prev) prev = f;
  }
  return bt;
}

int t5_bucket_from_thresholds(const BucketThresholds& bt, int delta) {
  const int d = delta < 0 ? -delta : delta;
  int f = 0;
  for (int v = 1; v < bt.half; ++v) f += (d >= bt.thr[v]) ? 1 : 0;
  return f + (delta > 0 ? bt.half : 0);
}

}  // namespace wc
