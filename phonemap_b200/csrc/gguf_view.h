// gguf_view.h -- read-only view of a GGUF v2/v3 file held in memory.
//
// Reads what SlipStream's loader reads (SlipStream/src/core/gguf_loader.c:
// 250-431): the KV keys that size a llama model, the tensor infos (dims are
// [ne0 = cols, ne1 = rows]) and the data section, which starts at the first
// 32-byte boundary after the tensor infos (gguf_loader.c:426).  Defaults for
// missing keys follow gguf_loader.c:370-379.
#pragma once
#include <stdint.h>
#include <string.h>

#include <string>
#include <unordered_map>
#include <vector>

namespace ss {

struct GgufTensor {
  std::string name;
  uint32_t n_dims = 0;
  uint64_t dims[4] = {1, 1, 1, 1};
  int type = -1;
  uint64_t offset = 0;  // absolute offset in the file
  uint64_t bytes = 0;
  const uint8_t* data = nullptr;
  uint64_t cols() const { return dims[0]; }
  uint64_t rows() const { return n_dims > 1 ? dims[1] : 1; }
};

struct GgufModel {
  std::string arch;
  uint32_t hidden = 0, n_heads = 0, n_kv_heads = 0, context_length = 0, ffn = 0,
           n_layers = 0, vocab = 0, key_length = 0, rope_dim = 0;
  float rope_theta = 0.0f, rms_eps = 0.0f;
  std::vector<GgufTensor> tensors;
  std::unordered_map<std::string, size_t> by_name;

  const GgufTensor* find(const std::string& n) const {
    auto it = by_name.find(n);
    return it == by_name.end() ? nullptr : &tensors[it->second];
  }
};

inline size_t ggml_type_size(int t) {
  switch (t) {
    case 0: return 4;
    case 1: return 2;
    case 2: return 18;
    case 8: return 34;
    default: return 0;
  }
}
inline int ggml_block_size(int t) { return (t == 2 || t == 8) ? 32 : 1; }

class GgufReader {
 public:
  GgufReader(const uint8_t* p, uint64_t n) : base_(p), p_(p), end_(p + n) {}
  bool ok() const { return ok_; }
  uint64_t pos() const { return (uint64_t)(p_ - base_); }
  uint64_t u(int n) {
    uint64_t v = 0;
    if (!ok_ || (uint64_t)(end_ - p_) < (uint64_t)n) { ok_ = false; return 0; }
    memcpy(&v, p_, (size_t)n);
    p_ += n;
    return v;
  }
  std::string str() {
    uint64_t len = u(8);
    if (!ok_ || (uint64_t)(end_ - p_) < len) { ok_ = false; return std::string(); }
    std::string s((const char*)p_, (size_t)len);
    p_ += len;
    return s;
  }
  void skip(uint32_t type, int depth = 0) {
    static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (type == 8) { uint64_t len = u(8); adv(len); return; }
    if (type == 9) {
      if (depth > 4) { ok_ = false; return; }
      uint32_t at = (uint32_t)u(4);
      uint64_t n = u(8);
      if (at < 13 && at != 8 && at != 9) { adv(n * (uint64_t)sz[at]); return; }
      for (uint64_t i = 0; i < n && ok_; i++) skip(at, depth + 1);
      return;
    }
    if (type < 13) adv((uint64_t)sz[type]); else ok_ = false;
  }

 private:
  void adv(uint64_t n) {
    if ((uint64_t)(end_ - p_) < n) { ok_ = false; return; }
    p_ += n;
  }
  const uint8_t* base_;
  const uint8_t* p_;
  const uint8_t* end_;
  bool ok_ = true;
};

inline bool ends_with(const std::string& s, const char* suf) {
  size_t m = strlen(suf);
  return s.size() >= m && s.compare(s.size() - m, m, suf) == 0;
}

// Parses the header; returns false with a message on malformed input.
inline bool gguf_parse(const uint8_t* base, uint64_t size, GgufModel* m, std::string* err) {
  GgufReader r(base, size);
  if (r.u(4) != 0x46554747u) { *err = "not a GGUF file (bad magic)"; return false; }
  uint32_t version = (uint32_t)r.u(4);
  if (version < 2 || version > 3) { *err = "unsupported GGUF version"; return false; }
  uint64_t n_t = r.u(8), n_kv = r.u(8);
  if (!r.ok() || n_t > (1u << 24) || n_kv > (1u << 24)) { *err = "corrupt GGUF header"; return false; }
  for (uint64_t i = 0; i < n_kv && r.ok(); i++) {
    std::string k = r.str();
    uint32_t t = (uint32_t)r.u(4);
    if (k == "general.architecture" && t == 8) m->arch = r.str();
    else if (t == 4 && ends_with(k, ".embedding_length")) m->hidden = (uint32_t)r.u(4);
    else if (t == 4 && ends_with(k, ".attention.head_count_kv")) m->n_kv_heads = (uint32_t)r.u(4);
    else if (t == 4 && ends_with(k, ".attention.head_count")) m->n_heads = (uint32_t)r.u(4);
    else if (t == 4 && ends_with(k, ".context_length")) m->context_length = (uint32_t)r.u(4);
    else if (t == 4 && ends_with(k, ".feed_forward_length")) m->ffn = (uint32_t)r.u(4);
    else if (t == 4 && ends_with(k, ".block_count")) m->n_layers = (uint32_t)r.u(4);
    else if (t == 4 && ends_with(k, ".vocab_size")) m->vocab = (uint32_t)r.u(4);
    else if (t == 4 && ends_with(k, ".attention.key_length")) m->key_length = (uint32_t)r.u(4);
    else if (t == 4 && ends_with(k, ".rope.dimension_count")) m->rope_dim = (uint32_t)r.u(4);
    else if (t == 6 && ends_with(k, ".rope.freq_base")) { uint32_t b = (uint32_t)r.u(4); memcpy(&m->rope_theta, &b, 4); }
    else if (t == 6 && ends_with(k, ".attention.layer_norm_rms_epsilon")) { uint32_t b = (uint32_t)r.u(4); memcpy(&m->rms_eps, &b, 4); }
    else r.skip(t);
  }
  if (!r.ok()) { *err = "corrupt GGUF metadata"; return false; }
  if (m->rms_eps == 0.0f) m->rms_eps = 1e-5f;
  if (m->rope_theta == 0.0f) m->rope_theta = 10000.0f;
  if (m->context_length == 0) m->context_length = 2048;
  m->tensors.resize((size_t)n_t);
  for (uint64_t i = 0; i < n_t && r.ok(); i++) {
    GgufTensor& t = m->tensors[(size_t)i];
    t.name = r.str();
    t.n_dims = (uint32_t)r.u(4);
    if (t.n_dims > 4) { *err = "tensor with more than 4 dims"; return false; }
    for (uint32_t d = 0; d < t.n_dims; d++) t.dims[d] = r.u(8);
    t.type = (int)r.u(4);
    t.offset = r.u(8);
  }
  if (!r.ok()) { *err = "corrupt GGUF tensor infos"; return false; }
  const uint64_t data_off = (r.pos() + 31) & ~(uint64_t)31;
  for (size_t i = 0; i < m->tensors.size(); i++) {
    GgufTensor& t = m->tensors[i];
    uint64_t n = 1;
    for (uint32_t d = 0; d < t.n_dims; d++) n *= t.dims[d];
    const size_t ts = ggml_type_size(t.type);
    const int bs = ggml_block_size(t.type);
    t.bytes = ts ? n / (uint64_t)bs * ts : 0;
    t.offset += data_off;
    if (ts && (t.offset > size || t.bytes > size - t.offset)) {
      *err = "tensor " + t.name + " extends past the end of the file";
      return false;
    }
    t.data = base + t.offset;
    m->by_name[t.name] = i;
    if (m->vocab == 0 && t.name == "token_embd.weight" && t.n_dims == 2) m->vocab = (uint32_t)t.dims[1];
  }
  return true;
}

}  // namespace ss
