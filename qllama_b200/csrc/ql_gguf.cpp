// ql_gguf.cpp -- GGUF reader and ql_llama_load_gguf (qllama_model.h).
//
// Reads the GGUF container (version 2 or 3, little-endian) and assembles a
// device model from it, as the reference does on the CPU:
//   GgufFile::from_reader: magic, version checks, metadata, tensor infos, the
//     data section at the next multiple of general.alignment (default 32)
//                                          src/gguf/parser.rs:52-99, 101-147
//   metadata value types 0-12 and arrays   src/gguf/parser.rs:193-237, types.rs:20-50
//   load_tensor: F32 as is, F16 widened exactly, quantised types rejected;
//     dimensions reversed (ggml's ne[0] is the contiguous one)
//                                          src/gguf/loader.rs:1-132
//   TransformerConfig::from_gguf           src/transformer/config.rs:71-164
//   Transformer::from_gguf (tensor names, tied lm_head)
//                                          src/transformer/transformer.rs:142-197
// The file is read with plain stdio; every size and offset from the file is
// checked before use.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/qllama_model.h"
#include "ql_internal.h"

namespace {

enum : uint32_t {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32v = 6, kBool = 7,
  kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12,
};
enum : uint32_t { kGgmlF32 = 0, kGgmlF16 = 1 };
constexpr uint32_t kMaxVersion = 3;

struct Value {
  uint32_t type = 0;
  uint64_t u = 0;     // unsigned integers and bool
  int64_t i = 0;      // signed integers
  double f = 0.0;     // floats
  std::string s;      // strings
  uint32_t elem = 0;  // arrays: element type and count (the items are skipped)
  uint64_t count = 0;
};

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;  // ggml order: dims[0] contiguous
  uint32_t type = 0;
  uint64_t offset = 0;
};

struct File {
  FILE* f = nullptr;
  std::string path;
  std::map<std::string, Value> meta;
  std::vector<TensorInfo> tensors;
  uint64_t data_start = 0;
  uint64_t size = 0;
  ~File() {
    if (f) std::fclose(f);
  }
  const TensorInfo* find(const std::string& n) const {
    for (const auto& t : tensors)
      if (t.name == n) return &t;
    return nullptr;
  }
};

struct Reader {
  File& file;
  std::string err;
  bool read(void* p, size_t n) {
    if (std::fread(p, 1, n, file.f) != n) {
      err = "unexpected end of file";
      return false;
    }
    return true;
  }
  template <typename T>
  bool get(T& v) {
    return read(&v, sizeof v);
  }
  bool str(std::string& s) {
    uint64_t n = 0;
    if (!get(n)) return false;
    if (n > (1ull << 24)) {
      err = "string length " + std::to_string(n) + " is implausible";
      return false;
    }
    s.resize(n);
    return n == 0 || read(&s[0], n);
  }
  bool skip(uint64_t n) {
    if (std::fseek(file.f, static_cast<long>(n), SEEK_CUR) != 0) {
      err = "seek failed";
      return false;
    }
    return true;
  }
  static int scalar_size(uint32_t t) {
    switch (t) {
      case kU8: case kI8: case kBool: return 1;
      case kU16: case kI16: return 2;
      case kU32: case kI32: case kF32v: return 4;
      case kU64: case kI64: case kF64: return 8;
      default: return 0;
    }
  }
  bool scalar(uint32_t t, Value& v) {
    v.type = t;
    switch (t) {
      case kU8: { uint8_t x; if (!get(x)) return false; v.u = x; v.i = x; v.f = x; return true; }
      case kI8: { int8_t x; if (!get(x)) return false; v.i = x; v.f = x; return true; }
      case kU16: { uint16_t x; if (!get(x)) return false; v.u = x; v.i = x; v.f = x; return true; }
      case kI16: { int16_t x; if (!get(x)) return false; v.i = x; v.f = x; return true; }
      case kU32: { uint32_t x; if (!get(x)) return false; v.u = x; v.i = x; v.f = x; return true; }
      case kI32: { int32_t x; if (!get(x)) return false; v.i = x; v.f = x; return true; }
      case kU64: { uint64_t x; if (!get(x)) return false; v.u = x; v.i = static_cast<int64_t>(x); v.f = static_cast<double>(x); return true; }
      case kI64: { int64_t x; if (!get(x)) return false; v.i = x; v.f = static_cast<double>(x); return true; }
      case kF32v: { float x; if (!get(x)) return false; v.f = x; return true; }
      case kF64: { double x; if (!get(x)) return false; v.f = x; return true; }
      case kBool: {
        uint8_t x;
        if (!get(x)) return false;
        if (x > 1) {
          err = "invalid bool value " + std::to_string(x);
          return false;
        }
        v.u = x;
        return true;
      }
      default: err = "unknown metadata value type " + std::to_string(t); return false;
    }
  }
  bool value(uint32_t t, Value& v, int depth = 0) {
    if (t == kString) {
      v.type = t;
      return str(v.s);
    }
    if (t == kArray) {
      v.type = t;
      if (!get(v.elem) || !get(v.count)) return false;
      if (depth > 4) {
        err = "metadata arrays nested too deeply";
        return false;
      }
      const int sz = scalar_size(v.elem);
      if (sz > 0) return skip(v.count * static_cast<uint64_t>(sz));
      for (uint64_t i = 0; i < v.count; ++i) {
        Value item;
        if (!value(v.elem, item, depth + 1)) return false;
      }
      return true;
    }
    return scalar(t, v);
  }
};

int parse(File& file, const char* path) {
  file.path = path;
  file.f = std::fopen(path, "rb");
  if (!file.f) return ql_fail(QL_ERR_INVALID, "cannot open %s", path);
  std::fseek(file.f, 0, SEEK_END);
  file.size = static_cast<uint64_t>(std::ftell(file.f));
  std::fseek(file.f, 0, SEEK_SET);
  Reader rd{file, {}};
  char magic[4];
  uint32_t version = 0;
  uint64_t n_tensors = 0, n_kv = 0;
  if (!rd.read(magic, 4) || !rd.get(version))
    return ql_fail(QL_ERR_INVALID, "GGUF header: %s", rd.err.c_str());
  if (std::memcmp(magic, "GGUF", 4) != 0) return ql_fail(QL_ERR_INVALID, "Invalid GGUF magic");
  if (version == 0) return ql_fail(QL_ERR_INVALID, "Bad GGUF version: 0");
  if ((version & 0xFFFFu) == 0)
    return ql_fail(QL_ERR_INVALID,
                   "GGUF version %u has a zero low half; the file may be big-endian", version);
  if (version == 1) return ql_fail(QL_ERR_UNSUPPORTED, "GGUF version 1 is not supported");
  if (version > kMaxVersion)
    return ql_fail(QL_ERR_UNSUPPORTED, "GGUF version %u exceeds supported version %u", version,
                   kMaxVersion);
  if (!rd.get(n_tensors) || !rd.get(n_kv))
    return ql_fail(QL_ERR_INVALID, "GGUF header: %s", rd.err.c_str());
  if (n_tensors > (1u << 20) || n_kv > (1u << 20))
    return ql_fail(QL_ERR_INVALID, "GGUF counts are implausible (%llu tensors, %llu keys)",
                   (unsigned long long)n_tensors, (unsigned long long)n_kv);
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key;
    uint32_t t = 0;
    Value v;
    if (!rd.str(key) || !rd.get(t) || !rd.value(t, v))
      return ql_fail(QL_ERR_INVALID, "GGUF metadata: %s", rd.err.c_str());
    file.meta[key] = v;
  }
  for (uint64_t i = 0; i < n_tensors; ++i) {
    TensorInfo ti;
    uint32_t nd = 0;
    if (!rd.str(ti.name) || !rd.get(nd))
      return ql_fail(QL_ERR_INVALID, "GGUF tensor info: %s", rd.err.c_str());
    if (nd == 0 || nd > 4) return ql_fail(QL_ERR_INVALID, "tensor %s has %u dimensions", ti.name.c_str(), nd);
    ti.dims.resize(nd);
    for (uint32_t d = 0; d < nd; ++d)
      if (!rd.get(ti.dims[d])) return ql_fail(QL_ERR_INVALID, "GGUF tensor info: %s", rd.err.c_str());
    if (!rd.get(ti.type) || !rd.get(ti.offset))
      return ql_fail(QL_ERR_INVALID, "GGUF tensor info: %s", rd.err.c_str());
    file.tensors.push_back(ti);
  }
  uint64_t align = 32;
  auto it = file.meta.find("general.alignment");
  if (it != file.meta.end()) {
    if (it->second.type != kU32 || it->second.u == 0 || it->second.u % 8 != 0)
      return ql_fail(QL_ERR_INVALID, "general.alignment must be a nonzero UINT32 multiple of 8");
    align = it->second.u;
  }
  const uint64_t pos = static_cast<uint64_t>(std::ftell(file.f));
  file.data_start = pos + (align - pos % align) % align;
  return QL_OK;
}

// Reads one tensor as f32 in the reference's logical layout (dims reversed):
// the element order in the file already is that layout, row-major.
int load_f32(File& file, const std::string& name, std::vector<float>& out, std::vector<uint64_t>& dims) {
  const TensorInfo* ti = file.find(name);
  if (!ti) return ql_fail(QL_ERR_INVALID, "Tensor not found: %s", name.c_str());
  if (ti->type != kGgmlF32 && ti->type != kGgmlF16) {
    if (ti->type >= 2 && ti->type <= 15)
      return ql_fail(QL_ERR_UNSUPPORTED, "Quantized type %u of tensor %s not yet supported",
                     ti->type, name.c_str());
    return ql_fail(QL_ERR_UNSUPPORTED,
                   "Unsupported tensor type %u of %s; only F32 and F16 are supported", ti->type,
                   name.c_str());
  }
  uint64_t n = 1;
  for (uint64_t d : ti->dims) {
    if (d == 0 || n > (1ull << 40) / d) return ql_fail(QL_ERR_INVALID, "tensor %s is too large", name.c_str());
    n *= d;
  }
  const uint64_t es = ti->type == kGgmlF32 ? 4 : 2;
  const uint64_t begin = file.data_start + ti->offset;
  if (ti->offset > file.size || begin + n * es > file.size)
    return ql_fail(QL_ERR_INVALID, "tensor %s lies outside the file", name.c_str());
  dims.assign(ti->dims.rbegin(), ti->dims.rend());
  out.resize(n);
  if (std::fseek(file.f, static_cast<long>(begin), SEEK_SET) != 0)
    return ql_fail(QL_ERR_INVALID, "seek to tensor %s failed", name.c_str());
  if (es == 4) {
    if (std::fread(out.data(), 4, n, file.f) != n)
      return ql_fail(QL_ERR_INVALID, "short read of tensor %s", name.c_str());
    return QL_OK;
  }
  std::vector<uint16_t> h(n);
  if (std::fread(h.data(), 2, n, file.f) != n)
    return ql_fail(QL_ERR_INVALID, "short read of tensor %s", name.c_str());
  for (uint64_t i = 0; i < n; ++i) {  // IEEE half -> single, exact
    const uint32_t sgn = (h[i] & 0x8000u) << 16, ex = (h[i] >> 10) & 0x1fu, man = h[i] & 0x3ffu;
    uint32_t bits;
    if (ex == 0) {
      if (man == 0) {
        bits = sgn;
      } else {  // subnormal: normalise
        int e = -1;
        uint32_t m = man;
        do {
          ++e;
          m <<= 1;
        } while ((m & 0x400u) == 0);
        bits = sgn | (static_cast<uint32_t>(127 - 15 - e) << 23) | ((m & 0x3ffu) << 13);
      }
    } else if (ex == 31) {
      bits = sgn | 0x7f800000u | (man << 13);
    } else {
      bits = sgn | ((ex + 127 - 15) << 23) | (man << 13);
    }
    std::memcpy(&out[i], &bits, 4);
  }
  return QL_OK;
}

int read_dim(const File& f, const std::string& key, bool optional, int64_t* out, bool* found) {
  auto it = f.meta.find(key);
  if (found) *found = it != f.meta.end();
  if (it == f.meta.end()) {
    if (optional) return QL_OK;
    return ql_fail(QL_ERR_INVALID, "Missing metadata key: %s", key.c_str());
  }
  const Value& v = it->second;
  const bool is_uint = v.type == kU8 || v.type == kU16 || v.type == kU32 || v.type == kU64;
  const bool is_int = v.type == kI8 || v.type == kI16 || v.type == kI32 || v.type == kI64;
  if (!is_uint && !is_int) return ql_fail(QL_ERR_INVALID, "Metadata key %s is not an integer", key.c_str());
  const int64_t x = is_uint ? static_cast<int64_t>(v.u) : v.i;
  if (x <= 0 || x > (1ll << 31) - 1)
    return ql_fail(QL_ERR_INVALID, "Metadata key %s must be a positive dimension, got %lld",
                   key.c_str(), (long long)x);
  *out = x;
  return QL_OK;
}

int read_positive_f32(const File& f, const std::string& key, float* out) {
  auto it = f.meta.find(key);
  if (it == f.meta.end()) return ql_fail(QL_ERR_INVALID, "Missing metadata key: %s", key.c_str());
  const Value& v = it->second;
  if (v.type != kF32v && v.type != kF64)
    return ql_fail(QL_ERR_INVALID, "Metadata key %s is not a float", key.c_str());
  const float x = static_cast<float>(v.f);
  if (!std::isfinite(x) || x <= 0.f)
    return ql_fail(QL_ERR_INVALID, "Metadata key %s must be finite and positive", key.c_str());
  *out = x;
  return QL_OK;
}

}  // namespace

extern "C" int ql_llama_load_gguf(ql_ctx* ctx, const char* path, ql_llama** out) {
  if (!path || !out) return ql_fail(QL_ERR_INVALID, "ql_llama_load_gguf: NULL argument");
  *out = nullptr;
  File file;
  int r = parse(file, path);
  if (r != QL_OK) return r;
  auto arch_it = file.meta.find("general.architecture");
  if (arch_it == file.meta.end() || arch_it->second.type != kString)
    return ql_fail(QL_ERR_INVALID, "Missing or invalid metadata key: general.architecture");
  const std::string arch = arch_it->second.s;
  auto key = [&](const char* k) { return arch + "." + k; };
  const TensorInfo* emb = file.find("token_embd.weight");
  if (!emb) return ql_fail(QL_ERR_INVALID, "Missing tensor: token_embd.weight");
  if (emb->dims.size() != 2)
    return ql_fail(QL_ERR_INVALID, "token_embd.weight must be 2D [vocab_size, hidden_size]");
  ql_llama_config cfg{};
  cfg.vocab_size = static_cast<int32_t>(emb->dims[1]);
  cfg.hidden_size = static_cast<int32_t>(emb->dims[0]);
  auto tok = file.meta.find("tokenizer.ggml.tokens");
  if (tok != file.meta.end() && tok->second.type == kArray &&
      tok->second.count != static_cast<uint64_t>(cfg.vocab_size))
    return ql_fail(QL_ERR_INVALID,
                   "tokenizer.ggml.tokens has %llu entries but token_embd.weight has %d rows",
                   (unsigned long long)tok->second.count, cfg.vocab_size);
  int64_t heads = 0, kv_heads = 0, rot = 0, ff = 0, blocks = 0, ctx_len = 0;
  bool have_kv = false, have_rot = false;
  if ((r = read_dim(file, key("attention.head_count"), false, &heads, nullptr)) != QL_OK) return r;
  if (cfg.hidden_size % heads != 0)
    return ql_fail(QL_ERR_INVALID, "embedding_length %d is not divisible by attention.head_count %lld",
                   cfg.hidden_size, (long long)heads);
  if ((r = read_dim(file, key("attention.head_count_kv"), true, &kv_heads, &have_kv)) != QL_OK) return r;
  if (!have_kv) kv_heads = heads;
  if (kv_heads > heads)
    return ql_fail(QL_ERR_INVALID, "attention.head_count_kv %lld must not exceed attention.head_count %lld",
                   (long long)kv_heads, (long long)heads);
  if (heads % kv_heads != 0)
    return ql_fail(QL_ERR_INVALID, "attention.head_count %lld must be divisible by attention.head_count_kv %lld",
                   (long long)heads, (long long)kv_heads);
  if ((r = read_dim(file, key("rope.dimension_count"), true, &rot, &have_rot)) != QL_OK) return r;
  if (have_rot && rot != cfg.hidden_size / heads)
    return ql_fail(QL_ERR_UNSUPPORTED,
                   "rope.dimension_count %lld does not match head_dim %lld; partial RoPE is not "
                   "supported yet", (long long)rot, (long long)(cfg.hidden_size / heads));
  if ((r = read_positive_f32(file, key("attention.layer_norm_rms_epsilon"), &cfg.rms_norm_eps)) != QL_OK)
    return r;
  cfg.rope_theta = 10000.0f;  // llama.cpp's default when rope.freq_base is absent
  if (file.meta.count(key("rope.freq_base")) &&
      (r = read_positive_f32(file, key("rope.freq_base"), &cfg.rope_theta)) != QL_OK)
    return r;
  if ((r = read_dim(file, key("feed_forward_length"), false, &ff, nullptr)) != QL_OK) return r;
  if ((r = read_dim(file, key("block_count"), false, &blocks, nullptr)) != QL_OK) return r;
  if ((r = read_dim(file, key("context_length"), false, &ctx_len, nullptr)) != QL_OK) return r;
  cfg.num_heads = static_cast<int32_t>(heads);
  cfg.num_kv_heads = static_cast<int32_t>(kv_heads);
  cfg.intermediate_size = static_cast<int32_t>(ff);
  cfg.num_layers = static_cast<int32_t>(blocks);
  cfg.max_position_embeddings = static_cast<int32_t>(ctx_len);

  // every check on the file is done: only now is a device needed
  if (!ctx) return ql_fail(QL_ERR_INVALID, "ql_llama_load_gguf: NULL context");
  ql_llama* m = nullptr;
  if ((r = ql_llama_create(ctx, &cfg, &m)) != QL_OK) return r;
  std::vector<float> data;
  std::vector<uint64_t> dims;
  auto load = [&](const std::string& name) -> int {
    int rc = load_f32(file, name, data, dims);
    if (rc == QL_OK) rc = ql_llama_set_tensor(m, name.c_str(), data.data(),
                                              static_cast<int64_t>(data.size()));
    return rc;
  };
  std::vector<std::string> names = {"token_embd.weight", "output_norm.weight"};
  if (file.find("output.weight")) names.push_back("output.weight");
  for (int l = 0; l < cfg.num_layers; ++l)
    for (const char* s : {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm",
                          "ffn_gate", "ffn_up", "ffn_down"})
      names.push_back("blk." + std::to_string(l) + "." + s + ".weight");
  for (const auto& n : names) {
    if ((r = load(n)) != QL_OK) {
      const std::string msg = ql_last_error();
      ql_llama_destroy(m);
      return ql_fail(r, "%s", msg.c_str());
    }
  }
  *out = m;
  return QL_OK;
}
