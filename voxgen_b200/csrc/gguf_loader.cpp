// GGUF reader and BaseLM config validation; see gguf_loader.h for citations.
#include "gguf_loader.h"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "../../include/voxgen_cuda.h"

namespace vg {

static std::string fmt(const char *f, ...) __attribute__((format(printf, 1, 2)));
static std::string fmt(const char *f, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, sizeof buf, f, ap);
  va_end(ap);
  return buf;
}

[[noreturn]] static void fail(int code, const std::string &msg) { throw Error{code, msg}; }

const TensorInfo *GgufSummary::find(const std::string &name) const {
  for (const auto &t : tensors)
    if (t.name == name) return &t;
  return nullptr;
}

static const char *type_name(uint32_t t) {
  switch (t) {
    case GGML_F32: return "F32";
    case GGML_F16: return "F16";
    case GGML_Q8_0: return "Q8_0";
    default: return "GGML_TYPE_OTHER";
  }
}

uint64_t storage_bytes(uint32_t type, uint64_t elements) {
  switch (type) {
    case GGML_F32:
      if (elements > UINT64_MAX / 4) fail(VG_EFORMAT, "F32 tensor size overflow");
      return elements * 4;
    case GGML_F16:
      if (elements > UINT64_MAX / 2) fail(VG_EFORMAT, "F16 tensor size overflow");
      return elements * 2;
    case GGML_Q8_0:
      // ggml Q8_0: blocks of 32 values = fp16 scale (2 B) + 32 int8 quants.
      if (elements % 32) fail(VG_EFORMAT, fmt("Q8_0 tensor has %llu elements, not divisible by 32",
                                              (unsigned long long)elements));
      return elements / 32 * 34;
    default:
      fail(VG_EUNSUPPORTED, fmt("unsupported GGML tensor type %u", type));
  }
}

namespace {
struct Reader {
  const uint8_t *p, *begin, *end;
  void need(size_t n) {
    if ((size_t)(end - p) < n)
      fail(VG_EFORMAT, fmt("unexpected EOF while reading GGUF at byte %zu", (size_t)(p - begin)));
  }
  template <class T> T get() {
    need(sizeof(T));
    T v;
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t n = get<uint64_t>();
    need(n);
    std::string s(reinterpret_cast<const char *>(p), (size_t)n);
    p += n;
    return s;
  }
};

// read_meta_value, src/gguf.rs:190-220
MetaValue read_value(Reader &r, uint32_t ty, int depth) {
  if (depth > 8) fail(VG_EFORMAT, "GGUF metadata nesting too deep");
  MetaValue v;
  switch (ty) {
    case 0: v.number = r.get<uint8_t>(); v.integral = true; break;
    case 1: v.number = r.get<int8_t>(); v.integral = true; break;
    case 2: v.number = r.get<uint16_t>(); v.integral = true; break;
    case 3: v.number = r.get<int16_t>(); v.integral = true; break;
    case 4: v.number = r.get<uint32_t>(); v.integral = true; break;
    case 5: v.number = r.get<int32_t>(); v.integral = true; break;
    case 6: v.number = r.get<float>(); break;
    case 7: v.number = r.get<uint8_t>() != 0; v.integral = true; break;
    case 8: v.kind = MetaValue::TEXT; v.text = r.str(); break;
    case 9: {
      uint32_t et = r.get<uint32_t>();
      uint64_t n = r.get<uint64_t>();
      for (uint64_t i = 0; i < n; ++i) (void)read_value(r, et, depth + 1);
      v.kind = MetaValue::ARRAY;
      break;
    }
    case 10: v.number = (double)r.get<uint64_t>(); v.integral = true; break;
    case 11: v.number = (double)r.get<int64_t>(); v.integral = true; break;
    case 12: v.number = r.get<double>(); break;
    default: fail(VG_EFORMAT, fmt("unknown GGUF metadata value type %u", ty));
  }
  return v;
}

struct Mapping {
  void *addr = MAP_FAILED;
  size_t len = 0;
  ~Mapping() {
    if (addr != MAP_FAILED && len) munmap(addr, len);
  }
};
}  // namespace

GgufSummary load_summary(const std::string &path) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) fail(VG_EIO, fmt("open %s failed", path.c_str()));
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    fail(VG_EIO, fmt("stat %s failed", path.c_str()));
  }
  Mapping map;
  map.len = (size_t)st.st_size;
  if (map.len) map.addr = mmap(nullptr, map.len, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map.len == 0 || map.addr == MAP_FAILED) fail(VG_EFORMAT, fmt("%s is not a GGUF file", path.c_str()));
  const uint8_t *base = static_cast<const uint8_t *>(map.addr);
  Reader r{base, base, base + map.len};
  GgufSummary s;
  s.path = path;
  s.file_bytes = map.len;
  if (r.get<uint32_t>() != 0x46554747u) fail(VG_EFORMAT, fmt("%s is not a GGUF file", path.c_str()));
  s.version = r.get<uint32_t>();
  if (s.version < 2 || s.version > 3)
    fail(VG_EFORMAT, fmt("unsupported GGUF version %u; expected v2/v3", s.version));
  uint64_t tensor_count = r.get<uint64_t>();
  uint64_t metadata_count = r.get<uint64_t>();
  for (uint64_t i = 0; i < metadata_count; ++i) {
    std::string key = r.str();
    uint32_t ty = r.get<uint32_t>();
    MetaValue v = read_value(r, ty, 0);
    if (key == "general.alignment" && v.kind == MetaValue::NUMBER && (ty == 4 || ty == 10))
      s.alignment = v.number >= 1 ? (uint64_t)v.number : 1;
    s.metadata[key] = v;
  }
  if (tensor_count > 200000) fail(VG_EFORMAT, "GGUF tensor count is implausible");
  s.tensors.reserve((size_t)tensor_count);
  for (uint64_t i = 0; i < tensor_count; ++i) {
    TensorInfo t;
    t.name = r.str();
    uint32_t n_dims = r.get<uint32_t>();
    if (n_dims == 0 || n_dims > 8) fail(VG_EFORMAT, fmt("invalid tensor rank %u for %s", n_dims, t.name.c_str()));
    t.elements = 1;
    for (uint32_t d = 0; d < n_dims; ++d) {
      uint64_t v = r.get<uint64_t>();
      if (v && t.elements > UINT64_MAX / v) fail(VG_EFORMAT, fmt("element-count overflow for %s", t.name.c_str()));
      t.elements *= v;
      t.dims.push_back(v);
    }
    t.type = r.get<uint32_t>();
    t.offset = r.get<uint64_t>();
    try {
      t.bytes = storage_bytes(t.type, t.elements);
    } catch (Error &e) {
      e.msg = "tensor " + t.name + ": " + e.msg;
      throw;
    }
    s.tensors.push_back(std::move(t));
  }
  uint64_t pos = (uint64_t)(r.p - base);
  s.data_offset = (pos + s.alignment - 1) / s.alignment * s.alignment;
  for (const auto &t : s.tensors) {
    uint64_t end = s.data_offset + t.offset;
    if (end < t.offset || end + t.bytes < end) fail(VG_EFORMAT, "tensor absolute offset overflow");
    if (end + t.bytes > s.file_bytes)
      fail(VG_EFORMAT, fmt("tensor %s extends beyond end of %s", t.name.c_str(), path.c_str()));
  }
  return s;
}

uint32_t primary_base_format(const GgufSummary &s) {
  // Look only at sizeable multi-dimensional tensors (src/gguf.rs:118-129).
  uint64_t q8 = 0, f16 = 0;
  for (const auto &t : s.tensors) {
    if (t.dims.size() < 2 || t.elements < 4096) continue;
    if (t.type == GGML_Q8_0) q8 += t.bytes;
    if (t.type == GGML_F16) f16 += t.bytes;
  }
  if (q8 > 0 && q8 >= f16) return GGML_Q8_0;
  if (f16 > 0) return GGML_F16;
  fail(VG_EUNSUPPORTED, "could not identify BaseLM as Q8_0 or F16 from the tensor table");
}

static const MetaValue *meta(const GgufSummary &s, std::initializer_list<const char *> keys) {
  for (const char *k : keys) {
    auto it = s.metadata.find(k);
    if (it != s.metadata.end()) return &it->second;
  }
  return nullptr;
}
static bool meta_u32(const GgufSummary &s, std::initializer_list<const char *> keys, uint32_t &out) {
  for (const char *k : keys) {
    auto it = s.metadata.find(k);
    if (it == s.metadata.end()) continue;
    const MetaValue &v = it->second;
    if (v.kind == MetaValue::NUMBER && v.integral && v.number >= 0 && v.number <= 4294967295.0) {
      out = (uint32_t)v.number;
      return true;
    }
    if (v.kind == MetaValue::TEXT) {  // the reference parses metadata text (src/baselm.rs:274-276)
      char *e = nullptr;
      unsigned long long x = strtoull(v.text.c_str(), &e, 10);
      if (e && *e == 0 && !v.text.empty() && x <= 4294967295ull) {
        out = (uint32_t)x;
        return true;
      }
    }
  }
  return false;
}
static bool meta_f32(const GgufSummary &s, std::initializer_list<const char *> keys, float &out) {
  for (const char *k : keys) {
    auto it = s.metadata.find(k);
    if (it == s.metadata.end()) continue;
    const MetaValue &v = it->second;
    if (v.kind == MetaValue::NUMBER) {
      out = (float)v.number;
      return true;
    }
    if (v.kind == MetaValue::TEXT) {
      char *e = nullptr;
      float x = strtof(v.text.c_str(), &e);
      if (e && *e == 0 && !v.text.empty()) {
        out = x;
        return true;
      }
    }
  }
  return false;
}
static std::string join(std::initializer_list<const char *> keys) {
  std::string o;
  for (const char *k : keys) o += (o.empty() ? "" : " or ") + std::string(k);
  return o;
}
#define REQ_U32(dst, ...)                                                               \
  do {                                                                                  \
    if (!meta_u32(s, {__VA_ARGS__}, dst))                                              \
      fail(VG_EUNSUPPORTED, "missing required metadata: " + join({__VA_ARGS__}));      \
  } while (0)
#define REQ_F32(dst, ...)                                                               \
  do {                                                                                  \
    if (!meta_f32(s, {__VA_ARGS__}, dst))                                              \
      fail(VG_EUNSUPPORTED, "missing required metadata: " + join({__VA_ARGS__}));      \
  } while (0)

static const TensorInfo &tensor(const GgufSummary &s, const std::string &name) {
  const TensorInfo *t = s.find(name);
  if (!t) fail(VG_EUNSUPPORTED, fmt("required GGUF tensor \"%s\" is missing from %s", name.c_str(), s.path.c_str()));
  return *t;
}
static std::string dims_str(const std::vector<uint64_t> &d) {
  std::string o = "[";
  for (size_t i = 0; i < d.size(); ++i) o += (i ? ", " : "") + std::to_string(d[i]);
  return o + "]";
}
static void require_dims(const TensorInfo &t, std::vector<uint64_t> dims) {
  if (t.dims != dims)
    fail(VG_EUNSUPPORTED, "tensor " + t.name + " has dimensions " + dims_str(t.dims) + ", expected " + dims_str(dims));
}
static void require_f32(const TensorInfo &t) {
  if (t.type != GGML_F32) fail(VG_EUNSUPPORTED, fmt("tensor %s is %s, expected F32", t.name.c_str(), type_name(t.type)));
}
static void require_matrix_type(const TensorInfo &t) {
  if (t.type != GGML_F16 && t.type != GGML_Q8_0)
    fail(VG_EUNSUPPORTED, fmt("matrix %s uses unsupported %s", t.name.c_str(), type_name(t.type)));
  if (t.type == GGML_Q8_0 && t.dims[0] % 32 != 0)
    fail(VG_EUNSUPPORTED, fmt("Q8_0 matrix %s has row width %llu, not divisible by 32", t.name.c_str(),
                              (unsigned long long)t.dims[0]));
}

float BaseLmConfig::rope_scaling_factor() const {
  // src/baselm.rs:194-205
  if (rope_scaling_type != "longrope" || context_length <= rope_original_context_length ||
      rope_original_context_length <= 1)
    return 1.0f;
  float mx = (float)context_length, orig = (float)rope_original_context_length;
  return std::sqrt(1.0f + std::log(mx / orig) / std::log(orig));
}

BaseLmConfig config_from_gguf(const GgufSummary &s, uint32_t requested) {
  // validate_baselm, src/gguf.rs:135-148
  for (const auto &t : s.tensors)
    if (t.type != GGML_F32 && t.type != GGML_F16 && t.type != GGML_Q8_0)
      fail(VG_EUNSUPPORTED, fmt("Unsupported BaseLM tensor type %s in %s", type_name(t.type), t.name.c_str()));
  BaseLmConfig c;
  c.format = primary_base_format(s);
  if (requested != 0 && requested != c.format)
    fail(VG_EUNSUPPORTED, fmt("BaseLM format mismatch: requested %s, GGUF tensor table looks like %s",
                              requested == GGML_Q8_0 ? "q8_0" : "f16", c.format == GGML_Q8_0 ? "q8_0" : "f16"));
  const MetaValue *arch = meta(s, {"general.architecture"});
  if (!arch) fail(VG_EUNSUPPORTED, "required GGUF metadata key \"general.architecture\" is missing");
  if (arch->kind != MetaValue::TEXT || arch->text != "minicpm4")
    fail(VG_EUNSUPPORTED, "VoxGen BaseLM expects general.architecture=minicpm4, got \"" + arch->text + "\"");
  REQ_U32(c.context_length, "minicpm4.context_length");
  REQ_U32(c.embedding_length, "minicpm4.embedding_length");
  REQ_U32(c.block_count, "minicpm4.block_count");
  REQ_U32(c.feed_forward_length, "minicpm4.feed_forward_length");
  REQ_U32(c.head_count, "minicpm4.attention.head_count");
  REQ_U32(c.head_count_kv, "minicpm4.attention.head_count_kv");
  REQ_U32(c.head_dim, "minicpm4.attention.key_length", "minicpm4.rope.dimension_count");
  uint32_t rope_dim = 0;
  REQ_U32(rope_dim, "minicpm4.rope.dimension_count");
  REQ_F32(c.rms_epsilon, "minicpm4.attention.layer_norm_rms_epsilon");
  REQ_F32(c.rope_theta, "minicpm4.rope.freq_base");
  const MetaValue *st = meta(s, {"minicpm4.rope.scaling.type"});
  c.rope_scaling_type = (st && st->kind == MetaValue::TEXT) ? st->text : "none";
  c.rope_original_context_length = c.context_length;
  meta_u32(s, {"minicpm4.rope.scaling.original_context_length", "minicpm4.rope.scaling.original_context_len"},
           c.rope_original_context_length);
  meta_f32(s, {"minicpm4.embedding_scale"}, c.embedding_scale);
  meta_f32(s, {"minicpm4.residual_scale"}, c.residual_scale);
  meta_f32(s, {"minicpm4.logit_scale"}, c.logit_scale);
  if (c.head_count_kv == 0 || c.head_count == 0)
    fail(VG_EUNSUPPORTED, "head_count and head_count_kv must be positive");
  if (c.head_count % c.head_count_kv != 0)
    fail(VG_EUNSUPPORTED, fmt("head_count %u is not divisible by head_count_kv %u", c.head_count, c.head_count_kv));
  if (rope_dim != c.head_dim)
    fail(VG_EUNSUPPORTED, fmt("partial RoPE is not implemented: rope_dimension_count=%u, head_dim=%u", rope_dim, c.head_dim));
  if (c.rope_scaling_type != "longrope" && c.rope_scaling_type != "none")
    fail(VG_EUNSUPPORTED, "unsupported RoPE scaling type \"" + c.rope_scaling_type + "\"; expected longrope");
  if ((uint64_t)c.head_count * c.head_dim != c.embedding_length)
    fail(VG_EUNSUPPORTED, fmt("head_count*head_dim = %u does not equal embedding_length %u",
                              c.head_count * c.head_dim, c.embedding_length));
  c.kv_dim = c.head_count_kv * c.head_dim;

  const TensorInfo &tok = tensor(s, "token_embd.weight");
  if (tok.dims.size() != 2) fail(VG_EUNSUPPORTED, "token_embd.weight must be rank 2, got " + dims_str(tok.dims));
  if (tok.dims[1] > 0xFFFFFFFFull) fail(VG_EUNSUPPORTED, "vocabulary size exceeds u32");
  c.vocab_size = (uint32_t)tok.dims[1];
  require_dims(tok, {c.embedding_length, c.vocab_size});
  require_matrix_type(tok);
  if (const TensorInfo *o = s.find("output.weight")) {
    require_dims(*o, {c.embedding_length, c.vocab_size});
    require_matrix_type(*o);
    c.tied_output = false;
    c.output_tensor = "output.weight";
  } else {
    c.tied_output = true;
    c.output_tensor = "token_embd.weight";
  }
  require_dims(tensor(s, "output_norm.weight"), {c.embedding_length});
  if (c.rope_scaling_type == "longrope") {
    require_dims(tensor(s, "rope_factors_short.weight"), {c.head_dim / 2});
    require_dims(tensor(s, "rope_factors_long.weight"), {c.head_dim / 2});
    require_f32(tensor(s, "rope_factors_short.weight"));
    require_f32(tensor(s, "rope_factors_long.weight"));
  }
  // validate_layer, src/baselm.rs:215-247
  for (uint32_t i = 0; i < c.block_count; ++i) {
    auto nm = [&](const char *suffix) { return fmt("blk.%u.%s", i, suffix); };
    const TensorInfo &an = tensor(s, nm("attn_norm.weight"));
    const TensorInfo &fn = tensor(s, nm("ffn_norm.weight"));
    require_dims(an, {c.embedding_length});
    require_dims(fn, {c.embedding_length});
    require_f32(an);
    require_f32(fn);
    const uint64_t E = c.embedding_length, F = c.feed_forward_length, K = c.kv_dim;
    struct { const char *suffix; std::vector<uint64_t> dims; } mats[] = {
        {"attn_q.weight", {E, E}},  {"attn_k.weight", {E, K}},  {"attn_v.weight", {E, K}},
        {"attn_output.weight", {E, E}}, {"ffn_gate.weight", {E, F}}, {"ffn_up.weight", {E, F}},
        {"ffn_down.weight", {F, E}}};
    for (auto &m : mats) {
      const TensorInfo &t = tensor(s, nm(m.suffix));
      require_dims(t, m.dims);
      require_matrix_type(t);
    }
  }
  require_f32(tensor(s, "output_norm.weight"));
  // validate_format_consistency, src/baselm.rs:1266-1293
  for (const auto &t : s.tensors) {
    if (t.dims.size() < 2 || t.elements < 4096 || t.name.find("rope_factors") != std::string::npos) continue;
    if (c.format == GGML_F16 && t.type != GGML_F16)
      fail(VG_EUNSUPPORTED, fmt("F16 BaseLM has non-F16 matrix %s (%s)", t.name.c_str(), type_name(t.type)));
    if (c.format == GGML_Q8_0 && t.type != GGML_Q8_0 && t.type != GGML_F16)
      fail(VG_EUNSUPPORTED, fmt("Q8_0 BaseLM has unsupported matrix %s (%s)", t.name.c_str(), type_name(t.type)));
  }
  return c;
}

void check_kernel_support(const GgufSummary &s, const BaseLmConfig &c) {
  const uint32_t hd = c.head_dim;
  if (hd != 32 && hd != 64 && hd != 128 && hd != 256)
    fail(VG_EUNSUPPORTED, fmt("head_dim %u is not supported by the CUDA attention kernel (32, 64, 128 or 256)", hd));
  if (c.head_count / c.head_count_kv > 32)
    fail(VG_EUNSUPPORTED, "more than 32 query heads per KV head is not supported");
  auto cols_ok = [](uint32_t type, uint64_t cols) {
    return type == GGML_Q8_0 ? cols % 32 == 0 : cols % 8 == 0;
  };
  for (uint32_t i = 0; i < c.block_count; ++i) {
    auto nm = [&](const char *suffix) { return fmt("blk.%u.%s", i, suffix); };
    const TensorInfo &q = *s.find(nm("attn_q.weight"));
    const TensorInfo &k = *s.find(nm("attn_k.weight"));
    const TensorInfo &v = *s.find(nm("attn_v.weight"));
    if (q.type != k.type || q.type != v.type)
      fail(VG_EUNSUPPORTED, fmt("layer %u: Q/K/V projections of different types are not supported by the fused QKV kernel", i));
    const TensorInfo &g = *s.find(nm("ffn_gate.weight"));
    const TensorInfo &u = *s.find(nm("ffn_up.weight"));
    if (g.type != u.type)
      fail(VG_EUNSUPPORTED, fmt("SwiGLU gate/up dtypes differ: %s vs %s", type_name(g.type), type_name(u.type)));
    for (const char *suffix : {"attn_q.weight", "attn_output.weight", "ffn_gate.weight", "ffn_down.weight"}) {
      const TensorInfo &t = *s.find(nm(suffix));
      if (!cols_ok(t.type, t.dims[0]))
        fail(VG_EUNSUPPORTED, fmt("matrix %s has row width %llu; F16 rows must be a multiple of 8 columns",
                                  t.name.c_str(), (unsigned long long)t.dims[0]));
    }
  }
  const TensorInfo &tok = *s.find("token_embd.weight");
  if (!cols_ok(tok.type, tok.dims[0])) fail(VG_EUNSUPPORTED, "token_embd.weight row width not supported");
}

AcousticConfig acoustic_from_gguf(const GgufSummary &s, const BaseLmConfig &base) {
  AcousticConfig a;
  const MetaValue *arch = meta(s, {"general.architecture"});
  a.architecture = arch && arch->kind == MetaValue::TEXT ? arch->text : std::string();
  if (a.architecture != "voxcpm-acoustic")  // src/acoustic.rs:64-67
    fail(VG_EINVAL, "expected general.architecture=voxcpm-acoustic for the acoustic GGUF, got \"" + a.architecture + "\"");
  if (!meta_f32(s, {"voxcpm.model_version"}, a.model_version) || std::fabs(a.model_version - 2.0f) > 0.01f)
    fail(VG_EUNSUPPORTED, "the acoustic GGUF must be VoxCPM2 acoustic v2.0 (voxcpm.model_version)");
  const MetaValue *nr = meta(s, {"voxcpm.residual_lm.no_rope"});
  if (!meta_u32(s, {"voxcpm.residual_lm.n_layer"}, a.residual_block_count) ||
      !meta_u32(s, {"voxcpm.residual_lm.n_embd"}, a.embedding_length) ||
      !meta_u32(s, {"voxcpm.fsq.latent_dim"}, a.fsq_latent_dim) || !meta_f32(s, {"voxcpm.fsq.scale"}, a.fsq_scale) ||
      !nr || nr->kind != MetaValue::NUMBER)
    fail(VG_EINVAL, "acoustic GGUF metadata is missing voxcpm.residual_lm.* or voxcpm.fsq.* keys");
  a.no_rope = nr->number != 0;
  if (!a.no_rope) fail(VG_EUNSUPPORTED, "VoxCPM2 ResidualLM must run with no_rope=true");  // src/acoustic.rs:969
  if (a.residual_block_count == 0 || a.fsq_latent_dim == 0)
    fail(VG_EINVAL, "acoustic GGUF declares an empty ResidualLM or FSQ latent");
  if (a.embedding_length != base.embedding_length)  // src/acoustic.rs:92-99
    fail(VG_EINVAL, fmt("BaseLM geometry is incompatible with ResidualLM: n_embd %u vs BaseLM %u",
                         a.embedding_length, base.embedding_length));
  if (!std::isfinite(a.fsq_scale) || a.fsq_scale <= 0.0f) fail(VG_EINVAL, fmt("invalid FSQ scale %g", a.fsq_scale));
  for (const auto &t : s.tensors)  // validate_acoustic_f16, src/gguf.rs:150-160
    if (t.type != GGML_F32 && t.type != GGML_F16)
      fail(VG_EUNSUPPORTED, "unsupported acoustic tensor type in " + t.name + "; the F16 acoustic GGUF is required");
  const uint32_t H = a.embedding_length, L = a.fsq_latent_dim, KV = base.kv_dim, F = base.feed_forward_length;
  auto need = [&](const std::string &name) -> const TensorInfo & {
    const TensorInfo *t = s.find(name);
    if (!t) fail(VG_EINVAL, "acoustic GGUF is missing tensor " + name);
    return *t;
  };
  auto matrix = [&](const std::string &name, uint32_t cols, uint32_t rows) {  // require_matrix, :189-205
    const TensorInfo &t = need(name);
    if (t.dims.size() != 2 || t.dims[0] != cols || t.dims[1] != rows)
      fail(VG_EINVAL, fmt("tensor %s does not have dimensions [%u, %u]", name.c_str(), cols, rows));
    if (t.type != GGML_F16) fail(VG_EUNSUPPORTED, "tensor " + name + " must be F16");
  };
  auto vector = [&](const std::string &name, uint32_t n, bool f32_only, bool allow_f32) {  // require_vector, :207-216
    const TensorInfo &t = need(name);
    if (t.dims.size() != 1 || t.dims[0] != n) fail(VG_EINVAL, fmt("tensor %s does not have dimensions [%u]", name.c_str(), n));
    if (f32_only ? t.type != GGML_F32 : !(t.type == GGML_F16 || (allow_f32 && t.type == GGML_F32)))
      fail(VG_EUNSUPPORTED, "tensor " + name + " has an unsupported type");
  };
  matrix("fsq.in_proj.weight", H, L);
  vector("fsq.in_proj.bias", L, false, false);
  matrix("fsq.out_proj.weight", L, H);
  vector("fsq.out_proj.bias", H, false, false);
  matrix("projections.res_fusion_proj.weight", 2 * H, H);
  vector("projections.res_fusion_proj.bias", H, false, false);
  vector("residual_lm.output_norm.weight", H, true, true);
  for (uint32_t l = 0; l < a.residual_block_count; ++l) {
    auto p = [&](const char *sfx) { return fmt("residual_lm.blk.%u.%s", l, sfx); };
    vector(p("attn_norm.weight"), H, true, true);
    vector(p("ffn_norm.weight"), H, true, true);
    matrix(p("attn_q.weight"), H, base.head_count * base.head_dim);
    matrix(p("attn_k.weight"), H, KV);
    matrix(p("attn_v.weight"), H, KV);
    matrix(p("attn_output.weight"), base.head_count * base.head_dim, H);
    matrix(p("ffn_gate.weight"), H, F);
    matrix(p("ffn_up.weight"), H, F);
    matrix(p("ffn_down.weight"), F, H);
  }
  return a;
}

}  // namespace vg
