// GGUF reader and BaseLM config validation (host only, no CUDA).
//
// Restates gguf::load_summary (src/gguf.rs:222-286), GgmlType::storage_bytes
// (:37-48), primary_base_format (:117-133), validate_baselm (:135-148) and
// BaseLmConfig::from_gguf (src/baselm.rs:60-180) without its fixed-geometry
// gate (:102-113): any geometry the CUDA kernels support is accepted.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace vg {

enum GgmlType : uint32_t { GGML_F32 = 0, GGML_F16 = 1, GGML_Q8_0 = 8 };

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;  // GGUF order: dims[0] is the contiguous extent
  uint32_t type = 0;
  uint64_t offset = 0;  // relative to the data region
  uint64_t elements = 0;
  uint64_t bytes = 0;
};

struct MetaValue {
  enum Kind { NUMBER, TEXT, ARRAY } kind = NUMBER;
  double number = 0;
  bool integral = false;
  std::string text;
};

struct GgufSummary {
  std::string path;
  uint32_t version = 0;
  uint64_t alignment = 32;
  uint64_t data_offset = 0;
  uint64_t file_bytes = 0;
  std::map<std::string, MetaValue> metadata;
  std::vector<TensorInfo> tensors;

  const TensorInfo *find(const std::string &name) const;
};

struct BaseLmConfig {
  uint32_t context_length = 0, embedding_length = 0, block_count = 0,
           feed_forward_length = 0, vocab_size = 0, head_count = 0, head_count_kv = 0,
           head_dim = 0, kv_dim = 0, rope_original_context_length = 0;
  float rms_epsilon = 0, rope_theta = 0, embedding_scale = 0, residual_scale = 0,
        logit_scale = 0;
  std::string rope_scaling_type;
  bool tied_output = true;
  std::string output_tensor;
  uint32_t format = GGML_Q8_0;  // primary format
  float rope_scaling_factor() const;
  bool rope_long() const { return context_length > rope_original_context_length; }
};

// The ResidualLM + FSQ + fusion part of an acoustic GGUF (AcousticConfig,
// src/acoustic.rs:59-187), checked against the BaseLM it follows. The
// reference accepts only 8 layers, 2048 wide, a 512-wide FSQ latent; this
// loader takes any geometry the kernels support and the same tensor table.
struct AcousticConfig {
  std::string architecture;
  float model_version = 0;
  uint32_t residual_block_count = 0, embedding_length = 0, fsq_latent_dim = 0;
  bool no_rope = false;
  float fsq_scale = 0;
};

// Thrown (inside the library only) with a VG_* status and message.
struct Error {
  int code;
  std::string msg;
};

uint64_t storage_bytes(uint32_t type, uint64_t elements);  // throws Error
GgufSummary load_summary(const std::string &path);          // throws Error
uint32_t primary_base_format(const GgufSummary &s);         // throws Error
// requested: 0 (auto) or GGML_Q8_0 / GGML_F16
BaseLmConfig config_from_gguf(const GgufSummary &s, uint32_t requested_format);
// Geometry limits of the CUDA kernels (head_dim, alignment of row widths, ...).
void check_kernel_support(const GgufSummary &s, const BaseLmConfig &c);
// Parses and validates the acoustic GGUF's ResidualLM/FSQ/fusion tensors
// against the BaseLM geometry (heads, head_dim, FFN width, epsilon).
AcousticConfig acoustic_from_gguf(const GgufSummary &s, const BaseLmConfig &base);

}  // namespace vg
