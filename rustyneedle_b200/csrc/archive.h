// archive.h — reader of rustyneedle's `.cact` archives (host side).
//
// Format: docs/format.md of the reference; parsing follows
// crates/cact/src/{geometry.rs:41-115, record.rs:38-85, archive.rs:43-70} and
// the canonical positional walk of layout.rs:190-293.
#pragma once

#include <cstdint>
#include <string>
#include <array>
#include <vector>

namespace nba {

struct ArchiveError {
  int status;  // nb_status
  std::string message;
};

enum Kind : uint8_t { HALF = 1, SINGLE = 2, CODEBOOK = 3, RAW = 4 };

struct Record {
  uint8_t kind = 0;
  std::vector<uint64_t> shape;
  uint64_t offset = 0, byte_len = 0;
  uint32_t group_size = 0, bits = 0;
  uint64_t rows() const { return shape.empty() ? 0 : shape[0]; }
  uint64_t columns() const { return shape.size() > 1 ? shape[1] : 1; }
  uint64_t group() const { return group_size ? group_size : 1; }
  uint64_t padded_columns() const { return (columns() + group() - 1) / group() * group(); }
  uint32_t index_bits() const { return bits == 5 ? 2 : bits; }
  uint64_t packed_row_bytes() const { return padded_columns() * index_bits() / 8; }
  uint64_t packed_bytes() const { return rows() * packed_row_bytes(); }
  uint64_t groups_per_row() const { return padded_columns() / group(); }
};

struct Geometry {
  uint32_t tensor_count, codebook_len, kv_window, kv_bits, vocab, out_vocab, d_model, num_heads, num_kv_heads, num_layers,
      qk_head_dim, v_head_dim, max_seq_len, hada_n, mhc_lanes, sliding_window, qkv_conv_taps, engram_slots, engram_sub_dim,
      engram_tables, engram_conv_taps, engram_conv_dilation, engram_seed_heads;
  uint64_t global_layers;
  std::vector<uint32_t> engram_orders, engram_sites;
  float rope_theta;
  uint32_t output_vocab() const { return out_vocab == 0 ? vocab : out_vocab; }
  bool is_global_layer(uint32_t layer) const { return layer < 64 && ((global_layers >> layer) & 1u); }
};

struct HadamardIdx { uint32_t d1, d2, b2, d3, d4, w1a, w1b, w2a, w2b, w3a, w3b, cond_v, cond_u; };
struct LayerIdx {
  uint32_t norm_in, q, k, v, q_norm, k_norm, gate, out, post_norm, attn_gate, pre_hada;
  bool has_taps = false;
  uint32_t taps[3]{};  // q, k, v causal convolution gains (when has_taps)
  HadamardIdx hada;
};
struct LanesIdx { uint32_t a_pre, a_post, a_res, b_pre, b_post, b_res, phi_pre, phi_post, phi_res; };

struct Layout {
  uint32_t embedding = 0;
  std::vector<LayerIdx> layers;
  LanesIdx lanes{};
  uint32_t perms[2]{};
  uint32_t engram_sites = 0;
  std::vector<std::array<uint32_t, 4>> engrams;  // per site: tables, key_proj, value_proj, taps
  uint32_t final_norm = 0;
  uint32_t probe_heads = 0;
  struct HeadIdx { uint32_t code, probes, gain, query, row_bias, proj, bias; };
  std::vector<HeadIdx> heads;  // crates/cact/src/layout.rs:236-254
  bool audio = false;
  std::vector<std::array<uint32_t, 10>> cross;  // per decoder layer: norm, q, k, v, gate, out, q_norm, k_norm, post_norm, gate
  uint32_t position_gate = 0;
  uint32_t text_vocab = 0;
  uint32_t tokenizer = 0;
};

class Archive {
 public:
  // Throws ArchiveError.
  explicit Archive(const char* path);
  ~Archive();
  Archive(const Archive&) = delete;
  Archive& operator=(const Archive&) = delete;

  const Geometry& geometry() const { return geo_; }
  const std::vector<float>& codebook() const { return codebook_; }
  const Record& record(uint32_t i) const { return records_.at(i); }
  uint32_t count() const { return (uint32_t)records_.size(); }
  const uint8_t* data(uint32_t i) const { return base_ + records_.at(i).offset; }
  std::vector<float> floats(uint32_t i) const;  // kinds 1 and 2 (crates/model/src/tensors.rs:3-9)
  Layout resolve() const;
  void validate_tokenizer(uint32_t index) const;  // crates/tokenizer/src/vocabulary.rs:66-99

 private:
  const uint8_t* base_ = nullptr;
  size_t size_ = 0;
  Geometry geo_{};
  std::vector<float> codebook_;
  std::vector<Record> records_;
};

float half_to_f32(uint16_t bits);

}  // namespace nba
