// needle_oracle.cpp — CPU restatement of rustyneedle's Needle-3 token loop.
//
// TEST INFRASTRUCTURE ONLY: the checker the B200 kernels are compared with and
// the CPU baseline bench.py times. Nothing in rustyneedle_b200 links or calls it.
//
// Every routine names the reference function it restates (path:line inside the
// rustyneedle workspace). Float association order follows the reference exactly;
// the file is compiled with -ffp-contract=off so no multiply-add is fused unless
// the reference fuses it (panel.rs:187 vfmaq_f32, ops.rs:243/274 vfmaq_laneq_f32),
// where std::fma is written out.
//
// Rust's float `Iterator::sum` starts from -0.0 (toolchain >= 1.83; the workspace
// pins rust-version 1.87); explicit `let mut total = 0.0` loops start from +0.0.
// Both are mirrored below.

#include "needle_oracle.h"

#include <omp.h>

#include <algorithm>
#include <array>
#include <cfenv>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <deque>
#include <fstream>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace nbo {

static thread_local std::string g_error;

struct Failure : std::runtime_error {
  int status;
  Failure(int s, const std::string& m) : std::runtime_error(m), status(s) {}
};

enum Status { OK = 0, ERR_IO = -1, ERR_ARCHIVE = -2, ERR_DEPTH = -3, ERR_ARGUMENT = -4, ERR_UNSUPPORTED = -5 };

constexpr float NORM_EPSILON = 1e-6f;
constexpr float COEFFICIENT_LEVELS = 2047.0f;
constexpr size_t LANES8 = 8;
constexpr float RUST_SUM_START = -0.0f;

// ---------------------------------------------------------------- cact crate

// crates/cact/src/layout.rs:323-339
float half_to_f32(uint16_t bits) {
  uint32_t sign = bits >> 15, exponent = (bits >> 10) & 0x1f, mantissa = bits & 0x3ff, value;
  if (exponent == 0 && mantissa == 0) {
    value = sign << 31;
  } else if (exponent == 0) {
    uint32_t shift = __builtin_clz(mantissa) - 21;
    uint32_t m = (mantissa << shift) & 0x3ff;
    value = sign << 31 | (113 - shift) << 23 | m << 13;
  } else if (exponent == 0x1f && mantissa == 0) {
    value = sign << 31 | 0x7f800000u;
  } else if (exponent == 0x1f) {
    value = sign << 31 | 0x7fc00000u | mantissa << 13;
  } else {
    value = sign << 31 | (exponent + 112) << 23 | mantissa << 13;
  }
  float f;
  std::memcpy(&f, &value, 4);
  return f;
}

enum Kind : uint8_t { HALF = 1, SINGLE = 2, CODEBOOK = 3, RAW = 4 };

// crates/cact/src/record.rs:27-85
struct Record {
  uint8_t kind = 0;
  std::vector<size_t> shape;
  size_t offset = 0, byte_len = 0, group_size = 0;
  uint32_t bits = 0;
  size_t rows() const { return shape.empty() ? 0 : shape[0]; }
  size_t columns() const { return shape.size() > 1 ? shape[1] : 1; }
  size_t group() const { return std::max<size_t>(group_size, 1); }
  size_t padded_columns() const { return (columns() + group() - 1) / group() * group(); }
  uint32_t index_bits() const { return bits == 5 ? 2 : bits; }
  size_t packed_row_bytes() const { return padded_columns() * index_bits() / 8; }
  size_t packed_bytes() const { return rows() * packed_row_bytes(); }
  size_t groups_per_row() const { return padded_columns() / group(); }
};

// crates/cact/src/geometry.rs:9-115
struct Geometry {
  size_t tensor_count, codebook_len, kv_window, vocab, out_vocab, d_model, num_heads, num_kv_heads, num_layers,
      qk_head_dim, v_head_dim, max_seq_len, hada_n, mhc_lanes, sliding_window, qkv_conv_taps, engram_slots,
      engram_sub_dim, engram_tables, engram_conv_taps, engram_conv_dilation, engram_seed_heads;
  uint32_t kv_bits;
  uint64_t global_layers;
  std::vector<size_t> engram_orders, engram_sites;
  float rope_theta;
  size_t output_vocab() const { return out_vocab == 0 ? vocab : out_vocab; }
  bool is_global_layer(size_t layer) const { return (global_layers >> layer & 1) == 1; }
};

struct Cursor {
  const std::vector<uint8_t>& bytes;
  size_t position;
  const char* what;
  template <typename T>
  T take() {
    if (position + sizeof(T) > bytes.size()) throw Failure(ERR_ARCHIVE, std::string("archive is truncated inside the ") + what);
    T v;
    std::memcpy(&v, bytes.data() + position, sizeof(T));
    position += sizeof(T);
    return v;
  }
};

struct Archive {
  std::vector<uint8_t> bytes;
  Geometry geo{};
  std::vector<float> codebook;
  std::vector<Record> records;
  const uint8_t* data(size_t index) const { return bytes.data() + records[index].offset; }
};

// crates/cact/src/archive.rs:37-70 and geometry.rs:41-115
std::shared_ptr<Archive> open_archive(const char* path) {
  auto archive = std::make_shared<Archive>();
  std::ifstream file(path, std::ios::binary);
  if (!file) throw Failure(ERR_IO, std::string("cannot open ") + path);
  archive->bytes.assign(std::istreambuf_iterator<char>(file), std::istreambuf_iterator<char>());
  Cursor c{archive->bytes, 0, "header"};
  uint32_t tag = c.take<uint32_t>();
  if (tag != 0x05E12A84u) {
    char m[96];
    std::snprintf(m, sizeof m, "not a Needle 3 archive (format tag 0x%08x)", tag);
    throw Failure(ERR_ARCHIVE, m);
  }
  Geometry& g = archive->geo;
  auto u = [&]() { return (size_t)c.take<uint32_t>(); };
  g.tensor_count = u();
  g.codebook_len = u();
  g.kv_window = u();
  g.kv_bits = (uint32_t)u();
  g.vocab = u();
  g.out_vocab = u();
  g.d_model = u();
  g.num_heads = u();
  g.num_kv_heads = u();
  g.num_layers = u();
  g.qk_head_dim = u();
  g.v_head_dim = u();
  g.max_seq_len = u();
  g.hada_n = u();
  g.mhc_lanes = u();
  g.sliding_window = u();
  uint64_t lo = u(), hi = u();
  g.global_layers = lo | (hi << 32);
  g.qkv_conv_taps = u();
  g.engram_slots = u();
  g.engram_sub_dim = u();
  g.engram_tables = u();
  g.engram_conv_taps = u();
  g.engram_conv_dilation = u();
  g.engram_seed_heads = u();
  size_t order_count = u();
  size_t orders[4];
  for (auto& o : orders) o = u();
  size_t site_count = u();
  size_t sites[16];
  for (auto& s : sites) s = u();
  g.rope_theta = c.take<float>();
  if (order_count > 4 || site_count > 16)
    throw Failure(ERR_ARCHIVE, "unexpected tensor layout: engram order or site count exceeds the header capacity");
  g.engram_orders.assign(orders, orders + order_count);
  g.engram_sites.assign(sites, sites + site_count);
  c.what = "codebook";
  for (size_t i = 0; i < g.codebook_len; ++i) archive->codebook.push_back(c.take<float>());
  c.what = "tensor directory";
  for (size_t i = 0; i < g.tensor_count; ++i) {
    Record r;
    r.kind = c.take<uint8_t>();
    if (r.kind < 1 || r.kind > 4) throw Failure(ERR_ARCHIVE, "unknown tensor element kind " + std::to_string(r.kind));
    size_t rank = c.take<uint8_t>();
    c.take<uint16_t>();
    size_t dims[4];
    for (auto& d : dims) d = c.take<uint32_t>();
    r.shape.assign(dims, dims + std::min<size_t>(rank, 4));
    r.offset = c.take<uint64_t>();
    r.byte_len = c.take<uint64_t>();
    r.group_size = c.take<uint32_t>();
    r.bits = c.take<uint32_t>();
    archive->records.push_back(r);
  }
  for (size_t i = 0; i < archive->records.size(); ++i) {
    const Record& r = archive->records[i];
    if (r.offset + r.byte_len < r.offset || r.offset + r.byte_len > archive->bytes.size())
      throw Failure(ERR_ARCHIVE, "tensor " + std::to_string(i) + " lies outside the archive");
    size_t width = r.kind == HALF ? 2 : r.kind == SINGLE ? 4 : 1;
    if (r.offset % width || r.byte_len % width)
      throw Failure(ERR_ARCHIVE, "unexpected tensor layout: tensor " + std::to_string(i) + " is not aligned to its element width");
  }
  return archive;
}

struct HadamardT { size_t d1, d2, b2, d3, d4, w1a, w1b, w2a, w2b, w3a, w3b, cond_v, cond_u; };
struct LayerT {
  size_t norm_in, q, k, v, q_norm, k_norm, gate, out, post_norm, attn_gate, pre_hada;
  bool has_taps = false;
  size_t taps[3]{};
  HadamardT hada;
};
struct LanesT { size_t a_pre, a_post, a_res, b_pre, b_post, b_res, phi_pre, phi_post, phi_res; };
struct Layout {
  size_t embedding;
  std::vector<LayerT> layers;
  LanesT lanes;
  size_t perms[2];
  size_t engram_count = 0;
  std::vector<std::array<size_t, 4>> engrams;  // tables, key_proj, value_proj, taps per site
  size_t final_norm;
  size_t head_count = 0;
  struct HeadT { uint8_t code; size_t probes, gain, query, row_bias, proj, bias; };
  std::vector<HeadT> heads;
  bool audio = false;
  std::vector<std::array<size_t, 10>> cross;  // per decoder layer: norm, q, k, v, gate, out, q_norm, k_norm, post_norm, gate scalar
  size_t position_gate = 0;
  size_t text_vocab = 0;
  size_t tokenizer;
};

// crates/cact/src/layout.rs:190-293 (the canonical positional walk)
Layout resolve_layout(const Archive& a) {
  Layout L{};
  size_t count = a.records.size();
  if (count == 0 || a.records[count - 1].kind != RAW) throw Failure(ERR_ARCHIVE, "unexpected tensor layout: no trailing tokenizer blob");
  L.tokenizer = count - 1;
  size_t next = 0, end = L.tokenizer;
  auto take = [&]() {
    if (next >= end) throw Failure(ERR_ARCHIVE, "unexpected tensor layout: directory ends before the canonical tensor list");
    return next++;
  };
  auto peek = [&]() -> int { return next < end ? a.records[next].kind : -1; };
  auto hada = [&]() {
    HadamardT h;
    size_t* f = &h.d1;
    for (int i = 0; i < 13; ++i) f[i] = take();
    return h;
  };
  L.embedding = take();
  for (size_t l = 0; l < a.geo.num_layers; ++l) {
    LayerT t{};
    t.norm_in = take();
    t.q = take();
    t.k = take();
    t.v = take();
    if (a.geo.qkv_conv_taps > 0) {
      t.has_taps = true;
      for (auto& x : t.taps) x = take();
    }
    t.q_norm = take();
    t.k_norm = take();
    t.gate = take();
    t.out = take();
    t.post_norm = take();
    t.attn_gate = take();
    t.pre_hada = take();
    t.hada = hada();
    L.layers.push_back(t);
  }
  size_t* lf = &L.lanes.a_pre;
  for (int i = 0; i < 9; ++i) lf[i] = take();
  L.perms[0] = take();
  L.perms[1] = take();
  for (size_t s = 0; s < a.geo.engram_sites.size(); ++s) {
    std::array<size_t, 4> e;
    for (size_t& i : e) i = take();
    L.engrams.push_back(e);
    L.engram_count++;
  }
  L.final_norm = take();
  if (peek() == HALF) {  // layout.rs:236-254 probe heads
    size_t manifest = take();
    const Record& r = a.records[manifest];
    const uint16_t* codes = reinterpret_cast<const uint16_t*>(a.data(manifest));
    for (size_t i = 0; i < r.byte_len / 2; ++i) {
      int code = (int)std::round(half_to_f32(codes[i]));
      if (code < 1 || code > 3) throw Failure(ERR_ARCHIVE, "unexpected tensor layout: unrecognised head manifest code");
      Layout::HeadT h;
      h.code = (uint8_t)code;
      h.probes = take();
      h.gain = take();
      h.query = take();
      h.row_bias = take();
      h.proj = take();
      h.bias = take();
      if (code == 3) take();  // calibration: not read by the model crate
      L.heads.push_back(h);
      L.head_count++;
    }
  }
  if (peek() == SINGLE) {  // layout.rs:256-293 audio encoder
    size_t manifest = take();
    const Record& r = a.records[manifest];
    const float* v = reinterpret_cast<const float*>(a.data(manifest));
    if (r.byte_len / 4 != 13 || v[0] != 3246.0f) throw Failure(ERR_ARCHIVE, "unexpected tensor layout: audio manifest is malformed");
    size_t encoder_layers = (size_t)v[3], stem_stages = (size_t)v[7];
    L.text_vocab = (size_t)v[2];
    for (size_t l = 0; l < a.geo.num_layers; ++l) {
      std::array<size_t, 10> c;
      for (size_t& x : c) x = take();
      L.cross.push_back(c);
    }
    L.position_gate = take();
    for (size_t l = 0; l < encoder_layers; ++l)
      for (int i = 0; i < 17 + 26; ++i) take();
    for (int i = 0; i < 9 + 1 + 1; ++i) take();
    for (size_t s = 1; s < stem_stages; ++s) { take(); take(); }
    take();
    take();
    L.audio = true;
  }
  if (next != L.tokenizer)
    throw Failure(ERR_ARCHIVE, "unexpected tensor layout: " + std::to_string(L.tokenizer - next) + " tensors are left over before the tokenizer");
  return L;
}

// crates/model/src/tensors.rs:3-13
std::vector<float> floats(const Archive& a, size_t index) {
  const Record& r = a.records[index];
  std::vector<float> out;
  if (r.kind == HALF) {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(a.data(index));
    for (size_t i = 0; i < r.byte_len / 2; ++i) out.push_back(half_to_f32(h[i]));
  } else if (r.kind == SINGLE) {
    out.resize(r.byte_len / 4);
    std::memcpy(out.data(), a.data(index), r.byte_len);
  } else {
    throw Failure(ERR_ARCHIVE, "tensor " + std::to_string(index) + " does not hold floating point values");
  }
  return out;
}

// ------------------------------------------------------------- kernels crate

// crates/kernels/src/walsh.rs:41-76 (the aarch64 group-of-128 path, walsh.rs:7-38,
// evaluates the same butterfly network in the same order).
void transform_in_place(float* v, size_t n) {
  size_t span = 1;
  if (n >= 4) {
    for (size_t q = 0; q + 4 <= n; q += 4) {
      float a = v[q], b = v[q + 1], c = v[q + 2], d = v[q + 3];
      float ls = a + b, ld = a - b, hs = c + d, hd = c - d;
      v[q] = ls + hs;
      v[q + 1] = ld + hd;
      v[q + 2] = ls - hs;
      v[q + 3] = ld - hd;
    }
    span = 4;
  }
  while (span < n) {
    for (size_t block = 0; block + 2 * span <= n; block += 2 * span)
      for (size_t i = 0; i < span; ++i) {
        float a = v[block + i], b = v[block + span + i];
        v[block + i] = a + b;
        v[block + span + i] = a - b;
      }
    span *= 2;
  }
  float scale = 1.0f / std::sqrt((float)n);
  for (size_t i = 0; i < n; ++i) v[i] *= scale;
}

// walsh.rs:78-80
void rotate_groups(float* v, size_t n, size_t group) {
  for (size_t g = 0; g + group <= n; g += group) transform_in_place(v + g, group);
}

// ops.rs:7-17
float sum_of_squares(const float* v, size_t n) {
  float lanes[LANES8] = {0};
  size_t whole = n / LANES8 * LANES8;
  for (size_t c = 0; c < whole; c += LANES8)
    for (size_t l = 0; l < LANES8; ++l) lanes[l] += v[c + l] * v[c + l];
  float tail = RUST_SUM_START;
  for (size_t i = whole; i < n; ++i) tail += v[i] * v[i];
  float s = RUST_SUM_START;
  for (size_t l = 0; l < LANES8; ++l) s += lanes[l];
  return s + tail;
}

// ops.rs:19-30
float dot_product(const float* a, const float* b, size_t n) {
  float lanes[LANES8] = {0};
  size_t whole = n / LANES8 * LANES8;
  for (size_t c = 0; c < whole; c += LANES8)
    for (size_t l = 0; l < LANES8; ++l) lanes[l] += a[c + l] * b[c + l];
  float tail = RUST_SUM_START;
  for (size_t i = whole; i < n; ++i) tail += a[i] * b[i];
  float s = RUST_SUM_START;
  for (size_t l = 0; l < LANES8; ++l) s += lanes[l];
  return s + tail;
}

// ops.rs:32-42 (f32::max ignores NaN, as fmaxf does)
float peak_magnitude(const float* v, size_t n) {
  float lanes[LANES8] = {0};
  size_t whole = n / LANES8 * LANES8;
  for (size_t c = 0; c < whole; c += LANES8)
    for (size_t l = 0; l < LANES8; ++l) lanes[l] = std::fmax(lanes[l], std::fabs(v[c + l]));
  float tail = 0.0f;
  for (size_t i = whole; i < n; ++i) tail = std::fmax(tail, std::fabs(v[i]));
  float acc = tail;
  for (size_t l = 0; l < LANES8; ++l) acc = std::fmax(acc, lanes[l]);
  return acc;
}

// ops.rs:44-50
void zero_centred_norm(const float* in, const float* gain, float* out, size_t n) {
  float ms = sum_of_squares(in, n) / (float)n;
  float inv = 1.0f / std::sqrt(ms + NORM_EPSILON);
  for (size_t i = 0; i < n; ++i) out[i] = (1.0f + gain[i]) * in[i] * inv;
}

// ops.rs:52-58
void zero_centred_norm_in_place(float* v, const float* gain, size_t n) {
  float ms = sum_of_squares(v, n) / (float)n;
  float inv = 1.0f / std::sqrt(ms + NORM_EPSILON);
  for (size_t i = 0; i < n; ++i) v[i] = (1.0f + gain[i]) * v[i] * inv;
}

// ops.rs:60-66
void unit_rms(const float* in, float* out, size_t n) {
  float ms = sum_of_squares(in, n) / (float)n;
  float inv = 1.0f / std::sqrt(ms + NORM_EPSILON);
  for (size_t i = 0; i < n; ++i) out[i] = in[i] * inv;
}

// ops.rs:69-71 — f32::exp is the platform libm expf.
float sigmoid(float v) { return 1.0f / (1.0f + std::exp(-v)); }

// ops.rs:83-90
float fast_exp(float value) {
  float c = value;
  if (c < -87.0f) c = -87.0f;
  if (c > 87.0f) c = 87.0f;
  float scaled = c * 1.44269504088896341f;
  float whole = std::round(scaled);
  float f = scaled - whole;
  float p = f * 0.0013333558f;
  p = 0.009618129f + p;
  p = f * p;
  p = 0.05550411f + p;
  p = f * p;
  p = 0.2402265f + p;
  p = f * p;
  p = 0.69314718055994531f + p;
  p = f * p;
  p = 1.0f + p;
  int32_t w = std::isnan(whole) ? 0 : (int32_t)whole;
  uint32_t bits = (uint32_t)((w + 127) << 23);
  float e;
  std::memcpy(&e, &bits, 4);
  return p * e;
}

// ops.rs:74-76
float silu(float v) { return v / (1.0f + fast_exp(-v)); }

// ops.rs:92-101
void softmax_in_place(float* v, size_t n) {
  float peak = -INFINITY;
  for (size_t i = 0; i < n; ++i) peak = std::fmax(peak, v[i]);
  float total = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    v[i] = fast_exp(v[i] - peak);
    total += v[i];
  }
  float inverse = 1.0f / total;
  for (size_t i = 0; i < n; ++i) v[i] *= inverse;
}

// ops.rs:103-110
float int8_scale(const float* v, size_t n) {
  float peak = peak_magnitude(v, n);
  return peak > 0.0f ? peak / 127.0f : 1.0f;
}

static inline float clampf(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }
// round_ties_even: nearbyint under the default round-to-nearest mode.
static inline float rne(float x) { return std::nearbyint(x); }

// ops.rs:112-118
float quantise_int8(const float* v, int8_t* codes, size_t n) {
  float scale = int8_scale(v, n);
  for (size_t i = 0; i < n; ++i) codes[i] = (int8_t)clampf(rne(v[i] / scale), -128.0f, 127.0f);
  return scale;
}

// ops.rs:120-125
void fake_quantise_int8(float* v, size_t n) {
  float scale = int8_scale(v, n);
  for (size_t i = 0; i < n; ++i) v[i] = clampf(rne(v[i] / scale), -128.0f, 127.0f) * scale;
}

// ops.rs:127-129
std::vector<float> rotary_frequencies(size_t head_dim, float theta) {
  std::vector<float> f;
  for (size_t i = 0; i < head_dim / 2; ++i) f.push_back(1.0f / std::pow(theta, 2.0f * (float)i / (float)head_dim));
  return f;
}

// ops.rs:131-141 (sin_cos of an f32 angle: libm sinf and cosf)
void apply_rotary(float* head, size_t dim, size_t position, const float* freq) {
  size_t half = dim / 2;
  for (size_t i = 0; i < half; ++i) {
    float angle = (float)position * freq[i];
    float s = std::sin(angle), c = std::cos(angle);
    float a = head[i], b = head[half + i];
    head[i] = a * c - b * s;
    head[half + i] = b * c + a * s;
  }
}

// ops.rs:143-164
void kronecker_fixed32(const float* in, const float* left, size_t left_size, const float* right, float* out) {
  const size_t R = 32;
  std::vector<float> mixed(left_size * R);
  for (size_t i = 0; i < left_size; ++i) {
    float acc[32] = {0};
    for (size_t j = 0; j < R; ++j) {
      float value = in[i * R + j];
      for (size_t c = 0; c < R; ++c) acc[c] += value * right[j * R + c];
    }
    std::memcpy(&mixed[i * R], acc, sizeof acc);
  }
  for (size_t k = 0; k < left_size; ++k) {
    float acc[32] = {0};
    for (size_t i = 0; i < left_size; ++i) {
      float gain = left[i * left_size + k];
      for (size_t c = 0; c < R; ++c) acc[c] += gain * mixed[i * R + c];
    }
    std::memcpy(&out[k * R], acc, sizeof acc);
  }
}

// ops.rs:219-299 — the aarch64 32x32 path fuses every multiply-add.
void kronecker_neon32(const float* in, const float* left, const float* right, float* out) {
  const size_t S = 32;
  float mixed[32 * 32];
  for (size_t r = 0; r < S; ++r)
    for (size_t c = 0; c < S; ++c) {
      float acc = 0.0f;
      for (size_t j = 0; j < S; ++j) acc = std::fma(right[j * S + c], in[r * S + j], acc);
      mixed[r * S + c] = acc;
    }
  for (size_t k = 0; k < S; ++k)
    for (size_t c = 0; c < S; ++c) {
      float acc = 0.0f;
      for (size_t i = 0; i < S; ++i) acc = std::fma(mixed[i * S + c], left[i * S + k], acc);
      out[k * S + c] = acc;
    }
}

// ops.rs:166-196
void kronecker_apply(const float* in, const float* left, size_t ls, const float* right, size_t rs, float* out, int mode) {
  if (mode == NBO_MODE_INT && rs == 32 && ls == 32) return kronecker_neon32(in, left, right, out);
  if (rs == 32) return kronecker_fixed32(in, left, ls, right, out);
  std::vector<float> mixed(ls * rs, 0.0f);
  for (size_t i = 0; i < ls; ++i)
    for (size_t j = 0; j < rs; ++j) {
      float value = in[i * rs + j];
      for (size_t c = 0; c < rs; ++c) mixed[i * rs + c] += value * right[j * rs + c];
    }
  for (size_t i = 0; i < ls * rs; ++i) out[i] = 0.0f;
  for (size_t i = 0; i < ls; ++i)
    for (size_t k = 0; k < ls; ++k) {
      float gain = left[i * ls + k];
      for (size_t c = 0; c < rs; ++c) out[k * rs + c] += gain * mixed[i * rs + c];
    }
}

// ops.rs:198-217
void sinkhorn_in_place(float* x, size_t size, size_t iterations) {
  const float MIN_POSITIVE = 1.17549435e-38f;
  for (size_t r = 0; r < size; ++r) {
    float peak = -INFINITY;
    for (size_t c = 0; c < size; ++c) peak = std::fmax(peak, x[r * size + c]);
    for (size_t c = 0; c < size; ++c) x[r * size + c] = std::exp(x[r * size + c] - peak);
  }
  for (size_t it = 0; it < iterations; ++it) {
    for (size_t r = 0; r < size; ++r) {
      float total = RUST_SUM_START;
      for (size_t c = 0; c < size; ++c) total += x[r * size + c];
      float inverse = 1.0f / std::fmax(total, MIN_POSITIVE);
      for (size_t c = 0; c < size; ++c) x[r * size + c] *= inverse;
    }
    for (size_t c = 0; c < size; ++c) {
      float total = RUST_SUM_START;
      for (size_t r = 0; r < size; ++r) total += x[r * size + c];
      float inverse = 1.0f / std::fmax(total, MIN_POSITIVE);
      for (size_t r = 0; r < size; ++r) x[r * size + c] *= inverse;
    }
  }
}

// crates/kernels/src/codebook.rs:1-43 and matrix.rs:499-514
struct LevelTable {
  uint32_t bits = 0;  // index width of the lookup (ternary crumbs read as 2 bits)
  float levels[16] = {0};
};

LevelTable lookup_table(uint32_t record_bits, const std::vector<float>& cb, size_t group) {
  LevelTable t;
  auto copy = [&](size_t from, size_t n) {
    if (cb.size() < from + n) throw Failure(ERR_ARCHIVE, "codebook is shorter than 28 values");
    for (size_t i = 0; i < n; ++i) t.levels[i] = cb[from + i];
  };
  switch (record_bits) {
    case 1: {
      float level = std::sqrt(2.0f / 3.14159265358979323846f) / std::sqrt((float)group);
      t.bits = 1;
      t.levels[0] = -level;
      t.levels[1] = level;
      break;
    }
    case 2: t.bits = 2; copy(0, 4); break;
    case 3: t.bits = 3; copy(4, 8); break;
    case 4: t.bits = 4; copy(12, 16); break;
    case 5: {
      float level = 1.2240064f / std::sqrt((float)group);
      t.bits = 2;
      t.levels[0] = 0.0f;
      t.levels[1] = level;
      t.levels[2] = 0.0f;
      t.levels[3] = -level;
      break;
    }
    default: throw Failure(ERR_UNSUPPORTED, "unsupported codebook width " + std::to_string(record_bits));
  }
  return t;
}

// crates/kernels/src/neon.rs:108-124
struct IntegerLevels {
  bool present = false;
  int8_t table[16] = {0};
  float scale = 1.0f;
};

IntegerLevels integer_levels(const LevelTable& t) {
  IntegerLevels il;
  if (t.bits != 2 && t.bits != 4) return il;
  size_t count = (size_t)1 << t.bits;
  float peak = 0.0f;
  for (size_t i = 0; i < count; ++i) peak = std::fmax(peak, std::fabs(t.levels[i]));
  il.scale = peak > 0.0f ? peak / 127.0f : 1.0f;
  for (size_t i = 0; i < count; ++i) il.table[i] = (int8_t)std::round(t.levels[i] / il.scale);
  il.present = true;
  return il;
}

// Per-group int8 activation: neon.rs:22-46 (vrndnq ties-to-even, clamp ±127),
// panel.rs:46-65 (NaturalInput::new), neon.rs:58-105 (PlaneInput).
struct GroupInput {
  std::vector<int8_t> codes;
  std::vector<float> scales;
};

GroupInput quantise_groups(const float* rotated, size_t columns, size_t group) {
  GroupInput in;
  size_t groups = columns / group;
  in.codes.resize(columns);
  in.scales.resize(groups);
  for (size_t g = 0; g < groups; ++g) {
    const float* s = rotated + g * group;
    float peak = peak_magnitude(s, group);
    float scale = peak > 0.0f ? peak / 127.0f : 1.0f;
    in.scales[g] = scale;
    for (size_t i = 0; i < group; ++i) in.codes[g * group + i] = (int8_t)clampf(rne(s[i] / scale), -127.0f, 127.0f);
  }
  return in;
}

// crates/kernels/src/matrix.rs:18-441
struct QMatrix {
  const uint8_t* packed = nullptr;
  size_t rows = 0, columns = 0, padded = 0, group = 0, row_bytes = 0, groups = 0;
  uint32_t record_bits = 0;
  LevelTable table;
  IntegerLevels ilevels;
  std::vector<float> norms;

  // matrix.rs:113-121: panels exist for 2-bit records whose group is a multiple of 16.
  bool panel() const { return ilevels.present && record_bits == 2 && group % 16 == 0; }
  // neon.rs:13-19
  bool plane() const {
    if (!ilevels.present) return false;
    return (table.bits == 2 && group % 64 == 0) || (table.bits == 4 && group % 32 == 0);
  }
  bool integer_path(int mode) const { return mode == NBO_MODE_INT && (panel() || plane()); }

  const uint8_t* row_packed(size_t row) const { return packed + row * row_bytes; }

  // matrix.rs:622-631
  uint32_t index_at(const uint8_t* p, size_t index) const {
    size_t bit = index * table.bits, byte = bit / 8, shift = bit % 8;
    uint32_t mask = (1u << table.bits) - 1;
    uint32_t raw = shift + table.bits > 8 ? (((uint32_t)p[byte]) | ((uint32_t)p[byte + 1] << 8)) >> shift : ((uint32_t)p[byte]) >> shift;
    return raw & mask;
  }
  float value(const uint8_t* p, size_t index) const { return table.levels[index_at(p, index)]; }

  // matrix.rs:123-128
  std::vector<float> prepare(const float* input) const {
    std::vector<float> r(padded, 0.0f);
    std::memcpy(r.data(), input, columns * sizeof(float));
    rotate_groups(r.data(), padded, group);
    return r;
  }

  // matrix.rs:140-153
  std::vector<float> dequantise_row(size_t row) const {
    std::vector<float> out(padded, 0.0f);
    const uint8_t* p = row_packed(row);
    for (size_t g = 0; g < groups; ++g) {
      float norm = norms[row * groups + g];
      for (size_t i = 0; i < group; ++i) out[g * group + i] = value(p, g * group + i) * norm;
      transform_in_place(&out[g * group], group);
    }
    out.resize(columns);
    return out;
  }

  int32_t group_sum(size_t row, size_t g, const int8_t* codes) const {
    const uint8_t* p = row_packed(row);
    int32_t acc = 0;
    for (size_t i = 0; i < group; ++i) acc += (int32_t)ilevels.table[index_at(p, g * group + i)] * (int32_t)codes[g * group + i];
    return acc;
  }

  // INT mode, one row. Panels (panel.rs:153-197): fma(f32(acc), (norm*level_scale)*act_scale, total).
  // Planes (neon.rs:138-183): total += f32(acc) * norm * level_scale * act_scale.
  float row_integer(size_t row, const GroupInput& in, int32_t* sums) const {
    float total = 0.0f;
    bool fused = panel();
    for (size_t g = 0; g < groups; ++g) {
      int32_t acc = group_sum(row, g, in.codes.data());
      if (sums) sums[g] = acc;
      float norm = norms[row * groups + g];
      if (fused) {
        float scaled = (norm * ilevels.scale) * in.scales[g];
        total = std::fma((float)acc, scaled, total);
      } else {
        total += (float)acc * norm * ilevels.scale * in.scales[g];
      }
    }
    return total;
  }

  // FLOAT mode, one row: matrix.rs:427-440 with the byte tables of 524-552/610-620.
  float row_float(size_t row, const float* rotated) const {
    const uint8_t* p = row_packed(row);
    float total = 0.0f;
    size_t per_byte = table.bits == 1 ? 8 : table.bits == 2 ? 4 : table.bits == 4 ? 2 : 0;
    uint32_t mask = (1u << table.bits) - 1;
    for (size_t g = 0; g < groups; ++g) {
      const float* in = rotated + g * group;
      float partial = RUST_SUM_START;
      if (per_byte) {
        float lanes[8] = {0};
        size_t nbytes = group / per_byte;
        const uint8_t* bytes = p + g * nbytes;
        for (size_t j = 0; j < nbytes; ++j)
          for (size_t l = 0; l < per_byte; ++l) lanes[l] += table.levels[(bytes[j] >> (l * table.bits)) & mask] * in[j * per_byte + l];
        for (size_t l = 0; l < per_byte; ++l) partial += lanes[l];
      } else {
        for (size_t i = 0; i < group; ++i) partial += value(p, g * group + i) * in[i];
      }
      total += partial * norms[row * groups + g];
    }
    return total;
  }

  // matrix.rs:391-399 + 489-497 (the non-aarch64 multiply_batch inner loop)
  void expand_row_scaled(size_t row, float* out) const {
    const uint8_t* p = row_packed(row);
    for (size_t g = 0; g < groups; ++g) {
      float norm = norms[row * groups + g];
      for (size_t i = 0; i < group; ++i) out[g * group + i] = value(p, g * group + i) * norm;
    }
  }
};

static inline float dot8(const float* a, const float* b, size_t n) {
  float lanes[8] = {0};
  for (size_t c = 0; c + 8 <= n; c += 8)
    for (size_t l = 0; l < 8; ++l) lanes[l] += a[c + l] * b[c + l];
  float s = RUST_SUM_START;
  for (size_t l = 0; l < 8; ++l) s += lanes[l];
  return s;
}

QMatrix load_matrix(const Archive& a, size_t index) {
  const Record& r = a.records[index];
  if (r.kind != CODEBOOK) throw Failure(ERR_ARCHIVE, "tensor " + std::to_string(index) + " is not codebook-quantised");
  QMatrix m;
  m.packed = a.data(index);
  m.rows = r.rows();
  m.columns = r.columns();
  m.padded = r.padded_columns();
  m.group = r.group();
  m.record_bits = r.bits;
  m.row_bytes = r.packed_row_bytes();
  m.groups = r.groups_per_row();
  m.table = lookup_table(r.bits, a.codebook, r.group_size);
  m.ilevels = integer_levels(m.table);
  size_t packed = r.packed_bytes();
  if (packed + m.rows * m.groups * 2 > r.byte_len) throw Failure(ERR_ARCHIVE, "codebook tensor " + std::to_string(index) + " is shorter than its shape");
  const uint16_t* h = reinterpret_cast<const uint16_t*>(m.packed + packed);
  m.norms.resize(m.rows * m.groups);
  for (size_t i = 0; i < m.norms.size(); ++i) m.norms[i] = half_to_f32(h[i]);
  return m;
}

// --------------------------------------------------------------- model crate

struct Hadamard {
  size_t size = 0, rank = 0;
  std::vector<float> d1, d2, b2, d3, d4, cond_v, cond_u;
  std::vector<float> left[3], right[3];
  size_t left_size[3]{}, right_size[3]{};
  const std::vector<size_t>* perm1 = nullptr;
  const std::vector<size_t>* perm2 = nullptr;
};

struct LayerW {
  std::vector<float> norm_in, post_norm, pre_hada, q_norm, k_norm;
  float attention_gate = 0.0f;
  QMatrix q, k, v, gate, out;
  std::vector<float> taps[3];  // q, k, v causal convolution gains [tap][width]; empty without taps
  Hadamard hada;
};

struct LanesW {
  size_t lanes = 0;
  std::vector<float> a_pre, a_post, a_res, b_pre, b_post, b_res;
  QMatrix phi_pre, phi_post, phi_res;
};

// model/src/engram.rs:12-28
struct EngramW {
  QMatrix tables, key_proj, value_proj;
  std::vector<float> taps;  // [conv_taps][d]
};

// model/src/heads.rs:6-18, loaded for every row (the embedding cell and one
// cell per layer); a depth selects rows (ProbeHead::with_rows, heads.rs:52-78).
struct ProbeHeadW {
  uint8_t code = 0;
  size_t rows = 0, ppl = 0, queries = 0, width = 0;
  std::vector<float> probes, gain, query, row_bias, bias;  // probes [rows][ppl][width], query [queries][width]
  QMatrix projection;
};

// whistle/src/cross.rs:8-19
struct CrossLayerW {
  std::vector<float> norm, q_norm, k_norm, post_norm;
  QMatrix q, k, v, gate, out;
  float gate_scalar = 0.0f;
};

struct Weights {
  QMatrix embedding;
  std::vector<LayerW> layers;
  std::vector<CrossLayerW> cross;  // a Whistle archive's cross attention, per decoder layer
  float position_gate = 0.0f;
  size_t text_vocab = 0;
  LanesW lanes;
  std::vector<EngramW> engrams;  // one per engram site
  std::vector<ProbeHeadW> heads;
  std::vector<float> final_norm;
  std::vector<size_t> perm1, perm2;
};

}  // namespace nbo

struct nbo_model {
  std::shared_ptr<nbo::Archive> archive;
  nbo::Layout layout;
  std::shared_ptr<nbo::Weights> weights;
  std::vector<size_t> active;
  int mode = NBO_MODE_INT;
  int threads = 1;
};

namespace nbo {

// crates/model/src/ladder.rs:1-29
std::vector<int32_t> ladder_order(int layers) {
  std::vector<int32_t> order;
  if (layers <= 1) {
    for (int i = 0; i < layers; ++i) order.push_back(i);
    return order;
  }
  std::vector<int32_t> selected{0, layers - 1};
  order = selected;
  while ((int)order.size() < layers) {
    std::sort(selected.begin(), selected.end());
    int best_gap = -1, best_left = 0, best_right = 0;
    for (size_t i = 0; i + 1 < selected.size(); ++i) {
      int gap = selected[i + 1] - selected[i];
      if (gap <= 1) continue;
      // max_by_key((gap, Reverse(left))): widest gap, the leftmost among equals.
      if (gap > best_gap || (gap == best_gap && selected[i] < best_left)) {
        best_gap = gap;
        best_left = selected[i];
        best_right = selected[i + 1];
      }
    }
    int candidate = (best_left + best_right) / 2;
    selected.push_back(candidate);
    order.push_back(candidate);
  }
  return order;
}

bool ladder_select(int layers, int depth, std::vector<int32_t>& out) {
  if (depth < std::min(2, layers) || depth > layers) return false;
  auto order = ladder_order(layers);
  out.assign(order.begin(), order.begin() + depth);
  std::sort(out.begin(), out.end());
  return true;
}

// hadamard.rs:228-258
Hadamard load_hadamard(const Archive& a, const HadamardT& t, const std::vector<size_t>* p1, const std::vector<size_t>* p2, size_t size) {
  Hadamard h;
  h.size = size;
  h.d1 = floats(a, t.d1);
  h.d2 = floats(a, t.d2);
  h.b2 = floats(a, t.b2);
  h.d3 = floats(a, t.d3);
  h.d4 = floats(a, t.d4);
  h.cond_v = floats(a, t.cond_v);
  h.cond_u = floats(a, t.cond_u);
  h.rank = h.cond_u.size() / size;
  size_t lr[3][2] = {{t.w1a, t.w1b}, {t.w2a, t.w2b}, {t.w3a, t.w3b}};
  for (int i = 0; i < 3; ++i) {
    h.left[i] = floats(a, lr[i][0]);
    h.right[i] = floats(a, lr[i][1]);
    h.left_size[i] = (size_t)std::llround(std::sqrt((double)h.left[i].size()));
    h.right_size[i] = (size_t)std::llround(std::sqrt((double)h.right[i].size()));
  }
  h.perm1 = p1;
  h.perm2 = p2;
  return h;
}

// hadamard.rs:260-311
std::vector<float> hadamard_apply(const Hadamard& h, const float* input, size_t width, int mode) {
  std::vector<float> weights(h.rank, 0.0f);
  if (h.rank == 8) {
    float chains[4][8] = {{0}};
    for (size_t g = 0; g * 4 < width && g * 32 < h.cond_v.size(); ++g) {
      for (size_t j = 0; j < 4 && g * 4 + j < width; ++j) {
        if (g * 32 + (j + 1) * 8 > h.cond_v.size()) break;
        float value = input[g * 4 + j];
        const float* row = &h.cond_v[g * 32 + j * 8];
        for (size_t r = 0; r < 8; ++r) chains[j][r] += value * row[r];
      }
    }
    for (int c = 0; c < 4; ++c)
      for (size_t r = 0; r < 8; ++r) weights[r] += chains[c][r];
  } else {
    for (size_t d = 0; d < width; ++d)
      for (size_t r = 0; r < h.rank; ++r) weights[r] += input[d] * h.cond_v[d * h.rank + r];
  }
  softmax_in_place(weights.data(), weights.size());
  std::vector<float> modulation(h.size, 1.0f);
  for (size_t r = 0; r < h.rank; ++r)
    for (size_t i = 0; i < h.size; ++i) modulation[i] += weights[r] * h.cond_u[r * h.size + i];
  std::vector<float> scaled(h.size, 0.0f), first(h.size), second(h.size), third(h.size), gathered(h.size);
  for (size_t i = 0; i < h.size; ++i) scaled[i] = (i < width ? input[i] : 0.0f) * h.d1[i];
  kronecker_apply(scaled.data(), h.left[0].data(), h.left_size[0], h.right[0].data(), h.right_size[0], first.data(), mode);
  for (size_t i = 0; i < h.size; ++i) gathered[i] = first[(*h.perm1)[i]];
  for (size_t i = 0; i < h.size; ++i) scaled[i] = silu(h.d2[i] * modulation[i] * gathered[i] + h.b2[i]);
  kronecker_apply(scaled.data(), h.left[1].data(), h.left_size[1], h.right[1].data(), h.right_size[1], second.data(), mode);
  for (size_t i = 0; i < h.size; ++i) scaled[i] = second[(*h.perm2)[i]] * h.d3[i];
  kronecker_apply(scaled.data(), h.left[2].data(), h.left_size[2], h.right[2].data(), h.right_size[2], third.data(), mode);
  std::vector<float> out(width);
  for (size_t i = 0; i < width; ++i) out[i] = third[i] * h.d4[i];
  return out;
}

std::shared_ptr<Weights> load_weights(const Archive& a, const Layout& L) {
  const Geometry& g = a.geo;
  if (!g.engram_sites.empty() && (g.engram_orders.empty() || g.engram_tables % g.engram_orders.size() != 0 || g.engram_slots == 0))
    throw Failure(ERR_ARCHIVE, "engram tables are not a multiple of the orders");
  if (!g.engram_sites.empty() && g.engram_conv_taps == 0) throw Failure(ERR_UNSUPPORTED, "engram sites without value taps");
  if (g.num_heads % std::max<size_t>(g.num_kv_heads, 1) != 0) throw Failure(ERR_ARCHIVE, "query heads are not a multiple of kv heads");
  auto w = std::make_shared<Weights>();
  auto perm = [&](size_t index) {
    std::vector<size_t> p;
    for (float v : floats(a, index)) p.push_back((size_t)v);
    for (size_t v : p)
      if (v >= g.hada_n) throw Failure(ERR_ARCHIVE, "hadamard permutation entry out of range");
    return p;
  };
  w->perm1 = perm(L.perms[0]);
  w->perm2 = perm(L.perms[1]);
  w->embedding = load_matrix(a, L.embedding);
  for (const LayerT& t : L.layers) {
    LayerW lw;
    lw.norm_in = floats(a, t.norm_in);
    lw.q = load_matrix(a, t.q);
    lw.k = load_matrix(a, t.k);
    lw.v = load_matrix(a, t.v);
    lw.gate = load_matrix(a, t.gate);
    lw.out = load_matrix(a, t.out);
    if (t.has_taps) {
      // model/src/attention.rs:30 (floats of the three tap tensors)
      const size_t widths[3] = {lw.q.rows, lw.k.rows, lw.v.rows};
      for (int i = 0; i < 3; ++i) {
        lw.taps[i] = floats(a, t.taps[i]);
        if (lw.taps[i].size() < g.qkv_conv_taps * widths[i]) throw Failure(ERR_ARCHIVE, "conv tap tensor is shorter than taps x width");
      }
    }
    lw.q_norm = floats(a, t.q_norm);
    lw.k_norm = floats(a, t.k_norm);
    lw.post_norm = floats(a, t.post_norm);
    lw.attention_gate = floats(a, t.attn_gate).at(0);
    lw.pre_hada = floats(a, t.pre_hada);
    lw.hada = load_hadamard(a, t.hada, &w->perm1, &w->perm2, g.hada_n);
    w->layers.push_back(std::move(lw));
  }
  LanesW& ln = w->lanes;
  ln.lanes = g.mhc_lanes;
  ln.a_pre = floats(a, L.lanes.a_pre);
  ln.a_post = floats(a, L.lanes.a_post);
  ln.a_res = floats(a, L.lanes.a_res);
  ln.b_pre = floats(a, L.lanes.b_pre);
  ln.b_post = floats(a, L.lanes.b_post);
  ln.b_res = floats(a, L.lanes.b_res);
  ln.phi_pre = load_matrix(a, L.lanes.phi_pre);
  ln.phi_post = load_matrix(a, L.lanes.phi_post);
  ln.phi_res = load_matrix(a, L.lanes.phi_res);
  for (const auto& e : L.engrams) {  // engram.rs:19-28
    EngramW ew;
    ew.tables = load_matrix(a, e[0]);
    ew.key_proj = load_matrix(a, e[1]);
    ew.value_proj = load_matrix(a, e[2]);
    ew.taps = floats(a, e[3]);
    if (ew.tables.rows < g.engram_tables * g.engram_slots || ew.tables.columns != g.engram_sub_dim ||
        ew.key_proj.columns != g.engram_tables * g.engram_sub_dim || ew.value_proj.columns != ew.key_proj.columns ||
        ew.key_proj.rows != g.d_model || ew.value_proj.rows != g.d_model || ew.taps.size() < g.engram_conv_taps * g.d_model)
      throw Failure(ERR_ARCHIVE, "engram tensors do not match the header");
    w->engrams.push_back(std::move(ew));
  }
  for (const Layout::HeadT& h : L.heads) {  // heads.rs:29-50
    ProbeHeadW hw;
    hw.code = h.code;
    QMatrix probes = load_matrix(a, h.probes), query = load_matrix(a, h.query);
    hw.rows = g.num_layers + 1;
    hw.width = probes.columns;
    hw.ppl = probes.rows / hw.rows;
    hw.queries = query.rows;
    for (size_t r = 0; r < probes.rows; ++r) {  // dense() (heads.rs:20-28)
      std::vector<float> row = probes.dequantise_row(r);
      hw.probes.insert(hw.probes.end(), row.begin(), row.end());
    }
    for (size_t r = 0; r < query.rows; ++r) {
      std::vector<float> row = query.dequantise_row(r);
      hw.query.insert(hw.query.end(), row.begin(), row.end());
    }
    hw.gain = floats(a, h.gain);
    hw.row_bias = floats(a, h.row_bias);
    hw.projection = load_matrix(a, h.proj);
    hw.bias = floats(a, h.bias);
    const size_t slots = hw.rows * hw.ppl;
    if (hw.ppl == 0 || hw.gain.size() < slots || hw.row_bias.size() < hw.queries * slots || query.columns != hw.width ||
        hw.projection.columns != hw.queries * hw.width || hw.bias.size() < hw.projection.rows)
      throw Failure(ERR_ARCHIVE, "probe head tensors do not match one another");
    w->heads.push_back(std::move(hw));
  }
  for (const auto& c : L.cross) {  // CrossWeights::load (cross.rs:38-56)
    CrossLayerW cw;
    cw.norm = floats(a, c[0]);
    cw.q = load_matrix(a, c[1]);
    cw.k = load_matrix(a, c[2]);
    cw.v = load_matrix(a, c[3]);
    cw.gate = load_matrix(a, c[4]);
    cw.out = load_matrix(a, c[5]);
    cw.q_norm = floats(a, c[6]);
    cw.k_norm = floats(a, c[7]);
    cw.post_norm = floats(a, c[8]);
    cw.gate_scalar = floats(a, c[9]).at(0);
    w->cross.push_back(std::move(cw));
  }
  if (L.audio) {
    w->position_gate = floats(a, L.position_gate).at(0);
    w->text_vocab = L.text_vocab;
  }
  w->final_norm = floats(a, L.final_norm);
  return w;
}

// A fork-join section over `tasks` items (the reference's spin pool, pool.rs:137-161).
template <typename F>
void fork(int threads, size_t tasks, bool parallel, F&& f) {
  if (!parallel || threads <= 1 || tasks <= 1 || omp_in_parallel()) {
    for (size_t i = 0; i < tasks; ++i) f(i);
    return;
  }
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
  for (size_t i = 0; i < tasks; ++i) f(i);
}

constexpr size_t ROWS_PER_TASK = 64;          // matrix.rs:10
constexpr size_t PARALLEL_VECTOR_ROWS = 512;  // matrix.rs:9
constexpr size_t PARALLEL_ROW_THRESHOLD = 256;  // matrix.rs:8
constexpr size_t PARALLEL_POSITIONS = 128;    // model/src/attention.rs:9

struct Job {
  const QMatrix* m;
  size_t first_row;
  float* out;
  size_t rows;
};

// matrix.rs:155-202 (multiply_vector, multiply_fused, multiply_rows) for one token.
void multiply_jobs(const std::vector<Job>& jobs, const float* rotated, int mode, int threads, bool fused_threshold = true) {
  // One shared integer input per (bits, group) format (matrix.rs:168-174).
  std::vector<std::pair<std::pair<uint32_t, size_t>, GroupInput>> shared;
  if (mode == NBO_MODE_INT)
    for (const Job& j : jobs)
      if (j.m->integer_path(mode)) {
        auto key = std::make_pair(j.m->record_bits, j.m->group);
        bool known = false;
        for (auto& s : shared) known |= s.first == key;
        if (!known) shared.push_back({key, quantise_groups(rotated, j.m->padded, j.m->group)});
      }
  struct Task { const Job* job; size_t first; size_t count; const GroupInput* in; };
  std::vector<Task> tasks;
  size_t total_rows = 0;
  for (const Job& j : jobs) {
    const GroupInput* in = nullptr;
    for (auto& s : shared)
      if (s.first == std::make_pair(j.m->record_bits, j.m->group)) in = &s.second;
    for (size_t r = 0; r < j.rows; r += ROWS_PER_TASK) tasks.push_back({&j, r, std::min(ROWS_PER_TASK, j.rows - r), in});
    total_rows += j.rows;
  }
  bool parallel = fused_threshold && total_rows >= PARALLEL_VECTOR_ROWS;
  fork(threads, tasks.size(), parallel, [&](size_t t) {
    const Task& task = tasks[t];
    for (size_t i = 0; i < task.count; ++i) {
      size_t row = task.job->first_row + task.first + i;
      task.job->out[task.first + i] = task.in ? task.job->m->row_integer(row, *task.in, nullptr) : task.job->m->row_float(row, rotated);
    }
  });
}

// matrix.rs:330-389, the non-aarch64 batched product (FLOAT-mode prefill).
void multiply_batch_float(const QMatrix& m, const float* rotated, size_t count, float* output, int threads) {
  size_t width = m.padded;
  std::vector<float> transposed(m.rows * count);
  size_t chunks = (m.rows + ROWS_PER_TASK - 1) / ROWS_PER_TASK;
  fork(threads, chunks, m.rows >= PARALLEL_ROW_THRESHOLD, [&](size_t chunk) {
    size_t first = chunk * ROWS_PER_TASK, tile_rows = std::min(ROWS_PER_TASK, m.rows - first);
    std::vector<float> tile(8 * width);
    for (size_t done = 0; done < tile_rows; done += 8) {
      size_t take = std::min<size_t>(8, tile_rows - done);
      for (size_t o = 0; o < take; ++o) m.expand_row_scaled(first + done + o, &tile[o * width]);
      for (size_t t = 0; t < count; ++t)
        for (size_t o = 0; o < take; ++o) transposed[(first + done + o) * count + t] = dot8(&tile[o * width], rotated + t * width, width);
    }
  });
  for (size_t t = 0; t < count; ++t)
    for (size_t r = 0; r < m.rows; ++r) output[t * m.rows + r] = transposed[r * count + t];
}

struct Cache {
  std::vector<int8_t> keys, values;               // [position][kv][dim]
  std::vector<std::vector<float>> key_scales, value_scales;  // [kv][position]
  std::deque<std::vector<float>> raw_history[3];  // q, k, v projections before the taps, newest first
};

// model/src/attention.rs:83-93 (mix_taps): Σ over tap < min(taps, position + 1)
// of gain[tap] · history[tap], from +0.0, one multiply and one add per term.
void mix_taps(const std::vector<float>& gains, const std::deque<std::vector<float>>& history, size_t taps, size_t position,
              float* out, size_t width) {
  for (size_t i = 0; i < width; ++i) out[i] = 0.0f;
  for (size_t tap = 0; tap < std::min(taps, position + 1); ++tap) {
    const float* g = &gains[tap * width];
    const std::vector<float>& sample = history.at(tap);
    for (size_t i = 0; i < width; ++i) out[i] += g[i] * sample[i];
  }
}

// crates/kernels/src/attention.rs:251-280 for one head over positions [first, total).
void attend_head(const int8_t* query, float query_scale, const Cache& cache, size_t kv, size_t kv_heads, size_t qk, size_t vd,
                 size_t first, size_t total, int mode, float* out) {
  size_t count = total - first;
  std::vector<int32_t> scores(count);
  for (size_t p = 0; p < count; ++p) {
    const int8_t* key = &cache.keys[((first + p) * kv_heads + kv) * qk];
    int32_t s = 0;
    for (size_t i = 0; i < qk; ++i) s += (int32_t)query[i] * (int32_t)key[i];
    scores[p] = s;
  }
  const float* key_scales = cache.key_scales[kv].data() + first;
  const float* value_scales = cache.value_scales[kv].data() + first;
  std::vector<float> coef(count);
  float total_weight;
  if (mode == NBO_MODE_INT) {
    // neon.rs:277-307: four-lane partial sums, then (l0+l1)+(l2+l3), then the tail.
    size_t vector_count = count - count % 4;
    float peak = -INFINITY;
    for (size_t i = 0; i < count; ++i) {
      coef[i] = (float)scores[i] * key_scales[i] * query_scale;
      peak = std::fmax(peak, coef[i]);
    }
    float lanes[4] = {0, 0, 0, 0};
    for (size_t i = 0; i < vector_count; ++i) {
      float e = fast_exp(coef[i] - peak);
      lanes[i % 4] += e;
      coef[i] = e * value_scales[i];
    }
    total_weight = (lanes[0] + lanes[1]) + (lanes[2] + lanes[3]);
    for (size_t i = vector_count; i < count; ++i) {
      float e = fast_exp(coef[i] - peak);
      total_weight += e;
      coef[i] = e * value_scales[i];
    }
  } else {
    float peak = -INFINITY;
    for (size_t i = 0; i < count; ++i) {
      coef[i] = (float)scores[i] * key_scales[i] * query_scale;
      peak = std::fmax(peak, coef[i]);
    }
    total_weight = 0.0f;
    for (size_t i = 0; i < count; ++i) {
      float e = fast_exp(coef[i] - peak);
      total_weight += e;
      coef[i] = e * value_scales[i];
    }
  }
  // Twelve-bit softmax weights, exact integer sums (attention.rs:294-328;
  // neon.rs:348-437 splits the same integers into two 6-bit halves).
  float peak = 0.0f;
  for (size_t i = 0; i < count; ++i) peak = std::fmax(peak, std::fabs(coef[i]));
  if (peak <= 0.0f) {
    for (size_t d = 0; d < vd; ++d) out[d] = 0.0f;
  } else {
    float scale = peak / COEFFICIENT_LEVELS;
    std::vector<int64_t> totals(vd, 0);
    for (size_t i = 0; i < count; ++i) {
      int32_t w = (int32_t)std::round(coef[i] / scale);
      if (w == 0) continue;
      const int8_t* v = &cache.values[((first + i) * kv_heads + kv) * vd];
      for (size_t d = 0; d < vd; ++d) totals[d] += (int64_t)w * v[d];
    }
    for (size_t d = 0; d < vd; ++d) out[d] = (float)totals[d] * scale;
  }
  float inverse = 1.0f / total_weight;
  for (size_t d = 0; d < vd; ++d) out[d] *= inverse;
}

struct Routing {
  std::vector<float> input, post, residual;
};

}  // namespace nbo

struct nbo_session {
  const nbo_model* model;
  std::vector<uint32_t> tokens;
  std::vector<nbo::Cache> caches;
  std::vector<std::deque<std::vector<float>>> engram_history;  // per site: raw values, newest first (engram.rs:45-48)
  struct Accumulator { std::vector<float> peak, total, weighted; };  // heads.rs:151-156
  std::vector<Accumulator> accumulators;                            // per probe head
  std::vector<float> frequencies;
  std::vector<float> hidden;
};

namespace nbo {

// crates/model/src/lanes.rs:146-181
Routing route(const nbo_model* M, size_t layer, size_t slot, const float* stream, size_t width) {
  const LanesW& L = M->weights->lanes;
  size_t lanes = L.lanes;
  std::vector<float> normalised(lanes * width);
  unit_rms(stream, normalised.data(), lanes * width);
  fake_quantise_int8(normalised.data(), normalised.size());
  std::vector<float> rotated = L.phi_pre.prepare(normalised.data());
  Routing r;
  std::vector<float> pre(lanes), post(lanes), residual(lanes * lanes);
  std::vector<Job> jobs{{&L.phi_pre, layer * lanes, pre.data(), lanes},
                        {&L.phi_post, layer * lanes, post.data(), lanes},
                        {&L.phi_res, layer * lanes * lanes, residual.data(), lanes * lanes}};
  multiply_jobs(jobs, rotated.data(), M->mode, M->threads);
  size_t own = slot % lanes;
  r.input.assign(width, 0.0f);
  for (size_t lane = 0; lane < lanes; ++lane) {
    float pre_offset = lane == own ? 8.0f + -4.0f : -4.0f;
    float gate = sigmoid(L.a_pre[layer] * pre[lane] + L.b_pre[layer * lanes + lane] + pre_offset);
    for (size_t i = 0; i < width; ++i) r.input[i] += gate * stream[lane * width + i];
    float post_offset = lane == own ? 0.0f : -4.0f;
    post[lane] = 2.0f * sigmoid(L.a_post[layer] * post[lane] + L.b_post[layer * lanes + lane] + post_offset);
  }
  size_t base = layer * lanes * lanes;
  for (size_t i = 0; i < residual.size(); ++i) residual[i] = L.a_res[layer] * residual[i] + L.b_res[base + i];
  sinkhorn_in_place(residual.data(), lanes, 20);
  r.post = post;
  r.residual = residual;
  return r;
}

// lanes.rs:183-204 and session.rs:192-200
void combine_into(const Routing& r, const float* stream, const float* delta, size_t width, size_t lanes, float* next) {
  for (size_t lane = 0; lane < lanes; ++lane) {
    float* out = next + lane * width;
    for (size_t i = 0; i < width; ++i) out[i] = 0.0f;
    for (size_t s = 0; s < lanes; ++s) {
      float w = r.residual[lane * lanes + s];
      for (size_t i = 0; i < width; ++i) out[i] += w * stream[s * width + i];
    }
    for (size_t i = 0; i < width; ++i) out[i] += r.post[lane] * delta[i];
  }
}

std::vector<float> lane_mean(const float* stream, size_t width, size_t lanes) {
  std::vector<float> mean(width, 0.0f);
  for (size_t l = 0; l < lanes; ++l)
    for (size_t i = 0; i < width; ++i) mean[i] += stream[l * width + i] / (float)lanes;
  return mean;
}

// After the fused projections: per-head norm, rotary and int8 codes, and the cache
// append (model/src/attention.rs:118-143). Returns query codes and scales.
void heads_and_cache(const nbo_model* M, const LayerW& W, Cache& cache, const float* freq, size_t position, float* q, float* k,
                     const float* v, std::vector<int8_t>& qcodes, std::vector<float>& qscales) {
  const Geometry& g = M->archive->geo;
  size_t qk = g.qk_head_dim, vd = g.v_head_dim, H = g.num_heads, KV = g.num_kv_heads;
  qcodes.assign(H * qk, 0);
  qscales.resize(H);
  for (size_t h = 0; h < H; ++h) {
    zero_centred_norm_in_place(q + h * qk, W.q_norm.data(), qk);
    apply_rotary(q + h * qk, qk, position, freq);
    qscales[h] = quantise_int8(q + h * qk, &qcodes[h * qk], qk);
  }
  for (size_t h = 0; h < KV; ++h) {
    zero_centred_norm_in_place(k + h * qk, W.k_norm.data(), qk);
    apply_rotary(k + h * qk, qk, position, freq);
  }
  cache.key_scales.resize(KV);
  cache.value_scales.resize(KV);
  for (size_t h = 0; h < KV; ++h) {
    std::vector<int8_t> codes(qk);
    float s = quantise_int8(k + h * qk, codes.data(), qk);
    cache.keys.insert(cache.keys.end(), codes.begin(), codes.end());
    cache.key_scales[h].push_back(s);
  }
  for (size_t h = 0; h < KV; ++h) {
    std::vector<int8_t> codes(vd);
    float s = quantise_int8(v + h * vd, codes.data(), vd);
    cache.values.insert(cache.values.end(), codes.begin(), codes.end());
    cache.value_scales[h].push_back(s);
  }
}

// model/src/attention.rs:156-213 for one token
std::vector<float> attend_heads(const nbo_model* M, size_t layer, const Cache& cache, size_t position, const std::vector<int8_t>& qcodes,
                                const std::vector<float>& qscales, bool parallel) {
  const Geometry& g = M->archive->geo;
  size_t qk = g.qk_head_dim, vd = g.v_head_dim, H = g.num_heads, KV = g.num_kv_heads;
  size_t total = position + 1;
  size_t first = (g.sliding_window > 0 && !g.is_global_layer(layer)) ? (total > g.sliding_window ? total - g.sliding_window : 0) : 0;
  size_t group = H / KV;
  float inverse_root = 1.0f / std::sqrt((float)qk);
  std::vector<float> out(H * vd);
  fork(M->threads, H, parallel && total - first >= PARALLEL_POSITIONS, [&](size_t h) {
    attend_head(&qcodes[h * qk], qscales[h] * inverse_root, cache, h / group, KV, qk, vd, first, total, M->mode, &out[h * vd]);
  });
  return out;
}

// model/src/attention.rs:96-154
std::vector<float> attend(const nbo_model* M, const LayerW& W, size_t layer, Cache& cache, const float* freq, size_t position, const float* hidden) {
  const Geometry& g = M->archive->geo;
  size_t d = g.d_model;
  std::vector<float> quantised(hidden, hidden + d);
  fake_quantise_int8(quantised.data(), d);
  std::vector<float> rotated = W.q.prepare(quantised.data());
  std::vector<float> q(W.q.rows), k(W.k.rows), v(W.v.rows), gate(W.gate.rows);
  std::vector<Job> jobs{{&W.q, 0, q.data(), W.q.rows}, {&W.k, 0, k.data(), W.k.rows}, {&W.v, 0, v.data(), W.v.rows}, {&W.gate, 0, gate.data(), W.gate.rows}};
  multiply_jobs(jobs, rotated.data(), M->mode, M->threads);
  if (!W.taps[0].empty()) {
    // attention.rs:105-111: the raw rows join the history, then each is mixed
    size_t taps = g.qkv_conv_taps;
    std::vector<float>* rows[3] = {&q, &k, &v};
    for (int i = 0; i < 3; ++i) {
      cache.raw_history[i].push_front(*rows[i]);
      while (cache.raw_history[i].size() > taps) cache.raw_history[i].pop_back();
    }
    for (int i = 0; i < 3; ++i) mix_taps(W.taps[i], cache.raw_history[i], taps, position, rows[i]->data(), rows[i]->size());
  }
  std::vector<int8_t> qcodes;
  std::vector<float> qscales;
  heads_and_cache(M, W, cache, freq, position, q.data(), k.data(), v.data(), qcodes, qscales);
  std::vector<float> attended = attend_heads(M, layer, cache, position, qcodes, qscales, true);
  for (size_t i = 0; i < attended.size(); ++i) attended[i] *= sigmoid(gate[i]);
  fake_quantise_int8(attended.data(), attended.size());
  std::vector<float> rot_out = W.out.prepare(attended.data());
  std::vector<float> output(W.out.rows);
  std::vector<Job> oj{{&W.out, 0, output.data(), W.out.rows}};
  multiply_jobs(oj, rot_out.data(), M->mode, M->threads);
  return output;
}

// The post-attention half of a block (session.rs:121-137): post norm, gated
// residual, Hadamard MLP, lane delta and lane combine.
struct CrossMemory;
void cross_apply(const nbo_model* M, const CrossMemory& mem, size_t layer, float* x);

void finish_block(const nbo_model* M, const LayerW& W, const Routing& r, std::vector<float>& x, std::vector<float>& attended,
                  const float* stream, float* next, const CrossMemory* cross = nullptr, size_t layer = 0) {
  const Geometry& g = M->archive->geo;
  size_t d = g.d_model, lanes = g.mhc_lanes;
  zero_centred_norm_in_place(attended.data(), W.post_norm.data(), d);
  float gate = sigmoid(W.attention_gate);
  for (size_t i = 0; i < d; ++i) x[i] += gate * attended[i];
  if (cross) cross_apply(M, *cross, layer, x.data());  // session.rs:126-128
  std::vector<float> pre(d);
  zero_centred_norm(x.data(), W.pre_hada.data(), pre.data(), d);
  std::vector<float> mlp = hadamard_apply(W.hada, pre.data(), d, M->mode);
  for (size_t i = 0; i < d; ++i) x[i] += mlp[i];
  std::vector<float> delta(d);
  for (size_t i = 0; i < d; ++i) delta[i] = x[i] - r.input[i];
  combine_into(r, stream, delta.data(), d, lanes, next);
}

// ---------------------------------------------------------------- engram sites
// engram.rs:30-46: per (order, head) table a multiplicative hash of the last
// `order` token ids (0 before the start), xor-shifted, modulo the slots.
std::vector<size_t> table_indices(const Geometry& g, const std::vector<uint32_t>& tokens, size_t position) {
  const uint32_t HASH_SEED = 0x9E3779B9u, HASH_PRIME = 0x01000193u;
  const size_t hpo = g.engram_tables / g.engram_orders.size();
  const size_t stride = g.engram_seed_heads == 0 ? hpo : g.engram_seed_heads;
  std::vector<size_t> out;
  for (size_t oi = 0; oi < g.engram_orders.size(); ++oi)
    for (size_t head = 0; head < hpo; ++head) {
      uint32_t acc = HASH_SEED * (uint32_t)(oi * stride + head + 1);
      for (size_t back = 0; back < g.engram_orders[oi]; ++back) {
        uint32_t token = position >= back ? tokens[position - back] : 0u;
        acc = (acc ^ token) * HASH_PRIME;
      }
      acc ^= acc >> 15;
      out.push_back(acc % (uint32_t)g.engram_slots);
    }
  return out;
}

// engram.rs:72-83: table t's row, or zeros while the position is shorter
// than the table's order, concatenated and fake-quantised.
std::vector<float> engram_gather(const nbo_model* M, const EngramW& E, const std::vector<size_t>& idx, size_t position) {
  const Geometry& g = M->archive->geo;
  const size_t sub = g.engram_sub_dim, hpo = g.engram_tables / g.engram_orders.size();
  std::vector<float> gathered(g.engram_tables * sub, 0.0f);
  for (size_t t = 0; t < g.engram_tables; ++t)
    if (position + 1 >= g.engram_orders[t / hpo]) {
      std::vector<float> row = E.tables.dequantise_row(t * g.engram_slots + idx[t]);
      std::copy(row.begin(), row.end(), gathered.begin() + t * sub);
    }
  fake_quantise_int8(gathered.data(), gathered.size());
  return gathered;
}

// Σ over taps whose reach (tap · dilation) the position covers of
// gain[tap] · raw[position - tap · dilation], from +0.0 (engram.rs:92-103).
template <typename Source>
void engram_conv(const Geometry& g, const EngramW& E, size_t position, size_t width, Source&& raw_at, float* value) {
  for (size_t i = 0; i < width; ++i) value[i] = 0.0f;
  for (size_t tap = 0; tap < g.engram_conv_taps; ++tap) {
    size_t back = tap * g.engram_conv_dilation;
    if (position < back) continue;
    const float* past = raw_at(back);
    const float* gn = &E.taps[tap * width];
    for (size_t i = 0; i < width; ++i) value[i] += gn[i] * past[i];
  }
}

size_t engram_keep(const Geometry& g) { return (g.engram_conv_taps - 1) * g.engram_conv_dilation + 1; }

// EngramSiteState::contribute (engram.rs:68-105) for one token.
void engram_contribute(const nbo_model* M, size_t site, std::deque<std::vector<float>>& history, const std::vector<size_t>& idx,
                       size_t position, std::vector<float>& key, std::vector<float>& value) {
  const Geometry& g = M->archive->geo;
  const EngramW& E = M->weights->engrams[site];
  std::vector<float> gathered = engram_gather(M, E, idx, position);
  std::vector<float> rotated = E.key_proj.prepare(gathered.data());
  key.assign(E.key_proj.rows, 0.0f);
  std::vector<float> raw(E.value_proj.rows, 0.0f);
  std::vector<Job> jobs{{&E.key_proj, 0, key.data(), E.key_proj.rows}, {&E.value_proj, 0, raw.data(), E.value_proj.rows}};
  multiply_jobs(jobs, rotated.data(), M->mode, M->threads);
  const size_t width = raw.size();
  history.push_front(raw);
  while (history.size() > engram_keep(g)) history.pop_back();
  value.assign(width, 0.0f);
  engram_conv(g, E, position, width, [&](size_t back) { return history.at(back).data(); }, value.data());
}

// session.rs:180-190
void add_engram(float* x, const float* key, const float* value, size_t width) {
  std::vector<float> ux(width), uk(width);
  unit_rms(x, ux.data(), width);
  unit_rms(key, uk.data(), width);
  float dot = -0.0f;  // Iterator::sum
  for (size_t i = 0; i < width; ++i) dot += ux[i] * uk[i];
  float alpha = sigmoid(dot / std::sqrt((float)width));
  for (size_t i = 0; i < width; ++i) x[i] += alpha * value[i];
}

// ModelConfig::engram_site_at (config.rs:87-89): the first site on the layer.
int engram_site_at(const Geometry& g, size_t layer) {
  for (size_t i = 0; i < g.engram_sites.size(); ++i)
    if (g.engram_sites[i] == layer) return (int)i;
  return -1;
}

bool layer_active(const nbo_model* M, size_t layer) { return std::find(M->active.begin(), M->active.end(), layer) != M->active.end(); }

// ---------------------------------------------------------------- probe heads
// The head's rows for this model: the embedding cell and one per active layer
// (model.rs:69-70).
std::vector<size_t> head_rows(const nbo_model* M) {
  std::vector<size_t> rows{0};
  for (size_t l : M->active) rows.push_back(l + 1);
  return rows;
}

// ProbeHead::observe (heads.rs:127-148): per (cell, probe) an online softmax
// pool of the cells, weighted by exp(score - running peak).
void observe(const ProbeHeadW& h, const std::vector<size_t>& rows, nbo_session::Accumulator& acc, const std::vector<std::vector<float>>& cells) {
  const size_t width = h.width;
  const float root = std::sqrt((float)width);
  for (size_t c = 0; c < cells.size(); ++c)
    for (size_t k = 0; k < h.ppl; ++k) {
      const size_t slot = c * h.ppl + k;
      const float* direction = &h.probes[(rows[c] * h.ppl + k) * width];
      const float score = dot_product(cells[c].data(), direction, width) / root;
      const float peak = std::fmax(acc.peak[slot], score);
      const float rescale = acc.peak[slot] == -INFINITY ? 0.0f : std::exp(acc.peak[slot] - peak);
      const float weight = std::exp(score - peak);
      acc.total[slot] = acc.total[slot] * rescale + weight;
      float* target = &acc.weighted[slot * width];
      for (size_t i = 0; i < width; ++i) target[i] = target[i] * rescale + weight * cells[c][i];
      acc.peak[slot] = peak;
    }
}

// ProbeHead::pooled (heads.rs:85-115)
std::vector<float> pooled(const ProbeHeadW& h, const std::vector<size_t>& rows, const nbo_session::Accumulator& acc) {
  const size_t width = h.width, slots = rows.size() * h.ppl, all = h.rows * h.ppl;
  std::vector<float> readouts(slots * width), averaged(width);
  for (size_t slot = 0; slot < slots; ++slot) {
    const float inverse = 1.0f / acc.total[slot];
    for (size_t i = 0; i < width; ++i) averaged[i] = acc.weighted[slot * width + i] * inverse;
    unit_rms(averaged.data(), &readouts[slot * width], width);
    const float gain = h.gain[rows[slot / h.ppl] * h.ppl + slot % h.ppl];
    for (size_t i = 0; i < width; ++i) readouts[slot * width + i] *= gain;
  }
  const float root = std::sqrt((float)width);
  std::vector<float> out(h.queries * width, 0.0f), weights(slots);
  for (size_t q = 0; q < h.queries; ++q) {
    for (size_t slot = 0; slot < slots; ++slot)
      weights[slot] = dot_product(&readouts[slot * width], &h.query[q * width], width) / root +
                      h.row_bias[q * all + rows[slot / h.ppl] * h.ppl + slot % h.ppl];
    softmax_in_place(weights.data(), slots);
    for (size_t slot = 0; slot < slots; ++slot)
      for (size_t i = 0; i < width; ++i) out[q * width + i] += weights[slot] * readouts[slot * width + i];
  }
  return out;
}

// ProbeHead::project (heads.rs:117-125)
std::vector<float> project_head(const nbo_model* M, const ProbeHeadW& h, const std::vector<float>& pooled_values) {
  std::vector<float> rotated = h.projection.prepare(pooled_values.data());
  std::vector<float> out(h.projection.rows, 0.0f);
  std::vector<Job> jobs{{&h.projection, 0, out.data(), h.projection.rows}};
  multiply_jobs(jobs, rotated.data(), M->mode, M->threads);
  for (size_t i = 0; i < out.size(); ++i) out[i] += h.bias[i];
  return out;
}

// ---------------------------------------------------------- Whistle cross attention
// whistle/src/cross.rs:29-35: per decoder layer the int8 keys [frame][head][qk]
// with their scales [frame][head], and the values likewise.
struct CrossMemory {
  size_t frames = 0;
  std::vector<std::vector<int8_t>> keys, values;
  std::vector<std::vector<float>> key_scales, value_scales;
};

// CrossWeights::memory (cross.rs:58-99).
CrossMemory cross_memory(const nbo_model* M, const float* encoded, size_t frames) {
  const Geometry& g = M->archive->geo;
  const Weights& W = *M->weights;
  const size_t dim = g.d_model, half = dim / 2, qk = g.qk_head_dim, vd = g.v_head_dim, heads = dim / vd;
  const float gate = sigmoid(W.position_gate);
  const float rate = -std::log(10000.0f) / ((float)half - 1.0f);
  std::vector<float> memory(frames * dim);
  for (size_t t = 0; t < frames; ++t) {
    const float* row = encoded + t * dim;
    float* out = &memory[t * dim];
    for (size_t j = 0; j < half; ++j) {
      const float angle = (float)t * std::exp(rate * (float)j);
      out[j] = row[j] + gate * std::sin(angle);
      out[half + j] = row[half + j] + gate * std::cos(angle);
    }
    fake_quantise_int8(out, dim);
  }
  CrossMemory mem;
  mem.frames = frames;
  for (const CrossLayerW& layer : W.cross) {
    const size_t kr = layer.k.rows, vr = layer.v.rows;
    std::vector<float> k(frames * kr), v(frames * vr);
    if (M->mode == NBO_MODE_INT) {  // the integer batched product computes each row as the single-row one does
      for (size_t t = 0; t < frames; ++t) {
        std::vector<float> rotated = layer.k.prepare(&memory[t * dim]);
        std::vector<Job> jobs{{&layer.k, 0, &k[t * kr], kr}, {&layer.v, 0, &v[t * vr], vr}};
        multiply_jobs(jobs, rotated.data(), M->mode, M->threads);
      }
    } else {
      const size_t padded = layer.k.padded;
      std::vector<float> rotated(frames * padded);
      for (size_t t = 0; t < frames; ++t) {
        std::vector<float> r = layer.k.prepare(&memory[t * dim]);
        std::memcpy(&rotated[t * padded], r.data(), padded * sizeof(float));
      }
      multiply_batch_float(layer.k, rotated.data(), frames, k.data(), M->threads);
      multiply_batch_float(layer.v, rotated.data(), frames, v.data(), M->threads);
    }
    std::vector<int8_t> kc(k.size()), vc(v.size());
    std::vector<float> ks(frames * heads), vs(frames * heads);
    for (size_t i = 0; i < frames * heads; ++i) {
      zero_centred_norm_in_place(&k[i * qk], layer.k_norm.data(), qk);
      ks[i] = quantise_int8(&k[i * qk], &kc[i * qk], qk);
      vs[i] = quantise_int8(&v[i * vd], &vc[i * vd], vd);
    }
    mem.keys.push_back(std::move(kc));
    mem.key_scales.push_back(std::move(ks));
    mem.values.push_back(std::move(vc));
    mem.value_scales.push_back(std::move(vs));
  }
  return mem;
}

// CrossState::apply (cross.rs:121-182) on x after the layer's attention residual.
void cross_apply(const nbo_model* M, const CrossMemory& mem, size_t layer_index, float* x) {
  const Geometry& g = M->archive->geo;
  const CrossLayerW& layer = M->weights->cross.at(layer_index);
  const size_t dim = g.d_model, qk = g.qk_head_dim, vd = g.v_head_dim, heads = dim / vd, frames = mem.frames;
  std::vector<float> normed(dim);
  zero_centred_norm(x, layer.norm.data(), normed.data(), dim);
  fake_quantise_int8(normed.data(), dim);
  std::vector<float> rotated = layer.q.prepare(normed.data());
  std::vector<float> q(layer.q.rows), gate(layer.gate.rows);
  multiply_jobs({{&layer.q, 0, q.data(), layer.q.rows}}, rotated.data(), M->mode, M->threads);
  multiply_jobs({{&layer.gate, 0, gate.data(), layer.gate.rows}}, rotated.data(), M->mode, M->threads);
  const float inverse_root = 1.0f / std::sqrt((float)qk);
  std::vector<float> context(heads * vd, 0.0f), scores(frames);
  for (size_t head = 0; head < heads; ++head) {
    float* query = &q[head * qk];
    zero_centred_norm_in_place(query, layer.q_norm.data(), qk);
    std::vector<int8_t> codes(qk);
    const float query_scale = quantise_int8(query, codes.data(), qk) * inverse_root;
    for (size_t f = 0; f < frames; ++f) {
      const int8_t* key = &mem.keys[layer_index][(f * heads + head) * qk];
      int32_t dot = 0;
      for (size_t i = 0; i < qk; ++i) dot += (int32_t)codes[i] * (int32_t)key[i];
      scores[f] = (float)dot * mem.key_scales[layer_index][f * heads + head] * query_scale;
    }
    softmax_in_place(scores.data(), frames);
    float* out = &context[head * vd];
    for (size_t f = 0; f < frames; ++f) {
      const float scale = mem.value_scales[layer_index][f * heads + head] * scores[f];
      const int8_t* value = &mem.values[layer_index][(f * heads + head) * vd];
      for (size_t i = 0; i < vd; ++i) out[i] += scale * (float)value[i];
    }
  }
  for (size_t i = 0; i < context.size(); ++i) context[i] *= sigmoid(gate[i]);
  fake_quantise_int8(context.data(), context.size());
  std::vector<float> rotated_out = layer.out.prepare(context.data());
  std::vector<float> attended(layer.out.rows);
  multiply_jobs({{&layer.out, 0, attended.data(), layer.out.rows}}, rotated_out.data(), M->mode, M->threads);
  zero_centred_norm_in_place(attended.data(), layer.post_norm.data(), dim);
  const float gain = sigmoid(layer.gate_scalar);
  for (size_t i = 0; i < dim; ++i) x[i] += gain * attended[i];
}

std::vector<float> embed(const nbo_model* M, uint32_t token) {
  const Geometry& g = M->archive->geo;
  if (token >= M->weights->embedding.rows) throw Failure(ERR_ARGUMENT, "token id outside the embedding");
  std::vector<float> row = M->weights->embedding.dequantise_row(token);
  float scale = std::sqrt((float)g.d_model);
  std::vector<float> stream;
  for (size_t l = 0; l < g.mhc_lanes; ++l)
    for (float v : row) stream.push_back(v * scale);
  return stream;
}

// session.rs:76-148
void push(nbo_session* s, uint32_t token, float* trace, const CrossMemory* cross = nullptr) {
  const nbo_model* M = s->model;
  const Geometry& g = M->archive->geo;
  size_t d = g.d_model, lanes = g.mhc_lanes;
  size_t position = s->tokens.size();
  std::vector<float> stream = embed(M, token);
  s->tokens.push_back(token);
  // session.rs:93-102: every site on an active layer contributes
  const size_t sites = g.engram_sites.size();
  std::vector<std::vector<float>> ekey(sites), evalue(sites);
  if (sites) {
    std::vector<size_t> idx = table_indices(g, s->tokens, position);
    for (size_t i = 0; i < sites; ++i)
      if (layer_active(M, g.engram_sites[i])) engram_contribute(M, i, s->engram_history[i], idx, position, ekey[i], evalue[i]);
  }
  std::vector<float> next(stream.size());
  std::vector<float> normed(d);
  std::vector<std::vector<float>> cells{lane_mean(stream.data(), d, lanes)};  // session.rs:91-92, 139
  for (size_t slot = 0; slot < M->active.size(); ++slot) {
    size_t layer = M->active[slot];
    const LayerW& W = M->weights->layers[layer];
    Routing r = route(M, layer, slot, stream.data(), d);
    std::vector<float> x = r.input;
    const int site = engram_site_at(g, layer);
    if (site >= 0 && !ekey[site].empty()) add_engram(x.data(), ekey[site].data(), evalue[site].data(), d);
    zero_centred_norm(x.data(), W.norm_in.data(), normed.data(), d);
    std::vector<float> attended = attend(M, W, layer, s->caches[layer], s->frequencies.data(), position, normed.data());
    finish_block(M, W, r, x, attended, stream.data(), next.data(), cross, layer);
    std::swap(stream, next);
    if (trace) std::memcpy(trace + slot * lanes * d, stream.data(), lanes * d * sizeof(float));
    if (!M->weights->heads.empty()) cells.push_back(lane_mean(stream.data(), d, lanes));
  }
  std::vector<float> mean = lane_mean(stream.data(), d, lanes);
  s->hidden.assign(d, 0.0f);
  zero_centred_norm(mean.data(), M->weights->final_norm.data(), s->hidden.data(), d);
  const std::vector<size_t> rows = head_rows(M);
  for (size_t h = 0; h < M->weights->heads.size(); ++h) observe(M->weights->heads[h], rows, s->accumulators[h], cells);  // session.rs:144-146
}

// crates/model/src/prefill.rs:10-99 with the non-aarch64 attend_batch
// (model/src/attention.rs:216-369). INT mode never comes here: its batched
// products and attention reproduce push() exactly (panel.rs tiles compute each
// token lane as the single-token tile does), so feed() steps token by token.
void prefill_float(nbo_session* s, const uint32_t* tokens, size_t count) {
  const nbo_model* M = s->model;
  const Geometry& g = M->archive->geo;
  size_t d = g.d_model, lanes = g.mhc_lanes, frame = lanes * d;
  size_t qk = g.qk_head_dim, vd = g.v_head_dim, H = g.num_heads, KV = g.num_kv_heads;
  size_t first = s->tokens.size();
  for (size_t t = 0; t < count; ++t)
    if (tokens[t] >= M->weights->embedding.rows) throw Failure(ERR_ARGUMENT, "token id outside the embedding");
  s->tokens.insert(s->tokens.end(), tokens, tokens + count);
  std::vector<float> stream(count * frame), next(count * frame);
  fork(M->threads, count, true, [&](size_t t) {
    std::vector<float> e = embed(M, tokens[t]);
    std::memcpy(&stream[t * frame], e.data(), frame * sizeof(float));
  });
  // EngramSiteState::contribute_batch (engram.rs:112-160) per active site
  const size_t sites = g.engram_sites.size();
  std::vector<std::vector<float>> ekeys(sites), evalues(sites);
  for (size_t i = 0; i < sites; ++i) {
    if (!layer_active(M, g.engram_sites[i])) continue;
    const EngramW& E = M->weights->engrams[i];
    const size_t padded = E.key_proj.padded, kw = E.key_proj.rows, vw = E.value_proj.rows;
    std::vector<float> rotated(count * padded);
    fork(M->threads, count, true, [&](size_t t) {
      std::vector<float> gathered = engram_gather(M, E, table_indices(g, s->tokens, first + t), first + t);
      std::vector<float> r = E.key_proj.prepare(gathered.data());
      std::memcpy(&rotated[t * padded], r.data(), padded * sizeof(float));
    });
    ekeys[i].assign(count * kw, 0.0f);
    std::vector<float> raw(count * vw);
    multiply_batch_float(E.key_proj, rotated.data(), count, ekeys[i].data(), M->threads);
    multiply_batch_float(E.value_proj, rotated.data(), count, raw.data(), M->threads);
    const std::deque<std::vector<float>> previous = s->engram_history[i];
    evalues[i].assign(count * vw, 0.0f);
    fork(M->threads, count, true, [&](size_t t) {
      engram_conv(g, E, first + t, vw,
                  [&](size_t back) { return back <= t ? &raw[(t - back) * vw] : previous.at(back - t - 1).data(); }, &evalues[i][t * vw]);
    });
    const size_t keep = engram_keep(g);
    for (size_t t = count > keep ? count - keep : 0; t < count; ++t)
      s->engram_history[i].push_front(std::vector<float>(raw.begin() + t * vw, raw.begin() + (t + 1) * vw));
    while (s->engram_history[i].size() > keep) s->engram_history[i].pop_back();
  }
  const bool heads = !M->weights->heads.empty();
  std::vector<std::vector<std::vector<float>>> cells(count);  // prefill.rs:31, 86-88
  if (heads)
    for (size_t t = 0; t < count; ++t) cells[t].push_back(lane_mean(&stream[t * frame], d, lanes));
  for (size_t slot = 0; slot < M->active.size(); ++slot) {
    size_t layer = M->active[slot];
    const LayerW& W = M->weights->layers[layer];
    Cache& cache = s->caches[layer];
    std::vector<Routing> routings(count);
    std::vector<float> x(count * d), normed(count * d);
    const int site = engram_site_at(g, layer);
    fork(M->threads, count, true, [&](size_t t) {
      routings[t] = route(M, layer, slot, &stream[t * frame], d);
      std::memcpy(&x[t * d], routings[t].input.data(), d * sizeof(float));
      if (site >= 0 && !ekeys[site].empty()) add_engram(&x[t * d], &ekeys[site][t * d], &evalues[site][t * d], d);
      zero_centred_norm(&x[t * d], W.norm_in.data(), &normed[t * d], d);
    });
    // attend_batch: fake-quantise, rotate and multiply every token at once.
    std::vector<float> quantised = normed;
    fork(M->threads, count, true, [&](size_t t) { fake_quantise_int8(&quantised[t * d], d); });
    size_t padded = W.q.padded;
    std::vector<float> rotated(count * padded, 0.0f);
    for (size_t t = 0; t < count; ++t) {
      std::memcpy(&rotated[t * padded], &quantised[t * d], d * sizeof(float));
      rotate_groups(&rotated[t * padded], padded, W.q.group);
    }
    std::vector<float> q(count * W.q.rows), k(count * W.k.rows), v(count * W.v.rows), gate(count * W.gate.rows);
    multiply_batch_float(W.q, rotated.data(), count, q.data(), M->threads);
    multiply_batch_float(W.k, rotated.data(), count, k.data(), M->threads);
    multiply_batch_float(W.v, rotated.data(), count, v.data(), M->threads);
    multiply_batch_float(W.gate, rotated.data(), count, gate.data(), M->threads);
    if (!W.taps[0].empty()) {
      // attention.rs:243-276: token t's tap j reads row t - j of this chunk, or
      // the history before it; the history keeps the newest rows
      size_t taps = g.qkv_conv_taps;
      std::vector<float>* rows[3] = {&q, &k, &v};
      for (int i = 0; i < 3; ++i) {
        size_t width = rows[i]->size() / count;
        std::vector<float> mixed(count * width, 0.0f);
        const std::deque<std::vector<float>> previous = cache.raw_history[i];
        for (size_t t = 0; t < count; ++t) {
          size_t position = first + t;
          for (size_t tap = 0; tap < std::min(taps, position + 1); ++tap) {
            const float* src = tap <= t ? &(*rows[i])[(t - tap) * width] : previous.at(tap - t - 1).data();
            const float* gn = &W.taps[i][tap * width];
            for (size_t c = 0; c < width; ++c) mixed[t * width + c] += gn[c] * src[c];
          }
        }
        size_t newest = std::min(count, taps);
        for (size_t t = count - newest; t < count; ++t)
          cache.raw_history[i].push_front(std::vector<float>(rows[i]->begin() + t * width, rows[i]->begin() + (t + 1) * width));
        while (cache.raw_history[i].size() > taps) cache.raw_history[i].pop_back();
        *rows[i] = std::move(mixed);
      }
    }
    std::vector<int8_t> qcodes(count * H * qk);
    std::vector<float> qscales(count * H);
    for (size_t t = 0; t < count; ++t) {
      std::vector<int8_t> codes;
      std::vector<float> scales;
      heads_and_cache(M, W, cache, s->frequencies.data(), first + t, &q[t * H * qk], &k[t * KV * qk], &v[t * KV * vd], codes, scales);
      std::memcpy(&qcodes[t * H * qk], codes.data(), codes.size());
      std::memcpy(&qscales[t * H], scales.data(), scales.size() * sizeof(float));
    }
    std::vector<float> attended(count * H * vd);
    fork(M->threads, count, true, [&](size_t t) {
      std::vector<int8_t> codes(&qcodes[t * H * qk], &qcodes[(t + 1) * H * qk]);
      std::vector<float> scales(&qscales[t * H], &qscales[(t + 1) * H]);
      std::vector<float> o = attend_heads(M, layer, cache, first + t, codes, scales, false);
      std::memcpy(&attended[t * H * vd], o.data(), o.size() * sizeof(float));
    });
    size_t aw = H * vd;
    fork(M->threads, count, true, [&](size_t t) {
      for (size_t i = 0; i < aw; ++i) attended[t * aw + i] *= sigmoid(gate[t * aw + i]);
      fake_quantise_int8(&attended[t * aw], aw);
    });
    size_t opad = W.out.padded;
    std::vector<float> rot_out(count * opad, 0.0f);
    for (size_t t = 0; t < count; ++t) {
      std::memcpy(&rot_out[t * opad], &attended[t * aw], aw * sizeof(float));
      rotate_groups(&rot_out[t * opad], opad, W.out.group);
    }
    std::vector<float> output(count * d);
    multiply_batch_float(W.out, rot_out.data(), count, output.data(), M->threads);
    fork(M->threads, count, true, [&](size_t t) {
      std::vector<float> xt(&x[t * d], &x[(t + 1) * d]);
      std::vector<float> at(&output[t * d], &output[(t + 1) * d]);
      finish_block(M, W, routings[t], xt, at, &stream[t * frame], &next[t * frame]);
    });
    std::swap(stream, next);
    if (heads)
      for (size_t t = 0; t < count; ++t) cells[t].push_back(lane_mean(&stream[t * frame], d, lanes));
  }
  const std::vector<size_t> rows = head_rows(M);
  for (size_t t = 0; t < count && heads; ++t)  // prefill.rs:90-94
    for (size_t h = 0; h < M->weights->heads.size(); ++h) observe(M->weights->heads[h], rows, s->accumulators[h], cells[t]);
  std::vector<float> mean = lane_mean(&stream[(count - 1) * frame], d, lanes);
  s->hidden.assign(d, 0.0f);
  zero_centred_norm(mean.data(), M->weights->final_norm.data(), s->hidden.data(), d);
}

// session.rs:56-70
void feed(nbo_session* s, const uint32_t* tokens, size_t count) {
  const size_t BATCH_THRESHOLD = 4, PREFILL_CHUNK = 128;
  if (count >= BATCH_THRESHOLD) {
    for (size_t at = 0; at < count; at += PREFILL_CHUNK) {
      size_t n = std::min(PREFILL_CHUNK, count - at);
      if (n >= BATCH_THRESHOLD && s->model->mode == NBO_MODE_FLOAT) {
        prefill_float(s, tokens + at, n);
      } else {
        for (size_t i = 0; i < n; ++i) push(s, tokens[at + i], nullptr);
      }
    }
  } else {
    for (size_t i = 0; i < count; ++i) push(s, tokens[i], nullptr);
  }
}

// session.rs:166-177
void logits(const nbo_session* s, float* out) {
  const nbo_model* M = s->model;
  const QMatrix& E = M->weights->embedding;
  size_t d = M->archive->geo.d_model;
  std::vector<float> q = s->hidden;
  if (q.size() != d) q.assign(d, 0.0f);
  fake_quantise_int8(q.data(), d);
  std::vector<float> rotated = E.prepare(q.data());
  std::vector<Job> jobs{{&E, 0, out, M->archive->geo.output_vocab()}};
  multiply_jobs(jobs, rotated.data(), M->mode, M->threads);
}

template <typename F>
int guard(F&& f) {
  try {
    f();
    return OK;
  } catch (const Failure& e) {
    g_error = e.what();
    return e.status;
  } catch (const std::exception& e) {
    g_error = e.what();
    return ERR_ARGUMENT;
  }
}

}  // namespace nbo

using namespace nbo;

extern "C" {

const char* nbo_last_error(void) { return g_error.c_str(); }

int nbo_model_open(const char* path, int mode, int threads, nbo_model** out) {
  *out = nullptr;
  return guard([&] {
    auto m = std::make_unique<nbo_model>();
    m->archive = open_archive(path);
    m->layout = resolve_layout(*m->archive);
    m->weights = load_weights(*m->archive, m->layout);
    for (size_t i = 0; i < m->archive->geo.num_layers; ++i) m->active.push_back(i);
    m->mode = mode;
    m->threads = threads > 0 ? threads : omp_get_num_procs();
    *out = m.release();
  });
}

int nbo_model_with_depth(const nbo_model* model, int depth, nbo_model** out) {
  *out = nullptr;
  std::vector<int32_t> layers;
  if (!ladder_select((int)model->archive->geo.num_layers, depth, layers)) {
    g_error = "depth " + std::to_string(depth) + " is outside the 2 to " + std::to_string(model->archive->geo.num_layers) + " layers this model offers";
    return ERR_DEPTH;
  }
  auto m = std::make_unique<nbo_model>(*model);
  m->active.assign(layers.begin(), layers.end());
  *out = m.release();
  return OK;
}

void nbo_model_free(nbo_model* model) { delete model; }

int nbo_model_active_layers(const nbo_model* model, int32_t* out, int cap) {
  int n = (int)model->active.size();
  for (int i = 0; i < n && i < cap; ++i) out[i] = (int32_t)model->active[i];
  return n;
}

void nbo_model_geometry(const nbo_model* m, int32_t* o) {
  const Geometry& g = m->archive->geo;
  o[0] = (int32_t)g.vocab;
  o[1] = (int32_t)g.output_vocab();
  o[2] = (int32_t)g.d_model;
  o[3] = (int32_t)g.num_heads;
  o[4] = (int32_t)g.num_kv_heads;
  o[5] = (int32_t)g.num_layers;
  o[6] = (int32_t)g.qk_head_dim;
  o[7] = (int32_t)g.max_seq_len;
}

void nbo_model_set_threads(nbo_model* model, int threads) { model->threads = threads > 0 ? threads : omp_get_num_procs(); }

nbo_session* nbo_session_new(const nbo_model* model) {
  auto* s = new nbo_session();
  s->model = model;
  s->caches.resize(model->archive->geo.num_layers);
  s->engram_history.resize(model->archive->geo.engram_sites.size());
  for (const nbo::ProbeHeadW& h : model->weights->heads) {  // ProbeHead::accumulator (heads.rs:80-83)
    const size_t slots = (model->active.size() + 1) * h.ppl;
    s->accumulators.push_back({std::vector<float>(slots, -INFINITY), std::vector<float>(slots, 0.0f), std::vector<float>(slots * h.width, 0.0f)});
  }
  s->frequencies = rotary_frequencies(model->archive->geo.qk_head_dim, model->archive->geo.rope_theta);
  return s;
}

nbo_session* nbo_session_clone(const nbo_session* s) { return new nbo_session(*s); }
void nbo_session_free(nbo_session* s) { delete s; }
size_t nbo_session_len(const nbo_session* s) { return s->tokens.size(); }

// Session::head_output / pooled_readout (session.rs:150-160): the values
// written (at most `cap`), or -1 when the model has no head with `code`.
static long head_values(const nbo_session* s, int code, float* out, size_t cap, bool project) {
  const nbo_model* M = s->model;
  for (size_t h = 0; h < M->weights->heads.size(); ++h)
    if (M->weights->heads[h].code == code) {
      std::vector<float> v = nbo::pooled(M->weights->heads[h], nbo::head_rows(M), s->accumulators[h]);
      if (project) v = nbo::project_head(M, M->weights->heads[h], v);
      std::memcpy(out, v.data(), std::min(cap, v.size()) * sizeof(float));
      return (long)v.size();
    }
  return -1;
}
long nbo_session_head_output(const nbo_session* s, int code, float* out, size_t cap) { return head_values(s, code, out, cap, true); }
long nbo_session_pooled_readout(const nbo_session* s, int code, float* out, size_t cap) { return head_values(s, code, out, cap, false); }

void nbo_session_push(nbo_session* s, uint32_t token) { guard([&] { push(s, token, nullptr); }); }

// Whistle: CrossWeights::memory of an encoder output [frames][d_model], and
// Session::push_with(token, CrossState) (session.rs:76-148 with the hook).
struct nbo_cross_memory {
  nbo::CrossMemory m;
};
int nbo_cross_memory_new(const nbo_model* model, const float* encoded, size_t frames, nbo_cross_memory** out) {
  *out = nullptr;
  return guard([&] {
    if (model->weights->cross.empty()) throw nbo::Failure(nbo::ERR_ARGUMENT, "the archive carries no cross attention");
    auto* m = new nbo_cross_memory();
    m->m = nbo::cross_memory(model, encoded, frames);
    *out = m;
  });
}
void nbo_cross_memory_free(nbo_cross_memory* memory) { delete memory; }
size_t nbo_cross_memory_read(const nbo_cross_memory* memory, int layer, int8_t* keys, float* key_scales, int8_t* values, float* value_scales) {
  const nbo::CrossMemory& m = memory->m;
  std::memcpy(keys, m.keys[layer].data(), m.keys[layer].size());
  std::memcpy(key_scales, m.key_scales[layer].data(), m.key_scales[layer].size() * 4);
  std::memcpy(values, m.values[layer].data(), m.values[layer].size());
  std::memcpy(value_scales, m.value_scales[layer].data(), m.value_scales[layer].size() * 4);
  return m.frames;
}
int nbo_session_push_cross(nbo_session* s, uint32_t token, const nbo_cross_memory* memory) {
  return guard([&] { push(s, token, nullptr, &memory->m); });
}
size_t nbo_model_text_vocab(const nbo_model* model) { return model->weights->text_vocab; }
void nbo_session_push_traced(nbo_session* s, uint32_t token, float* trace) { guard([&] { push(s, token, trace); }); }
void nbo_session_feed(nbo_session* s, const uint32_t* tokens, size_t count) { guard([&] { feed(s, tokens, count); }); }
void nbo_session_logits(const nbo_session* s, float* out) { guard([&] { logits(s, out); }); }
void nbo_session_hidden(const nbo_session* s, float* out) {
  for (size_t i = 0; i < s->hidden.size(); ++i) out[i] = s->hidden[i];
}

size_t nbo_session_cache(const nbo_session* s, int layer, int8_t* keys, float* key_scales, int8_t* values, float* value_scales) {
  const Cache& c = s->caches.at(layer);
  const Geometry& g = s->model->archive->geo;
  size_t n = c.key_scales.empty() ? 0 : c.key_scales[0].size();
  if (keys) std::memcpy(keys, c.keys.data(), c.keys.size());
  if (values) std::memcpy(values, c.values.data(), c.values.size());
  for (size_t h = 0; h < c.key_scales.size(); ++h) {
    if (key_scales) std::memcpy(key_scales + h * n, c.key_scales[h].data(), n * sizeof(float));
    if (value_scales) std::memcpy(value_scales + h * n, c.value_scales[h].data(), n * sizeof(float));
  }
  (void)g;
  return n;
}

void nbo_sessions_step(nbo_session** sessions, size_t count, const uint32_t* tokens, float* out, int threads) {
  if (threads <= 0) threads = omp_get_num_procs();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
  for (size_t i = 0; i < count; ++i) {
    nbo_session* s = sessions[i];
    size_t vocab = s->model->archive->geo.output_vocab();
    guard([&] {
      push(s, tokens[i], nullptr);
      if (out) logits(s, out + i * vocab);
    });
  }
}

int32_t nbo_argmax(const float* v, size_t n) {
  size_t best = 0;
  for (size_t i = 0; i < n; ++i)
    if (v[i] > v[best]) best = i;
  return (int32_t)best;
}

int32_t nbo_argmax_allowed(const float* v, const uint8_t* allowed, size_t n) {
  long best = -1;
  for (size_t i = 0; i < n; ++i)
    if (allowed[i] && (best < 0 || v[i] > v[best])) best = (long)i;
  return (int32_t)best;
}

void nbo_allowed_statistics(const float* logits, size_t n, uint32_t token, const uint8_t* allowed, float* probability, float* mass) {
  float peak_all = -INFINITY, peak_allowed = -INFINITY;
  for (size_t i = 0; i < n; ++i) peak_all = std::fmax(peak_all, logits[i]);
  for (size_t i = 0; i < n; ++i) peak_allowed = std::fmax(peak_allowed, allowed[i] ? logits[i] : -INFINITY);
  float total_all = 0.0f, total_allowed = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    total_all += fast_exp(logits[i] - peak_all);
    total_allowed += fast_exp(logits[i] - peak_allowed) * (allowed[i] ? 1.0f : 0.0f);
  }
  *probability = fast_exp(logits[token] - peak_allowed) / total_allowed;
  *mass = total_allowed * fast_exp(peak_allowed - peak_all) / total_all;
}

void nbo_walsh(float* values, size_t count) { transform_in_place(values, count); }
float nbo_fast_exp(float value) { return fast_exp(value); }
float nbo_sigmoid(float value) { return sigmoid(value); }
void nbo_softmax(float* values, size_t count) { softmax_in_place(values, count); }
void nbo_kronecker(const float* input, const float* left, size_t ls, const float* right, size_t rs, float* output, int mode) {
  kronecker_apply(input, left, ls, right, rs, output, mode);
}
void nbo_sinkhorn(float* logits, size_t size, size_t iterations) { sinkhorn_in_place(logits, size, iterations); }
void nbo_zero_centred_norm(const float* input, const float* gains, float* output, size_t count) {
  zero_centred_norm(input, gains, output, count);
}
void nbo_fake_quantise_int8(float* values, size_t count) { fake_quantise_int8(values, count); }
float nbo_quantise_int8(const float* values, int8_t* codes, size_t count) { return quantise_int8(values, codes, count); }
void nbo_rotary(float* head, size_t dim, size_t position, float theta) {
  std::vector<float> f = rotary_frequencies(dim, theta);
  apply_rotary(head, dim, position, f.data());
}
int nbo_ladder_order(int layers, int32_t* out) {
  auto o = ladder_order(layers);
  std::copy(o.begin(), o.end(), out);
  return (int)o.size();
}
int nbo_ladder_select(int layers, int depth, int32_t* out) {
  std::vector<int32_t> s;
  if (!ladder_select(layers, depth, s)) return ERR_DEPTH;
  std::copy(s.begin(), s.end(), out);
  return (int)s.size();
}
float nbo_half_to_f32(uint16_t bits) { return half_to_f32(bits); }

int nbo_matrix_product(const nbo_model* model, int tensor, const float* input, size_t first_row, size_t rows, float* out, int32_t* sums) {
  return guard([&] {
    QMatrix m = load_matrix(*model->archive, (size_t)tensor);
    if (first_row + rows > m.rows) throw Failure(ERR_ARGUMENT, "row range outside the matrix");
    std::vector<float> rotated = m.prepare(input);
    if (model->mode == NBO_MODE_INT && m.integer_path(NBO_MODE_INT)) {
      GroupInput in = quantise_groups(rotated.data(), m.padded, m.group);
      for (size_t r = 0; r < rows; ++r) out[r] = m.row_integer(first_row + r, in, sums ? sums + r * m.groups : nullptr);
    } else {
      for (size_t r = 0; r < rows; ++r) out[r] = m.row_float(first_row + r, rotated.data());
    }
  });
}

// The product of a matrix given in the archive's representation (packed
// bits-wide indices per row, the 2^bits codebook levels, fp16 norms per
// 128-column group) through the same QMatrix code as the archive path.
int nbo_product_raw(int mode, uint32_t bits, const uint8_t* packed, const float* levels, const uint16_t* norms, size_t rows,
                    size_t cols, const float* input, float* out, int32_t* sums) {
  return guard([&] {
    if ((bits != 2 && bits != 4) || cols % 128 != 0 || !packed || !levels || !norms || !input || !out)
      throw Failure(ERR_ARGUMENT, "a raw product takes 2- or 4-bit codes and a multiple of 128 columns");
    std::vector<float> cb(28, 0.0f);
    for (uint32_t i = 0; i < (1u << bits); ++i) cb[(bits == 2 ? 0 : 12) + i] = levels[i];
    QMatrix m;
    m.packed = packed;
    m.rows = rows;
    m.columns = m.padded = cols;
    m.group = 128;
    m.record_bits = bits;
    m.row_bytes = cols * bits / 8;
    m.groups = cols / 128;
    m.table = lookup_table(bits, cb, 128);
    m.ilevels = integer_levels(m.table);
    m.norms.resize(rows * m.groups);
    for (size_t i = 0; i < m.norms.size(); ++i) m.norms[i] = half_to_f32(norms[i]);
    std::vector<float> rotated = m.prepare(input);
    if (mode == NBO_MODE_INT && m.integer_path(NBO_MODE_INT)) {
      GroupInput in = quantise_groups(rotated.data(), m.padded, m.group);
      for (size_t r = 0; r < rows; ++r) out[r] = m.row_integer(r, in, sums ? sums + r * m.groups : nullptr);
    } else {
      for (size_t r = 0; r < rows; ++r) out[r] = m.row_float(r, rotated.data());
    }
  });
}

// One head's attention (attend_head) over `count` cached positions given
// directly: keys and values [count][dim] int8, their scales [count].
int nbo_attend_head_raw(int mode, const int8_t* query, float query_scale, const int8_t* keys, const float* key_scales,
                        const int8_t* values, const float* value_scales, size_t count, size_t dim, float* out) {
  return guard([&] {
    if (!query || !keys || !key_scales || !values || !value_scales || !out || count == 0 || dim == 0)
      throw Failure(ERR_ARGUMENT, "a raw attention takes a query, at least one position and a head width");
    Cache cache;
    cache.keys.assign(keys, keys + count * dim);
    cache.values.assign(values, values + count * dim);
    cache.key_scales.assign(1, std::vector<float>(key_scales, key_scales + count));
    cache.value_scales.assign(1, std::vector<float>(value_scales, value_scales + count));
    attend_head(query, query_scale, cache, 0, 1, dim, dim, 0, count, mode, out);
  });
}

int nbo_matrix_dequantise_row(const nbo_model* model, int tensor, size_t row, float* out) {
  return guard([&] {
    QMatrix m = load_matrix(*model->archive, (size_t)tensor);
    if (row >= m.rows) throw Failure(ERR_ARGUMENT, "row outside the matrix");
    std::vector<float> r = m.dequantise_row(row);
    std::memcpy(out, r.data(), r.size() * sizeof(float));
  });
}

int nbo_tensor_info(const nbo_model* model, int tensor, int64_t* o) {
  if (tensor < 0 || (size_t)tensor >= model->archive->records.size()) return ERR_ARGUMENT;
  const Record& r = model->archive->records[tensor];
  o[0] = r.kind;
  o[1] = (int64_t)r.rows();
  o[2] = (int64_t)r.columns();
  o[3] = (int64_t)r.group_size;
  o[4] = (int64_t)r.bits;
  return OK;
}

int nbo_route(const nbo_model* model, int layer, int slot, const float* stream, float* input, float* post, float* residual) {
  return guard([&] {
    if (!model || !stream || !input || !post || !residual || layer < 0 || slot < 0)
      throw Failure(ERR_ARGUMENT, "a route takes a model, a layer, a slot, the lane stream and three outputs");
    Routing r = route(model, (size_t)layer, (size_t)slot, stream, model->archive->geo.d_model);
    std::memcpy(input, r.input.data(), r.input.size() * sizeof(float));
    std::memcpy(post, r.post.data(), r.post.size() * sizeof(float));
    std::memcpy(residual, r.residual.data(), r.residual.size() * sizeof(float));
  });
}

int nbo_hadamard_apply(const nbo_model* model, int layer, const float* input, float* out) {
  return guard([&] {
    const LayerW& W = model->weights->layers.at((size_t)layer);
    std::vector<float> r = hadamard_apply(W.hada, input, model->archive->geo.d_model, model->mode);
    std::memcpy(out, r.data(), r.size() * sizeof(float));
  });
}

}  // extern "C"
