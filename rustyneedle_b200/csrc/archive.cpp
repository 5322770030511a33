// archive.cpp — `.cact` reader: memory-mapped, bounds- and alignment-checked,
// every failure reported as a status instead of a panic.
#include "archive.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>

#include "../../include/needle_b200.h"

namespace nba {

namespace {

constexpr uint32_t FORMAT_TAG = 0x05E12A84u;
constexpr size_t HEADER_BYTES = 196;
constexpr size_t RECORD_BYTES = 44;

[[noreturn]] void fail(int status, const std::string& message) { throw ArchiveError{status, message}; }

struct Reader {
  const uint8_t* base;
  size_t size, at;
  const char* what;
  template <typename T>
  T take() {
    if (at + sizeof(T) > size) fail(NB_ERR_ARCHIVE, std::string("archive is truncated inside the ") + what);
    T v;
    std::memcpy(&v, base + at, sizeof(T));
    at += sizeof(T);
    return v;
  }
};

}  // namespace

// crates/cact/src/layout.rs:323-339
float half_to_f32(uint16_t bits) {
  uint32_t sign = bits >> 15, exponent = (bits >> 10) & 0x1f, mantissa = bits & 0x3ff, value;
  if (exponent == 0 && mantissa == 0) {
    value = sign << 31;
  } else if (exponent == 0) {
    uint32_t shift = (uint32_t)__builtin_clz(mantissa) - 21;
    value = sign << 31 | (113 - shift) << 23 | ((mantissa << shift) & 0x3ff) << 13;
  } else if (exponent == 0x1f) {
    value = sign << 31 | 0x7f800000u | (mantissa ? 0x00400000u | mantissa << 13 : 0);
  } else {
    value = sign << 31 | (exponent + 112) << 23 | mantissa << 13;
  }
  float f;
  std::memcpy(&f, &value, 4);
  return f;
}

Archive::Archive(const char* path) {
  int fd = ::open(path, O_RDONLY);
  if (fd < 0) fail(NB_ERR_IO, std::string("cannot open ") + path + ": " + std::strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    fail(NB_ERR_IO, std::string("cannot stat ") + path);
  }
  size_ = (size_t)st.st_size;
  if (size_ > 0) {
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) fail(NB_ERR_IO, std::string("cannot map ") + path);
    base_ = static_cast<const uint8_t*>(m);
  } else {
    ::close(fd);
  }
  try {
    Reader r{base_, size_, 0, "header"};
    uint32_t tag = r.take<uint32_t>();
    if (tag != FORMAT_TAG) {
      char m[80];
      std::snprintf(m, sizeof m, "not a Needle 3 archive (format tag 0x%08x)", tag);
      fail(NB_ERR_ARCHIVE, m);
    }
    uint32_t fields[26];
    for (auto& f : fields) f = r.take<uint32_t>();
    Geometry& g = geo_;
    g.tensor_count = fields[0];
    g.codebook_len = fields[1];
    g.kv_window = fields[2];
    g.kv_bits = fields[3];
    g.vocab = fields[4];
    g.out_vocab = fields[5];
    g.d_model = fields[6];
    g.num_heads = fields[7];
    g.num_kv_heads = fields[8];
    g.num_layers = fields[9];
    g.qk_head_dim = fields[10];
    g.v_head_dim = fields[11];
    g.max_seq_len = fields[12];
    g.hada_n = fields[13];
    g.mhc_lanes = fields[14];
    g.sliding_window = fields[15];
    g.global_layers = (uint64_t)fields[16] | ((uint64_t)fields[17] << 32);
    g.qkv_conv_taps = fields[18];
    g.engram_slots = fields[19];
    g.engram_sub_dim = fields[20];
    g.engram_tables = fields[21];
    g.engram_conv_taps = fields[22];
    g.engram_conv_dilation = fields[23];
    g.engram_seed_heads = fields[24];
    uint32_t order_count = fields[25], orders[4], sites[16];
    for (auto& o : orders) o = r.take<uint32_t>();
    uint32_t site_count = r.take<uint32_t>();
    for (auto& s : sites) s = r.take<uint32_t>();
    g.rope_theta = r.take<float>();
    if (order_count > 4 || site_count > 16)
      fail(NB_ERR_ARCHIVE, "unexpected tensor layout: engram order or site count exceeds the header capacity");
    g.engram_orders.assign(orders, orders + order_count);
    g.engram_sites.assign(sites, sites + site_count);
    r.what = "codebook";
    for (uint32_t i = 0; i < g.codebook_len; ++i) codebook_.push_back(r.take<float>());
    r.what = "tensor directory";
    records_.reserve(g.tensor_count);
    for (uint32_t i = 0; i < g.tensor_count; ++i) {
      Record rec;
      rec.kind = r.take<uint8_t>();
      if (rec.kind < 1 || rec.kind > 4) fail(NB_ERR_ARCHIVE, "unknown tensor element kind " + std::to_string(rec.kind));
      uint32_t rank = r.take<uint8_t>();
      r.take<uint16_t>();
      uint32_t dims[4];
      for (auto& d : dims) d = r.take<uint32_t>();
      rec.shape.assign(dims, dims + (rank < 4 ? rank : 4));
      rec.offset = r.take<uint64_t>();
      rec.byte_len = r.take<uint64_t>();
      rec.group_size = r.take<uint32_t>();
      rec.bits = r.take<uint32_t>();
      records_.push_back(rec);
    }
    (void)HEADER_BYTES;
    (void)RECORD_BYTES;
    for (size_t i = 0; i < records_.size(); ++i) {
      const Record& rec = records_[i];
      if (rec.offset + rec.byte_len < rec.offset || rec.offset + rec.byte_len > size_)
        fail(NB_ERR_ARCHIVE, "tensor " + std::to_string(i) + " lies outside the archive");
      uint64_t width = rec.kind == HALF ? 2 : rec.kind == SINGLE ? 4 : 1;
      if (rec.offset % width || rec.byte_len % width)
        fail(NB_ERR_ARCHIVE, "unexpected tensor layout: tensor " + std::to_string(i) + " is not aligned to its element width");
    }
  } catch (...) {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_);
    base_ = nullptr;
    throw;
  }
}

Archive::~Archive() {
  if (base_) munmap(const_cast<uint8_t*>(base_), size_);
}

std::vector<float> Archive::floats(uint32_t i) const {
  const Record& r = record(i);
  std::vector<float> out;
  if (r.kind == HALF) {
    out.resize(r.byte_len / 2);
    for (size_t k = 0; k < out.size(); ++k) {
      uint16_t h;
      std::memcpy(&h, data(i) + 2 * k, 2);
      out[k] = half_to_f32(h);
    }
  } else if (r.kind == SINGLE) {
    out.resize(r.byte_len / 4);
    std::memcpy(out.data(), data(i), r.byte_len);
  } else {
    fail(NB_ERR_ARCHIVE, "tensor " + std::to_string(i) + " holds no floating point values");
  }
  return out;
}

// crates/cact/src/layout.rs:190-293
Layout Archive::resolve() const {
  Layout L;
  uint32_t count = this->count();
  if (count == 0 || records_.back().kind != RAW) fail(NB_ERR_ARCHIVE, "unexpected tensor layout: no trailing tokenizer blob");
  L.tokenizer = count - 1;
  uint32_t next = 0, end = L.tokenizer;
  auto take = [&]() -> uint32_t {
    if (next >= end) fail(NB_ERR_ARCHIVE, "unexpected tensor layout: directory ends before the canonical tensor list");
    return next++;
  };
  auto peek = [&]() -> int { return next < end ? records_[next].kind : -1; };
  L.embedding = take();
  for (uint32_t l = 0; l < geo_.num_layers; ++l) {
    LayerIdx t{};
    t.norm_in = take();
    t.q = take();
    t.k = take();
    t.v = take();
    if (geo_.qkv_conv_taps > 0) {
      t.has_taps = true;
      for (uint32_t& x : t.taps) x = take();
    }
    t.q_norm = take();
    t.k_norm = take();
    t.gate = take();
    t.out = take();
    t.post_norm = take();
    t.attn_gate = take();
    t.pre_hada = take();
    uint32_t* h = &t.hada.d1;
    for (int i = 0; i < 13; ++i) h[i] = take();
    L.layers.push_back(t);
  }
  uint32_t* lanes = &L.lanes.a_pre;
  for (int i = 0; i < 9; ++i) lanes[i] = take();
  L.perms[0] = take();
  L.perms[1] = take();
  for (size_t s = 0; s < geo_.engram_sites.size(); ++s) {
    std::array<uint32_t, 4> e;
    for (uint32_t& i : e) i = take();
    L.engrams.push_back(e);
    L.engram_sites++;
  }
  L.final_norm = take();
  if (peek() == HALF) {
    uint32_t manifest = take();
    const Record& r = records_[manifest];
    for (uint64_t i = 0; i < r.byte_len / 2; ++i) {
      uint16_t h;
      std::memcpy(&h, data(manifest) + 2 * i, 2);
      long code = std::lround(half_to_f32(h));
      if (code < 1 || code > 3) fail(NB_ERR_ARCHIVE, "unexpected tensor layout: unrecognised head manifest code");
      Layout::HeadIdx hi;
      hi.code = (uint32_t)code;
      hi.probes = take();
      hi.gain = take();
      hi.query = take();
      hi.row_bias = take();
      hi.proj = take();
      hi.bias = take();
      if (code == 3) take();  // calibration: not read by the model crate
      L.heads.push_back(hi);
      L.probe_heads++;
    }
  }
  if (peek() == SINGLE) {
    uint32_t manifest = take();
    const Record& r = records_[manifest];
    float v[13];
    if (r.byte_len != 13 * 4) fail(NB_ERR_ARCHIVE, "unexpected tensor layout: audio manifest is malformed");
    std::memcpy(v, data(manifest), sizeof v);
    if (v[0] != 3246.0f) fail(NB_ERR_ARCHIVE, "unexpected tensor layout: audio manifest is malformed");
    uint32_t encoder_layers = (uint32_t)v[3], stem_stages = (uint32_t)v[7];
    L.text_vocab = (uint32_t)v[2];
    for (uint32_t l = 0; l < geo_.num_layers; ++l) {
      std::array<uint32_t, 10> c;
      for (uint32_t& x : c) x = take();
      L.cross.push_back(c);
    }
    L.position_gate = take();
    for (uint32_t l = 0; l < encoder_layers; ++l)
      for (int i = 0; i < 6 + 11 + 26; ++i) take();
    for (int i = 0; i < 9 + 1 + 1; ++i) take();
    for (uint32_t s = 1; s < stem_stages; ++s) {
      take();
      take();
    }
    take();
    take();
    L.audio = true;
  }
  if (next != L.tokenizer)
    fail(NB_ERR_ARCHIVE, "unexpected tensor layout: " + std::to_string(L.tokenizer - next) + " tensors are left over before the tokenizer");
  return L;
}

// crates/tokenizer/src/vocabulary.rs:66-99: a 24-byte header, then per piece
// f32 score, u8 kind (0-4), u16 length and the piece bytes.
void Archive::validate_tokenizer(uint32_t index) const {
  const Record& r = record(index);
  const uint8_t* p = data(index);
  uint64_t n = r.byte_len;
  if (n < 24) fail(NB_ERR_ARCHIVE, "tokenizer blob is malformed: truncated header");
  uint32_t pieces;
  std::memcpy(&pieces, p, 4);
  uint64_t at = 24;
  for (uint32_t i = 0; i < pieces; ++i) {
    if (at + 7 > n) fail(NB_ERR_ARCHIVE, "tokenizer blob is malformed: truncated piece");
    if (p[at + 4] > 4) fail(NB_ERR_ARCHIVE, "tokenizer blob is malformed: unknown piece type");
    uint16_t len;
    std::memcpy(&len, p + at + 5, 2);
    if (at + 7 + len > n) fail(NB_ERR_ARCHIVE, "tokenizer blob is malformed: truncated piece text");
    at += 7 + len;
  }
}

}  // namespace nba
