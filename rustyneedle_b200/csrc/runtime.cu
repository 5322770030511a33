// runtime.cu — host runtime and C ABI of the B200 Needle-3 token loop.
//
// An Engine owns one opened archive on one GPU: the device weights, the KV
// page pool, the session slots and the forward-pass workspace, all driven on
// one CUDA stream. nb_model handles (Model::open, Model::with_depth) share an
// Engine and differ only in their active layers; sessions are slots of the
// Engine; batches capture one greedy decode step as a CUDA graph.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/needle_b200.h"
#include "archive.h"
#include "expf_table.h"
#include "kernels.h"
#include "layout.h"

using namespace nbl;

namespace nbr {

thread_local std::string g_error;

struct Failure {
  nb_status status;
  std::string message;
};

[[noreturn]] void fail(nb_status s, const std::string& m) { throw Failure{s, m}; }

#define NB_CUDA(call)                                                                                          \
  do {                                                                                                         \
    cudaError_t e_ = (call);                                                                                   \
    if (e_ != cudaSuccess) ::nbr::fail(NB_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));      \
  } while (0)

template <typename F>
nb_status guard(F&& f) {
  try {
    f();
    return NB_OK;
  } catch (const Failure& e) {
    g_error = e.message;
    return e.status;
  } catch (const nba::ArchiveError& e) {
    g_error = e.message;
    return (nb_status)e.status;
  } catch (const std::bad_alloc&) {
    g_error = "host allocation failed";
    return NB_ERR_ARGUMENT;
  } catch (const std::exception& e) {
    g_error = e.what();
    return NB_ERR_ARGUMENT;
  }
}

// ------------------------------------------------------------ level tables
// crates/kernels/src/codebook.rs:1-43 and matrix.rs:499-514
struct Levels {
  uint32_t bits = 0;  // lookup width (ternary crumbs read as 2 bits)
  float values[16] = {0};
  int8_t ints[16] = {0};  // IntegerLevels::table (neon.rs:114-123)
  float int_scale = 1.0f;
  bool fused = false;  // 2-bit panels: fma combine (panel.rs:184-187)
};

Levels levels_for(uint32_t record_bits, const std::vector<float>& cb, uint32_t group) {
  Levels L;
  auto copy = [&](size_t from, size_t n) {
    if (cb.size() < from + n) fail(NB_ERR_ARCHIVE, "codebook is shorter than 28 values");
    for (size_t i = 0; i < n; ++i) L.values[i] = cb[from + i];
  };
  switch (record_bits) {
    case 2:
      L.bits = 2;
      copy(0, 4);
      L.fused = group % 16 == 0;
      break;
    case 4:
      L.bits = 4;
      copy(12, 16);
      break;
    case 5: {
      float level = 1.2240064f / std::sqrt((float)group);
      L.bits = 2;
      L.values[1] = level;
      L.values[3] = -level;
      break;
    }
    default:
      fail(NB_ERR_UNSUPPORTED, "codebook width " + std::to_string(record_bits) +
                                   " runs on the reference's float kernel, which this build does not implement");
  }
  if ((L.bits == 2 && group % 64 != 0) || (L.bits == 4 && group % 32 != 0))
    fail(NB_ERR_UNSUPPORTED, "group size " + std::to_string(group) + " has no integer kernel in the reference");
  uint32_t count = 1u << L.bits;
  float peak = 0.0f;
  for (uint32_t i = 0; i < count; ++i) peak = std::fmax(peak, std::fabs(L.values[i]));
  L.int_scale = peak > 0.0f ? peak / 127.0f : 1.0f;
  for (uint32_t i = 0; i < count; ++i) L.ints[i] = (int8_t)std::round(L.values[i] / L.int_scale);
  return L;
}

static inline uint32_t code_at(const uint8_t* row, uint64_t i, uint32_t bits) {
  uint64_t bit = i * bits, byte = bit >> 3, shift = bit & 7;
  uint32_t raw = row[byte];
  if (shift + bits > 8) raw |= (uint32_t)row[byte + 1] << 8;
  return (raw >> shift) & ((1u << bits) - 1);
}

// ----------------------------------------------------------------- engine
struct Engine;

struct DeviceArena {
  std::vector<void*> blocks;
  ~DeviceArena() {
    for (void* p : blocks) cudaFree(p);
  }
  template <typename T>
  T* alloc(size_t count) {
    void* p = nullptr;
    size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) fail(NB_ERR_CUDA, "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    blocks.push_back(p);
    return static_cast<T*>(p);
  }
  template <typename T>
  T* upload(const std::vector<T>& v, cudaStream_t st) {
    T* p = alloc<T>(v.size());
    if (!v.empty()) NB_CUDA(cudaMemcpyAsync(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, st));
    return p;
  }
};

struct PinnedBuffer {
  void* p = nullptr;
  size_t bytes = 0;
  ~PinnedBuffer() {
    if (p) cudaFreeHost(p);
  }
  void ensure(size_t n) {
    if (n <= bytes) return;
    if (p) cudaFreeHost(p);
    p = nullptr;
    NB_CUDA(cudaMallocHost(&p, n));
    bytes = n;
  }
  template <typename T>
  T* as() {
    return static_cast<T*>(p);
  }
};

// A batched step can split its sequences into up to this many groups whose
// forward passes run as independent chains of the step's graph (see
// step_groups for the default).
constexpr int MAX_STEP_GROUPS = 8;

struct Engine {
  int device = 0;
  cudaStream_t stream = nullptr, side = nullptr;
  cudaStream_t group_streams[MAX_STEP_GROUPS] = {};
  std::mutex mutex;
  nba::Geometry geo;
  ModelDev md{};
  std::vector<LayerDev> layers;
  DeviceArena arena;
  // sessions and KV pages
  uint32_t max_sessions = 0, max_pages = 0, num_pages = 0;
  uint8_t* pool = nullptr;
  int32_t* d_page_table = nullptr;
  PinnedBuffer h_table;               // pinned mirror: [slots][layers][max_pages] int32
  bool copies_in_flight = false;      // asynchronous copies still read pinned staging memory
  std::vector<uint32_t> refcount;     // per physical page
  std::vector<uint32_t> free_pages;
  std::vector<uint32_t> free_slots;
  std::vector<uint8_t> slot_dirty;
  // per slot: the page index whose page is private to the slot at every layer
  // of its session (-1: not known); sharing a page (a clone) or releasing the
  // slot forgets it
  std::vector<int32_t> slot_private;
  float* d_hidden = nullptr;  // [slots][d]
  size_t conv_ring_floats = 0;  // per slot: md.conv_ring's [layers][taps - 1][q | k | v]
  std::vector<EngramDev> engram_sites;  // host copies (the layers point at the device copies)
  std::vector<HeadDev> heads;           // host copies of md.heads
  std::vector<CrossLayerDev> cross_layers;  // Whistle: host copies of md.cross
  float position_gate = 0.0f;               // sigmoid of the archive's position gate
  uint32_t text_vocab = 0;
  const CrossMemDev** d_slot_cross = nullptr;  // md.slot_cross
  const CrossLayerDev* cross_of(int layer) const { return cross_layers.empty() ? nullptr : &cross_layers[layer]; }
  uint32_t act_groups = 0;  // act_scale floats per token: the widest product's groups
  // probe heads: (head, probe) pairs, the widest projection K, the most slots per session
  uint32_t head_pairs = 0, head_k = 0;
  size_t head_slots = 0;
  int32_t* d_head_rows = nullptr;
  float *d_head_readouts = nullptr, *d_head_weights = nullptr, *d_head_pooled = nullptr, *d_head_scale = nullptr, *d_head_out = nullptr;
  int8_t* d_head_act = nullptr;
  PinnedBuffer h_head;
  // forward workspace
  uint32_t capacity = 0;
  Work work{};
  uint32_t* d_tokens = nullptr;
  TokenMeta* d_meta = nullptr;
  PinnedBuffer h_tokens, h_meta, h_misc, h_error;
  // logits of single-session calls
  int8_t* d_logit_act = nullptr;
  float* d_logit_scale = nullptr;
  float* d_logits = nullptr;  // [max_sessions][V]
  int32_t* d_slots = nullptr;
  uint32_t* d_next = nullptr;
  float* d_peaks = nullptr;
  float* d_stats = nullptr;
  uint32_t* d_mask = nullptr;
  int32_t* d_active = nullptr;
  int* d_error = nullptr;  // set by a device wait that gave up
  int t_cap = 0;

  KvDev kv() const { return KvDev{pool, d_page_table, max_pages, geo.num_layers}; }
  const EngramDev* engram_of(int layer) const {
    const int site = layers[layer].engram_site;
    return site >= 0 ? &engram_sites[site] : nullptr;
  }

  ~Engine() {
    if (device >= 0) cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    if (side) cudaStreamDestroy(side);
    for (cudaStream_t g : group_streams)
      if (g) cudaStreamDestroy(g);
    if (stream) cudaStreamDestroy(stream);
  }

  int32_t& page_entry(uint32_t slot, uint32_t layer, uint32_t index) {
    return h_table.as<int32_t>()[((size_t)slot * geo.num_layers + layer) * max_pages + index];
  }

  // Waits until no queued copy still reads the pinned staging buffers, so the
  // host may rewrite them.
  void settle() {
    if (copies_in_flight) {
      NB_CUDA(cudaStreamSynchronize(stream));
      copies_in_flight = false;
    }
  }

  uint32_t take_page() {
    if (free_pages.empty()) fail(NB_ERR_KV_EXHAUSTED, "the KV page pool is exhausted (" + std::to_string(num_pages) + " pages)");
    uint32_t p = free_pages.back();
    free_pages.pop_back();
    refcount[p] = 1;
    return p;
  }

  void drop_page(int32_t p) {
    if (p < 0) return;
    if (--refcount[p] == 0) free_pages.push_back((uint32_t)p);
  }

  // Makes the page that receives `position` of every active layer private to `slot`.
  void prepare_append(uint32_t slot, const std::vector<int32_t>& active, uint32_t position) {
    const uint32_t index = position / PAGE_POSITIONS;
    if (slot_private[slot] == (int32_t)index) return;  // most steps: nothing to allocate or copy
    settle();
    for (int32_t layer : active) {
      int32_t& e = page_entry(slot, (uint32_t)layer, index);
      if (e < 0) {
        e = (int32_t)take_page();
        slot_dirty[slot] = 1;
      } else if (refcount[e] > 1) {
        uint32_t fresh = take_page();
        NB_CUDA(cudaMemcpyAsync(pool + (size_t)fresh * md.page.page_bytes, pool + (size_t)e * md.page.page_bytes, md.page.page_bytes,
                                cudaMemcpyDeviceToDevice, stream));
        --refcount[e];
        e = (int32_t)fresh;
        slot_dirty[slot] = 1;
      }
    }
    slot_private[slot] = (int32_t)index;
  }

  void flush_page_tables() {
    size_t row = (size_t)geo.num_layers * max_pages;
    for (uint32_t s = 0; s < max_sessions; ++s) {
      if (!slot_dirty[s]) continue;
      NB_CUDA(cudaMemcpyAsync(d_page_table + s * row, h_table.as<int32_t>() + s * row, row * 4, cudaMemcpyHostToDevice, stream));
      copies_in_flight = true;
      slot_dirty[s] = 0;
    }
  }
};

// Path of the libm-exception table: $NEEDLE_B200_EXPF_TABLE, else beside this library.
static std::string expf_table_path() {
  if (const char* env = std::getenv("NEEDLE_B200_EXPF_TABLE")) return env;
  Dl_info info;
  if (dladdr(reinterpret_cast<void*>(&expf_table_path), &info) && info.dli_fname) {
    std::string so = info.dli_fname;
    size_t slash = so.rfind('/');
    return (slash == std::string::npos ? std::string(".") : so.substr(0, slash)) + "/glibc_expf_exceptions.bin";
  }
  return "glibc_expf_exceptions.bin";
}

static std::mutex g_table_mutex;
static std::shared_ptr<nbx::ExpfTable> g_table;
static std::map<int, nbx::ExceptionSet> g_device_exceptions;  // never freed: a device constant points at it

static std::shared_ptr<nbx::ExpfTable> load_expf_table() {
  std::lock_guard<std::mutex> lock(g_table_mutex);
  if (g_table) return g_table;
  auto table = std::make_shared<nbx::ExpfTable>();
  std::string path = expf_table_path();
  if (!nbx::read_expf_table(path.c_str(), *table) || !nbx::verify_expf_table(*table)) {
    *table = nbx::scan_expf_exceptions(0);
    if (table->unexplained) fail(NB_ERR_UNSUPPORTED, "the host expf has mismatches the device exponential cannot reproduce");
    try {
      nbx::write_expf_table(path.c_str(), *table);
    } catch (...) {
    }
  }
  g_table = table;
  return table;
}

// The exception set's hash slots on `device` (uploaded once per process).
static nbx::ExceptionSet device_exception_set(int device) {
  auto table = load_expf_table();
  std::lock_guard<std::mutex> lock(g_table_mutex);
  auto it = g_device_exceptions.find(device);
  if (it != g_device_exceptions.end()) return it->second;
  uint32_t mask = 0;
  const std::vector<uint32_t> slots = nbx::hash_slots(*table, mask);
  uint32_t* d_slots = nullptr;
  NB_CUDA(cudaMalloc(&d_slots, slots.size() * 4));
  NB_CUDA(cudaMemcpy(d_slots, slots.data(), slots.size() * 4, cudaMemcpyHostToDevice));
  const nbx::ExceptionSet set{d_slots, mask};
  g_device_exceptions.emplace(device, set);
  return set;
}

// Expands a codebook matrix to int8 through the integer level table, in the
// tensor-core core-matrix layout (rows padded to 128-row tiles) or row-major.
static void expand_matrix(const nba::Archive& a, uint32_t index, const Levels& lv, bool core, std::vector<int8_t>& codes,
                          std::vector<float>& scales, uint32_t row_offset, uint32_t total_rows) {
  const nba::Record& r = a.record(index);
  uint64_t rows = r.rows(), cols = r.padded_columns(), groups = r.groups_per_row(), rb = r.packed_row_bytes();
  const uint8_t* packed = a.data(index);
  const uint8_t* norms = packed + r.packed_bytes();
  if (r.packed_bytes() + rows * groups * 2 > r.byte_len) fail(NB_ERR_ARCHIVE, "codebook tensor " + std::to_string(index) + " is shorter than its shape");
  const uint64_t stored_rows = core ? (total_rows + 127) / 128 * 128 : total_rows;
  if (codes.size() < stored_rows * cols) codes.resize(stored_rows * cols, 0);
  if (scales.size() < (size_t)total_rows * groups) scales.resize((size_t)total_rows * groups, 0.0f);
  for (uint64_t row = 0; row < rows; ++row) {
    const uint8_t* src = packed + row * rb;
    const uint64_t out_row = row + row_offset;
    for (uint64_t c = 0; c < cols; ++c) {
      int8_t v = lv.ints[code_at(src, c, lv.bits)];
      codes[core ? chunked_offset(out_row, (uint32_t)c, stored_rows) : out_row * cols + c] = v;
    }
    for (uint64_t g = 0; g < groups; ++g) {
      uint16_t h;
      std::memcpy(&h, norms + 2 * (row * groups + g), 2);
      float norm = nba::half_to_f32(h);
      scales[(row + row_offset) * groups + g] = lv.fused ? norm * lv.int_scale : norm;
    }
  }
}

static void check_matrix(const nba::Archive& a, uint32_t index, uint64_t rows, uint64_t cols, const char* what) {
  const nba::Record& r = a.record(index);
  if (r.kind != nba::CODEBOOK) fail(NB_ERR_ARCHIVE, std::string(what) + " is not codebook-quantised");
  if (r.rows() != rows || r.columns() != cols || r.group() != GROUP)
    fail(NB_ERR_UNSUPPORTED, std::string(what) + " has shape " + std::to_string(r.rows()) + "x" + std::to_string(r.columns()) +
                                 " group " + std::to_string(r.group_size));
}

static std::vector<float> floats_of(const nba::Archive& a, uint32_t index, size_t expected, const char* what) {
  std::vector<float> v = a.floats(index);
  if (expected && v.size() < expected) fail(NB_ERR_ARCHIVE, std::string(what) + " holds " + std::to_string(v.size()) + " values, expected " + std::to_string(expected));
  return v;
}

std::shared_ptr<Engine> open_engine(const char* path, const nb_options* opt) {
  nba::Archive a(path);
  nba::Layout lay = a.resolve();
  a.validate_tokenizer(lay.tokenizer);
  const nba::Geometry& g = a.geometry();
  if (g.qkv_conv_taps > 64) fail(NB_ERR_UNSUPPORTED, "more than 64 qkv conv taps are not implemented");
  uint32_t max_order = 0;
  if (!g.engram_sites.empty()) {
    if (g.engram_orders.empty() || g.engram_tables == 0 || g.engram_tables % g.engram_orders.size() || g.engram_slots == 0)
      fail(NB_ERR_ARCHIVE, "engram tables are not a whole number per order");
    if (g.engram_tables > 16) fail(NB_ERR_UNSUPPORTED, "more than 16 engram tables are not implemented");
    if (g.engram_sub_dim == 0 || g.engram_sub_dim % GROUP || g.engram_tables * g.engram_sub_dim > 2048)
      fail(NB_ERR_UNSUPPORTED, "engram rows must be whole 128-groups, at most 2048 values in all");
    if (g.engram_conv_taps == 0 || g.engram_conv_taps > 16) fail(NB_ERR_UNSUPPORTED, "engram value taps must number 1 to 16");
    for (uint32_t o : g.engram_orders) max_order = std::max(max_order, o);
    if (max_order > 64) fail(NB_ERR_UNSUPPORTED, "engram orders above 64 are not implemented");
    for (uint32_t site : g.engram_sites)
      if (site >= g.num_layers) fail(NB_ERR_ARCHIVE, "an engram site names a layer the model does not have");
  }
  if (g.mhc_lanes != LANES) fail(NB_ERR_UNSUPPORTED, "only 4-lane models are implemented");
  if (g.qk_head_dim != HEAD_DIM || g.v_head_dim != HEAD_DIM) fail(NB_ERR_UNSUPPORTED, "head dims other than 64 are not implemented");
  if (g.d_model != 512)
    fail(NB_ERR_UNSUPPORTED, "d_model " + std::to_string(g.d_model) + " is not implemented (the tensor-core products take K = 512)");
  if (g.num_kv_heads == 0 || g.num_heads % g.num_kv_heads || g.num_heads / g.num_kv_heads > 4 ||
      (g.num_heads / g.num_kv_heads == 3) || g.num_heads > MAX_HEADS || g.num_heads * HEAD_DIM != g.d_model)
    fail(NB_ERR_UNSUPPORTED, "head layout is not implemented");
  if (g.hada_n != 2048 && g.hada_n != 1024) fail(NB_ERR_UNSUPPORTED, "hada_n must be 1024 or 2048");
  if (g.max_seq_len == 0 || g.max_seq_len > 8192) fail(NB_ERR_UNSUPPORTED, "max_seq_len must be in 1..8192");
  if (g.output_vocab() > g.vocab || g.output_vocab() % 32 || g.output_vocab() > 8192)
    fail(NB_ERR_UNSUPPORTED, "output vocab must be a multiple of 32 up to 8192");

  auto E = std::make_shared<Engine>();
  E->geo = g;
  int device = opt && opt->device >= 0 ? opt->device : -1;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) fail(NB_ERR_NO_DEVICE, "no CUDA device is visible");
  if (device < 0) NB_CUDA(cudaGetDevice(&device));
  if (device >= count) fail(NB_ERR_ARGUMENT, "device ordinal out of range");
  E->device = device;
  NB_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  NB_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) fail(NB_ERR_NO_DEVICE, std::string("this build targets sm_100a; device is ") + prop.name);
  NB_CUDA(cudaStreamCreateWithFlags(&E->stream, cudaStreamNonBlocking));
  NB_CUDA(cudaStreamCreateWithFlags(&E->side, cudaStreamNonBlocking));
  for (cudaStream_t& g : E->group_streams) NB_CUDA(cudaStreamCreateWithFlags(&g, cudaStreamNonBlocking));
  cudaStream_t st = E->stream;
  DeviceArena& A = E->arena;

  // libm-compatible exponential: the kernels read the exception set through a
  // per-device constant, so its device copy is one per device for the whole
  // process (every engine on the device uses the same table)
  const nbx::ExceptionSet exceptions = device_exception_set(device);
  nbx::ExpConstants constants = nbx::make_exp_constants();
  nbk::set_exp_constants(constants, exceptions, st);
  NB_CUDA(cudaGetLastError());

  const uint32_t d = g.d_model, H = g.num_heads, KV = g.num_kv_heads, L = g.num_layers, N = g.hada_n;
  const uint32_t qkvg_rows = 2 * H * HEAD_DIM + 2 * KV * HEAD_DIM;
  ModelDev& md = E->md;
  md.d_model = d;
  md.heads = H;
  md.kv_heads = KV;
  md.vocab = g.vocab;
  md.output_vocab = g.output_vocab();
  md.hada_n = N;
  md.hada_left = N / 32;
  md.max_seq_len = g.max_seq_len;
  md.num_layers = L;
  md.sliding_window = g.sliding_window;
  md.conv_taps = g.qkv_conv_taps;
  md.qkv_width = (H + 2 * KV) * HEAD_DIM;
  EngramConfig ecfg{};
  if (!g.engram_sites.empty()) {
    ecfg.slots = g.engram_slots;
    ecfg.sub_dim = g.engram_sub_dim;
    ecfg.tables = g.engram_tables;
    ecfg.orders = (uint32_t)g.engram_orders.size();
    ecfg.heads_per_order = g.engram_tables / ecfg.orders;
    ecfg.stride = g.engram_seed_heads ? g.engram_seed_heads : ecfg.heads_per_order;
    for (uint32_t i = 0; i < ecfg.orders; ++i) ecfg.order[i] = g.engram_orders[i];
    ecfg.conv_taps = g.engram_conv_taps;
    ecfg.dilation = g.engram_conv_dilation;
    ecfg.ring_rows = (g.engram_conv_taps - 1) * g.engram_conv_dilation;
    ecfg.k = g.engram_tables * g.engram_sub_dim <= 512 ? 512 : 2048;
    md.token_rows = max_order - 1;
  }
  md.sqrt_d = std::sqrt((float)d);
  md.inv_sqrt_group = 1.0f / std::sqrt((float)GROUP);
  md.inv_root_qk = 1.0f / std::sqrt((float)HEAD_DIM);
  md.page = page_geometry(KV);

  // embedding: packed rows for the gather, int8 rows for the tied logits
  check_matrix(a, lay.embedding, g.vocab, d, "the embedding");
  const nba::Record& er = a.record(lay.embedding);
  Levels elv = levels_for(er.bits, a.codebook(), er.group_size);
  {
    std::vector<uint8_t> packed(a.data(lay.embedding), a.data(lay.embedding) + er.packed_bytes());
    md.embed_packed = A.upload(packed, st);
    md.embed_bits = elv.bits;
    md.embed_row_bytes = (uint32_t)er.packed_row_bytes();
    md.embed_levels = A.upload(std::vector<float>(elv.values, elv.values + 16), st);
    std::vector<float> norms((size_t)g.vocab * (d / GROUP));
    const uint8_t* nb = a.data(lay.embedding) + er.packed_bytes();
    for (size_t i = 0; i < norms.size(); ++i) {
      uint16_t h;
      std::memcpy(&h, nb + 2 * i, 2);
      norms[i] = nba::half_to_f32(h);
    }
    md.embed_norms = A.upload(norms, st);
    std::vector<int8_t> codes;
    std::vector<float> scales;
    expand_matrix(a, lay.embedding, elv, true, codes, scales, 0, g.vocab);
    // only the first output_vocab rows take part in the logits (session.rs:174-175)
    md.logits = QMat{A.upload(codes, st), A.upload(scales, st), elv.int_scale, md.output_vocab, d, d / GROUP, elv.fused ? 1 : 0};
  }
  // lanes
  {
    const uint32_t n = LANES * d;
    auto phi = [&](uint32_t index, uint32_t rows, const char* what) {
      check_matrix(a, index, rows, n, what);
      const nba::Record& r = a.record(index);
      Levels lv = levels_for(r.bits, a.codebook(), r.group_size);
      if (lv.fused) fail(NB_ERR_UNSUPPORTED, std::string(what) + " is 2-bit; the lane maps are implemented for 4-bit codes");
      std::vector<int8_t> codes;
      std::vector<float> scales;
      expand_matrix(a, index, lv, false, codes, scales, 0, rows);
      return QMat{A.upload(codes, st), A.upload(scales, st), lv.int_scale, rows, n, n / GROUP, 0};
    };
    md.phi_pre = phi(lay.lanes.phi_pre, L * LANES, "phi_pre");
    md.phi_post = phi(lay.lanes.phi_post, L * LANES, "phi_post");
    md.phi_res = phi(lay.lanes.phi_res, L * LANES * LANES, "phi_res");
    md.a_pre = A.upload(floats_of(a, lay.lanes.a_pre, L, "a_pre"), st);
    md.a_post = A.upload(floats_of(a, lay.lanes.a_post, L, "a_post"), st);
    md.a_res = A.upload(floats_of(a, lay.lanes.a_res, L, "a_res"), st);
    md.b_pre = A.upload(floats_of(a, lay.lanes.b_pre, L * LANES, "b_pre"), st);
    md.b_post = A.upload(floats_of(a, lay.lanes.b_post, L * LANES, "b_post"), st);
    md.b_res = A.upload(floats_of(a, lay.lanes.b_res, L * LANES * LANES, "b_res"), st);
  }
  md.final_norm = A.upload(floats_of(a, lay.final_norm, d, "final_norm"), st);
  for (int which = 0; which < 2; ++which) {
    std::vector<float> p = floats_of(a, lay.perms[which], N, "hadamard permutation");
    std::vector<int32_t> perm(N);
    for (uint32_t i = 0; i < N; ++i) {
      if (!(p[i] >= 0.0f) || p[i] >= (float)N) fail(NB_ERR_ARCHIVE, "hadamard permutation entry out of range");
      perm[i] = (int32_t)p[i];
    }
    (which == 0 ? md.perm1 : md.perm2) = A.upload(perm, st);
  }
  // rotary table: angle = position as f32 * frequency (ops.rs:127-141), sin/cos of the host libm
  {
    std::vector<float> freq(HEAD_DIM / 2);
    for (int i = 0; i < HEAD_DIM / 2; ++i) freq[i] = 1.0f / std::pow(g.rope_theta, 2.0f * (float)i / (float)HEAD_DIM);
    std::vector<float2> rot((size_t)g.max_seq_len * (HEAD_DIM / 2));
    for (uint32_t p = 0; p < g.max_seq_len; ++p)
      for (int i = 0; i < HEAD_DIM / 2; ++i) {
        float angle = (float)p * freq[i];
        rot[(size_t)p * (HEAD_DIM / 2) + i] = make_float2(std::sin(angle), std::cos(angle));
      }
    md.rotary = A.upload(rot, st);
  }
  // layers
  for (uint32_t l = 0; l < L; ++l) {
    const nba::LayerIdx& t = lay.layers[l];
    LayerDev D{};
    check_matrix(a, t.q, H * HEAD_DIM, d, "q_proj");
    check_matrix(a, t.k, KV * HEAD_DIM, d, "k_proj");
    check_matrix(a, t.v, KV * HEAD_DIM, d, "v_proj");
    check_matrix(a, t.gate, H * HEAD_DIM, d, "gate_proj");
    check_matrix(a, t.out, d, H * HEAD_DIM, "out_proj");
    Levels lq = levels_for(a.record(t.q).bits, a.codebook(), GROUP);
    for (uint32_t m : {t.k, t.v, t.gate})
      if (levels_for(a.record(m).bits, a.codebook(), GROUP).fused != lq.fused)
        fail(NB_ERR_UNSUPPORTED, "q, k, v and gate projections must share one code width");
    std::vector<int8_t> codes;
    std::vector<float> scales;
    uint32_t offset = 0;
    for (uint32_t m : {t.q, t.k, t.v, t.gate}) {
      Levels lv = levels_for(a.record(m).bits, a.codebook(), GROUP);
      expand_matrix(a, m, lv, true, codes, scales, offset, qkvg_rows);
      offset += (uint32_t)a.record(m).rows();
    }
    D.qkvg = QMat{A.upload(codes, st), A.upload(scales, st), lq.int_scale, qkvg_rows, d, d / GROUP, lq.fused ? 1 : 0};
    Levels lo = levels_for(a.record(t.out).bits, a.codebook(), GROUP);
    codes.clear();
    scales.clear();
    expand_matrix(a, t.out, lo, true, codes, scales, 0, d);
    D.out = QMat{A.upload(codes, st), A.upload(scales, st), lo.int_scale, d, H * HEAD_DIM, (H * HEAD_DIM) / GROUP, lo.fused ? 1 : 0};
    D.norm_in = A.upload(floats_of(a, t.norm_in, d, "norm_in"), st);
    D.post_norm = A.upload(floats_of(a, t.post_norm, d, "post_norm"), st);
    D.pre_hada = A.upload(floats_of(a, t.pre_hada, d, "pre_hada"), st);
    D.q_norm = A.upload(floats_of(a, t.q_norm, HEAD_DIM, "q_norm"), st);
    D.k_norm = A.upload(floats_of(a, t.k_norm, HEAD_DIM, "k_norm"), st);
    D.attn_gate = floats_of(a, t.attn_gate, 1, "attn_gate")[0];
    const nba::HadamardIdx& h = t.hada;
    HadamardDev& HD = D.hada;
    HD.d1 = A.upload(floats_of(a, h.d1, N, "d1"), st);
    HD.d2 = A.upload(floats_of(a, h.d2, N, "d2"), st);
    HD.b2 = A.upload(floats_of(a, h.b2, N, "b2"), st);
    HD.d3 = A.upload(floats_of(a, h.d3, N, "d3"), st);
    HD.d4 = A.upload(floats_of(a, h.d4, N, "d4"), st);
    uint32_t pairs[3][2] = {{h.w1a, h.w1b}, {h.w2a, h.w2b}, {h.w3a, h.w3b}};
    for (int i = 0; i < 3; ++i) {
      std::vector<float> left = a.floats(pairs[i][0]), right = a.floats(pairs[i][1]);
      size_t ls = (size_t)std::llround(std::sqrt((double)left.size())), rs = (size_t)std::llround(std::sqrt((double)right.size()));
      if (rs != HADA_RIGHT || ls != md.hada_left || ls * rs != N)
        fail(NB_ERR_UNSUPPORTED, "hadamard factors must be (hada_n/32)^2 and 32^2");
      HD.left[i] = A.upload(left, st);
      HD.right[i] = A.upload(right, st);
    }
    std::vector<float> cv = floats_of(a, h.cond_v, 0, "cond_v"), cu = floats_of(a, h.cond_u, 0, "cond_u");
    if (cu.size() != (size_t)COND_RANK * N || cv.size() != (size_t)COND_RANK * d)
      fail(NB_ERR_UNSUPPORTED, "the Hadamard condition must have rank 8");
    HD.cond_v = A.upload(cv, st);
    HD.cond_u = A.upload(cu, st);
    D.global = (g.sliding_window == 0 || g.is_global_layer(l)) ? 1 : 0;
    D.index = (int)l;
    if (t.has_taps) {
      // model/src/attention.rs:30: the q, k and v gains, [tap][width] each,
      // interleaved into [tap][q | k | v] to match a projection row
      const uint32_t widths[3] = {H * HEAD_DIM, KV * HEAD_DIM, KV * HEAD_DIM}, T = g.qkv_conv_taps;
      std::vector<float> taps((size_t)T * md.qkv_width);
      uint32_t at = 0;
      for (int i = 0; i < 3; ++i) {
        std::vector<float> gains = floats_of(a, t.taps[i], (size_t)T * widths[i], "conv taps");
        for (uint32_t k = 0; k < T; ++k)
          std::copy(gains.begin() + (size_t)k * widths[i], gains.begin() + (size_t)(k + 1) * widths[i], taps.begin() + (size_t)k * md.qkv_width + at);
        at += widths[i];
      }
      D.taps = A.upload(taps, st);
    }
    E->layers.push_back(D);
  }

  // engram sites (engram.rs:19-28): tables as packed rows for the gather,
  // key_proj and value_proj as one product, value taps
  std::vector<EngramDev> sites;
  for (size_t si = 0; si < g.engram_sites.size(); ++si) {
    const std::array<uint32_t, 4>& e = lay.engrams.at(si);
    EngramDev S{};
    S.cfg = ecfg;
    const nba::Record& tr = a.record(e[0]);
    if (tr.kind != nba::CODEBOOK || tr.rows() < (uint64_t)g.engram_tables * g.engram_slots || tr.columns() != g.engram_sub_dim ||
        tr.group() != GROUP)
      fail(NB_ERR_UNSUPPORTED, "engram tables must be codebook rows of sub_dim values in 128-groups, tables x slots of them");
    Levels tl = levels_for(tr.bits, a.codebook(), GROUP);
    S.packed = A.upload(std::vector<uint8_t>(a.data(e[0]), a.data(e[0]) + tr.packed_bytes()), st);
    S.row_bytes = (uint32_t)tr.packed_row_bytes();
    S.bits = tl.bits;
    S.levels = A.upload(std::vector<float>(tl.values, tl.values + 16), st);
    {
      const uint64_t n = tr.rows() * tr.groups_per_row();
      if (tr.packed_bytes() + n * 2 > tr.byte_len) fail(NB_ERR_ARCHIVE, "engram tables are shorter than their shape");
      std::vector<float> norms(n);
      const uint8_t* nb = a.data(e[0]) + tr.packed_bytes();
      for (uint64_t i = 0; i < n; ++i) {
        uint16_t h;
        std::memcpy(&h, nb + 2 * i, 2);
        norms[i] = nba::half_to_f32(h);
      }
      S.norms = A.upload(norms, st);
    }
    const uint32_t K = g.engram_tables * g.engram_sub_dim, KP = ecfg.k, kg = K / GROUP, pg = KP / GROUP;
    check_matrix(a, e[1], d, K, "engram key_proj");
    check_matrix(a, e[2], d, K, "engram value_proj");
    Levels lk = levels_for(a.record(e[1]).bits, a.codebook(), GROUP);
    if (levels_for(a.record(e[2]).bits, a.codebook(), GROUP).fused != lk.fused)
      fail(NB_ERR_UNSUPPORTED, "engram key_proj and value_proj must share one code width");
    // K-chunk-major codes do not depend on the total K, so the padded columns
    // simply stay zero; the scales are re-strided to the padded groups
    std::vector<int8_t> codes((size_t)((2 * d + 127) / 128 * 128) * KP, 0);
    std::vector<float> scales;
    expand_matrix(a, e[1], lk, true, codes, scales, 0, 2 * d);
    expand_matrix(a, e[2], levels_for(a.record(e[2]).bits, a.codebook(), GROUP), true, codes, scales, d, 2 * d);
    std::vector<float> padded((size_t)2 * d * pg, 0.0f);
    for (uint32_t r = 0; r < 2 * d; ++r)
      for (uint32_t gi = 0; gi < kg; ++gi) padded[(size_t)r * pg + gi] = scales[(size_t)r * kg + gi];
    S.kv = QMat{A.upload(codes, st), A.upload(padded, st), lk.int_scale, 2 * d, KP, pg, lk.fused ? 1 : 0};
    S.taps = A.upload(floats_of(a, e[3], (size_t)g.engram_conv_taps * d, "engram taps"), st);
    sites.push_back(S);
  }

  // probe heads (heads.rs:29-50): directions and queries dequantised to f32
  // on the device, gains and biases, the projection as a product
  if (lay.heads.size() > (size_t)MAX_PROBE_HEADS) fail(NB_ERR_UNSUPPORTED, "more than 4 probe heads are not implemented");
  md.num_probe_heads = (uint32_t)lay.heads.size();
  E->heads.resize(lay.heads.size());
  for (size_t hi = 0; hi < lay.heads.size(); ++hi) {
    const nba::Layout::HeadIdx& t = lay.heads[hi];
    HeadDev& H = E->heads[hi];
    H.code = (int)t.code;
    auto dense = [&](uint32_t index, const char* what) {
      const nba::Record& r = a.record(index);
      if (r.kind != nba::CODEBOOK || r.columns() != d || r.group() != GROUP)
        fail(NB_ERR_UNSUPPORTED, std::string("probe head ") + what + " must be codebook rows of d_model values in 128-groups");
      Levels lv = levels_for(r.bits, a.codebook(), GROUP);
      const uint64_t n = r.rows() * r.groups_per_row();
      if (r.packed_bytes() + n * 2 > r.byte_len) fail(NB_ERR_ARCHIVE, std::string("probe head ") + what + " is shorter than its shape");
      std::vector<float> norms(n);
      const uint8_t* nb = a.data(index) + r.packed_bytes();
      for (uint64_t i = 0; i < n; ++i) {
        uint16_t h;
        std::memcpy(&h, nb + 2 * i, 2);
        norms[i] = nba::half_to_f32(h);
      }
      const uint8_t* packed = A.upload(std::vector<uint8_t>(a.data(index), a.data(index) + r.packed_bytes()), st);
      const float* levels = A.upload(std::vector<float>(lv.values, lv.values + 16), st);
      float* out = A.alloc<float>((size_t)r.rows() * d);
      nbk::dense_rows(packed, (uint32_t)r.packed_row_bytes(), lv.bits, levels, A.upload(norms, st), (int)r.rows(), (int)d, md.inv_sqrt_group,
                      out, st);
      return std::make_pair(out, (uint32_t)r.rows());
    };
    auto probes = dense(t.probes, "probes");
    if (probes.second % (L + 1)) fail(NB_ERR_ARCHIVE, "probe head rows are not a whole number per layer");
    H.probes = probes.second / (L + 1);
    H.directions = probes.first;
    auto query = dense(t.query, "query");
    H.queries = query.second;
    H.query = query.first;
    const uint32_t all = (L + 1) * H.probes, K = H.queries * d;
    H.gain = A.upload(floats_of(a, t.gain, all, "probe head gain"), st);
    H.row_bias = A.upload(floats_of(a, t.row_bias, (size_t)H.queries * all, "probe head row_bias"), st);
    const nba::Record& pr = a.record(t.proj);
    if (pr.kind != nba::CODEBOOK || pr.columns() != K || pr.group() != GROUP || K > 2048)
      fail(NB_ERR_UNSUPPORTED, "probe head projection must take queries x d_model <= 2048 columns in 128-groups");
    H.outputs = (uint32_t)pr.rows();
    if (H.outputs == 0 || H.outputs > 4096) fail(NB_ERR_UNSUPPORTED, "probe head projections of more than 4096 outputs are not implemented");
    Levels lp = levels_for(pr.bits, a.codebook(), GROUP);
    const uint32_t KP = K <= 512 ? 512 : 2048, kg = K / GROUP, pg = KP / GROUP;
    std::vector<int8_t> codes((size_t)((H.outputs + 127) / 128 * 128) * KP, 0);
    std::vector<float> scales;
    expand_matrix(a, t.proj, lp, true, codes, scales, 0, H.outputs);
    std::vector<float> padded((size_t)H.outputs * pg, 0.0f);
    for (uint32_t r = 0; r < H.outputs; ++r)
      for (uint32_t gi = 0; gi < kg; ++gi) padded[(size_t)r * pg + gi] = scales[(size_t)r * kg + gi];
    H.proj = QMat{A.upload(codes, st), A.upload(padded, st), lp.int_scale, H.outputs, KP, pg, lp.fused ? 1 : 0};
    H.bias = A.upload(floats_of(a, t.bias, H.outputs, "probe head bias"), st);
  }

  // Whistle cross attention (CrossWeights::load, whistle/src/cross.rs:38-56)
  if (lay.audio) {
    if (lay.cross.size() != L) fail(NB_ERR_ARCHIVE, "the audio section does not carry cross attention for every decoder layer");
    auto stacked = [&](uint32_t first_idx, uint32_t second_idx, const char* what) {
      check_matrix(a, first_idx, H * HEAD_DIM, d, what);
      check_matrix(a, second_idx, H * HEAD_DIM, d, what);
      Levels l1 = levels_for(a.record(first_idx).bits, a.codebook(), GROUP), l2 = levels_for(a.record(second_idx).bits, a.codebook(), GROUP);
      if (l1.fused != l2.fused) fail(NB_ERR_UNSUPPORTED, std::string(what) + ": both products must share one code width");
      std::vector<int8_t> codes;
      std::vector<float> scales;
      expand_matrix(a, first_idx, l1, true, codes, scales, 0, 2 * H * HEAD_DIM);
      expand_matrix(a, second_idx, l2, true, codes, scales, H * HEAD_DIM, 2 * H * HEAD_DIM);
      return QMat{A.upload(codes, st), A.upload(scales, st), l1.int_scale, 2 * H * HEAD_DIM, d, d / GROUP, l1.fused ? 1 : 0};
    };
    auto sig = [](float v) { return 1.0f / (1.0f + std::exp(-v)); };  // ops.rs:69-71 in f32
    for (uint32_t l = 0; l < L; ++l) {
      const std::array<uint32_t, 10>& c = lay.cross[l];
      CrossLayerDev C{};
      C.norm = A.upload(floats_of(a, c[0], d, "cross norm"), st);
      C.qg = stacked(c[1], c[4], "cross q/gate");
      C.kv = stacked(c[2], c[3], "cross k/v");
      check_matrix(a, c[5], d, H * HEAD_DIM, "cross out_proj");
      Levels lo = levels_for(a.record(c[5]).bits, a.codebook(), GROUP);
      std::vector<int8_t> codes;
      std::vector<float> scales;
      expand_matrix(a, c[5], lo, true, codes, scales, 0, d);
      C.out = QMat{A.upload(codes, st), A.upload(scales, st), lo.int_scale, d, H * HEAD_DIM, (H * HEAD_DIM) / GROUP, lo.fused ? 1 : 0};
      C.q_norm = A.upload(floats_of(a, c[6], HEAD_DIM, "cross q_norm"), st);
      C.k_norm = A.upload(floats_of(a, c[7], HEAD_DIM, "cross k_norm"), st);
      C.post_norm = A.upload(floats_of(a, c[8], d, "cross post_norm"), st);
      C.gain = sig(floats_of(a, c[9], 1, "cross gate")[0]);
      E->cross_layers.push_back(C);
    }
    md.cross = A.upload(E->cross_layers, st);
    E->position_gate = sig(floats_of(a, lay.position_gate, 1, "position gate")[0]);
    E->text_vocab = lay.text_vocab;
  }

  // sessions, KV pool, workspace
  E->max_sessions = opt && opt->max_sessions ? opt->max_sessions : 256;
  E->max_pages = (g.max_seq_len + PAGE_POSITIONS - 1) / PAGE_POSITIONS;
  uint64_t default_pages = (uint64_t)E->max_sessions * L * E->max_pages;
  size_t free_bytes = 0, total_bytes = 0;
  NB_CUDA(cudaMemGetInfo(&free_bytes, &total_bytes));
  uint64_t cap_pages = (uint64_t)(free_bytes * 0.6) / md.page.page_bytes;
  E->num_pages = (uint32_t)(opt && opt->kv_pages ? opt->kv_pages : std::min<uint64_t>(default_pages, cap_pages));
  if (E->num_pages == 0) fail(NB_ERR_ARGUMENT, "the KV pool holds no page");
  E->pool = A.alloc<uint8_t>((size_t)E->num_pages * md.page.page_bytes);
  E->refcount.assign(E->num_pages, 0);
  for (uint32_t p = E->num_pages; p-- > 0;) E->free_pages.push_back(p);
  const size_t table_entries = (size_t)E->max_sessions * L * E->max_pages;
  E->h_table.ensure(table_entries * 4);
  std::fill(E->h_table.as<int32_t>(), E->h_table.as<int32_t>() + table_entries, -1);
  E->d_page_table = A.alloc<int32_t>(table_entries);
  NB_CUDA(cudaMemcpyAsync(E->d_page_table, E->h_table.p, table_entries * 4, cudaMemcpyHostToDevice, st));
  E->slot_dirty.assign(E->max_sessions, 0);
  E->slot_private.assign(E->max_sessions, -1);
  for (uint32_t s = E->max_sessions; s-- > 0;) E->free_slots.push_back(s);
  E->d_hidden = A.alloc<float>((size_t)E->max_sessions * d);
  NB_CUDA(cudaMemsetAsync(E->d_hidden, 0, (size_t)E->max_sessions * d * 4, st));
  for (uint32_t hi = 0; hi < md.num_probe_heads; ++hi) {  // ProbeAccumulator (heads.rs:151-156) per slot
    HeadDev& H = E->heads[hi];
    const size_t all = (size_t)(L + 1) * H.probes;
    H.peak = A.alloc<float>(E->max_sessions * all);
    H.total = A.alloc<float>(E->max_sessions * all);
    H.weighted = A.alloc<float>(E->max_sessions * all * d);
    E->head_pairs += H.probes;
    E->head_k = std::max<uint32_t>(E->head_k, H.proj.cols);
    E->head_slots = std::max<size_t>(E->head_slots, all);
  }
  if (md.num_probe_heads) {
    md.probe_heads = A.upload(E->heads, st);
    E->d_head_rows = A.alloc<int32_t>(L + 1);
    E->d_head_readouts = A.alloc<float>(E->head_slots * d);
    E->d_head_weights = A.alloc<float>(E->head_slots);
    E->d_head_pooled = A.alloc<float>(E->head_k);
    E->d_head_act = A.alloc<int8_t>((size_t)128 * E->head_k);
    NB_CUDA(cudaMemsetAsync(E->d_head_act, 0, (size_t)128 * E->head_k, st));
    E->d_head_scale = A.alloc<float>(E->head_k / GROUP);
    NB_CUDA(cudaMemsetAsync(E->d_head_scale, 0, (E->head_k / GROUP) * 4, st));
    E->d_head_out = A.alloc<float>(std::max<size_t>(E->head_k, 4096));
    E->h_head.ensure(std::max<size_t>(E->head_k, 4096) * 4);
  }
  if (md.cross) {
    E->d_slot_cross = A.alloc<const CrossMemDev*>(E->max_sessions);
    NB_CUDA(cudaMemsetAsync(E->d_slot_cross, 0, E->max_sessions * sizeof(void*), st));
    md.slot_cross = E->d_slot_cross;
  }
  for (EngramDev& S : sites)
    if (ecfg.ring_rows) {
      S.ring = A.alloc<float>((size_t)E->max_sessions * ecfg.ring_rows * d);
      NB_CUDA(cudaMemsetAsync(S.ring, 0, (size_t)E->max_sessions * ecfg.ring_rows * d * 4, st));
    }
  const EngramDev* d_sites = sites.empty() ? nullptr : A.upload(sites, st);
  if (md.token_rows) {
    md.token_ring = A.alloc<uint32_t>((size_t)E->max_sessions * md.token_rows);
    NB_CUDA(cudaMemsetAsync(md.token_ring, 0, (size_t)E->max_sessions * md.token_rows * 4, st));
  }
  for (uint32_t l = 0; l < L; ++l) {  // ModelConfig::engram_site_at: the first site listed on the layer
    E->layers[l].engram_site = -1;
    E->layers[l].engram = nullptr;
    for (size_t si = 0; si < sites.size() && E->layers[l].engram_site < 0; ++si)
      if (g.engram_sites[si] == l) {
        E->layers[l].engram_site = (int)si;
        E->layers[l].engram = d_sites + si;
      }
  }
  E->engram_sites = sites;
  if (g.qkv_conv_taps > 1) {
    E->conv_ring_floats = (size_t)L * (g.qkv_conv_taps - 1) * md.qkv_width;  // per slot
    md.conv_ring = A.alloc<float>(E->max_sessions * E->conv_ring_floats);
    NB_CUDA(cudaMemsetAsync(md.conv_ring, 0, E->max_sessions * E->conv_ring_floats * 4, st));
  }

  E->capacity = std::max<uint32_t>(opt && opt->max_batch_tokens ? opt->max_batch_tokens : 1024, E->max_sessions);
  const uint32_t M = E->capacity, AW = H * HEAD_DIM, actw = std::max({d, AW, ecfg.k});
  E->act_groups = actw / GROUP;
  Work& w = E->work;
  w.capacity = M;
  E->d_tokens = A.alloc<uint32_t>(M);
  E->d_meta = A.alloc<TokenMeta>(M);
  w.tokens = E->d_tokens;
  w.meta = E->d_meta;
  w.stream = A.alloc<float>((size_t)M * LANES * d);
  w.next_stream = A.alloc<float>((size_t)M * LANES * d);
  w.x = A.alloc<float>((size_t)M * d);
  w.route = A.alloc<float>((size_t)M * (LANES + LANES * LANES));
  const size_t act_rows = ((size_t)M + 127) / 128 * 128;
  w.act_rows = (uint32_t)act_rows;
  if (!sites.empty()) {
    w.engram_kv = A.alloc<float>((size_t)M * 2 * d);
    w.xin = A.alloc<float>((size_t)M * d);
  }
  if (md.cross) {
    w.xr = A.alloc<float>((size_t)M * d);
    w.cq = A.alloc<float>((size_t)M * 2 * d);
  }
  if (md.num_probe_heads) {
    if (M > 0xffff) fail(NB_ERR_ARGUMENT, "passes of more than 65535 tokens are not supported with probe heads");
    w.cells = A.alloc<float>((size_t)M * d);
    w.scores = A.alloc<float>((size_t)M * E->head_pairs);
    w.scan = A.alloc<float>((size_t)M * E->head_pairs * 2);
  }
  w.act = A.alloc<int8_t>(act_rows * actw);
  NB_CUDA(cudaMemsetAsync(w.act, 0, act_rows * actw, st));
  w.act_scale = A.alloc<float>((size_t)M * (actw / GROUP));
  w.proj = A.alloc<float>((size_t)M * qkvg_rows);
  w.qcodes = A.alloc<int8_t>((size_t)M * H * HEAD_DIM);
  w.qscale = A.alloc<float>((size_t)M * H);
  w.attn = A.alloc<float>((size_t)M * AW);
  w.outp = A.alloc<float>((size_t)M * d);
  w.arrivals = A.alloc<int>(M);
  NB_CUDA(cudaMemsetAsync(w.arrivals, 0, (size_t)M * sizeof(int), st));
  const uint32_t B = E->max_sessions, V = md.output_vocab;
  const size_t logit_rows = ((size_t)B + 127) / 128 * 128;
  E->d_logit_act = A.alloc<int8_t>(logit_rows * d);
  NB_CUDA(cudaMemsetAsync(E->d_logit_act, 0, logit_rows * d, st));
  E->d_error = A.alloc<int>(1);
  NB_CUDA(cudaMemsetAsync(E->d_error, 0, sizeof(int), st));
  E->md.error = E->d_error;
  E->h_error.ensure(sizeof(int));
  E->d_logit_scale = A.alloc<float>((size_t)B * (d / GROUP));
  E->d_logits = A.alloc<float>((size_t)B * V);
  // [slots][active flags][masks (B rows of V/32 words)]: a step's slots,
  // flags and host masks arrive in one upload
  E->d_slots = A.alloc<int32_t>(2 * (size_t)B + (size_t)B * (V / 32));
  E->d_active = E->d_slots + B;
  E->d_mask = reinterpret_cast<uint32_t*>(E->d_slots + 2 * (size_t)B);
  E->d_next = A.alloc<uint32_t>(B);
  E->d_peaks = A.alloc<float>((size_t)2 * B);
  E->d_stats = A.alloc<float>((size_t)2 * B);
  E->h_tokens.ensure((size_t)M * 4);
  E->h_meta.ensure((size_t)M * sizeof(TokenMeta));
  E->t_cap = (int)((g.max_seq_len + 3) / 4 * 4);
  NB_CUDA(nbk::configure(md, E->t_cap));
  NB_CUDA(cudaStreamSynchronize(st));
  return E;
}

// ------------------------------------------------------------ forward pass
struct TokenSpec {
  uint32_t token;
  uint32_t slot;
  uint32_t position;
  bool last;
};

// Runs the forward pass of up to `capacity` tokens on the engine's stream
// (embedding, every active layer, final norm into the sequences' hidden rows).
void forward(Engine& E, const std::vector<int32_t>& active, const TokenSpec* specs, uint32_t count) {
  E.settle();
  for (uint32_t i = 0; i < count; ++i) E.prepare_append(specs[i].slot, active, specs[i].position);
  E.flush_page_tables();
  uint32_t* ht = E.h_tokens.as<uint32_t>();
  TokenMeta* hm = E.h_meta.as<TokenMeta>();
  for (uint32_t i = 0; i < count; ++i) {
    ht[i] = specs[i].token;
    const bool continues = i > 0 && specs[i - 1].slot == specs[i].slot && specs[i - 1].position + 1 == specs[i].position;
    const int32_t run = continues ? (hm[i - 1].run & 0xffff) + 1 : 0;
    hm[i] = TokenMeta{(int32_t)specs[i].slot, (int32_t)specs[i].position, specs[i].last ? 1 : 0, run};
  }
  for (uint32_t i = count; i-- > 0;) {  // the run's length into every token of it
    const bool ends = i + 1 == count || (hm[i + 1].run & 0xffff) == 0;
    const int32_t len = ends ? (hm[i].run & 0xffff) + 1 : hm[i + 1].run >> 16;
    hm[i].run = (hm[i].run & 0xffff) | (len << 16);
  }
  NB_CUDA(cudaMemcpyAsync(E.d_tokens, ht, count * 4, cudaMemcpyHostToDevice, E.stream));
  NB_CUDA(cudaMemcpyAsync(E.d_meta, hm, count * sizeof(TokenMeta), cudaMemcpyHostToDevice, E.stream));
  E.copies_in_flight = true;
  Work w = E.work;
  KvDev kv = E.kv();
  // one token per sequence: the attention may do the head step itself
  bool distinct = true;
  std::vector<char> seen(E.max_sessions, 0);
  for (uint32_t i = 0; i < count && distinct; ++i) {
    distinct = !seen[specs[i].slot];
    seen[specs[i].slot] = 1;
  }
  nbk::launch_embed(E.md, w, (int)count, E.stream);
  if (E.md.num_probe_heads) nbk::launch_observe(E.md, w, w.stream, (int)count, 0, E.stream);
  for (size_t slot = 0; slot < active.size(); ++slot) {
    int layer = active[slot];
    nbk::launch_layer(E.md, E.layers[layer], E.engram_of(layer), E.cross_of(layer), w, kv, (int)count, layer, (int)slot, E.t_cap, distinct, E.stream);
    std::swap(w.stream, w.next_stream);
    if (E.md.num_probe_heads) nbk::launch_observe(E.md, w, w.stream, (int)count, layer + 1, E.stream);
  }
  nbk::launch_final(E.md, w, E.d_hidden, (int)count, E.stream);
  NB_CUDA(cudaGetLastError());
  // the pass alternates stream buffers; keep the engine's pair consistent
  E.work.stream = w.stream;
  E.work.next_stream = w.next_stream;
}

}  // namespace nbr

using namespace nbr;

// A device buffer freed on scope exit.
struct DevTemp {
  void* p = nullptr;
  explicit DevTemp(size_t bytes) { NB_CUDA(cudaMalloc(&p, bytes)); }
  ~DevTemp() { cudaFree(p); }
  template <typename T>
  T* as() { return static_cast<T*>(p); }
};

// ------------------------------------------------------------------- C ABI
struct nb_model {
  std::shared_ptr<Engine> engine;
  std::vector<int32_t> active;
};

// Whistle: the cross-attention memory of one encoder output (CrossMemory,
// whistle/src/cross.rs:29-35), in device memory of its own.
struct CrossMem {
  std::shared_ptr<Engine> engine;
  int frames = 0;
  int8_t *keys = nullptr, *values = nullptr;
  float *kscale = nullptr, *vscale = nullptr;
  CrossMemDev* dev = nullptr;
  ~CrossMem() {
    if (!engine) return;
    cudaSetDevice(engine->device);
    cudaStreamSynchronize(engine->stream);  // no queued pass still reads it
    cudaFree(keys);
    cudaFree(values);
    cudaFree(kscale);
    cudaFree(vscale);
    cudaFree(dev);
  }
};

struct nb_cross_memory {
  std::shared_ptr<CrossMem> mem;
};

struct nb_token_automaton {
  std::shared_ptr<Engine> engine;
  nbk::AutomatonDev dev;
  void *transitions = nullptr, *complete = nullptr, *bytes = nullptr, *offsets = nullptr, *error = nullptr;
  ~nb_token_automaton() {
    if (!engine) return;
    cudaSetDevice(engine->device);
    cudaStreamSynchronize(engine->stream);  // no queued mask or advance still reads it
    cudaFree(transitions);
    cudaFree(complete);
    cudaFree(bytes);
    cudaFree(offsets);
    cudaFree(error);
  }
};

struct nb_session {
  std::shared_ptr<Engine> engine;
  std::vector<int32_t> active;
  uint32_t slot = 0;
  uint32_t length = 0;
  std::shared_ptr<CrossMem> cross;  // Whistle: the memory every pass of this session attends to
};

struct nb_batch {
  std::shared_ptr<Engine> engine;
  std::vector<nb_session*> sessions;
  std::vector<int32_t> active;
  std::map<int, cudaGraphExec_t> graphs;  // key: mask | stats << 1
  uint32_t* d_tokens = nullptr;           // the batch's token ids (= the chosen tokens)
  TokenMeta* d_meta = nullptr;
  int32_t* d_order = nullptr;             // per group: its sequences by decreasing context length
  PinnedBuffer h_meta, h_next, h_stats, h_active;
  DeviceArena arena;
  cudaEvent_t fork = nullptr, join[MAX_STEP_GROUPS] = {};
  int groups = 1;  // independent chains of the step (sequences split in runs of whole 32-row tiles)
  uint32_t step_kernels = 0;  // kernels in the last step graph recorded
  bool use_graphs = true;
  ~nb_batch() {
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
    if (fork) cudaEventDestroy(fork);
    for (cudaEvent_t e : join)
      if (e) cudaEventDestroy(e);
  }
};

extern "C" {

const char* nb_last_error(void) { return g_error.c_str(); }

nb_status nb_model_open(const char* path, const nb_options* options, nb_model** out) {
  if (!out) return NB_ERR_ARGUMENT;
  *out = nullptr;
  return guard([&] {
    if (!path) fail(NB_ERR_ARGUMENT, "path is null");
    auto engine = open_engine(path, options);
    auto* m = new nb_model();
    m->engine = engine;
    for (uint32_t l = 0; l < engine->geo.num_layers; ++l) m->active.push_back((int32_t)l);
    *out = m;
  });
}

// crates/model/src/ladder.rs:1-29
static std::vector<int32_t> ladder_order(int layers) {
  std::vector<int32_t> order;
  if (layers <= 1) {
    for (int i = 0; i < layers; ++i) order.push_back(i);
    return order;
  }
  std::vector<int32_t> selected{0, layers - 1};
  order = selected;
  while ((int)order.size() < layers) {
    std::sort(selected.begin(), selected.end());
    int best_gap = -1, left = 0, right = 0;
    for (size_t i = 0; i + 1 < selected.size(); ++i) {
      int gap = selected[i + 1] - selected[i];
      if (gap > 1 && (gap > best_gap || (gap == best_gap && selected[i] < left))) {
        best_gap = gap;
        left = selected[i];
        right = selected[i + 1];
      }
    }
    selected.push_back((left + right) / 2);
    order.push_back((left + right) / 2);
  }
  return order;
}

nb_status nb_model_with_depth(const nb_model* model, uint32_t depth, nb_model** out) {
  if (!model || !out) return NB_ERR_ARGUMENT;
  *out = nullptr;
  int layers = (int)model->engine->geo.num_layers;
  if ((int)depth < std::min(2, layers) || (int)depth > layers) {
    g_error = "depth " + std::to_string(depth) + " is outside the 2 to " + std::to_string(layers) + " layers this model offers";
    return NB_ERR_DEPTH;
  }
  auto order = ladder_order(layers);
  std::vector<int32_t> active(order.begin(), order.begin() + depth);
  std::sort(active.begin(), active.end());
  auto* m = new nb_model();
  m->engine = model->engine;
  m->active = active;
  *out = m;
  return NB_OK;
}

nb_status nb_model_get_config(const nb_model* model, nb_model_config* out) {
  if (!model || !out) return NB_ERR_ARGUMENT;
  const nba::Geometry& g = model->engine->geo;
  std::memset(out, 0, sizeof *out);
  out->vocab = g.vocab;
  out->output_vocab = g.output_vocab();
  out->d_model = g.d_model;
  out->num_heads = g.num_heads;
  out->num_kv_heads = g.num_kv_heads;
  out->num_layers = g.num_layers;
  out->head_dim = g.qk_head_dim;
  out->max_seq_len = g.max_seq_len;
  out->hada_n = g.hada_n;
  out->lanes = g.mhc_lanes;
  out->depth = (uint32_t)model->active.size();
  for (size_t i = 0; i < model->active.size() && i < 64; ++i) out->active_layers[i] = model->active[i];
  out->rope_theta = g.rope_theta;
  return NB_OK;
}

void nb_model_release(nb_model* model) { delete model; }

nb_status nb_model_synchronize(nb_model* model) {
  if (!model) return NB_ERR_ARGUMENT;
  return guard([&] {
    NB_CUDA(cudaSetDevice(model->engine->device));
    NB_CUDA(cudaStreamSynchronize(model->engine->stream));
  });
}

static void set_slot_cross(Engine& E, uint32_t slot, const CrossMemDev* p);

nb_status nb_session_create(nb_model* model, nb_session** out) {
  if (!model || !out) return NB_ERR_ARGUMENT;
  *out = nullptr;
  return guard([&] {
    Engine& E = *model->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    if (E.free_slots.empty()) fail(NB_ERR_ARGUMENT, "every session slot is in use (max_sessions " + std::to_string(E.max_sessions) + ")");
    NB_CUDA(cudaSetDevice(E.device));
    auto* s = new nb_session();
    s->engine = model->engine;
    s->active = model->active;
    s->slot = E.free_slots.back();
    E.free_slots.pop_back();
    NB_CUDA(cudaMemsetAsync(E.d_hidden + (size_t)s->slot * E.md.d_model, 0, E.md.d_model * 4, E.stream));
    for (uint32_t h = 0; h < E.md.num_probe_heads; ++h) {  // ProbeHead::accumulator (heads.rs:80-83)
      const HeadDev& H = E.heads[h];
      const size_t all = (size_t)(E.md.num_layers + 1) * H.probes;
      nbk::fill(H.peak + s->slot * all, all, -INFINITY, E.stream);
      NB_CUDA(cudaMemsetAsync(H.total + s->slot * all, 0, all * 4, E.stream));
      NB_CUDA(cudaMemsetAsync(H.weighted + s->slot * all * E.md.d_model, 0, all * E.md.d_model * 4, E.stream));
    }
    *out = s;
  });
}

nb_status nb_session_clone(const nb_session* session, nb_session** out) {
  if (!session || !out) return NB_ERR_ARGUMENT;
  *out = nullptr;
  return guard([&] {
    Engine& E = *session->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    if (E.free_slots.empty()) fail(NB_ERR_ARGUMENT, "every session slot is in use");
    NB_CUDA(cudaSetDevice(E.device));
    E.settle();
    auto* s = new nb_session(*session);
    s->slot = E.free_slots.back();
    E.free_slots.pop_back();
    for (uint32_t l = 0; l < E.geo.num_layers; ++l)
      for (uint32_t i = 0; i < E.max_pages; ++i) {
        int32_t p = E.page_entry(session->slot, l, i);
        E.page_entry(s->slot, l, i) = p;
        if (p >= 0) ++E.refcount[p];
      }
    E.slot_dirty[s->slot] = 1;
    E.slot_private[session->slot] = E.slot_private[s->slot] = -1;  // every page is shared now
    NB_CUDA(cudaMemcpyAsync(E.d_hidden + (size_t)s->slot * E.md.d_model, E.d_hidden + (size_t)session->slot * E.md.d_model,
                            E.md.d_model * 4, cudaMemcpyDeviceToDevice, E.stream));
    const size_t d = E.md.d_model;
    set_slot_cross(E, s->slot, s->cross ? s->cross->dev : nullptr);  // the clone attends to the same memory
    for (uint32_t h = 0; h < E.md.num_probe_heads; ++h) {  // the probe accumulators are part of the session (session.rs:26)
      const HeadDev& H = E.heads[h];
      const size_t all = (size_t)(E.md.num_layers + 1) * H.probes;
      NB_CUDA(cudaMemcpyAsync(H.peak + s->slot * all, H.peak + session->slot * all, all * 4, cudaMemcpyDeviceToDevice, E.stream));
      NB_CUDA(cudaMemcpyAsync(H.total + s->slot * all, H.total + session->slot * all, all * 4, cudaMemcpyDeviceToDevice, E.stream));
      NB_CUDA(cudaMemcpyAsync(H.weighted + s->slot * all * d, H.weighted + session->slot * all * d, all * d * 4, cudaMemcpyDeviceToDevice,
                              E.stream));
    }
    for (const EngramDev& S : E.engram_sites)  // EngramSiteState is part of the session (session.rs:22)
      if (S.ring)
        NB_CUDA(cudaMemcpyAsync(S.ring + (size_t)s->slot * S.cfg.ring_rows * d, S.ring + (size_t)session->slot * S.cfg.ring_rows * d,
                                (size_t)S.cfg.ring_rows * d * 4, cudaMemcpyDeviceToDevice, E.stream));
    if (E.md.token_ring)
      NB_CUDA(cudaMemcpyAsync(E.md.token_ring + (size_t)s->slot * E.md.token_rows, E.md.token_ring + (size_t)session->slot * E.md.token_rows,
                              E.md.token_rows * 4, cudaMemcpyDeviceToDevice, E.stream));
    if (E.conv_ring_floats)  // the convolution history is part of the session (attention.rs:45, AttentionCache is Clone)
      NB_CUDA(cudaMemcpyAsync(E.md.conv_ring + s->slot * E.conv_ring_floats, E.md.conv_ring + session->slot * E.conv_ring_floats,
                              E.conv_ring_floats * 4, cudaMemcpyDeviceToDevice, E.stream));
    *out = s;
  });
}

void nb_session_release(nb_session* session) {
  if (!session) return;
  Engine& E = *session->engine;
  {
    std::lock_guard<std::mutex> lock(E.mutex);
    cudaSetDevice(E.device);
    try {
      E.settle();
    } catch (...) {
    }
    for (uint32_t l = 0; l < E.geo.num_layers; ++l)
      for (uint32_t i = 0; i < E.max_pages; ++i) {
        int32_t& p = E.page_entry(session->slot, l, i);
        E.drop_page(p);
        p = -1;
      }
    E.slot_dirty[session->slot] = 1;
    E.slot_private[session->slot] = -1;
    try {
      set_slot_cross(E, session->slot, nullptr);
    } catch (...) {
    }
    E.free_slots.push_back(session->slot);
  }
  delete session;
}

size_t nb_session_len(const nb_session* session) { return session ? session->length : 0; }

static void check_tokens(const Engine& E, const uint32_t* ids, size_t count) {
  for (size_t i = 0; i < count; ++i)
    if (ids[i] >= E.geo.vocab) fail(NB_ERR_ARGUMENT, "token id " + std::to_string(ids[i]) + " is outside the vocabulary");
}

// The engine's device error flag (a bounded device wait gave up): its read is
// queued with a pass's results and checked once the stream has synchronised.
static void queue_error_read(Engine& E) {
  NB_CUDA(cudaMemcpyAsync(E.h_error.p, E.d_error, sizeof(int), cudaMemcpyDeviceToHost, E.stream));
}
static void raise_device_error(Engine& E) {
  if (*E.h_error.as<int>()) {
    *E.h_error.as<int>() = 0;
    NB_CUDA(cudaMemsetAsync(E.d_error, 0, sizeof(int), E.stream));
    fail(NB_ERR_TIMEOUT, "a bounded device wait gave up");
  }
}

// Writes the session's entry of the slot-to-memory table.
static void set_slot_cross(Engine& E, uint32_t slot, const CrossMemDev* p) {
  if (E.d_slot_cross) NB_CUDA(cudaMemcpyAsync(E.d_slot_cross + slot, &p, sizeof p, cudaMemcpyHostToDevice, E.stream));
}

nb_status nb_cross_memory_create(nb_model* model, const float* encoded, size_t frames, nb_cross_memory** out) {
  if (!model || !out || !encoded) return NB_ERR_ARGUMENT;
  *out = nullptr;
  return guard([&] {
    Engine& E = *model->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    if (E.cross_layers.empty()) fail(NB_ERR_UNSUPPORTED, "the archive carries no audio section (cross attention)");
    if (frames == 0 || frames > (size_t)MAX_CROSS_FRAMES) fail(NB_ERR_ARGUMENT, "frames must be in 1.." + std::to_string(MAX_CROSS_FRAMES));
    NB_CUDA(cudaSetDevice(E.device));
    E.settle();
    const int d = (int)E.md.d_model, H = (int)E.md.heads, L = (int)E.geo.num_layers, half = d / 2, F = (int)frames;
    // the positional angles' sine and cosine (cross.rs:62-73), the platform
    // libm's as in the reference, like the rotary table
    std::vector<float> sin_t((size_t)F * half), cos_t((size_t)F * half);
    const float rate = -std::log(10000.0f) / ((float)half - 1.0f);
    for (int t = 0; t < F; ++t)
      for (int j = 0; j < half; ++j) {
        const float angle = (float)t * std::exp(rate * (float)j);
        sin_t[(size_t)t * half + j] = std::sin(angle);
        cos_t[(size_t)t * half + j] = std::cos(angle);
      }
    auto m = std::make_shared<CrossMem>();
    const size_t codes = (size_t)L * F * H * HEAD_DIM, scales = (size_t)L * F * H;
    NB_CUDA(cudaMalloc(&m->keys, codes));
    NB_CUDA(cudaMalloc(&m->values, codes));
    NB_CUDA(cudaMalloc(&m->kscale, scales * 4));
    NB_CUDA(cudaMalloc(&m->vscale, scales * 4));
    NB_CUDA(cudaMalloc(&m->dev, sizeof(CrossMemDev)));
    m->engine = model->engine;
    m->frames = F;
    const int act_rows = (F + 127) / 128 * 128;
    DevTemp enc((size_t)F * d * 4), sn(sin_t.size() * 4), cs(cos_t.size() * 4), rows((size_t)F * d * 4), act((size_t)act_rows * d),
        act_scale((size_t)F * (d / GROUP) * 4), kv((size_t)F * 2 * d * 4);
    NB_CUDA(cudaMemcpyAsync(enc.p, encoded, (size_t)F * d * 4, cudaMemcpyHostToDevice, E.stream));
    NB_CUDA(cudaMemcpyAsync(sn.p, sin_t.data(), sin_t.size() * 4, cudaMemcpyHostToDevice, E.stream));
    NB_CUDA(cudaMemcpyAsync(cs.p, cos_t.data(), cos_t.size() * 4, cudaMemcpyHostToDevice, E.stream));
    NB_CUDA(nbk::cross_memory(E.md, E.cross_layers, enc.as<float>(), F, sn.as<float>(), cs.as<float>(), E.position_gate, rows.as<float>(),
                              act.as<int8_t>(), act_scale.as<float>(), act_rows, kv.as<float>(), m->keys, m->kscale, m->values, m->vscale,
                              E.stream));
    const CrossMemDev h{F, m->keys, m->kscale, m->values, m->vscale};
    NB_CUDA(cudaMemcpyAsync(m->dev, &h, sizeof h, cudaMemcpyHostToDevice, E.stream));
    queue_error_read(E);
    NB_CUDA(cudaStreamSynchronize(E.stream));
    E.copies_in_flight = false;  // the staging copies have completed
    raise_device_error(E);
    *out = new nb_cross_memory{m};
  });
}

void nb_cross_memory_release(nb_cross_memory* memory) { delete memory; }

nb_status nb_token_automaton_create(nb_model* model, const uint32_t* transitions, uint32_t num_states,
                                    const uint8_t* complete, uint32_t start_state, const uint8_t* token_bytes,
                                    const uint32_t* token_offsets, uint32_t vocab, uint32_t call_start,
                                    uint32_t call_end, nb_token_automaton** out) {
  if (!model || !out || !transitions || !complete || !token_offsets) return NB_ERR_ARGUMENT;
  *out = nullptr;
  return guard([&] {
    Engine& E = *model->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    if (vocab != E.md.output_vocab)
      fail(NB_ERR_ARGUMENT, "the automaton's vocabulary must cover the model's " + std::to_string(E.md.output_vocab) + " output ids");
    if (num_states < 2 || num_states > NB_AUTOMATON_MAX_STATES)
      fail(NB_ERR_ARGUMENT, "num_states must be in 2.." + std::to_string(NB_AUTOMATON_MAX_STATES));
    if (start_state == 0 || start_state >= num_states) fail(NB_ERR_ARGUMENT, "start_state must be in 1..num_states-1");
    if (call_start >= vocab || call_end >= vocab) fail(NB_ERR_ARGUMENT, "call_start and call_end must be output ids");
    if (complete[0]) fail(NB_ERR_ARGUMENT, "state 0 (no call machine) cannot be complete");
    const size_t cells = (size_t)num_states * 256;
    for (size_t i = 0; i < cells; ++i)
      if ((transitions[i] & 0x7FFFFFFFu) >= num_states) fail(NB_ERR_ARGUMENT, "a transition leads outside the automaton");
    if (token_offsets[0] != 0) fail(NB_ERR_ARGUMENT, "token_offsets[0] must be 0");
    for (uint32_t t = 0; t < vocab; ++t) {
      if (token_offsets[t + 1] < token_offsets[t]) fail(NB_ERR_ARGUMENT, "token_offsets must not decrease");
      if (token_offsets[t + 1] - token_offsets[t] > NB_AUTOMATON_MAX_PIECE)
        fail(NB_ERR_ARGUMENT, "a piece is longer than " + std::to_string(NB_AUTOMATON_MAX_PIECE) + " bytes");
    }
    const size_t nbytes = token_offsets[vocab];
    if (nbytes && !token_bytes) fail(NB_ERR_ARGUMENT, "token_bytes is null");
    NB_CUDA(cudaSetDevice(E.device));
    auto a = std::make_unique<nb_token_automaton>();
    a->engine = model->engine;
    NB_CUDA(cudaMalloc(&a->transitions, cells * 4));
    NB_CUDA(cudaMalloc(&a->complete, num_states));
    NB_CUDA(cudaMalloc(&a->bytes, nbytes ? nbytes : 1));
    NB_CUDA(cudaMalloc(&a->offsets, ((size_t)vocab + 1) * 4));
    NB_CUDA(cudaMalloc(&a->error, 4));
    NB_CUDA(cudaMemcpyAsync(a->transitions, transitions, cells * 4, cudaMemcpyHostToDevice, E.stream));
    NB_CUDA(cudaMemcpyAsync(a->complete, complete, num_states, cudaMemcpyHostToDevice, E.stream));
    if (nbytes) NB_CUDA(cudaMemcpyAsync(a->bytes, token_bytes, nbytes, cudaMemcpyHostToDevice, E.stream));
    NB_CUDA(cudaMemcpyAsync(a->offsets, token_offsets, ((size_t)vocab + 1) * 4, cudaMemcpyHostToDevice, E.stream));
    NB_CUDA(cudaMemsetAsync(a->error, 0, 4, E.stream));
    NB_CUDA(cudaStreamSynchronize(E.stream));  // the host arrays may go once this returns
    nbk::AutomatonDev& d = a->dev;
    d.transitions = static_cast<const uint32_t*>(a->transitions);
    d.complete = static_cast<const uint8_t*>(a->complete);
    d.bytes = static_cast<const uint8_t*>(a->bytes);
    d.offsets = static_cast<const uint32_t*>(a->offsets);
    d.error = static_cast<uint32_t*>(a->error);
    d.num_states = num_states;
    d.start = start_state;
    d.call_start = call_start;
    d.call_end = call_end;
    d.vocab = (int)vocab;
    *out = a.release();
  });
}

void nb_token_automaton_release(nb_token_automaton* automaton) { delete automaton; }

nb_status nb_token_automaton_mask(nb_token_automaton* automaton, const uint32_t* states_device, uint32_t count,
                                  uint32_t* mask_bits_device) {
  if (!automaton || (count && (!states_device || !mask_bits_device))) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *automaton->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    NB_CUDA(cudaSetDevice(E.device));
    NB_CUDA(nbk::automaton_mask(automaton->dev, states_device, (int)count, mask_bits_device, E.stream));
  });
}

nb_status nb_token_automaton_advance(nb_token_automaton* automaton, const uint32_t* next_device, uint32_t count,
                                     uint32_t* states_device) {
  if (!automaton || (count && (!states_device || !next_device))) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *automaton->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    NB_CUDA(cudaSetDevice(E.device));
    NB_CUDA(nbk::automaton_advance(automaton->dev, next_device, (int)count, states_device, E.stream));
  });
}

nb_status nb_token_automaton_check(nb_token_automaton* automaton) {
  if (!automaton) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *automaton->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    NB_CUDA(cudaSetDevice(E.device));
    uint32_t word = 0;
    NB_CUDA(cudaMemcpyAsync(&word, automaton->dev.error, 4, cudaMemcpyDeviceToHost, E.stream));
    NB_CUDA(cudaMemsetAsync(automaton->dev.error, 0, 4, E.stream));
    NB_CUDA(cudaStreamSynchronize(E.stream));
    if (word) fail(NB_ERR_ARGUMENT, "a sequence state was outside the automaton (masked as unconstrained, not advanced)");
  });
}

nb_status nb_session_set_cross(nb_session* session, nb_cross_memory* memory) {
  if (!session) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *session->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    if (memory && memory->mem->engine != session->engine) fail(NB_ERR_ARGUMENT, "the memory belongs to another model");
    NB_CUDA(cudaSetDevice(E.device));
    session->cross = memory ? memory->mem : nullptr;
    set_slot_cross(E, session->slot, session->cross ? session->cross->dev : nullptr);
  });
}

size_t nb_model_text_vocab(const nb_model* model) { return model ? model->engine->text_vocab : 0; }

nb_status nb_debug_cross_memory(const nb_cross_memory* memory, int layer, int8_t* keys, float* key_scales, int8_t* values,
                                float* value_scales) {
  if (!memory || !keys || !key_scales || !values || !value_scales) return NB_ERR_ARGUMENT;
  return guard([&] {
    const CrossMem& m = *memory->mem;
    Engine& E = *m.engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    if (layer < 0 || layer >= (int)E.geo.num_layers) fail(NB_ERR_ARGUMENT, "layer out of range");
    NB_CUDA(cudaSetDevice(E.device));
    NB_CUDA(cudaStreamSynchronize(E.stream));
    // the device keeps [head][frame]; the caller gets the reference's [frame][head]
    const size_t F = (size_t)m.frames, H = E.md.heads, n = F * H, at = (size_t)layer * n;
    std::vector<int8_t> k(n * HEAD_DIM), v(n * HEAD_DIM);
    std::vector<float> ks(n), vs(n);
    NB_CUDA(cudaMemcpy(k.data(), m.keys + at * HEAD_DIM, n * HEAD_DIM, cudaMemcpyDeviceToHost));
    NB_CUDA(cudaMemcpy(v.data(), m.values + at * HEAD_DIM, n * HEAD_DIM, cudaMemcpyDeviceToHost));
    NB_CUDA(cudaMemcpy(ks.data(), m.kscale + at, n * 4, cudaMemcpyDeviceToHost));
    NB_CUDA(cudaMemcpy(vs.data(), m.vscale + at, n * 4, cudaMemcpyDeviceToHost));
    for (size_t h = 0; h < H; ++h)
      for (size_t f = 0; f < F; ++f) {
        std::memcpy(keys + (f * H + h) * HEAD_DIM, &k[(h * F + f) * HEAD_DIM], HEAD_DIM);
        std::memcpy(values + (f * H + h) * HEAD_DIM, &v[(h * F + f) * HEAD_DIM], HEAD_DIM);
        key_scales[f * H + h] = ks[h * F + f];
        value_scales[f * H + h] = vs[h * F + f];
      }
  });
}

// Session::head_output / pooled_readout (session.rs:150-160).
static nb_status head_values(nb_session* session, uint32_t code, float* out, size_t capacity, size_t* count, bool project_out) {
  if (!session || (!out && capacity)) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *session->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    int h = -1;
    for (uint32_t i = 0; i < E.md.num_probe_heads && h < 0; ++i)
      if ((uint32_t)E.heads[i].code == code) h = (int)i;
    if (h < 0) fail(NB_ERR_ARGUMENT, "the model has no probe head with code " + std::to_string(code));
    NB_CUDA(cudaSetDevice(E.device));
    E.settle();
    const HeadDev& H = E.heads[h];
    std::vector<int32_t> rows{0};
    for (int32_t l : session->active) rows.push_back(l + 1);
    int32_t* hr = E.h_head.as<int32_t>();
    std::copy(rows.begin(), rows.end(), hr);
    NB_CUDA(cudaMemcpyAsync(E.d_head_rows, hr, rows.size() * 4, cudaMemcpyHostToDevice, E.stream));
    nbk::head_output(E.md, H, h, (int)session->slot, E.d_head_rows, (int)rows.size(), E.d_head_readouts, E.d_head_weights, E.d_head_pooled,
                     E.d_head_act, E.d_head_scale, 128, E.d_head_out, project_out, E.stream);
    const size_t n = project_out ? H.outputs : (size_t)H.queries * E.md.d_model;
    float* staged = E.h_head.as<float>();
    NB_CUDA(cudaMemcpyAsync(staged, project_out ? E.d_head_out : E.d_head_pooled, n * 4, cudaMemcpyDeviceToHost, E.stream));
    queue_error_read(E);
    NB_CUDA(cudaStreamSynchronize(E.stream));
    E.copies_in_flight = false;  // the staging copies have completed
    raise_device_error(E);
    std::copy(staged, staged + std::min(n, capacity), out);
    if (count) *count = n;
  });
}

nb_status nb_session_head_output(nb_session* session, uint32_t code, float* out, size_t capacity, size_t* count) {
  return head_values(session, code, out, capacity, count, true);
}

nb_status nb_session_pooled_readout(nb_session* session, uint32_t code, float* out, size_t capacity, size_t* count) {
  return head_values(session, code, out, capacity, count, false);
}

static void run_tokens(nb_session* s, const uint32_t* ids, size_t count) {
  Engine& E = *s->engine;
  if (s->length + count > E.geo.max_seq_len)
    fail(NB_ERR_CONTEXT_OVERFLOW, "the session would exceed max_seq_len " + std::to_string(E.geo.max_seq_len));
  NB_CUDA(cudaSetDevice(E.device));
  std::vector<TokenSpec> specs;
  size_t done = 0;
  while (done < count) {
    size_t n = std::min<size_t>(E.capacity, count - done);
    specs.resize(n);
    for (size_t i = 0; i < n; ++i) specs[i] = TokenSpec{ids[done + i], s->slot, (uint32_t)(s->length + done + i), i + 1 == n};
    forward(E, s->active, specs.data(), (uint32_t)n);
    done += n;
  }
  queue_error_read(E);
  NB_CUDA(cudaStreamSynchronize(E.stream));
  raise_device_error(E);
  s->length += (uint32_t)count;
}

nb_status nb_session_feed(nb_session* session, const uint32_t* ids, size_t count) {
  if (!session || (!ids && count)) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *session->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    check_tokens(E, ids, count);
    if (count) run_tokens(session, ids, count);
  });
}

nb_status nb_sessions_feed(nb_session* const* sessions, const uint32_t* const* ids, const size_t* counts, size_t n) {
  if (n == 0) return NB_OK;
  if (!sessions || !ids || !counts || !sessions[0]) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *sessions[0]->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    for (size_t i = 0; i < n; ++i) {
      nb_session* s = sessions[i];
      if (!s || s->engine.get() != &E) fail(NB_ERR_ARGUMENT, "the sessions must belong to one model");
      if (s->active != sessions[0]->active) fail(NB_ERR_ARGUMENT, "the sessions must share the model's active layers");
      for (size_t j = 0; j < i; ++j)
        if (sessions[j] == s) fail(NB_ERR_ARGUMENT, "a session appears twice");
      if (!ids[i] && counts[i]) fail(NB_ERR_ARGUMENT, "a session's ids are null");
      check_tokens(E, ids[i], counts[i]);
      if (s->length + counts[i] > E.geo.max_seq_len)
        fail(NB_ERR_CONTEXT_OVERFLOW, "a session would exceed max_seq_len " + std::to_string(E.geo.max_seq_len));
    }
    NB_CUDA(cudaSetDevice(E.device));
    // the prompts in session order, packed into passes of up to the engine's
    // capacity; a prompt may continue into the next pass (exact, as chunked
    // feeding is), and each pass marks the last token of every sequence in it
    std::vector<TokenSpec> specs;
    specs.reserve(E.capacity);
    size_t si = 0, done = 0;
    while (si < n) {
      specs.clear();
      while (si < n && specs.size() < E.capacity) {
        nb_session* s = sessions[si];
        const size_t take = std::min<size_t>(E.capacity - specs.size(), counts[si] - done);
        for (size_t k = 0; k < take; ++k)
          specs.push_back(TokenSpec{ids[si][done + k], s->slot, (uint32_t)(s->length + done + k), k + 1 == take});
        done += take;
        if (done == counts[si]) {
          ++si;
          done = 0;
        }
      }
      if (!specs.empty()) forward(E, sessions[0]->active, specs.data(), (uint32_t)specs.size());
    }
    queue_error_read(E);
    NB_CUDA(cudaStreamSynchronize(E.stream));
    E.copies_in_flight = false;  // the staging copies have completed
    raise_device_error(E);
    for (size_t i = 0; i < n; ++i) sessions[i]->length += (uint32_t)counts[i];
  });
}

nb_status nb_session_push(nb_session* session, uint32_t id) {
  if (!session) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *session->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    check_tokens(E, &id, 1);
    run_tokens(session, &id, 1);
  });
}

nb_status nb_session_logits(nb_session* session, float* out, size_t capacity) {
  if (!session || !out) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *session->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    uint32_t V = E.md.output_vocab;
    if (capacity < V) fail(NB_ERR_ARGUMENT, "the logits buffer holds fewer than output_vocab floats");
    NB_CUDA(cudaSetDevice(E.device));
    int32_t slot = (int32_t)session->slot;
    NB_CUDA(cudaMemcpyAsync(E.d_slots, &slot, 4, cudaMemcpyHostToDevice, E.stream));
    nbk::launch_logits(E.md, E.d_hidden, E.d_slots, 1, E.d_logit_act, E.d_logit_scale, E.d_logits, E.stream);
    NB_CUDA(cudaGetLastError());
    NB_CUDA(cudaMemcpyAsync(out, E.d_logits, (size_t)V * 4, cudaMemcpyDeviceToHost, E.stream));
    queue_error_read(E);
    NB_CUDA(cudaStreamSynchronize(E.stream));
    E.copies_in_flight = false;  // the staging copies have completed
    raise_device_error(E);
  });
}

// ------------------------------------------------------------------ batches
// The workspace rows [b0, capacity) as a workspace of their own. b0 is a
// multiple of 32, so the int8 activations (core-matrix layout, 8-row blocks
// of K bytes; K = d_model for both products that read them) start on a whole
// 32-token tile of the tensor-core product.
static Work work_rows(const Engine& E, const Work& w, uint32_t b0) {
  const size_t d = E.md.d_model, H = E.md.heads, KV = E.md.kv_heads, actw = d;  // act: the K-chunk-major chunk 0 block
  Work s = w;
  s.capacity = w.capacity - b0;
  s.tokens = w.tokens + b0;
  s.meta = w.meta + b0;
  s.order = w.order ? w.order + b0 : nullptr;
  s.stream = w.stream + b0 * LANES * d;
  s.next_stream = w.next_stream + b0 * LANES * d;
  s.x = w.x + b0 * d;
  s.route = w.route + b0 * (LANES + LANES * LANES);
  s.act = w.act + b0 * actw;
  s.act_scale = w.act_scale + b0 * E.act_groups;
  s.engram_kv = w.engram_kv ? w.engram_kv + b0 * 2 * d : nullptr;
  s.xin = w.xin ? w.xin + b0 * d : nullptr;
  s.cells = w.cells ? w.cells + b0 * d : nullptr;
  s.scores = w.scores ? w.scores + b0 * E.head_pairs : nullptr;
  s.scan = w.scan ? w.scan + b0 * E.head_pairs * 2 : nullptr;
  s.xr = w.xr ? w.xr + b0 * d : nullptr;
  s.cq = w.cq ? w.cq + b0 * 2 * d : nullptr;
  s.proj = w.proj + b0 * (2 * H + 2 * KV) * HEAD_DIM;
  s.qcodes = w.qcodes + b0 * H * HEAD_DIM;
  s.qscale = w.qscale + b0 * H;
  s.attn = w.attn + b0 * H * HEAD_DIM;
  s.outp = w.outp + b0 * d;
  s.arrivals = w.arrivals + b0;
  return s;
}

// Sequences [b0, b0 + count) of the step: tied logits, selection (and
// statistics), then the forward pass of the chosen tokens, on stream `st`.
static void build_group(nb_batch* b, bool masked, bool stats, uint32_t b0, uint32_t count, cudaStream_t st) {
  Engine& E = *b->engine;
  const uint32_t V = E.md.output_vocab, d = E.md.d_model;
  const int n = (int)count;
  uint32_t* mask = masked ? E.d_mask + (size_t)b0 * (V / 32) : nullptr;
  nbk::launch_logits(E.md, E.d_hidden, E.d_slots + b0, n, E.d_logit_act + (size_t)b0 * d, E.d_logit_scale + (size_t)b0 * (d / GROUP),
                     E.d_logits + (size_t)b0 * V, st);
  nbk::launch_select(E.d_logits + (size_t)b0 * V, (int)V, mask, E.d_active + b0, b->d_tokens + b0, E.d_peaks + 2 * b0, n, st);
  if (stats)
    nbk::launch_stats(E.d_logits + (size_t)b0 * V, (int)V, mask, E.d_active + b0, b->d_tokens + b0, E.d_peaks + 2 * b0,
                      E.d_stats + 2 * b0, 2, n, st);
  Work base = E.work;
  base.tokens = b->d_tokens;
  base.meta = b->d_meta;
  base.order = b->d_order;
  Work w = work_rows(E, base, b0);
  KvDev kv = E.kv();
  nbk::launch_embed(E.md, w, n, st);
  if (E.md.num_probe_heads) nbk::launch_observe(E.md, w, w.stream, n, 0, st);
  for (size_t slot = 0; slot < b->active.size(); ++slot) {
    int layer = b->active[slot];
    nbk::launch_layer(E.md, E.layers[layer], E.engram_of(layer), E.cross_of(layer), w, kv, n, layer, (int)slot, E.t_cap, true, st);
    std::swap(w.stream, w.next_stream);
    if (E.md.num_probe_heads) nbk::launch_observe(E.md, w, w.stream, n, layer + 1, st);
  }
  nbk::launch_final(E.md, w, E.d_hidden, n, st);
  nbk::launch_advance(b->d_meta + b0, n, st);
}

// Sequences per group: whole 32-sequence tiles.
static uint32_t group_rows(uint32_t B, int groups) { return groups <= 1 ? B : std::min(B, ((B + groups - 1) / groups + 31) / 32 * 32); }

static void build_step(nb_batch* b, bool masked, bool stats) {
  Engine& E = *b->engine;
  const uint32_t B = (uint32_t)b->sessions.size();
  const uint32_t per = group_rows(B, b->groups);
  if (per >= B) {
    build_group(b, masked, stats, 0, B, E.stream);
    return;
  }
  NB_CUDA(cudaEventRecord(b->fork, E.stream));
  int g = 0;
  for (uint32_t b0 = 0; b0 < B; b0 += per, ++g) {
    cudaStream_t st = E.group_streams[g];
    NB_CUDA(cudaStreamWaitEvent(st, b->fork, 0));
    build_group(b, masked, stats, b0, std::min(per, B - b0), st);
    NB_CUDA(cudaEventRecord(b->join[g], st));
  }
  for (int i = 0; i < g; ++i) NB_CUDA(cudaStreamWaitEvent(E.stream, b->join[i], 0));
}

// Two independent chains when each keeps at least STEP_GROUP_MIN sequences:
// one group's HBM-bound attention then runs beside the other's FP32-bound
// block finish (B = 256: 177k vs 172k tokens/s on one B200). Smaller groups
// would fall to the small-pass kernels (four groups of 64: 110k).
// $NEEDLE_B200_STEP_GROUPS=N forces N.
constexpr uint32_t STEP_GROUP_MIN = 128;
static int step_groups(uint32_t count) {
  int groups = count >= 2 * STEP_GROUP_MIN ? 2 : 1;
  if (const char* env = std::getenv("NEEDLE_B200_STEP_GROUPS")) groups = std::atoi(env);
  return std::max(1, std::min(groups, MAX_STEP_GROUPS));
}

nb_status nb_batch_create(nb_model* model, nb_session* const* sessions, uint32_t count, nb_batch** out) {
  if (!model || !out || (!sessions && count)) return NB_ERR_ARGUMENT;
  *out = nullptr;
  return guard([&] {
    Engine& E = *model->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    if (count == 0 || count > E.max_sessions || count > E.capacity) fail(NB_ERR_ARGUMENT, "batch size must be in 1..max_sessions");
    NB_CUDA(cudaSetDevice(E.device));
    auto b = std::make_unique<nb_batch>();
    b->engine = model->engine;
    b->active = model->active;
    for (uint32_t i = 0; i < count; ++i) {
      if (!sessions[i] || sessions[i]->engine != model->engine) fail(NB_ERR_ARGUMENT, "every session must belong to the batch's model");
      if (sessions[i]->active != model->active) fail(NB_ERR_ARGUMENT, "every session must run the batch model's depth");
      for (uint32_t j = 0; j < i; ++j)
        if (sessions[j] == sessions[i]) fail(NB_ERR_ARGUMENT, "a session appears twice in the batch");
      b->sessions.push_back(sessions[i]);
    }
    b->d_tokens = b->arena.alloc<uint32_t>(count);
    b->d_meta = b->arena.alloc<TokenMeta>(count);
    b->h_meta.ensure(count * sizeof(TokenMeta));
    b->h_next.ensure(count * 4);
    b->h_stats.ensure(count * 8);
    b->h_active.ensure(count * 4);
    NB_CUDA(cudaEventCreateWithFlags(&b->fork, cudaEventDisableTiming));
    for (cudaEvent_t& e : b->join) NB_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    b->groups = step_groups(count);
    // attention CTAs of each group in decreasing context length: the longest
    // sequences start first and the last wave holds the short ones (every
    // sequence advances one position per step, so the order holds)
    {
      const uint32_t per = group_rows(count, b->groups);
      std::vector<int32_t> order(count);
      for (uint32_t g0 = 0; g0 < count; g0 += per) {
        const uint32_t n = std::min(per, count - g0);
        for (uint32_t i = 0; i < n; ++i) order[g0 + i] = (int32_t)i;
        std::stable_sort(order.begin() + g0, order.begin() + g0 + n, [&](int32_t a, int32_t c) {
          return b->sessions[g0 + a]->length > b->sessions[g0 + c]->length;
        });
      }
      b->d_order = b->arena.alloc<int32_t>(count);
      NB_CUDA(cudaMemcpy(b->d_order, order.data(), count * 4, cudaMemcpyHostToDevice));
    }
    *out = b.release();
  });
}

void nb_batch_release(nb_batch* batch) {
  if (!batch) return;
  {
    std::lock_guard<std::mutex> lock(batch->engine->mutex);
    cudaSetDevice(batch->engine->device);
    cudaStreamSynchronize(batch->engine->stream);
  }
  delete batch;
}

// Host part of a step: which sequences can grow, their pages, their metadata.
// mask_bits (host, B rows of output_vocab/32 words, or null) joins the upload
// of the slots and flags.
static uint32_t stage_step(nb_batch* b, const uint32_t* mask_bits = nullptr) {
  Engine& E = *b->engine;
  E.settle();
  const uint32_t B = (uint32_t)b->sessions.size();
  TokenMeta* hm = b->h_meta.as<TokenMeta>();
  int32_t* ha = b->h_active.as<int32_t>();
  // the slots at [0, B), the active flags at [max_sessions, max_sessions + B)
  // and the masks from 2 · max_sessions on: d_slots, d_active and d_mask are
  // one device array
  const size_t flags = E.max_sessions, words = E.md.output_vocab / 32;
  E.h_misc.ensure((2 * flags + (size_t)B * words) * 4);
  int32_t* slots = E.h_misc.as<int32_t>();
  uint32_t live = 0;
  for (uint32_t i = 0; i < B; ++i) {
    nb_session* s = b->sessions[i];
    slots[i] = (int32_t)s->slot;
    // generator.rs:99: a step needs session.len() + 1 < max_seq_len
    bool ok = s->length + 1 < E.geo.max_seq_len;
    ha[i] = ok ? 1 : 0;
    hm[i] = TokenMeta{ok ? (int32_t)s->slot : -1, (int32_t)s->length, 1, 1 << 16};
    if (ok) {
      E.prepare_append(s->slot, b->active, s->length);
      ++live;
    }
  }
  E.flush_page_tables();
  std::memcpy(slots + flags, ha, B * 4);
  size_t upload = flags + B;
  if (mask_bits) {
    std::memcpy(slots + 2 * flags, mask_bits, (size_t)B * words * 4);
    upload = 2 * flags + (size_t)B * words;
  }
  NB_CUDA(cudaMemcpyAsync(E.d_slots, slots, upload * 4, cudaMemcpyHostToDevice, E.stream));
  NB_CUDA(cudaMemcpyAsync(b->d_meta, hm, B * sizeof(TokenMeta), cudaMemcpyHostToDevice, E.stream));
  E.copies_in_flight = true;
  return live;
}

static void launch_step(nb_batch* b, bool masked, bool stats) {
  Engine& E = *b->engine;
  if (!b->use_graphs) {
    build_step(b, masked, stats);
    NB_CUDA(cudaGetLastError());
    return;
  }
  int key = (masked ? 1 : 0) | (stats ? 2 : 0);
  auto it = b->graphs.find(key);
  if (it == b->graphs.end()) {
    cudaGraph_t graph;
    NB_CUDA(cudaStreamBeginCapture(E.stream, cudaStreamCaptureModeThreadLocal));
    const long before = nbk::launch_counter();
    try {
      build_step(b, masked, stats);
    } catch (...) {
      cudaStreamEndCapture(E.stream, &graph);
      throw;
    }
    b->step_kernels = (uint32_t)(nbk::launch_counter() - before);
    NB_CUDA(cudaStreamEndCapture(E.stream, &graph));
    cudaGraphExec_t exec;
    cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) fail(NB_ERR_CUDA, std::string("cudaGraphInstantiate: ") + cudaGetErrorString(e));
    it = b->graphs.emplace(key, exec).first;
  }
  NB_CUDA(cudaGraphLaunch(it->second, E.stream));
}

static void finish_step(nb_batch* b) {
  for (size_t i = 0; i < b->sessions.size(); ++i)
    if (b->h_active.as<int32_t>()[i]) b->sessions[i]->length += 1;
}

nb_status nb_batch_step(nb_batch* batch, const uint32_t* mask_bits, uint32_t* next, nb_step_stats* stats) {
  if (!batch || !next) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *batch->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    NB_CUDA(cudaSetDevice(E.device));
    const uint32_t B = (uint32_t)batch->sessions.size(), words = E.md.output_vocab / 32;
    stage_step(batch, mask_bits);
    launch_step(batch, mask_bits != nullptr, stats != nullptr);
    NB_CUDA(cudaMemcpyAsync(batch->h_next.p, batch->d_tokens, B * 4, cudaMemcpyDeviceToHost, E.stream));
    if (stats) NB_CUDA(cudaMemcpyAsync(batch->h_stats.p, E.d_stats, (size_t)B * 8, cudaMemcpyDeviceToHost, E.stream));
    queue_error_read(E);
    NB_CUDA(cudaStreamSynchronize(E.stream));
    E.copies_in_flight = false;  // the staging copies have completed
    raise_device_error(E);
    const int32_t* ha = batch->h_active.as<int32_t>();
    for (uint32_t i = 0; i < B; ++i) {
      next[i] = ha[i] ? batch->h_next.as<uint32_t>()[i] : 0xffffffffu;
      if (stats) {
        stats[i].probability = ha[i] ? batch->h_stats.as<float>()[2 * i] : 0.0f;
        stats[i].mass = ha[i] ? batch->h_stats.as<float>()[2 * i + 1] : 1.0f;
        stats[i].status = ha[i] ? NB_OK : NB_ERR_CONTEXT_OVERFLOW;
      }
    }
    finish_step(batch);
  });
}

nb_status nb_batch_step_device(nb_batch* batch, const uint32_t* mask_bits_device, uint32_t* next_device, nb_step_stats* stats_device) {
  if (!batch || !next_device || stats_device) {
    g_error = "nb_batch_step_device takes device pointers for next and mask, and no stats";
    return NB_ERR_ARGUMENT;
  }
  return guard([&] {
    Engine& E = *batch->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    NB_CUDA(cudaSetDevice(E.device));
    const uint32_t B = (uint32_t)batch->sessions.size(), words = E.md.output_vocab / 32;
    stage_step(batch);
    if (mask_bits_device)
      NB_CUDA(cudaMemcpyAsync(E.d_mask, mask_bits_device, (size_t)B * words * 4, cudaMemcpyDeviceToDevice, E.stream));
    launch_step(batch, mask_bits_device != nullptr, false);
    NB_CUDA(cudaMemcpyAsync(next_device, batch->d_tokens, B * 4, cudaMemcpyDeviceToDevice, E.stream));
    queue_error_read(E);
    NB_CUDA(cudaStreamSynchronize(E.stream));
    E.copies_in_flight = false;  // the staging copies have completed
    raise_device_error(E);
    finish_step(batch);
  });
}

nb_status nb_batch_run(nb_batch* batch, uint32_t steps, const uint32_t* mask_bits_device, uint32_t* tokens_device,
                       float* elapsed_ms) {
  if (!batch || steps == 0) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *batch->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    NB_CUDA(cudaSetDevice(E.device));
    const uint32_t B = (uint32_t)batch->sessions.size(), words = E.md.output_vocab / 32;
    for (nb_session* s : batch->sessions)
      if (s->length + steps >= E.geo.max_seq_len)
        fail(NB_ERR_CONTEXT_OVERFLOW, "a session of the batch cannot take " + std::to_string(steps) + " more tokens");
    // pages for every position the run will write, then the usual staging
    for (nb_session* s : batch->sessions)
      for (uint32_t k = 1; k < steps; ++k)
        if ((s->length + k) % PAGE_POSITIONS == 0) E.prepare_append(s->slot, batch->active, s->length + k);
    stage_step(batch);
    cudaEvent_t start, stop;
    NB_CUDA(cudaEventCreate(&start));
    NB_CUDA(cudaEventCreate(&stop));
    NB_CUDA(cudaEventRecord(start, E.stream));
    for (uint32_t k = 0; k < steps; ++k) {
      if (mask_bits_device)
        NB_CUDA(cudaMemcpyAsync(E.d_mask, mask_bits_device + (size_t)k * B * words, (size_t)B * words * 4, cudaMemcpyDeviceToDevice,
                                E.stream));
      launch_step(batch, mask_bits_device != nullptr, false);
      if (tokens_device)
        NB_CUDA(cudaMemcpyAsync(tokens_device + (size_t)k * B, batch->d_tokens, B * 4, cudaMemcpyDeviceToDevice, E.stream));
    }
    NB_CUDA(cudaEventRecord(stop, E.stream));
    queue_error_read(E);  // after the timed region
    NB_CUDA(cudaEventSynchronize(stop));
    float ms = 0.0f;
    NB_CUDA(cudaEventElapsedTime(&ms, start, stop));
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    NB_CUDA(cudaStreamSynchronize(E.stream));
    E.copies_in_flight = false;
    raise_device_error(E);
    if (elapsed_ms) *elapsed_ms = ms;
    for (nb_session* s : batch->sessions) s->length += steps;
  });
}

nb_status nb_session_step(nb_session* session, const uint32_t* mask_bits, uint32_t* next, nb_step_stats* stats) {
  if (!session || !next) return NB_ERR_ARGUMENT;
  nb_model m;
  m.engine = session->engine;
  m.active = session->active;
  nb_batch* b = nullptr;
  nb_status s = nb_batch_create(&m, &session, 1, &b);
  if (s != NB_OK) return s;
  b->use_graphs = false;
  nb_step_stats st{};
  s = nb_batch_step(b, mask_bits, next, stats ? &st : nullptr);
  if (stats) *stats = st;
  if (s == NB_OK && stats && st.status != NB_OK) {
    g_error = "the session's context is full";
    s = NB_ERR_CONTEXT_OVERFLOW;
  }
  nb_batch_release(b);
  return s;
}

// Allocates nothing on the device (its scratch is the file-scope array of
// kernels.cu) and, on success, nothing on the host either; see the header
// for the callers it serves.
nb_status nb_model_project_static(nb_model* model, int which, uint32_t layer, const float* in_device, uint32_t count,
                                  float* out_device, void* stream) {
  if (!model || !in_device || !out_device || count == 0 || which < 0 || which > 2) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *model->engine;
    if (which < 2 && layer >= E.layers.size()) fail(NB_ERR_ARGUMENT, "no such layer");
    if (count > (uint32_t)nbk::STATIC_MAX_TOKENS)
      fail(NB_ERR_ARGUMENT, "count " + std::to_string(count) + " is above the " + std::to_string(nbk::STATIC_MAX_TOKENS) +
                                " tokens the static scratch holds");
    if (reinterpret_cast<uintptr_t>(in_device) % 16 || reinterpret_cast<uintptr_t>(out_device) % 4)
      fail(NB_ERR_ARGUMENT, "in_device must be 16-byte and out_device 4-byte aligned");
    const QMat& W = which == 0 ? E.layers[layer].qkvg : which == 1 ? E.layers[layer].out : E.md.logits;
    NB_CUDA(cudaSetDevice(E.device));
    NB_CUDA(nbk::static_scratch_setup(E.device));
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : E.stream;
    int wait_failed = 0;
    NB_CUDA(nbk::launch_static_project(E.device, E.md, W, in_device, (int)count, out_device, st, &wait_failed));
    if (wait_failed) fail(NB_ERR_TIMEOUT, "a bounded wait of the tensor-core product gave up");
  });
}

nb_status nb_build_expf_table(const char* path) {
  if (!path) return NB_ERR_ARGUMENT;
  return guard([&] {
    nbx::ExpfTable table = nbx::scan_expf_exceptions(0);
    if (table.unexplained) fail(NB_ERR_UNSUPPORTED, "the host expf has mismatches the device exponential cannot reproduce");
    nbx::write_expf_table(path, table);
  });
}

}  // extern "C"

// ---------------------------------------------------------------- test hooks
#include "../../include/needle_b200_debug.h"

namespace nbr {
template <typename T>
struct DeviceTemp {
  T* p = nullptr;
  explicit DeviceTemp(size_t n) { NB_CUDA(cudaMalloc(&p, std::max<size_t>(n * sizeof(T), 16))); }
  ~DeviceTemp() { cudaFree(p); }
};
}  // namespace nbr

extern "C" {

nb_status nb_debug_math(nb_model* model, int op, const float* in, float* out, size_t count) {
  if (!model || !in || !out || op < 0 || op > 4) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *model->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    NB_CUDA(cudaSetDevice(E.device));
    E.settle();
    DeviceTemp<float> din(count), dout(count);
    NB_CUDA(cudaMemcpyAsync(din.p, in, count * 4, cudaMemcpyHostToDevice, E.stream));
    nbk::launch_debug_math(op, din.p, dout.p, (int)count, E.stream);
    NB_CUDA(cudaGetLastError());
    NB_CUDA(cudaMemcpyAsync(out, dout.p, count * 4, cudaMemcpyDeviceToHost, E.stream));
    NB_CUDA(cudaStreamSynchronize(E.stream));
  });
}

nb_status nb_debug_project(nb_model* model, int which, uint32_t layer, const float* in, size_t count, float* out) {
  if (!model || !in || !out || count == 0) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *model->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    if (layer >= E.layers.size() || which < 0 || which > 2) fail(NB_ERR_ARGUMENT, "no such matrix");
    const QMat& W = which == 0 ? E.layers[layer].qkvg : which == 1 ? E.layers[layer].out : E.md.logits;
    NB_CUDA(cudaSetDevice(E.device));
    E.settle();
    const uint32_t K = W.cols;
    // the tensor-core product reads whole 16..128-token tiles of activations
    const size_t tile_rows = (count + 127) / 128 * 128;
    DeviceTemp<float> din(count * K), dout(count * W.rows), dscale(tile_rows * W.groups);
    DeviceTemp<int8_t> dact(tile_rows * K);
    NB_CUDA(cudaMemsetAsync(dact.p, 0, tile_rows * K, E.stream));
    NB_CUDA(cudaMemcpyAsync(din.p, in, count * K * 4, cudaMemcpyHostToDevice, E.stream));
    nbk::launch_debug_project(E.md, W, din.p, (int)K, (int)count, dact.p, dscale.p, dout.p, (int)W.rows, E.stream);
    NB_CUDA(cudaGetLastError());
    NB_CUDA(cudaMemcpyAsync(out, dout.p, count * W.rows * 4, cudaMemcpyDeviceToHost, E.stream));
    NB_CUDA(cudaStreamSynchronize(E.stream));
  });
}

nb_status nb_debug_hadamard(nb_model* model, uint32_t layer, const float* in, size_t count, float* out) {
  if (!model || !in || !out || count == 0) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *model->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    if (layer >= E.layers.size()) fail(NB_ERR_ARGUMENT, "no such layer");
    NB_CUDA(cudaSetDevice(E.device));
    E.settle();
    const size_t d = E.md.d_model;
    DeviceTemp<float> din(count * d), dout(count * d);
    NB_CUDA(cudaMemcpyAsync(din.p, in, count * d * 4, cudaMemcpyHostToDevice, E.stream));
    nbk::launch_debug_hadamard(E.md, E.layers[layer], din.p, dout.p, (int)count, E.stream);
    NB_CUDA(cudaGetLastError());
    NB_CUDA(cudaMemcpyAsync(out, dout.p, count * d * 4, cudaMemcpyDeviceToHost, E.stream));
    NB_CUDA(cudaStreamSynchronize(E.stream));
  });
}

nb_status nb_debug_product(int device, uint32_t bits, const uint8_t* packed, const float* levels, const uint16_t* norms, uint32_t rows,
                           uint32_t cols, const float* in, uint32_t count, float* out, uint32_t reps, float* ms_per_product) {
  if (!packed || !levels || !norms || !in || !out || rows == 0 || count == 0 || (cols != 512 && cols != 2048) || (bits != 2 && bits != 4))
    return NB_ERR_ARGUMENT;
  return guard([&] {
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) fail(NB_ERR_NO_DEVICE, "no CUDA device");
    NB_CUDA(cudaSetDevice(device));
    std::vector<float> cb(28, 0.0f);
    for (uint32_t i = 0; i < (1u << bits); ++i) cb[(bits == 2 ? 0 : 12) + i] = levels[i];
    const Levels lv = levels_for(bits, cb, GROUP);
    const size_t rows_cap = ((size_t)rows + 127) / 128 * 128, groups = cols / GROUP, act_rows = ((size_t)count + 127) / 128 * 128;
    const size_t rb = (size_t)cols * bits / 8;
    std::vector<int8_t> codes(rows_cap * cols, 0);
    std::vector<float> scales((size_t)rows * groups);
    for (size_t r = 0; r < rows; ++r) {
      for (uint32_t c = 0; c < cols; ++c) codes[chunked_offset(r, c, rows_cap)] = lv.ints[code_at(packed + r * rb, c, lv.bits)];
      for (size_t g = 0; g < groups; ++g) {
        const float norm = nba::half_to_f32(norms[r * groups + g]);
        scales[r * groups + g] = lv.fused ? norm * lv.int_scale : norm;
      }
    }
    DeviceTemp<int8_t> dcodes(codes.size()), dact(act_rows * cols);
    DeviceTemp<float> dscales(scales.size()), din((size_t)count * cols), dact_scale((size_t)count * groups), dout((size_t)count * rows);
    DeviceTemp<int> derr(1);
    cudaStream_t st;
    NB_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    NB_CUDA(cudaMemcpyAsync(dcodes.p, codes.data(), codes.size(), cudaMemcpyHostToDevice, st));
    NB_CUDA(cudaMemcpyAsync(dscales.p, scales.data(), scales.size() * 4, cudaMemcpyHostToDevice, st));
    NB_CUDA(cudaMemcpyAsync(din.p, in, (size_t)count * cols * 4, cudaMemcpyHostToDevice, st));
    NB_CUDA(cudaMemsetAsync(dact.p, 0, act_rows * cols, st));
    NB_CUDA(cudaMemsetAsync(derr.p, 0, sizeof(int), st));
    const QMat W{dcodes.p, dscales.p, lv.int_scale, rows, cols, (uint32_t)groups, lv.fused ? 1 : 0};
    float ms = 0.0f;
    cudaError_t e = nbk::launch_product_bench(W, din.p, (int)count, dact.p, dact_scale.p, (int)act_rows, dout.p, derr.p, (int)reps, &ms, st);
    int err = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, dout.p, (size_t)count * rows * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&err, derr.p, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaStreamDestroy(st);
    NB_CUDA(e);
    if (err) fail(NB_ERR_TIMEOUT, "a bounded wait of the tensor-core product gave up");
    if (ms_per_product) *ms_per_product = ms;
  });
}

nb_status nb_debug_expire_waits(nb_model* model, uint32_t count) {
  if (!model) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *model->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    NB_CUDA(cudaSetDevice(E.device));
    NB_CUDA(nbk::set_expire_route((int)count, E.stream));
    NB_CUDA(cudaStreamSynchronize(E.stream));
  });
}

nb_status nb_debug_read_bandwidth(int device, size_t bytes, uint32_t passes, uint32_t reps, float* ms_per_read) {
  if (!ms_per_read || bytes < 16 || bytes % 16 != 0 || reps == 0 || passes == 0 || passes > 4096) return NB_ERR_ARGUMENT;
  return guard([&] {
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) fail(NB_ERR_NO_DEVICE, "no CUDA device");
    NB_CUDA(cudaSetDevice(device));
    DeviceTemp<uint8_t> buffer(bytes);
    DeviceTemp<uint32_t> sink(4);
    cudaStream_t st;
    NB_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    cudaError_t e = cudaMemsetAsync(buffer.p, 0x5A, bytes, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(sink.p, 0, 16, st);
    float ms = 0.0f;
    if (e == cudaSuccess) e = nbk::launch_read_bench(buffer.p, bytes, (int)passes, sink.p, (int)reps, &ms, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaStreamDestroy(st);
    NB_CUDA(e);
    *ms_per_read = ms / (float)passes;
  });
}

nb_status nb_debug_hidden(nb_session* session, float* out) {
  if (!session || !out) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *session->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    NB_CUDA(cudaSetDevice(E.device));
    NB_CUDA(cudaMemcpyAsync(out, E.d_hidden + (size_t)session->slot * E.md.d_model, E.md.d_model * 4, cudaMemcpyDeviceToHost,
                            E.stream));
    NB_CUDA(cudaStreamSynchronize(E.stream));
  });
}

nb_status nb_debug_kv(nb_session* session, uint32_t layer, int8_t* keys, float* key_scales, int8_t* values, float* value_scales) {
  if (!session) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *session->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    if (layer >= E.geo.num_layers) fail(NB_ERR_ARGUMENT, "no such layer");
    NB_CUDA(cudaSetDevice(E.device));
    E.settle();
    const PageGeometry& pg = E.md.page;
    const uint32_t n = session->length, KV = pg.kv_heads;
    std::vector<uint8_t> page(pg.page_bytes);
    for (uint32_t base = 0; base < n; base += PAGE_POSITIONS) {
      int32_t p = E.page_entry(session->slot, layer, base / PAGE_POSITIONS);
      if (p < 0) fail(NB_ERR_ARGUMENT, "the layer holds no page at this position");
      NB_CUDA(cudaMemcpy(page.data(), E.pool + (size_t)p * pg.page_bytes, pg.page_bytes, cudaMemcpyDeviceToHost));
      for (uint32_t i = 0; i < PAGE_POSITIONS && base + i < n; ++i) {
        uint32_t pos = base + i;
        for (uint32_t h = 0; h < KV; ++h) {
          for (uint32_t dim = 0; dim < HEAD_DIM; ++dim) {
            if (keys) keys[((size_t)pos * KV + h) * HEAD_DIM + dim] = (int8_t)page[((size_t)h * PAGE_POSITIONS + i) * HEAD_DIM + dim];
            if (values)
              values[((size_t)pos * KV + h) * HEAD_DIM + dim] =
                  (int8_t)page[pg.value_offset + (size_t)h * PAGE_POSITIONS * HEAD_DIM + (i / 4) * (HEAD_DIM * 4) + dim * 4 + i % 4];
          }
          float ks, vs;
          std::memcpy(&ks, &page[pg.kscale_offset + ((size_t)h * PAGE_POSITIONS + i) * 4], 4);
          std::memcpy(&vs, &page[pg.vscale_offset + ((size_t)h * PAGE_POSITIONS + i) * 4], 4);
          if (key_scales) key_scales[(size_t)h * n + pos] = ks;
          if (value_scales) value_scales[(size_t)h * n + pos] = vs;
        }
      }
    }
  });
}

}  // extern "C"

extern "C" nb_status nb_debug_step_kernels(nb_batch* batch, uint32_t* kernels) {
  if (!batch || !kernels) return NB_ERR_ARGUMENT;
  *kernels = batch->step_kernels;
  return NB_OK;
}

extern "C" nb_status nb_debug_time_attention(nb_batch* batch, uint32_t reps, float* ms_per_launch, double* bytes_per_launch) {
  if (!batch || reps == 0 || !ms_per_launch) return NB_ERR_ARGUMENT;
  return guard([&] {
    Engine& E = *batch->engine;
    std::lock_guard<std::mutex> lock(E.mutex);
    NB_CUDA(cudaSetDevice(E.device));
    E.settle();
    const uint32_t B = (uint32_t)batch->sessions.size();
    // the batch's current positions (the last step's tokens were appended at length-1)
    TokenMeta* hm = batch->h_meta.as<TokenMeta>();
    double bytes = 0.0;
    const double per_position = (double)E.md.kv_heads * (2 * HEAD_DIM + 8);
    for (uint32_t i = 0; i < B; ++i) {
      nb_session* s = batch->sessions[i];
      uint32_t pos = s->length ? s->length - 1 : 0;
      hm[i] = TokenMeta{(int32_t)s->slot, (int32_t)pos, 1, 1 << 16};
      bytes += (double)(pos + 1) * per_position;
    }
    NB_CUDA(cudaMemcpyAsync(batch->d_meta, hm, B * sizeof(TokenMeta), cudaMemcpyHostToDevice, E.stream));
    Work base = E.work;
    base.meta = batch->d_meta;
    base.order = batch->d_order;
    KvDev kv = E.kv();
    // the attention launches the step runs (one per group of sequences, each
    // over its rows in its launch order), with the output projection's
    // activation step fused in where it is; the head step (which the step
    // also fuses in) is left out, since replaying it would rewrite the cache
    const uint32_t per = group_rows(B, batch->groups);
    auto attend = [&](int32_t layer) {
      for (uint32_t b0 = 0; b0 < B; b0 += per) {
        const Work w = work_rows(E, base, b0);
        nbk::launch_attention(E.md, E.layers[layer], w, kv, (int)std::min(per, B - b0), layer, E.t_cap, false, E.stream);
      }
    };
    cudaEvent_t start, stop;
    NB_CUDA(cudaEventCreate(&start));
    NB_CUDA(cudaEventCreate(&stop));
    // one untimed round warms the caches the way the step does
    for (int32_t layer : batch->active) attend(layer);
    NB_CUDA(cudaEventRecord(start, E.stream));
    for (uint32_t r = 0; r < reps; ++r)
      for (int32_t layer : batch->active) attend(layer);
    NB_CUDA(cudaEventRecord(stop, E.stream));
    NB_CUDA(cudaEventSynchronize(stop));
    NB_CUDA(cudaGetLastError());
    float ms = 0.0f;
    NB_CUDA(cudaEventElapsedTime(&ms, start, stop));
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    *ms_per_launch = ms / (float)(reps * batch->active.size());
    if (bytes_per_launch) *bytes_per_launch = bytes;
  });
}
