// layout.h — device data layout of a loaded Needle-3 model, its KV pages and
// the per-pass workspace. Shared by the host runtime and the kernels.
//
// Weights. Every codebook-quantised matrix (crates/cact/src/record.rs, kind 3)
// is expanded once at load from its 2- or 4-bit indices to int8 through the
// reference's integer level table (crates/kernels/src/neon.rs:114-123). The
// matrices of the tensor-core products (fused q/k/v/gate, out_proj, the tied
// logits) are stored in the K-major core-matrix layout of core_offset() with
// rows padded to whole 128-row tiles; the lane maps stay row-major.
// Per (row, group) scales are f32: for 2-bit matrices the product
// norm*level_scale of the panel combine (panel.rs:184), for 4-bit matrices the
// norm alone (the row combine multiplies by level_scale after the norm,
// neon.rs:180).
//
// KV pages hold 64 positions of one layer of one sequence for every kv head:
//   keys    [kv][64 positions][head_dim] int8            (position-major rows)
//   values  [kv][16 blocks][head_dim][4 positions] int8  (the reference's
//           4-position value panels, model/src/attention.rs:54-69)
//   kscale  [kv][64] f32, vscale [kv][64] f32
//
// QKV causal convolution (models with qkv_conv_taps > 0): each layer's gains
// are [tap][q | k | v] (tap 0 = the current position), and the ring
// conv_ring[slot][layer][taps - 1][q | k | v] keeps a sequence's raw
// (pre-convolution) projections of its last taps - 1 positions, row
// position % (taps - 1).
//
// Engram sites (models/src/engram.rs): per site the hashed tables (packed
// code rows, dequantised on gather like the embedding), key_proj and
// value_proj stacked into one 2d-row product whose K (tables · sub_dim) is
// zero-padded to 512 or 2048, and the value convolution gains. A sequence's
// raw values of its last (taps - 1) · dilation positions sit in the site's
// ring [slots][rows][d] at row position % rows; its last (max order - 1)
// token ids in token_ring[slots][rows] at position % rows.
//
// Probe heads (models/src/heads.rs): per head the probe directions and query
// rows dequantised to f32 ([rows = layers + 1][probes][d], [queries][d]), the
// gains and row biases, the projection as a product (K = queries · d
// zero-padded to 512 or 2048), and per session slot the online-softmax
// accumulators peak, total [rows][probes] and weighted [rows][probes][d], all
// indexed by the archive row (0 = the embedding cell, layer + 1), so every
// depth uses its subset.
//
// Whistle cross attention (whistle/src/cross.rs): per decoder layer the q|gate
// and k|v products (k|v builds the memory) and the out product; a memory holds
// for every layer the int8 keys and values [head][frame][64] of one encoder
// output with their scales [head][frame]; slot_cross[slot] points at the
// memory a session attends to (null: none).
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifndef __CUDACC__
#define __host__
#define __device__
#endif

namespace nbl {

constexpr int GROUP = 128;
constexpr int HEAD_DIM = 64;
constexpr int PAGE_POSITIONS = 64;
constexpr int LANES = 4;
constexpr int MAX_D = 1024;
constexpr int MAX_HEADS = 16;
constexpr int HADA_RIGHT = 32;
constexpr int COND_RANK = 8;

struct PageGeometry {
  uint32_t kv_heads;
  uint32_t key_bytes;     // kv * 64 * head_dim
  uint32_t value_offset;  // == key_bytes
  uint32_t kscale_offset; // 2 * key_bytes
  uint32_t vscale_offset;
  uint32_t page_bytes;
};

inline PageGeometry page_geometry(uint32_t kv_heads) {
  PageGeometry p;
  p.kv_heads = kv_heads;
  p.key_bytes = kv_heads * PAGE_POSITIONS * HEAD_DIM;
  p.value_offset = p.key_bytes;
  p.kscale_offset = 2 * p.key_bytes;
  p.vscale_offset = p.kscale_offset + kv_heads * PAGE_POSITIONS * 4;
  p.page_bytes = p.vscale_offset + kv_heads * PAGE_POSITIONS * 4;
  return p;
}

// Canonical K-major core-matrix layout of the tensor-core operands: element
// (row r, byte k) of a matrix with `kchunks` 16-byte chunks per row sits in
// the 8-row × 16-byte core matrix (r/8, k/16), rows 16 bytes apart. A group of
// 8 rows is one contiguous block of kchunks·128 bytes.
__host__ __device__ inline size_t core_offset(size_t r, uint32_t k, uint32_t kchunks) {
  return ((r >> 3) * kchunks + (k >> 4)) * 128 + (r & 7) * 16 + (k & 15);
}

// Operands wider than 512 columns are stored K-chunk-major: chunk c (columns
// 512c .. 512c+511) of all rows (padded to rows_cap) is one block in the
// core-matrix layout above, so a 128-row tile of one chunk is 64 KB
// contiguous. For K = 512 this is the plain core-matrix layout.
constexpr uint32_t KCHUNK = 512;
__host__ __device__ inline size_t chunked_offset(size_t r, uint32_t k, size_t rows_cap) {
  return (size_t)(k / KCHUNK) * rows_cap * KCHUNK + core_offset(r, k % KCHUNK, KCHUNK / 16);
}

// A codebook-quantised matrix in device layout.
struct QMat {
  const int8_t* codes;   // int8, K-chunk-major core-matrix layout (rows padded to 128), or row-major (lane maps)
  const float* scales;   // [rows][groups]
  float level_scale;     // IntegerLevels::scale
  uint32_t rows, cols, groups;
  int fused;             // 1: 2-bit panel combine (fma); 0: 4-bit row combine
};

struct HadamardDev {
  const float *d1, *d2, *b2, *d3, *d4;
  const float* left[3];   // left_size x left_size
  const float* right[3];  // 32 x 32
  const float *cond_v, *cond_u;
};

// config.rs:4-14, the same for every site
struct EngramConfig {
  uint32_t slots, sub_dim, tables, orders, heads_per_order, stride;
  uint32_t order[4];
  uint32_t conv_taps, dilation, ring_rows, k;  // ring_rows = (conv_taps - 1) · dilation; k: the padded product K
};

struct EngramDev {
  EngramConfig cfg;
  const uint8_t* packed;   // tables · slots rows of packed codes
  uint32_t row_bytes, bits;
  const float* levels;     // 2^bits levels
  const float* norms;      // [rows][sub_dim / 128]
  QMat kv;                 // key_proj rows, then value_proj rows
  const float* taps;       // [conv_taps][d]
  float* ring;             // [slots][ring_rows][d]; null when ring_rows == 0
};

struct HeadDev {
  int code;
  uint32_t probes, queries, outputs;  // probes per row
  const float* directions;  // [layers + 1][probes][d]
  const float* gain;        // [layers + 1][probes]
  const float* query;       // [queries][d]
  const float* row_bias;    // [queries][(layers + 1) · probes]
  QMat proj;                // outputs × queries · d (padded)
  const float* bias;        // [outputs]
  float *peak, *total, *weighted;  // per slot: [(layers + 1) · probes], the same, × d
};
constexpr int MAX_PROBE_HEADS = 4;

struct CrossLayerDev {
  QMat qg;   // q_proj rows, then gate_proj rows
  QMat kv;   // k_proj rows, then v_proj rows (the memory)
  QMat out;
  const float *norm, *q_norm, *k_norm, *post_norm;
  float gain;  // sigmoid(gate)
};

struct CrossMemDev {
  int frames;
  const int8_t* keys;    // [layers][heads][frames][64] (head-major: one head's rows are contiguous)
  const float* kscale;   // [layers][heads][frames]
  const int8_t* values;  // [layers][heads][frames][64]
  const float* vscale;   // [layers][heads][frames]
};
constexpr int MAX_CROSS_FRAMES = 2048;  // a 30-second window is 1500 frames

struct LayerDev {
  QMat qkvg;  // q, k, v and gate_proj stacked row-wise (one fused product, matrix.rs:167-193)
  QMat out;
  const float *norm_in, *post_norm, *pre_hada, *q_norm, *k_norm;
  float attn_gate;
  HadamardDev hada;
  int global;  // 1 when the layer attends to the whole context
  int index;   // the layer's index in the archive
  const float* taps;  // [conv_taps][q | k | v] causal convolution gains; null without taps
  int engram_site;           // the engram site on this layer (the first listed), -1 for none
  const EngramDev* engram;   // that site's weights and ring (device memory); null for none
};

struct ModelDev {
  uint32_t d_model, heads, kv_heads, vocab, output_vocab, hada_n, hada_left, max_seq_len, num_layers;
  uint32_t sliding_window;
  float sqrt_d;          // (d_model as f32).sqrt()
  float inv_sqrt_group;  // 1 / sqrt(128)
  float inv_root_qk;     // 1 / sqrt(head_dim)
  // embedding: packed 4-bit (or 2-bit) rows for the gather, int8 for logits
  const uint8_t* embed_packed;
  uint32_t embed_bits, embed_row_bytes;
  const float* embed_levels;  // 16 float levels
  const float* embed_norms;   // [vocab][groups]
  QMat logits;                // the tied embedding as a product
  // lanes (crates/model/src/lanes.rs)
  QMat phi_pre, phi_post, phi_res;  // row-major int8, K = lanes * d_model
  const float *a_pre, *a_post, *a_res, *b_pre, *b_post, *b_res;
  const float* final_norm;
  const int32_t* perm1;
  const int32_t* perm2;
  const float2* rotary;       // [max_seq_len][head_dim/2] (sin, cos)
  PageGeometry page;
  int* error;                 // the engine's device flag: set when a bounded device wait gave up
  uint32_t conv_taps;         // QKV causal convolution taps (0 = none)
  uint32_t qkv_width;         // (heads + 2 kv_heads) * head_dim: the convolved part of a projection row
  float* conv_ring;           // [slots][layers][conv_taps - 1][qkv_width]; null when conv_taps < 2
  uint32_t* token_ring;       // [slots][token_rows] (engram sites); null when token_rows == 0
  uint32_t token_rows;        // max order - 1
  uint32_t num_probe_heads;
  const HeadDev* probe_heads;  // [num_probe_heads] (device memory)
  const CrossLayerDev* cross;              // [num_layers] (device memory); null without a Whistle section
  const CrossMemDev* const* slot_cross;    // [slots] the memory each session attends to (null: none)
};

// Per-token metadata of one forward pass.
struct TokenMeta {
  int32_t slot;      // session slot (page table row)
  int32_t position;  // absolute position of this token
  int32_t last;      // 1 when this is the sequence's last token in the pass
  int32_t run;       // bits 0-15: the token's index in its sequence's run of this pass; 16-31: the run's length
};

// Device workspace of a forward pass over at most `capacity` tokens.
struct Work {
  uint32_t capacity;
  const uint32_t* tokens;   // [M] token ids (device)
  const TokenMeta* meta;    // [M]
  const int32_t* order;     // [M] attention CTA row i serves token order[i] (longest contexts first); null = i
  float* stream;            // [M][4][d]
  float* next_stream;       // [M][4][d]
  float* x;                 // [M][d]      routing input, then the block's running value
  float* route;             // [M][4 + 16] post gates and Sinkhorn residual weights
  int8_t* act;              // int8 activations in the core-matrix layout (K = 512), capacity rounded to 128
  float* act_scale;         // [M][groups]
  float* proj;              // [M][q + k + v + gate]
  int8_t* qcodes;           // [M][heads][64]
  float* qscale;            // [M][heads]
  float* attn;              // [M][heads * 64]
  float* outp;              // [M][d]
  int* arrivals;            // [M] attention CTAs done per token (zero between passes)
  float* engram_kv;         // [M][2d] an engram site's key and raw value rows (null without sites)
  float* xin;               // [M][d] the routing input at an engram site layer (x holds it plus the engram term)
  float* cells;             // [M][d] a layer's lane means (probe heads)
  float* scores;            // [M][heads · probes] their probe scores / sqrt(d)
  float* scan;              // [M][heads · probes][2] the run's rescale and weight per token
  float* xr;                // [M][d] x after the attention residual and the cross attention (Whistle)
  float* cq;                // [M][2d] the cross attention's q and gate rows (Whistle)
  uint32_t act_rows;        // rows of the activation buffer's K-chunk-major layout
};

struct KvDev {
  uint8_t* pool;
  const int32_t* page_table;  // [slots][layers][max_pages]
  uint32_t max_pages;
  uint32_t num_layers;
};

}  // namespace nbl
