// kernels.cu — sm_100a kernels of the Needle-3 token loop.
//
// One forward pass runs over a batch of M tokens (any mix of sequences and
// positions; decode is one token per sequence, prefill many per sequence).
// Per active layer:
//   k_route       lane routing (crates/model/src/lanes.rs:146-181), norm_in and
//                 the int8 activation of the attention input
//   k_project     fused q/k/v/gate product (kernels/src/matrix.rs:167-193)
//   k_heads       per-head norm, rotary, int8 codes and the KV-page append
//                 (model/src/attention.rs:118-143)
//   k_attend      paged int8 attention with the 12-bit softmax weights
//                 (kernels/src/attention.rs:251-280, neon.rs:277-437)
//   k_prep        sigmoid gate and int8 activation of the output projection
//   k_project     out_proj
//   k_block       post norm, gated residual, Hadamard MLP and lane combine
//                 (model/src/session.rs:121-137, hadamard.rs:260-304)
// then k_final (lane mean and final norm) and, per generated token, the tied
// logits product and k_select (generator.rs:147-194).
#include <cuda_runtime.h>

#include "device.cuh"
#include "kernels.h"

namespace nbk {

using namespace nbl;

__device__ __forceinline__ void named_barrier(int id, int threads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory"); }

// index `i` of a packed little-endian row of `bits`-wide codes (matrix.rs:622-631)
__device__ __forceinline__ uint32_t code_at(const uint8_t* row, uint32_t i, uint32_t bits) {
  uint32_t bit = i * bits, byte = bit >> 3, shift = bit & 7;
  uint32_t raw = row[byte];
  if (shift + bits > 8) raw |= (uint32_t)row[byte + 1] << 8;
  return (raw >> shift) & ((1u << bits) - 1);
}

__device__ __forceinline__ uint8_t* page_base(const KvDev& kv, const PageGeometry& pg, int slot, int layer, int position) {
  int page = kv.page_table[((size_t)slot * kv.num_layers + layer) * kv.max_pages + position / PAGE_POSITIONS];
  return kv.pool + (size_t)page * pg.page_bytes;
}

// ----------------------------------------------------------------- embedding
// QuantisedMatrix::dequantise_row (matrix.rs:140-153) times sqrt(d), copied
// into every lane (session.rs:84-90). grid M, block 128.
__global__ void __launch_bounds__(128) k_embed(ModelDev md, Work w, int M) {
  int t = blockIdx.x;
  if (t >= M || w.meta[t].slot < 0) return;
  uint32_t token = w.tokens[t];
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int d = md.d_model, groups = d / GROUP;
  const uint8_t* row = md.embed_packed + (size_t)token * md.embed_row_bytes;
  float* out = w.stream + (size_t)t * LANES * d;
  for (int g = warp; g < groups; g += blockDim.x >> 5) {
    float norm = md.embed_norms[(size_t)token * groups + g];
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = fmul(md.embed_levels[code_at(row, g * GROUP + 4 * lane + j, md.embed_bits)], norm);
    fwht128(v, md.inv_sqrt_group);
    float4 o = make_float4(fmul(v[0], md.sqrt_d), fmul(v[1], md.sqrt_d), fmul(v[2], md.sqrt_d), fmul(v[3], md.sqrt_d));
#pragma unroll
    for (int l = 0; l < LANES; ++l) *reinterpret_cast<float4*>(out + l * d + g * GROUP + 4 * lane) = o;
  }
}

// ------------------------------------------------------------------- routing
// grid M, block 256 (8 warps). Warp 7 finishes the Sinkhorn mixing weights
// while warps 0-6 build the block input, norm it and quantise it.
__global__ void __launch_bounds__(256) k_route(ModelDev md, LayerDev L, Work w, int M, int layer, int slot) {
  extern __shared__ float sm[];
  int t = blockIdx.x;
  if (t >= M || w.meta[t].slot < 0) return;
  const int d = md.d_model, n = LANES * d, ng = n / GROUP;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* s_stream = sm;                               // n
  float* s_work = sm + n;                             // n (normalised stream, later x)
  int8_t* s_codes = reinterpret_cast<int8_t*>(sm + 2 * n);  // n bytes
  __shared__ float s_ascale[MAX_D * LANES / GROUP];
  __shared__ float s_red[8];
  __shared__ float s_phi[LANES + LANES + LANES * LANES];
  __shared__ float s_gate[LANES];
  __shared__ float s_inv;

  const float4* src = reinterpret_cast<const float4*>(w.stream + (size_t)t * n);
  for (int i = tid; i < n / 4; i += blockDim.x) reinterpret_cast<float4*>(s_stream)[i] = src[i];
  __syncthreads();
  // unit_rms over all lanes (ops.rs:60-66), then fake_quantise_int8 (ops.rs:120-125)
  if (warp == 0) {
    float ss = sum_of_squares_warp(s_stream, n);
    if (lane == 0) s_inv = inverse_rms(ss, n);
  }
  __syncthreads();
  float inv = s_inv, peak = 0.0f;
  for (int i = tid; i < n; i += blockDim.x) {
    float v = fmul(s_stream[i], inv);
    s_work[i] = v;
    peak = fmaxf(peak, fabsf(v));
  }
  float scale = int8_scale_of(block_max(peak, s_red));
  for (int i = tid; i < n; i += blockDim.x) s_work[i] = fake_quant(s_work[i], scale);
  __syncthreads();
  // rotate and quantise per 128-group (QuantisedMatrix::prepare + PlaneInput)
  for (int g = warp; g < ng; g += 8) {
    float v[4];
    *reinterpret_cast<float4*>(v) = *reinterpret_cast<const float4*>(s_work + g * GROUP + 4 * lane);
    fwht128(v, md.inv_sqrt_group);
    uint32_t packed;
    float sc = quantise_group(v, packed);
    *reinterpret_cast<uint32_t*>(s_codes + g * GROUP + 4 * lane) = packed;
    if (lane == 0) s_ascale[g] = sc;
  }
  __syncthreads();
  // phi products: 4 pre rows, 4 post rows, 16 residual rows of this layer
  // (lanes.rs:156-163), 4-bit row combine (neon.rs:164-183)
  for (int r = warp; r < 24; r += 8) {
    const QMat& P = r < 4 ? md.phi_pre : (r < 8 ? md.phi_post : md.phi_res);
    int row = r < 4 ? layer * LANES + r : (r < 8 ? layer * LANES + (r - 4) : layer * LANES * LANES + (r - 8));
    const uint32_t* wrow = reinterpret_cast<const uint32_t*>(P.codes + (size_t)row * n);
    const uint32_t* arow = reinterpret_cast<const uint32_t*>(s_codes);
    float total = 0.0f;
    for (int g = 0; g < ng; ++g) {
      int acc = dp4a(wrow[g * 32 + lane], arow[g * 32 + lane], 0);
      acc = warp_sum_int(acc);
      total = fadd(total, fmul(fmul(fmul((float)acc, P.scales[(size_t)row * ng + g]), P.level_scale), s_ascale[g]));
    }
    if (lane == 0) s_phi[r] = total;
  }
  __syncthreads();
  float* route_out = w.route + (size_t)t * (LANES + LANES * LANES);
  if (warp == 7) {
    // post gates and the Sinkhorn-normalised residual mixing (lanes.rs:166-179, ops.rs:198-217)
    if (lane < LANES) {
      float off = lane == (slot % LANES) ? 0.0f : -4.0f;
      float p = fadd(fadd(fmul(md.a_post[layer], s_phi[4 + lane]), md.b_post[layer * LANES + lane]), off);
      route_out[lane] = fmul(2.0f, sigmoid(p));
    }
    if (lane == 0) {
      float x[16];
      for (int i = 0; i < 16; ++i) x[i] = fadd(fmul(md.a_res[layer], s_phi[8 + i]), md.b_res[layer * 16 + i]);
      for (int r = 0; r < 4; ++r) {
        float pk = -INFINITY;
        for (int c = 0; c < 4; ++c) pk = fmaxf(pk, x[r * 4 + c]);
        for (int c = 0; c < 4; ++c) x[r * 4 + c] = expf_libm(fsub(x[r * 4 + c], pk));
      }
      const float MIN_POSITIVE = 1.17549435e-38f;
      for (int it = 0; it < 20; ++it) {
        for (int r = 0; r < 4; ++r) {
          float tot = fadd(fadd(fadd(fadd(SUM_START, x[r * 4]), x[r * 4 + 1]), x[r * 4 + 2]), x[r * 4 + 3]);
          float iv = frcp(fmaxf(tot, MIN_POSITIVE));
          for (int c = 0; c < 4; ++c) x[r * 4 + c] = fmul(x[r * 4 + c], iv);
        }
        for (int c = 0; c < 4; ++c) {
          float tot = fadd(fadd(fadd(fadd(SUM_START, x[c]), x[4 + c]), x[8 + c]), x[12 + c]);
          float iv = frcp(fmaxf(tot, MIN_POSITIVE));
          for (int r = 0; r < 4; ++r) x[r * 4 + c] = fmul(x[r * 4 + c], iv);
        }
      }
      for (int i = 0; i < 16; ++i) route_out[LANES + i] = x[i];
    }
    return;
  }
  // warps 0-6 (224 threads) from here on
  const int nthreads = 224;
  if (tid < LANES) {
    float off = tid == (slot % LANES) ? 8.0f + -4.0f : -4.0f;
    s_gate[tid] = sigmoid(fadd(fadd(fmul(md.a_pre[layer], s_phi[tid]), md.b_pre[layer * LANES + tid]), off));
  }
  named_barrier(1, nthreads);
  float* s_x = s_work;  // reuse: the block input x (lanes.rs:169-171)
  float* xg = w.x + (size_t)t * d;
  for (int i = tid; i < d; i += nthreads) {
    float acc = 0.0f;
#pragma unroll
    for (int l = 0; l < LANES; ++l) acc = fadd(acc, fmul(s_gate[l], s_stream[l * d + i]));
    s_x[i] = acc;
    xg[i] = acc;
  }
  named_barrier(1, nthreads);
  if (warp == 0) {
    float ss = sum_of_squares_warp(s_x, d);
    if (lane == 0) s_inv = inverse_rms(ss, d);
  }
  named_barrier(1, nthreads);
  // zero_centred_norm (ops.rs:44-50) then fake_quantise_int8 (attention.rs:99-100)
  float* s_y = s_stream;  // reuse
  inv = s_inv;
  peak = 0.0f;
  for (int i = tid; i < d; i += nthreads) {
    float v = fmul(fmul(fadd(1.0f, L.norm_in[i]), s_x[i]), inv);
    s_y[i] = v;
    peak = fmaxf(peak, fabsf(v));
  }
  peak = warp_max(peak);
  if (lane == 0) s_red[warp] = peak;
  named_barrier(1, nthreads);
  peak = s_red[0];
  for (int i = 1; i < 7; ++i) peak = fmaxf(peak, s_red[i]);
  scale = int8_scale_of(peak);
  const int dg = d / GROUP;
  int8_t* act = w.act + (size_t)t * d;
  for (int g = warp; g < dg; g += 7) {
    float v[4];
    for (int j = 0; j < 4; ++j) v[j] = fake_quant(s_y[g * GROUP + 4 * lane + j], scale);
    fwht128(v, md.inv_sqrt_group);
    uint32_t packed;
    float sc = quantise_group(v, packed);
    *reinterpret_cast<uint32_t*>(act + g * GROUP + 4 * lane) = packed;
    if (lane == 0) w.act_scale[(size_t)t * dg + g] = sc;
  }
}

// --------------------------------------------------------------- projection
// out[m][row] for rows of W and tokens m: per (row, 128-group) an exact int32
// dot product, then the groups combined in order — fused for 2-bit matrices
// (panel.rs:184-187), a product chain for 4-bit ones (neon.rs:180).
// Lane (r, g) of a warp owns group g of row 8·warp + r and keeps its 128
// weight codes in registers while it walks the tokens. grid (ceil(rows/64),
// token chunks), block 256.
template <int GK>
__global__ void __launch_bounds__(256) k_project(QMat W, const int8_t* __restrict__ act, const float* __restrict__ act_scale,
                                                 float* __restrict__ out, int M, int out_stride, int tokens_per_cta,
                                                 const TokenMeta* __restrict__ meta) {
  constexpr int RB = 32 / GK;
  constexpr int K = GK * GROUP;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rowblock = blockIdx.x * 8 + warp;
  if (rowblock * RB >= (int)W.rows) return;
  const int r = lane / GK, g = lane % GK;
  const int row = rowblock * RB + r;
  const bool valid = row < (int)W.rows;
  uint4 wv[8];
  const uint4* base = reinterpret_cast<const uint4*>(W.codes) + (size_t)rowblock * 8 * 32;
#pragma unroll
  for (int k = 0; k < 8; ++k) wv[k] = valid ? base[k * 32 + lane] : make_uint4(0, 0, 0, 0);
  const float wscale = valid ? W.scales[(size_t)row * GK + g] : 0.0f;
  const int m0 = blockIdx.y * tokens_per_cta, m1 = min(M, m0 + tokens_per_cta);
  const int leader = r * GK;
  for (int m = m0; m < m1; ++m) {
    if (meta && meta[m].slot < 0) continue;
    const uint4* a = reinterpret_cast<const uint4*>(act + (size_t)m * K + g * GROUP);
    int acc = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint4 av = a[k];
      acc = dp4a(wv[k].x, av.x, acc);
      acc = dp4a(wv[k].y, av.y, acc);
      acc = dp4a(wv[k].z, av.z, acc);
      acc = dp4a(wv[k].w, av.w, acc);
    }
    const float as = act_scale[(size_t)m * GK + g];
    float total = 0.0f;
#pragma unroll
    for (int gg = 0; gg < GK; ++gg) {
      int ag = __shfl_sync(FULL, acc, leader + gg);
      float ws = __shfl_sync(FULL, wscale, leader + gg);
      float asg = __shfl_sync(FULL, as, leader + gg);
      if (W.fused)
        total = __fmaf_rn((float)ag, fmul(ws, asg), total);
      else
        total = fadd(total, fmul(fmul(fmul((float)ag, ws), W.level_scale), asg));
    }
    if (g == 0 && valid) out[(size_t)m * out_stride + row] = total;
  }
}

// ------------------------------------------------------------------- heads
// grid M, block 32·(heads + 2·kv_heads). One warp per q, k or v head; lane l
// holds elements l and l+32, the two halves rotary pairs (ops.rs:131-141).
__global__ void k_heads(ModelDev md, LayerDev L, Work w, KvDev kv, int M, int layer) {
  int t = blockIdx.x;
  if (t >= M) return;
  TokenMeta meta = w.meta[t];
  if (meta.slot < 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = md.heads, KV = md.kv_heads;
  // proj rows: q [H*64] | k [KV*64] | v [KV*64] | gate [H*64]
  const float* row = w.proj + (size_t)t * (2 * H + 2 * KV) * HEAD_DIM;
  const int kind = warp < H ? 0 : (warp < H + KV ? 1 : 2);
  const int head = kind == 0 ? warp : (kind == 1 ? warp - H : warp - H - KV);
  const float* src = row + (kind == 0 ? 0 : (kind == 1 ? H * HEAD_DIM : (H + KV) * HEAD_DIM)) + head * HEAD_DIM;
  float e0 = src[lane], e1 = src[lane + 32];
  if (kind != 2) {
    // zero_centred_norm_in_place over the head (ops.rs:52-58): lane l < 8 runs
    // the chain over elements l, l+8, ..., l+56
    float acc = 0.0f;
    const int chain = lane & 7;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float v = __shfl_sync(FULL, e0, chain + 8 * c);
      acc = fadd(acc, fmul(v, v));
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float v = __shfl_sync(FULL, e1, chain + 8 * c);
      acc = fadd(acc, fmul(v, v));
    }
    float s = SUM_START;
#pragma unroll
    for (int l = 0; l < 8; ++l) s = fadd(s, __shfl_sync(FULL, acc, l));
    float inv = inverse_rms(s, HEAD_DIM);
    const float* gain = kind == 0 ? L.q_norm : L.k_norm;
    e0 = fmul(fmul(fadd(1.0f, gain[lane]), e0), inv);
    e1 = fmul(fmul(fadd(1.0f, gain[lane + 32]), e1), inv);
    float2 sc = md.rotary[(size_t)meta.position * (HEAD_DIM / 2) + lane];
    float a = e0, b = e1;
    e0 = fsub(fmul(a, sc.y), fmul(b, sc.x));
    e1 = fadd(fmul(b, sc.y), fmul(a, sc.x));
  }
  // quantise_int8 (ops.rs:112-118)
  float peak = warp_max(fmaxf(fabsf(e0), fabsf(e1)));
  float scale = int8_scale_of(peak);
  int8_t c0 = (int8_t)clampf(rintf(fdiv(e0, scale)), -128.0f, 127.0f);
  int8_t c1 = (int8_t)clampf(rintf(fdiv(e1, scale)), -128.0f, 127.0f);
  if (kind == 0) {
    int8_t* q = w.qcodes + ((size_t)t * H + head) * HEAD_DIM;
    q[lane] = c0;
    q[lane + 32] = c1;
    if (lane == 0) w.qscale[(size_t)t * H + head] = scale;
    return;
  }
  const PageGeometry& pg = md.page;
  uint8_t* page = page_base(kv, pg, meta.slot, layer, meta.position);
  int p = meta.position % PAGE_POSITIONS;
  if (kind == 1) {
    int8_t* key = reinterpret_cast<int8_t*>(page) + ((size_t)head * PAGE_POSITIONS + p) * HEAD_DIM;
    key[lane] = c0;
    key[lane + 32] = c1;
    if (lane == 0) reinterpret_cast<float*>(page + pg.kscale_offset)[head * PAGE_POSITIONS + p] = scale;
  } else {
    int8_t* panel = reinterpret_cast<int8_t*>(page + pg.value_offset) + (size_t)head * PAGE_POSITIONS * HEAD_DIM + (p / 4) * (HEAD_DIM * 4) + (p % 4);
    panel[lane * 4] = c0;
    panel[(lane + 32) * 4] = c1;
    if (lane == 0) reinterpret_cast<float*>(page + pg.vscale_offset)[head * PAGE_POSITIONS + p] = scale;
  }
}

// ---------------------------------------------------------------- attention
// grid (M, kv_heads), block 160: warps 0-3 score, weight and accumulate the
// values of the kv head's query heads; warp 4 forms the softmax totals in the
// reference's order (four running lanes, (l0+l1)+(l2+l3), then the tail;
// neon.rs:277-307) while warps 0-3 accumulate.
constexpr int ATT_THREADS = 128;
constexpr int MAX_GROUP = 4;

template <int G>
__global__ void __launch_bounds__(160) k_attend(ModelDev md, Work w, KvDev kv, int M, int layer, int global, int t_cap) {
  extern __shared__ float sm[];
  const int t = blockIdx.x, kvh = blockIdx.y;
  if (t >= M) return;
  const TokenMeta meta = w.meta[t];
  if (meta.slot < 0) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = meta.position + 1;
  int first = 0;
  if (md.sliding_window > 0 && !global) first = total > (int)md.sliding_window ? total - (int)md.sliding_window : 0;
  const int count = total - first;
  const int b0 = first / 4, nblk = (total - 1) / 4 - b0 + 1;
  float* s_coef = sm;                                   // [G][t_cap]
  float* s_e = sm + G * t_cap;                          // [G][t_cap]
  uint32_t* s_whi = reinterpret_cast<uint32_t*>(sm + 2 * G * t_cap);  // [G][t_cap/4 + 2]
  uint32_t* s_wlo = s_whi + G * (t_cap / 4 + 2);
  int* s_pv = reinterpret_cast<int*>(s_wlo + G * (t_cap / 4 + 2));     // [8][G][64]
  __shared__ uint32_t s_q[MAX_GROUP][16];
  __shared__ float s_qs[MAX_GROUP], s_peak[MAX_GROUP], s_scale2[MAX_GROUP], s_total[MAX_GROUP];
  __shared__ float s_red[MAX_GROUP][4];
  const PageGeometry& pg = md.page;
  const int* table = kv.page_table + ((size_t)meta.slot * kv.num_layers + layer) * kv.max_pages;

  if (tid < G * 16) {
    int h = tid / 16, k = tid % 16;
    s_q[h][k] = reinterpret_cast<const uint32_t*>(w.qcodes + ((size_t)t * md.heads + kvh * G + h) * HEAD_DIM)[k];
  }
  if (tid < G) s_qs[tid] = fmul(w.qscale[(size_t)t * md.heads + kvh * G + tid], md.inv_root_qk);
  __syncthreads();

  if (tid < ATT_THREADS) {
    // pass 1: integer scores, coefficients (s · key_scale) · query_scale and their peak
    float lmax[G];
#pragma unroll
    for (int h = 0; h < G; ++h) lmax[h] = -INFINITY;
    for (int i = tid; i < count; i += ATT_THREADS) {
      int p = first + i;
      const uint8_t* page = kv.pool + (size_t)table[p / PAGE_POSITIONS] * pg.page_bytes;
      const uint4* key = reinterpret_cast<const uint4*>(page + ((size_t)kvh * PAGE_POSITIONS + p % PAGE_POSITIONS) * HEAD_DIM);
      uint4 k0 = key[0], k1 = key[1], k2 = key[2], k3 = key[3];
      float ks = reinterpret_cast<const float*>(page + pg.kscale_offset)[kvh * PAGE_POSITIONS + p % PAGE_POSITIONS];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const uint32_t* q = s_q[h];
        int s = 0;
        s = dp4a(k0.x, q[0], s); s = dp4a(k0.y, q[1], s); s = dp4a(k0.z, q[2], s); s = dp4a(k0.w, q[3], s);
        s = dp4a(k1.x, q[4], s); s = dp4a(k1.y, q[5], s); s = dp4a(k1.z, q[6], s); s = dp4a(k1.w, q[7], s);
        s = dp4a(k2.x, q[8], s); s = dp4a(k2.y, q[9], s); s = dp4a(k2.z, q[10], s); s = dp4a(k2.w, q[11], s);
        s = dp4a(k3.x, q[12], s); s = dp4a(k3.y, q[13], s); s = dp4a(k3.z, q[14], s); s = dp4a(k3.w, q[15], s);
        float c = fmul(fmul((float)s, ks), s_qs[h]);
        s_coef[h * t_cap + i] = c;
        lmax[h] = fmaxf(lmax[h], c);
      }
    }
    for (int h = 0; h < G; ++h) {
      float m = warp_max(lmax[h]);
      if (lane == 0) s_red[h][warp] = m;
    }
  }
  __syncthreads();
  if (tid < G) s_peak[tid] = fmaxf(fmaxf(s_red[tid][0], s_red[tid][1]), fmaxf(s_red[tid][2], s_red[tid][3]));
  __syncthreads();
  if (tid < ATT_THREADS) {
    // pass 2: e = fast_exp(c - peak), weight = e · value_scale, and the weights' peak
    float lmax[G];
#pragma unroll
    for (int h = 0; h < G; ++h) lmax[h] = 0.0f;
    for (int i = tid; i < count; i += ATT_THREADS) {
      int p = first + i;
      const uint8_t* page = kv.pool + (size_t)table[p / PAGE_POSITIONS] * pg.page_bytes;
      float vs = reinterpret_cast<const float*>(page + pg.vscale_offset)[kvh * PAGE_POSITIONS + p % PAGE_POSITIONS];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float e = fast_exp(fsub(s_coef[h * t_cap + i], s_peak[h]));
        s_e[h * t_cap + i] = e;
        float c2 = fmul(e, vs);
        s_coef[h * t_cap + i] = c2;
        lmax[h] = fmaxf(lmax[h], fabsf(c2));
      }
    }
    for (int h = 0; h < G; ++h) {
      float m = warp_max(lmax[h]);
      if (lane == 0) s_red[h][warp] = m;
    }
  }
  __syncthreads();
  if (tid < G) {
    float pk = fmaxf(fmaxf(s_red[tid][0], s_red[tid][1]), fmaxf(s_red[tid][2], s_red[tid][3]));
    s_peak[tid] = pk;
    s_scale2[tid] = fdiv(pk, 2047.0f);
  }
  __syncthreads();
  if (warp == 4) {
    // softmax totals in the order of neon.rs:294-305
    int h = lane >> 2, j = lane & 3;
    int vc = count - count % 4;
    float acc = 0.0f;
    if (h < G)
      for (int i = j; i < vc; i += 4) acc = fadd(acc, s_e[h * t_cap + i]);
    float l0 = __shfl_sync(FULL, acc, (lane & ~3) + 0), l1 = __shfl_sync(FULL, acc, (lane & ~3) + 1);
    float l2 = __shfl_sync(FULL, acc, (lane & ~3) + 2), l3 = __shfl_sync(FULL, acc, (lane & ~3) + 3);
    if (h < G && j == 0) {
      float tot = fadd(fadd(l0, l1), fadd(l2, l3));
      for (int i = vc; i < count; ++i) tot = fadd(tot, s_e[h * t_cap + i]);
      s_total[h] = tot;
    }
  } else {
    // pass 3: 12-bit weights round(c / (peak / 2047)) (half away from zero),
    // split into 6-bit halves per absolute 4-position block (neon.rs:348-365)
    for (int b = tid; b < nblk; b += ATT_THREADS) {
      int pbase = (b0 + b) * 4;
      for (int h = 0; h < G; ++h) {
        uint32_t hi = 0, lo = 0;
        float sc = s_scale2[h];
        bool live = s_peak[h] > 0.0f;
        for (int j = 0; j < 4; ++j) {
          int p = pbase + j;
          int wgt = 0;
          if (live && p >= first && p < total) wgt = (int)roundf(fdiv(s_coef[h * t_cap + (p - first)], sc));
          hi |= (uint32_t)((wgt >> 6) & 0xff) << (8 * j);
          lo |= (uint32_t)((wgt & 63) & 0xff) << (8 * j);
        }
        s_whi[h * (t_cap / 4 + 2) + b] = hi;
        s_wlo[h * (t_cap / 4 + 2) + b] = lo;
      }
    }
    named_barrier(1, ATT_THREADS);
    // pass 4: exact integer sums over the value panels; thread (dq, slice) owns
    // four dimensions and every eighth block
    const int dq = tid & 15, slice = tid >> 4;
    int hi_acc[G][4], lo_acc[G][4];
#pragma unroll
    for (int h = 0; h < G; ++h)
      for (int k = 0; k < 4; ++k) hi_acc[h][k] = lo_acc[h][k] = 0;
    for (int b = slice; b < nblk; b += 8) {
      int p = (b0 + b) * 4;
      const uint8_t* page = kv.pool + (size_t)table[p / PAGE_POSITIONS] * pg.page_bytes;
      uint4 v = *reinterpret_cast<const uint4*>(page + pg.value_offset + (size_t)kvh * PAGE_POSITIONS * HEAD_DIM +
                                                ((p % PAGE_POSITIONS) / 4) * (HEAD_DIM * 4) + dq * 16);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        uint32_t whi = s_whi[h * (t_cap / 4 + 2) + b], wlo = s_wlo[h * (t_cap / 4 + 2) + b];
        hi_acc[h][0] = dp4a(v.x, whi, hi_acc[h][0]);
        hi_acc[h][1] = dp4a(v.y, whi, hi_acc[h][1]);
        hi_acc[h][2] = dp4a(v.z, whi, hi_acc[h][2]);
        hi_acc[h][3] = dp4a(v.w, whi, hi_acc[h][3]);
        lo_acc[h][0] = dp4a(v.x, wlo, lo_acc[h][0]);
        lo_acc[h][1] = dp4a(v.y, wlo, lo_acc[h][1]);
        lo_acc[h][2] = dp4a(v.z, wlo, lo_acc[h][2]);
        lo_acc[h][3] = dp4a(v.w, wlo, lo_acc[h][3]);
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int k = 0; k < 4; ++k) s_pv[(slice * G + h) * HEAD_DIM + dq * 4 + k] = (hi_acc[h][k] << 6) + lo_acc[h][k];
  }
  __syncthreads();
  if (tid < ATT_THREADS) {
    for (int o = tid; o < G * HEAD_DIM; o += ATT_THREADS) {
      int h = o / HEAD_DIM, dim = o % HEAD_DIM;
      int sum = 0;
      for (int s = 0; s < 8; ++s) sum += s_pv[(s * G + h) * HEAD_DIM + dim];
      float value = s_peak[h] > 0.0f ? fmul((float)sum, s_scale2[h]) : 0.0f;
      float inverse = fdiv(1.0f, s_total[h]);
      w.attn[(size_t)t * md.heads * HEAD_DIM + (kvh * G + h) * HEAD_DIM + dim] = fmul(value, inverse);
    }
  }
}

// ------------------------------------------------------ int8 activation prep
// in[m] (K values, optionally times sigmoid(gate[m])) → fake_quantise_int8 →
// per-group rotation and int8 codes. Used for out_proj (attention.rs:145-150)
// and the logits (session.rs:170-175). grid M, block 128.
__global__ void __launch_bounds__(128) k_prep(const float* __restrict__ in, int in_stride, const int32_t* __restrict__ rows,
                                              const float* __restrict__ gate, int gate_stride, int K, int8_t* __restrict__ act,
                                              float* __restrict__ act_scale, int M, const TokenMeta* __restrict__ meta,
                                              float inv_sqrt_group, int fake) {
  __shared__ float s_v[MAX_D];
  __shared__ float s_red[4];
  int t = blockIdx.x;
  if (t >= M || (meta && meta[t].slot < 0)) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* src = in + (size_t)(rows ? rows[t] : t) * in_stride;
  float peak = 0.0f;
  for (int i = tid; i < K; i += blockDim.x) {
    float v = src[i];
    if (gate) v = fmul(v, sigmoid(gate[(size_t)t * gate_stride + i]));
    s_v[i] = v;
    peak = fmaxf(peak, fabsf(v));
  }
  float scale = int8_scale_of(block_max(peak, s_red));
  const int groups = K / GROUP;
  for (int g = warp; g < groups; g += blockDim.x >> 5) {
    float v[4];
    for (int j = 0; j < 4; ++j) v[j] = fake ? fake_quant(s_v[g * GROUP + 4 * lane + j], scale) : s_v[g * GROUP + 4 * lane + j];
    fwht128(v, inv_sqrt_group);
    uint32_t packed;
    float sc = quantise_group(v, packed);
    *reinterpret_cast<uint32_t*>(act + (size_t)t * K + g * GROUP + 4 * lane) = packed;
    if (lane == 0) act_scale[(size_t)t * groups + g] = sc;
  }
}

// ------------------------------------------------------------ block finish
// grid M, block 512. Post norm, gated residual (session.rs:121-125), the
// Hadamard MLP (hadamard.rs:260-304) and the lane combine (lanes.rs:183-204).
template <int LEFT, bool FUSED32>
__device__ __forceinline__ void kronecker(const float* __restrict__ X, const float* __restrict__ Lf, const float* __restrict__ R,
                                          float* __restrict__ mixed, float* __restrict__ out) {
  // ops.rs:143-164: mixed = X·R (sequential over j), out = Lᵀ·mixed (sequential over i).
  // FUSED32 restates the aarch64 32×32 path, which fuses each step (ops.rs:219-299).
  constexpr int PER = LEFT * HADA_RIGHT / 512;
  const int tid = threadIdx.x, c = tid & 31, r0 = tid >> 5;
  float acc[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) acc[q] = 0.0f;
  for (int j = 0; j < HADA_RIGHT; ++j) {
    float rv = R[j * HADA_RIGHT + c];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      float xv = X[(r0 + 16 * q) * HADA_RIGHT + j];
      acc[q] = FUSED32 ? __fmaf_rn(rv, xv, acc[q]) : fadd(acc[q], fmul(xv, rv));
    }
  }
#pragma unroll
  for (int q = 0; q < PER; ++q) mixed[(r0 + 16 * q) * HADA_RIGHT + c] = acc[q];
  __syncthreads();
#pragma unroll
  for (int q = 0; q < PER; ++q) acc[q] = 0.0f;
  for (int i = 0; i < LEFT; ++i) {
    float mv = mixed[i * HADA_RIGHT + c];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      float lv = Lf[i * LEFT + r0 + 16 * q];
      acc[q] = FUSED32 ? __fmaf_rn(mv, lv, acc[q]) : fadd(acc[q], fmul(lv, mv));
    }
  }
#pragma unroll
  for (int q = 0; q < PER; ++q) out[(r0 + 16 * q) * HADA_RIGHT + c] = acc[q];
  __syncthreads();
}

template <int LEFT>
__global__ void __launch_bounds__(512) k_block(ModelDev md, LayerDev L, Work w, int M) {
  extern __shared__ float sm[];
  constexpr int N = LEFT * HADA_RIGHT;
  constexpr bool FUSED32 = LEFT == 32;
  const int t = blockIdx.x;
  if (t >= M || w.meta[t].slot < 0) return;
  const int d = md.d_model, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* s_a = sm;               // d
  float* s_x = sm + MAX_D;       // d
  float* s_pre = sm + 2 * MAX_D; // d
  float* s_buf0 = sm + 3 * MAX_D;       // N
  float* s_buf1 = s_buf0 + N;           // N
  float* s_mod = s_buf1 + N;            // N
  float* s_left = s_mod + N;            // LEFT*LEFT
  float* s_right = s_left + LEFT * LEFT;  // 32*32
  __shared__ float s_inv, s_gate, s_w[COND_RANK], s_chain[4][COND_RANK];

  for (int i = tid; i < d; i += blockDim.x) {
    s_a[i] = w.outp[(size_t)t * d + i];
    s_x[i] = w.x[(size_t)t * d + i];
  }
  if (tid == 0) s_gate = sigmoid(L.attn_gate);
  __syncthreads();
  if (warp == 0) {
    float ss = sum_of_squares_warp(s_a, d);
    if (lane == 0) s_inv = inverse_rms(ss, d);
  }
  __syncthreads();
  for (int i = tid; i < d; i += blockDim.x) {
    float a = fmul(fmul(fadd(1.0f, L.post_norm[i]), s_a[i]), s_inv);
    s_a[i] = fadd(s_x[i], fmul(s_gate, a));  // s_a now holds the running block value
  }
  __syncthreads();
  if (warp == 0) {
    float ss = sum_of_squares_warp(s_a, d);
    if (lane == 0) s_inv = inverse_rms(ss, d);
  }
  __syncthreads();
  for (int i = tid; i < d; i += blockDim.x) s_pre[i] = fmul(fmul(fadd(1.0f, L.pre_hada[i]), s_a[i]), s_inv);
  __syncthreads();
  const HadamardDev& Hd = L.hada;
  // condition weights: four chains of rank-8 partial sums (hadamard.rs:263-276)
  if (tid < 4 * COND_RANK) {
    int j = tid / COND_RANK, rr = tid % COND_RANK;
    float acc = 0.0f;
    for (int g = 0; 4 * g + j < d; ++g) acc = fadd(acc, fmul(s_pre[4 * g + j], Hd.cond_v[(4 * g + j) * COND_RANK + rr]));
    s_chain[j][rr] = acc;
  }
  __syncthreads();
  if (tid == 0) {
    float wv[COND_RANK], peak = -INFINITY;
    for (int rr = 0; rr < COND_RANK; ++rr) {
      wv[rr] = fadd(fadd(fadd(fadd(0.0f, s_chain[0][rr]), s_chain[1][rr]), s_chain[2][rr]), s_chain[3][rr]);
      peak = fmaxf(peak, wv[rr]);
    }
    float total = 0.0f;
    for (int rr = 0; rr < COND_RANK; ++rr) {
      wv[rr] = fast_exp(fsub(wv[rr], peak));
      total = fadd(total, wv[rr]);
    }
    float inverse = fdiv(1.0f, total);
    for (int rr = 0; rr < COND_RANK; ++rr) s_w[rr] = fmul(wv[rr], inverse);
  }
  __syncthreads();
  for (int i = tid; i < N; i += blockDim.x) {
    float m = 1.0f;
    for (int rr = 0; rr < COND_RANK; ++rr) m = fadd(m, fmul(s_w[rr], Hd.cond_u[rr * N + i]));
    s_mod[i] = m;
    s_buf0[i] = fmul(i < d ? s_pre[i] : 0.0f, Hd.d1[i]);
  }
  for (int i = tid; i < LEFT * LEFT; i += blockDim.x) s_left[i] = Hd.left[0][i];
  for (int i = tid; i < HADA_RIGHT * HADA_RIGHT; i += blockDim.x) s_right[i] = Hd.right[0][i];
  __syncthreads();
  kronecker<LEFT, FUSED32>(s_buf0, s_left, s_right, s_buf1, s_buf0);  // first = K1(d1 ⊙ x)
  for (int i = tid; i < N; i += blockDim.x) {
    float g = s_buf0[md.perm1[i]];
    s_buf1[i] = silu(fadd(fmul(fmul(Hd.d2[i], s_mod[i]), g), Hd.b2[i]));
  }
  for (int i = tid; i < LEFT * LEFT; i += blockDim.x) s_left[i] = Hd.left[1][i];
  for (int i = tid; i < HADA_RIGHT * HADA_RIGHT; i += blockDim.x) s_right[i] = Hd.right[1][i];
  __syncthreads();
  kronecker<LEFT, FUSED32>(s_buf1, s_left, s_right, s_mod, s_buf1);  // second (s_mod is free now)
  for (int i = tid; i < N; i += blockDim.x) s_buf0[i] = fmul(s_buf1[md.perm2[i]], Hd.d3[i]);
  for (int i = tid; i < LEFT * LEFT; i += blockDim.x) s_left[i] = Hd.left[2][i];
  for (int i = tid; i < HADA_RIGHT * HADA_RIGHT; i += blockDim.x) s_right[i] = Hd.right[2][i];
  __syncthreads();
  kronecker<LEFT, FUSED32>(s_buf0, s_left, s_right, s_buf1, s_buf0);  // third
  // x += mlp; delta = x - input; next lanes (lanes.rs:183-204)
  const float* route = w.route + (size_t)t * (LANES + LANES * LANES);
  const float* stream = w.stream + (size_t)t * LANES * d;
  float* next = w.next_stream + (size_t)t * LANES * d;
  for (int i = tid; i < d; i += blockDim.x) {
    float xv = fadd(s_a[i], fmul(s_buf0[i], Hd.d4[i]));
    float delta = fsub(xv, s_x[i]);
#pragma unroll
    for (int l = 0; l < LANES; ++l) {
      float acc = 0.0f;
#pragma unroll
      for (int s = 0; s < LANES; ++s) acc = fadd(acc, fmul(route[LANES + l * LANES + s], stream[s * d + i]));
      next[l * d + i] = fadd(acc, fmul(route[l], delta));
    }
  }
}

// ------------------------------------------------------------------- final
// lane_mean (session.rs:192-200) and the final zero-centred norm into the
// sequence's hidden state, for the last token of each sequence. grid M, block 128.
__global__ void __launch_bounds__(128) k_final(ModelDev md, Work w, float* __restrict__ hidden, int M) {
  __shared__ float s_mean[MAX_D];
  __shared__ float s_inv;
  int t = blockIdx.x;
  if (t >= M) return;
  TokenMeta meta = w.meta[t];
  if (meta.slot < 0 || !meta.last) return;
  const int d = md.d_model, tid = threadIdx.x;
  const float* stream = w.stream + (size_t)t * LANES * d;
  for (int i = tid; i < d; i += blockDim.x) {
    float m = 0.0f;
#pragma unroll
    for (int l = 0; l < LANES; ++l) m = fadd(m, fdiv(stream[l * d + i], (float)LANES));
    s_mean[i] = m;
  }
  __syncthreads();
  if (tid < 32) {
    float ss = sum_of_squares_warp(s_mean, d);
    if (tid == 0) s_inv = inverse_rms(ss, d);
  }
  __syncthreads();
  for (int i = tid; i < d; i += blockDim.x) hidden[(size_t)meta.slot * d + i] = fmul(fmul(fadd(1.0f, md.final_norm[i]), s_mean[i]), s_inv);
}

// ------------------------------------------------------------------ select
// argmax / argmax_allowed (generator.rs:147-165): the first index holding the
// maximum over the allowed ids, or over all ids when none is allowed.
// grid B, block 256.
__global__ void __launch_bounds__(256) k_select(const float* __restrict__ logits, int V, const uint32_t* __restrict__ mask,
                                                const int32_t* __restrict__ active, uint32_t* __restrict__ next,
                                                float* __restrict__ peaks) {
  __shared__ float s_red[8];
  __shared__ int s_idx[8];
  __shared__ int s_any;
  const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (active && active[b] == 0) {
    if (tid == 0) next[b] = 0xffffffffu;
    return;
  }
  const float* v = logits + (size_t)b * V;
  const uint32_t* m = mask ? mask + (size_t)b * (V / 32) : nullptr;
  float pk_all = -INFINITY, pk_allowed = -INFINITY;
  int any = 0;
  for (int i = tid; i < V; i += blockDim.x) {
    float x = v[i];
    pk_all = fmaxf(pk_all, x);
    bool ok = m ? ((m[i >> 5] >> (i & 31)) & 1u) : true;
    if (ok) {
      pk_allowed = fmaxf(pk_allowed, x);
      any = 1;
    }
  }
  if (tid == 0) s_any = 0;
  __syncthreads();
  if (any) s_any = 1;
  float all = block_max(pk_all, s_red);
  float allowed = block_max(pk_allowed, s_red);
  bool restricted = m && s_any;
  float target = restricted ? allowed : all;
  int best = 0x7fffffff;
  for (int i = tid; i < V; i += blockDim.x) {
    bool ok = restricted ? ((m[i >> 5] >> (i & 31)) & 1u) : true;
    if (ok && v[i] == target) {
      best = i;
      break;
    }
  }
  for (int s = 16; s > 0; s >>= 1) best = min(best, __shfl_xor_sync(FULL, best, s));
  __syncthreads();
  if (lane == 0) s_idx[warp] = best;
  __syncthreads();
  if (tid == 0) {
    int r = s_idx[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) r = min(r, s_idx[i]);
    if (r == 0x7fffffff) r = 0;  // every value NaN: argmax keeps index 0
    next[b] = (uint32_t)r;
    if (peaks) {
      peaks[2 * b] = all;
      peaks[2 * b + 1] = m ? allowed : all;
    }
  }
}

// allowed_statistics (generator.rs:182-194) with the reference's sequential
// sums. grid B, block 256: exponentials in parallel, then two ordered chains.
__global__ void __launch_bounds__(256) k_stats(const float* __restrict__ logits, int V, const uint32_t* __restrict__ mask,
                                               const int32_t* __restrict__ active, const uint32_t* __restrict__ next,
                                               const float* __restrict__ peaks, float* __restrict__ stats, int stats_stride) {
  extern __shared__ float sm[];
  const int b = blockIdx.x, tid = threadIdx.x;
  if (active && active[b] == 0) return;
  const float* v = logits + (size_t)b * V;
  const uint32_t* m = mask ? mask + (size_t)b * (V / 32) : nullptr;
  const float pk_all = peaks[2 * b], pk_allowed = peaks[2 * b + 1];
  float* e_all = sm;
  float* e_allowed = sm + V;
  for (int i = tid; i < V; i += blockDim.x) {
    bool ok = m ? ((m[i >> 5] >> (i & 31)) & 1u) : true;
    e_all[i] = fast_exp(fsub(v[i], pk_all));
    e_allowed[i] = fmul(fast_exp(fsub(v[i], pk_allowed)), ok ? 1.0f : 0.0f);
  }
  __syncthreads();
  if (tid == 0) {
    float total_all = 0.0f, total_allowed = 0.0f;
    for (int i = 0; i < V; ++i) {
      total_all = fadd(total_all, e_all[i]);
      total_allowed = fadd(total_allowed, e_allowed[i]);
    }
    uint32_t token = next[b];
    float probability = fdiv(fast_exp(fsub(v[token], pk_allowed)), total_allowed);
    float mass = fdiv(fmul(total_allowed, fast_exp(fsub(pk_allowed, pk_all))), total_all);
    stats[(size_t)b * stats_stride] = probability;
    stats[(size_t)b * stats_stride + 1] = mass;
  }
}

// After a decode pass: the chosen token becomes the next input at the next position.
__global__ void k_advance(TokenMeta* meta, int B) {
  int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B || meta[b].slot < 0) return;
  meta[b].position += 1;
}

// -------------------------------------------------------------------- host
void set_exp_constants(const nbx::ExpConstants& constants, const nbx::ExceptionSet& exceptions, cudaStream_t stream) {
  cudaMemcpyToSymbolAsync(c_exp, &constants, sizeof constants, 0, cudaMemcpyHostToDevice, stream);
  cudaMemcpyToSymbolAsync(c_exceptions, &exceptions, sizeof exceptions, 0, cudaMemcpyHostToDevice, stream);
}

size_t route_smem(const ModelDev& md) { return (size_t)LANES * md.d_model * 4 * 2 + LANES * md.d_model; }
size_t attend_smem(const ModelDev& md, int t_cap) {
  int G = md.heads / md.kv_heads;
  return (size_t)2 * G * t_cap * 4 + 2 * (size_t)G * (t_cap / 4 + 2) * 4 + (size_t)8 * G * HEAD_DIM * 4;
}
size_t block_smem(const ModelDev& md) {
  int N = md.hada_left * HADA_RIGHT;
  return (size_t)(3 * MAX_D + 3 * N + md.hada_left * md.hada_left + HADA_RIGHT * HADA_RIGHT) * 4;
}

cudaError_t configure(const ModelDev& md, int t_cap) {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(k_route, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)route_smem(md)))) return e;
  if ((e = cudaFuncSetAttribute(k_attend<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attend_smem(md, t_cap)))) return e;
  if ((e = cudaFuncSetAttribute(k_attend<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attend_smem(md, t_cap)))) return e;
  if ((e = cudaFuncSetAttribute(k_attend<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attend_smem(md, t_cap)))) return e;
  if ((e = cudaFuncSetAttribute(k_block<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)block_smem(md)))) return e;
  if ((e = cudaFuncSetAttribute(k_block<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)block_smem(md)))) return e;
  if ((e = cudaFuncSetAttribute(k_stats, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 8192 * 4))) return e;
  return cudaSuccess;
}

static void project(const QMat& W, const int8_t* act, const float* act_scale, float* out, int M, int out_stride,
                    const TokenMeta* meta, cudaStream_t st) {
  int rowblocks = (W.rows + 63) / 64;
  int chunk = M <= 8 ? M : 16;
  dim3 grid(rowblocks, (M + chunk - 1) / chunk);
  if (W.groups == 4)
    k_project<4><<<grid, 256, 0, st>>>(W, act, act_scale, out, M, out_stride, chunk, meta);
  else if (W.groups == 8)
    k_project<8><<<grid, 256, 0, st>>>(W, act, act_scale, out, M, out_stride, chunk, meta);
}

void launch_embed(const ModelDev& md, const Work& w, int M, cudaStream_t st) { k_embed<<<M, 128, 0, st>>>(md, w, M); }

void launch_layer(const ModelDev& md, const LayerDev& L, const Work& w, const KvDev& kv, int M, int layer, int slot, int t_cap,
                  cudaStream_t st) {
  const int d = md.d_model, H = md.heads, KV = md.kv_heads;
  const int proj_stride = (2 * H + 2 * KV) * HEAD_DIM;
  k_route<<<M, 256, route_smem(md), st>>>(md, L, w, M, layer, slot);
  project(L.qkvg, w.act, w.act_scale, w.proj, M, proj_stride, w.meta, st);
  k_heads<<<M, 32 * (H + 2 * KV), 0, st>>>(md, L, w, kv, M, layer);
  const int G = H / KV;
  if (G == 1)
    k_attend<1><<<dim3(M, KV), 160, attend_smem(md, t_cap), st>>>(md, w, kv, M, layer, L.global, t_cap);
  else if (G == 2)
    k_attend<2><<<dim3(M, KV), 160, attend_smem(md, t_cap), st>>>(md, w, kv, M, layer, L.global, t_cap);
  else
    k_attend<4><<<dim3(M, KV), 160, attend_smem(md, t_cap), st>>>(md, w, kv, M, layer, L.global, t_cap);
  k_prep<<<M, 128, 0, st>>>(w.attn, H * HEAD_DIM, nullptr, w.proj + (H + 2 * KV) * HEAD_DIM, proj_stride, H * HEAD_DIM, w.act,
                            w.act_scale, M, w.meta, md.inv_sqrt_group, 1);
  project(L.out, w.act, w.act_scale, w.outp, M, d, w.meta, st);
  if (md.hada_left == 64)
    k_block<64><<<M, 512, block_smem(md), st>>>(md, L, w, M);
  else
    k_block<32><<<M, 512, block_smem(md), st>>>(md, L, w, M);
}

void launch_final(const ModelDev& md, const Work& w, float* hidden, int M, cudaStream_t st) { k_final<<<M, 128, 0, st>>>(md, w, hidden, M); }

void launch_logits(const ModelDev& md, const float* hidden, const int32_t* slots, int B, int8_t* act, float* act_scale, float* logits,
                   cudaStream_t st) {
  k_prep<<<B, 128, 0, st>>>(hidden, md.d_model, slots, nullptr, 0, md.d_model, act, act_scale, B, nullptr, md.inv_sqrt_group, 1);
  project(md.logits, act, act_scale, logits, B, md.output_vocab, nullptr, st);
}

void launch_select(const float* logits, int V, const uint32_t* mask, const int32_t* active, uint32_t* next, float* peaks, int B,
                   cudaStream_t st) {
  k_select<<<B, 256, 0, st>>>(logits, V, mask, active, next, peaks);
}

void launch_stats(const float* logits, int V, const uint32_t* mask, const int32_t* active, const uint32_t* next, const float* peaks,
                  float* stats, int stats_stride, int B, cudaStream_t st) {
  k_stats<<<B, 256, (size_t)2 * V * 4, st>>>(logits, V, mask, active, next, peaks, stats, stats_stride);
}

void launch_advance(TokenMeta* meta, int B, cudaStream_t st) { k_advance<<<(B + 127) / 128, 128, 0, st>>>(meta, B); }

void launch_attend(const ModelDev& md, const LayerDev& L, const Work& w, const KvDev& kv, int M, int layer, int t_cap, cudaStream_t st) {
  const int G = md.heads / md.kv_heads, KV = md.kv_heads;
  if (G == 1)
    k_attend<1><<<dim3(M, KV), 160, attend_smem(md, t_cap), st>>>(md, w, kv, M, layer, L.global, t_cap);
  else if (G == 2)
    k_attend<2><<<dim3(M, KV), 160, attend_smem(md, t_cap), st>>>(md, w, kv, M, layer, L.global, t_cap);
  else
    k_attend<4><<<dim3(M, KV), 160, attend_smem(md, t_cap), st>>>(md, w, kv, M, layer, L.global, t_cap);
}

// ------------------------------------------------------------------- debug
// Element-wise device math for the kernel-level tests: 0 expf (f32::exp),
// 1 sigmoid, 2 fast_exp, 3 silu.
__global__ void k_debug_math(int op, const float* in, float* out, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float x = in[i];
  out[i] = op == 0 ? expf_libm(x) : op == 1 ? sigmoid(x) : op == 2 ? fast_exp(x) : silu(x);
}

void launch_debug_math(int op, const float* in, float* out, int n, cudaStream_t st) {
  k_debug_math<<<(n + 255) / 256, 256, 0, st>>>(op, in, out, n);
}

// One codebook product of K-wide inputs (rotated and quantised per group,
// without the whole-vector fake quantisation) — QuantisedMatrix::prepare +
// multiply_vector (matrix.rs:123-165).
void launch_debug_project(const ModelDev& md, const QMat& W, const float* in, int K, int M, int8_t* act, float* act_scale,
                          float* out, int out_stride, cudaStream_t st) {
  k_prep<<<M, 128, 0, st>>>(in, K, nullptr, nullptr, 0, K, act, act_scale, M, nullptr, md.inv_sqrt_group, 0);
  project(W, act, act_scale, out, M, out_stride, nullptr, st);
}

}  // namespace nbk
