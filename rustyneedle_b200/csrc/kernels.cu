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
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <type_traits>
#include <utility>

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

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Copies `floats` (a multiple of 4, 16-byte aligned) from global to shared
// memory, 16 bytes per request; completes at cp_async_wait_all().
__device__ __forceinline__ void stage_async(float* dst, const float* src, int floats) {
  for (int i = threadIdx.x; i < floats / 4; i += blockDim.x) cp_async16(dst + 4 * i, src + 4 * i);
}

__device__ __forceinline__ uint8_t* page_base(const KvDev& kv, const PageGeometry& pg, int slot, int layer, int position) {
  int page = __ldcg(kv.page_table + ((size_t)slot * kv.num_layers + layer) * kv.max_pages + position / PAGE_POSITIONS);
  return kv.pool + (size_t)page * pg.page_bytes;
}

// A token's meta through L2 (it may be read before pdl_wait; see device.cuh).
__device__ __forceinline__ TokenMeta load_meta(const TokenMeta* meta, int t) {
  const int4 m = __ldcg(reinterpret_cast<const int4*>(meta + t));
  return TokenMeta{m.x, m.y, m.z, m.w};
}

// ----------------------------------------------------------------- embedding
// QuantisedMatrix::dequantise_row (matrix.rs:140-153) times sqrt(d), copied
// into every lane (session.rs:84-90). grid M, block 128.
__global__ void __launch_bounds__(128) k_embed(ModelDev md, Work w, int M) {
  pdl_wait();
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

// -------------------------------------------------------------- engram sites
// The token id at `position` of row t's sequence: this pass's row when the
// pass holds it (a pass keeps each sequence's tokens contiguous and in
// order), else the sequence's token ring.
__device__ __forceinline__ uint32_t token_at(const ModelDev& md, const Work& w, int t, const TokenMeta& meta, int position) {
  const int back = meta.position - position;
  if (back == 0) return __ldcg(w.tokens + t);
  if (t - back >= 0) {
    const TokenMeta o = load_meta(w.meta, t - back);
    if (o.slot == meta.slot && o.position == position) return __ldcg(w.tokens + t - back);
  }
  return __ldcg(md.token_ring + (size_t)meta.slot * md.token_rows + position % md.token_rows);
}

// grid M, block 128. A site's gathered table rows for token t (engram.rs:30-46,
// 68-83): table i hashes the last order(i) token ids (0 before the start),
// xor-shifts and takes the slot modulo; its row is dequantised like the
// embedding (level · norm, the normalised Walsh transform per 128-group,
// matrix.rs:140-153), or zeros while the position is shorter than the order.
// Then fake_quantise_int8 over the whole vector and the product's per-group
// rotation and int8 codes (QuantisedMatrix::prepare); groups past
// tables · sub_dim up to the padded K stay zero.
constexpr int ENGRAM_MAX_K = 2048, ENGRAM_MAX_TABLES = 16, ENGRAM_MAX_TAPS = 16;
__global__ void __launch_bounds__(128) k_engram_gather(ModelDev md, EngramDev E, Work w, int M) {
  __shared__ __align__(16) float s_g[ENGRAM_MAX_K];
  __shared__ uint32_t s_row[ENGRAM_MAX_TABLES];
  __shared__ float s_red[4];
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  if (t >= M) return;
  const TokenMeta meta = load_meta(w.meta, t);
  if (meta.slot < 0) return;
  const EngramConfig& c = E.cfg;
  const int tables = (int)c.tables, sub = (int)c.sub_dim, K = tables * sub, gpt = sub / GROUP;
  if (tid < tables) {
    const int oi = tid / (int)c.heads_per_order, head = tid % (int)c.heads_per_order, order = (int)c.order[oi];
    uint32_t acc = 0x9E3779B9u * (uint32_t)(oi * (int)c.stride + head + 1);
    for (int back = 0; back < order; ++back) {
      const uint32_t token = meta.position >= back ? token_at(md, w, t, meta, meta.position - back) : 0u;
      acc = (acc ^ token) * 0x01000193u;
    }
    acc ^= acc >> 15;
    s_row[tid] = meta.position + 1 >= order ? (uint32_t)tid * c.slots + acc % c.slots : 0xffffffffu;
  }
  __syncthreads();
  float peak = 0.0f;
  for (int pair = warp; pair < tables * gpt; pair += 4) {
    const int tb = pair / gpt, g = pair % gpt;
    const uint32_t row = s_row[tb];
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (row != 0xffffffffu) {
      const uint8_t* codes = E.packed + (size_t)row * E.row_bytes;
      const float norm = E.norms[(size_t)row * gpt + g];
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = fmul(E.levels[code_at(codes, g * GROUP + 4 * lane + j, E.bits)], norm);
      fwht128(v, md.inv_sqrt_group);
    }
    *reinterpret_cast<float4*>(s_g + tb * sub + g * GROUP + 4 * lane) = make_float4(v[0], v[1], v[2], v[3]);
    peak = fmaxf(peak, fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
  }
  peak = warp_max(peak);
  if (lane == 0) s_red[warp] = peak;
  __syncthreads();
  const float scale = int8_scale_of(fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3])));
  pdl_trigger();
  const int groups = (int)c.k / GROUP;
  for (int g = warp; g < groups; g += 4) {
    uint32_t packed = 0;
    float sc = 0.0f;
    if (g * GROUP < K) {
      const float4 x = reinterpret_cast<const float4*>(s_g + g * GROUP)[lane];
      float v[4] = {fake_quant(x.x, scale), fake_quant(x.y, scale), fake_quant(x.z, scale), fake_quant(x.w, scale)};
      fwht128(v, md.inv_sqrt_group);
      sc = quantise_group(v, packed);
    }
    *reinterpret_cast<uint32_t*>(w.act + chunked_offset(t, g * GROUP + 4 * lane, w.act_rows)) = packed;
    if (lane == 0) w.act_scale[(size_t)t * groups + g] = sc;
  }
}

// At an engram site layer, k_route's x (the routing input, s_x) takes the
// site's term (session.rs:180-190): alpha = sigmoid(Σ unit_rms(x)·unit_rms(key)
// / sqrt(d)), the dot an ordered sum from -0.0, then x += alpha · value, the
// value the dilated causal convolution of the raw values (engram.rs:92-103,
// 146-159: this pass's rows, else the site's ring). Threads 0..nthreads-1 of
// the CTA; s_key and s_prod are d floats of free shared memory.
__device__ __forceinline__ void engram_add(const ModelDev& md, const EngramDev& E, const Work& w, int t, int nthreads, float* s_x,
                                           float* s_key, float* s_prod, float* xg) {
  __shared__ float s_e[2];
  __shared__ const float* s_src[ENGRAM_MAX_TAPS];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, d = (int)md.d_model;
  const TokenMeta meta = load_meta(w.meta, t);
  const float* kv = w.engram_kv + (size_t)t * 2 * d;
  for (int i = tid; i < d; i += nthreads) s_key[i] = __ldcg(kv + i);
  if (tid < (int)E.cfg.conv_taps) {  // each tap's raw value row (null: the position is too short)
    const int back = tid * (int)E.cfg.dilation, R = (int)E.cfg.ring_rows;
    const float* src = nullptr;
    if (meta.position >= back) {
      bool here = back == 0;
      if (!here && t - back >= 0) {
        const TokenMeta o = load_meta(w.meta, t - back);
        here = o.slot == meta.slot && o.position == meta.position - back;
      }
      src = here ? w.engram_kv + (size_t)(t - back) * 2 * d + d : E.ring + ((size_t)meta.slot * R + (meta.position - back) % R) * d;
    }
    s_src[tid] = src;
  }
  named_barrier(1, nthreads);
  if (warp < 2) {
    const float ss = sum_of_squares_warp(warp == 0 ? s_x : s_key, d);
    if (lane == 0) s_e[warp] = inverse_rms(ss, d);
  }
  named_barrier(1, nthreads);
  const float inv_x = s_e[0], inv_k = s_e[1];
  for (int i = tid; i < d; i += nthreads) s_prod[i] = fmul(fmul(s_x[i], inv_x), fmul(s_key[i], inv_k));
  named_barrier(1, nthreads);
  if (tid == 0) {
    float dot = SUM_START;
    for (int i = 0; i < d; ++i) dot = fadd(dot, s_prod[i]);
    s_e[0] = sigmoid(fdiv(dot, md.sqrt_d));
  }
  named_barrier(1, nthreads);
  const float alpha = s_e[0];
  for (int i = tid; i < d; i += nthreads) {
    float value = 0.0f;
    for (int tap = 0; tap < (int)E.cfg.conv_taps; ++tap) {
      const float* src = s_src[tap];
      if (src) value = fadd(value, fmul(__ldg(E.taps + (size_t)tap * d + i), __ldcg(src + i)));
    }
    const float x = fadd(s_x[i], fmul(alpha, value));
    s_x[i] = x;
    xg[i] = x;
  }
}

// ------------------------------------------------------------------- routing
// grid M, block 256 (8 warps). Warp 7 finishes the Sinkhorn mixing weights
// while warps 0-6 build the block input, norm it and quantise it. Every
// global operand the kernel needs is staged by one round of cp.async.
constexpr int PHI_ROWS = LANES + LANES + LANES * LANES;

// Shared memory of k_route, in floats: this layer's phi rows (PHI_ROWS × n
// bytes), the stream, a work row, the squares in chain-major order (8 chains
// of n/8, stride n/8 + 4), the int8 codes, the phi norms and the norm_in gains.
// Without the phi rows (LEAN: they are read through L2) the rest is the same.
__host__ __device__ inline size_t route_floats(int d, bool lean = false) {
  const size_t n = (size_t)LANES * d, ng = n / GROUP;
  return (lean ? 0 : PHI_ROWS * n / 4) + 2 * n + 8 * (n / 8 + 4) + n / 4 + PHI_ROWS * ng + d;
}

// Failure detection test hook: while g_expire_route > 0, each k_route CTA
// that takes one of its counts gives up a bounded wait on a barrier that no
// copy will complete (short poll limit), records the engine's error flag,
// waits for its own bulk copies (which do complete, so nothing asynchronous
// outlives it) and returns without touching the token. The host then reports
// NB_ERR_TIMEOUT like any expired wait. Set only by nb_debug_expire_waits; 0
// otherwise.
__device__ int g_expire_route = 0;
constexpr uint32_t EXPIRE_POLLS = 1u << 12;

__device__ __forceinline__ void expire_wait(int* error) {
  __shared__ __align__(8) uint64_t s_never;
  const uint32_t never = smem_u32(&s_never);
  bulk_start(never, 16);  // 16 bytes announced, no copy issued: the wait cannot complete
  if (!mbar_wait_polls(never, 0, EXPIRE_POLLS)) atomicExch(error, 1);
}

__device__ __forceinline__ bool take_expiry() {
  int v = *reinterpret_cast<volatile int*>(&g_expire_route);
  while (v > 0) {
    const int prev = atomicCAS(&g_expire_route, v, v - 1);
    if (prev == v) return true;
    v = prev;
  }
  return false;
}

// LEAN (large prefill passes): the phi rows stay in global memory and the
// products read them through L2, so a CTA takes 33 KB of shared memory
// instead of 81 KB and six CTAs fit an SM instead of two.
template <bool LEAN>
__global__ void __launch_bounds__(256) k_route(ModelDev md, LayerDev L, Work w, int M, int layer, int slot, int* error) {
  extern __shared__ __align__(16) float sm[];
  const int t = blockIdx.x;
  const int d = md.d_model, n = LANES * d, ng = n / GROUP, sqs = n / 8 + 4;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* s_phiw = reinterpret_cast<uint8_t*>(sm);              // PHI_ROWS × n bytes (not LEAN)
  float* s_stream = sm + (LEAN ? 0 : PHI_ROWS * n / 4);          // n
  float* s_work = s_stream + n;                                  // n: later x and the phi terms
  float* s_sq = s_work + n;                                      // 8 × sqs
  int8_t* s_codes = reinterpret_cast<int8_t*>(s_sq + 8 * sqs);  // n bytes
  float* s_norms = s_sq + 8 * sqs + n / 4;                       // PHI_ROWS × ng phi norms
  float* s_gain = s_norms + PHI_ROWS * ng;                       // d norm_in gains
  __shared__ float s_ascale[MAX_D * LANES / GROUP];
  __shared__ float s_red[8];
  __shared__ float s_phi[PHI_ROWS];
  __shared__ float s_gate[LANES];
  __shared__ float s_inv, s_peak;
  __shared__ __align__(8) uint64_t s_bar;
  const uint32_t bar = smem_u32(&s_bar);

  // the layer's constant weights first, then (once the previous kernel is
  // done) the token's stream. One thread arms the barrier and issues the bulk
  // copies: the pre, post and residual rows of this layer are contiguous in
  // their matrices (rows 4l.., 4l.., 16l..), so seven copies in all. The test
  // hook's count is read after the copies are issued, so its load overlaps
  // them instead of delaying them.
  __shared__ int s_expire;
  if (tid == 0) {
    bulk_start(bar, (LEAN ? 0 : PHI_ROWS * n) + (PHI_ROWS * ng + d) * 4);
    if (!LEAN) {
      bulk_copy(s_phiw, md.phi_pre.codes + (size_t)layer * LANES * n, LANES * n, bar);
      bulk_copy(s_phiw + (size_t)LANES * n, md.phi_post.codes + (size_t)layer * LANES * n, LANES * n, bar);
      bulk_copy(s_phiw + (size_t)2 * LANES * n, md.phi_res.codes + (size_t)layer * LANES * LANES * n, LANES * LANES * n, bar);
    }
    bulk_copy(s_norms, md.phi_pre.scales + (size_t)layer * LANES * ng, LANES * ng * 4, bar);
    bulk_copy(s_norms + LANES * ng, md.phi_post.scales + (size_t)layer * LANES * ng, LANES * ng * 4, bar);
    bulk_copy(s_norms + 2 * LANES * ng, md.phi_res.scales + (size_t)layer * LANES * LANES * ng, LANES * LANES * ng * 4, bar);
    bulk_copy(s_gain, L.norm_in, d * 4, bar);
    s_expire = take_expiry();
  }
  // the routing parameters of this layer (constant): the pre/post gate
  // threads' scale and bias, and warp 7's residual-mixing ones
  float gate_a = 0.0f, gate_b = 0.0f, res_a = 0.0f, res_b = 0.0f;
  if (tid < 2 * LANES) {
    const int l = tid % LANES;
    gate_a = tid < LANES ? md.a_pre[layer] : md.a_post[layer];
    gate_b = tid < LANES ? md.b_pre[layer * LANES + l] : md.b_post[layer * LANES + l];
  }
  if (warp == 7 && lane < LANES * LANES) {
    res_a = md.a_res[layer];
    res_b = md.b_res[layer * LANES * LANES + lane];
  }
  pdl_wait();
  if (t >= M || w.meta[t].slot < 0) {
    if (tid == 0) {
      if (s_expire) expire_wait(error);
      if (!mbar_wait(bar, 0)) atomicExch(error, 1);  // no copy outlives the CTA
    }
    return;
  }
  stage_async(s_stream, w.stream + (size_t)t * n, n);
  cp_async_wait_all();
  __syncthreads();
  if (s_expire) {
    if (tid == 0) {
      expire_wait(error);
      if (!mbar_wait(bar, 0)) atomicExch(error, 1);
    }
    return;
  }
  // unit_rms over all lanes (ops.rs:60-66): the squares, placed chain-major
  // (value v joins chain v % 8 at place v / 8), and the peak |x|, which the
  // positive scale keeps: max |x·inv| = max|x| · inv
  {
    float pk = 0.0f;
    for (int v = tid; v < n; v += blockDim.x) {
      const float x = s_stream[v];
      s_sq[(v & 7) * sqs + (v >> 3)] = fmul(x, x);
      pk = fmaxf(pk, fabsf(x));
    }
    pk = warp_max(pk);
    if (lane == 0) s_red[warp] = pk;
  }
  __syncthreads();
  if (warp == 0) {
    // eight ordered chains over n/8 squares each, then the lanes in order from -0.0 (ops.rs:7-17)
    float acc = 0.0f;
    if (lane < 8) {
      const float4* q = reinterpret_cast<const float4*>(s_sq + lane * sqs);
      for (int m = 0; m < n / 32; m += 8) {
        float4 b[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) b[k] = q[m + k];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc = fadd(fadd(fadd(fadd(acc, b[k].x), b[k].y), b[k].z), b[k].w);
      }
    }
    float ss = SUM_START;
#pragma unroll
    for (int l = 0; l < 8; ++l) ss = fadd(ss, __shfl_sync(FULL, acc, l));
    if (lane == 0) {
      float pk = s_red[0];
      for (int i = 1; i < 8; ++i) pk = fmaxf(pk, s_red[i]);
      s_inv = inverse_rms(ss, n);
      s_peak = pk;
    }
  }
  __syncthreads();
  // fake_quantise_int8 (ops.rs:120-125) of the normalised stream, then rotate
  // and quantise per 128-group (QuantisedMatrix::prepare + PlaneInput)
  // (a warp takes groups g and g + 8 together, so their shuffle chains overlap)
  const float inv = s_inv;
  float scale = int8_scale_of(fmul(s_peak, inv));
  for (int g = warp; g < ng; g += 16) {
    const int g2 = g + 8;
    const bool two = g2 < ng;  // warp-uniform
    const float4 x = reinterpret_cast<const float4*>(s_stream + g * GROUP)[lane];
    const float4 y = reinterpret_cast<const float4*>(s_stream + (two ? g2 : g) * GROUP)[lane];
    float v[4] = {fake_quant(fmul(x.x, inv), scale), fake_quant(fmul(x.y, inv), scale), fake_quant(fmul(x.z, inv), scale),
                  fake_quant(fmul(x.w, inv), scale)};
    float u[4] = {fake_quant(fmul(y.x, inv), scale), fake_quant(fmul(y.y, inv), scale), fake_quant(fmul(y.z, inv), scale),
                  fake_quant(fmul(y.w, inv), scale)};
    fwht128(v, md.inv_sqrt_group);
    fwht128(u, md.inv_sqrt_group);
    uint32_t pv, pu;
    const float sv = quantise_group(v, pv), su = quantise_group(u, pu);
    *reinterpret_cast<uint32_t*>(s_codes + g * GROUP + 4 * lane) = pv;
    if (lane == 0) s_ascale[g] = sv;
    if (two) {
      *reinterpret_cast<uint32_t*>(s_codes + g2 * GROUP + 4 * lane) = pu;
      if (lane == 0) s_ascale[g2] = su;
    }
  }
  if (!mbar_wait(bar, 0) && tid == 0) atomicExch(error, 1);  // the phi rows, norms and gains
  __syncthreads();
  // phi products: 4 pre rows, 4 post rows, 16 residual rows of this layer
  // (lanes.rs:156-163). One thread per (row r, group g) pair sums the group's
  // 128 products exactly in int32 (dp4a), visiting its eight 16-byte chunks
  // from chunk tid % 8 on, so the eight threads of a shared-memory phase read
  // eight different bank quads; it then forms the scaled term
  // acc·norm·level_scale·act_scale. One thread per row adds the terms in
  // group order, the 4-bit row chain (neon.rs:164-183).
  float* s_term = s_work;  // [ng][PHI_ROWS]; s_work is free again
  {
    const float ls_pre = md.phi_pre.level_scale, ls_post = md.phi_post.level_scale, ls_res = md.phi_res.level_scale;
    for (int pair = tid; pair < PHI_ROWS * ng; pair += blockDim.x) {
      const int g = pair / PHI_ROWS, r = pair % PHI_ROWS;
      const uint8_t* wrow;
      if (LEAN)
        wrow = reinterpret_cast<const uint8_t*>(r < LANES ? md.phi_pre.codes + ((size_t)layer * LANES + r) * n
                          : (r < 2 * LANES ? md.phi_post.codes + ((size_t)layer * LANES + r - LANES) * n
                                           : md.phi_res.codes + ((size_t)layer * LANES * LANES + r - 2 * LANES) * n)) +
               g * GROUP;
      else
        wrow = s_phiw + (size_t)r * n + g * GROUP;
      const int8_t* arow = s_codes + g * GROUP;
      int acc0 = 0, acc1 = 0;
      uint4 wl[8];
      if (LEAN) {
#pragma unroll
        for (int k = 0; k < 8; ++k) wl[k] = __ldg(reinterpret_cast<const uint4*>(wrow + ((k + tid) & 7) * 16));
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int kk = (k + tid) & 7;
        const uint4 wv = LEAN ? wl[k] : *reinterpret_cast<const uint4*>(wrow + kk * 16);
        const uint4 a = *reinterpret_cast<const uint4*>(arow + kk * 16);
        acc0 = dp4a(wv.x, a.x, acc0);
        acc1 = dp4a(wv.y, a.y, acc1);
        acc0 = dp4a(wv.z, a.z, acc0);
        acc1 = dp4a(wv.w, a.w, acc1);
      }
      const float ls = r < LANES ? ls_pre : (r < 2 * LANES ? ls_post : ls_res);
      s_term[pair] = fmul(fmul(fmul((float)(acc0 + acc1), s_norms[r * ng + g]), ls), s_ascale[g]);
    }
  }
  __syncthreads();
  if (tid < PHI_ROWS) {
    float total = 0.0f;
#pragma unroll 16
    for (int g = 0; g < ng; ++g) total = fadd(total, s_term[g * PHI_ROWS + tid]);
    s_phi[tid] = total;
  }
  __syncthreads();
  float* route_out = w.route + (size_t)t * (LANES + LANES * LANES);
  if (warp == 7) {
    // the Sinkhorn-normalised residual mixing (lanes.rs:166-179, ops.rs:198-217):
    // lane 4r + c forms element (r, c) and its exponential, then every one of
    // the 16 lanes holds the whole matrix in registers and runs the 20
    // iterations itself; each row or column total is the reference's ordered
    // sum from -0.0, and the four totals of a phase are independent
    if (lane < LANES * LANES) {
      constexpr unsigned M16 = 0xffffu;
      const int r = lane / LANES;
      const float v = fadd(fmul(res_a, s_phi[2 * LANES + lane]), res_b);
      float pk = -INFINITY;
#pragma unroll
      for (int k = 0; k < LANES; ++k) pk = fmaxf(pk, __shfl_sync(M16, v, LANES * r + k));
      const float e = expf_libm(fsub(v, pk));
      float x[LANES * LANES];
#pragma unroll
      for (int i = 0; i < LANES * LANES; ++i) x[i] = __shfl_sync(M16, e, i);
      const float MIN_POSITIVE = 1.17549435e-38f;
#pragma unroll 1
      for (int it = 0; it < 20; ++it) {
#pragma unroll
        for (int rr = 0; rr < LANES; ++rr) {
          float total = SUM_START;
#pragma unroll
          for (int c = 0; c < LANES; ++c) total = fadd(total, x[LANES * rr + c]);
          const float inverse = rcp_positive(fmaxf(total, MIN_POSITIVE));  // total <= 4
#pragma unroll
          for (int c = 0; c < LANES; ++c) x[LANES * rr + c] = fmul(x[LANES * rr + c], inverse);
        }
#pragma unroll
        for (int c = 0; c < LANES; ++c) {
          float total = SUM_START;
#pragma unroll
          for (int rr = 0; rr < LANES; ++rr) total = fadd(total, x[LANES * rr + c]);
          const float inverse = rcp_positive(fmaxf(total, MIN_POSITIVE));  // total <= 4
#pragma unroll
          for (int rr = 0; rr < LANES; ++rr) x[LANES * rr + c] = fmul(x[LANES * rr + c], inverse);
        }
      }
      if (lane == 0) {
        float4* dst = reinterpret_cast<float4*>(route_out + LANES);
#pragma unroll
        for (int q = 0; q < LANES; ++q) dst[q] = make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
      }
    }
    return;
  }
  // warps 0-6 (224 threads) from here on; threads 0-3 form the pre gates,
  // threads 4-7 the post gates (2 · sigmoid, lanes.rs:166-179)
  const int nthreads = 224;
  if (tid < 2 * LANES) {
    const int l = tid % LANES;
    const bool pre = tid < LANES;
    const float off = pre ? (l == (slot % LANES) ? 8.0f + -4.0f : -4.0f) : (l == (slot % LANES) ? 0.0f : -4.0f);
    const float g = sigmoid(fadd(fadd(fmul(gate_a, s_phi[pre ? l : 4 + l]), gate_b), off));
    if (pre)
      s_gate[l] = g;
    else
      route_out[l] = fmul(2.0f, g);
  }
  named_barrier(1, nthreads);
  float* s_x = s_work;  // the block input x (lanes.rs:169-171)
  float* xg = w.x + (size_t)t * d;
  const bool engram = L.engram_site >= 0;
  float* xin = engram ? w.xin + (size_t)t * d : xg;  // the routing input; x adds the engram term to it
  for (int i = tid; i < d; i += nthreads) {
    float acc = 0.0f;
#pragma unroll
    for (int l = 0; l < LANES; ++l) acc = fadd(acc, fmul(s_gate[l], s_stream[l * d + i]));
    s_x[i] = acc;
    xin[i] = acc;
  }
  named_barrier(1, nthreads);
  if (engram) {
    engram_add(md, *L.engram, w, t, nthreads, s_x, s_stream, s_stream + d, xg);  // the lanes are no longer needed
    named_barrier(1, nthreads);
  }
  if (warp == 0) {
    float ss = sum_of_squares_warp(s_x, d);
    if (lane == 0) s_inv = inverse_rms(ss, d);
  }
  named_barrier(1, nthreads);
  // zero_centred_norm (ops.rs:44-50) then fake_quantise_int8 (attention.rs:99-100)
  float* s_y = s_stream;
  const float inv_x = s_inv;
  float peak = 0.0f;
  for (int i = tid; i < d; i += nthreads) {
    float v = fmul(fmul(fadd(1.0f, s_gain[i]), s_x[i]), inv_x);
    s_y[i] = v;
    peak = fmaxf(peak, fabsf(v));
  }
  peak = warp_max(peak);
  if (lane == 0) s_red[warp] = peak;
  named_barrier(1, nthreads);
  peak = s_red[0];
  for (int i = 1; i < 7; ++i) peak = fmaxf(peak, s_red[i]);
  scale = int8_scale_of(peak);
  pdl_trigger();  // the tail of the kernel overlaps the next one's prologue
  const int dg = d / GROUP;
  for (int g = warp; g < dg; g += 7) {
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = fake_quant(s_y[g * GROUP + 4 * lane + j], scale);
    fwht128(v, md.inv_sqrt_group);
    uint32_t packed;
    float sc = quantise_group(v, packed);
    *reinterpret_cast<uint32_t*>(w.act + core_offset(t, g * GROUP + 4 * lane, d / 16)) = packed;
    if (lane == 0) w.act_scale[(size_t)t * dg + g] = sc;
  }
}

// ------------------------------------------------------- tensor-core product
// out[m][row] = Σ_g combine(acc_g[row][m]) for a K = 512 codebook matrix on
// the 5th-generation tensor cores: tcgen05.mma kind::i8 with int32
// accumulators in TMEM, one accumulator per 128-column group (the reference
// scales every group separately, neon.rs:158 / panel.rs:184-187), four
// K = 32 steps per group. Operands live in global memory in the canonical
// K-major core-matrix layout (core_offset, layout.h) so a 128-row weight tile
// and an NT-token activation tile are each one contiguous block, fetched by
// cp.async.bulk onto an mbarrier. In the epilogue warp w reads TMEM lane
// quadrant w%4 (thread = weight row) for its share of the tokens, each group's
// accumulators with tcgen05.ld, and combines them in group order: fma for
// 2-bit panels, the product chain for 4-bit rows. Small token tiles keep the
// epilogue short and spread a projection over many CTAs.
// grid (ceil(rows/128), ceil(M/NT)), block 16·NT (8 tokens per warp slice).
constexpr int GEMM_ROWS = 128;
constexpr int GEMM_K = 512;
constexpr int GEMM_KC = GEMM_K / 16;  // 16-byte chunks per row

// UMMA shared-memory descriptor (K-major, no swizzle): start address, the byte
// offset between the two 16-byte K halves of a K = 32 step (LBO) and between
// 8-row core-matrix groups (SBO), descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3fff) | ((uint64_t)((lbo >> 4) & 0x3fff) << 16) | ((uint64_t)((sbo >> 4) & 0x3fff) << 32) |
         (1ull << 46);
}

// K = 512 · KCH (KCH chunks of the K-chunk-major layout, one after another:
// the weight tile and the activation block of chunk c are copied, its 16 MMAs
// accumulate groups 4c..4c+3, and the next chunk's copy starts once they have
// completed). The epilogue combines the groups in order.
constexpr int GEMM_THREADS_PER_TOKEN = 16;  // 4 TMEM lane quadrants × NT/8 token slices of 32 threads

template <int NT, int KCH>
__global__ void __launch_bounds__(GEMM_THREADS_PER_TOKEN * NT) k_gemm(QMat W, const int8_t* __restrict__ act, const float* __restrict__ act_scale,
                                              float* __restrict__ out, int M, int out_stride, const TokenMeta* __restrict__ meta,
                                              int* __restrict__ error, int act_rows) {
  constexpr int GK = KCH * (GEMM_K / GROUP);
  constexpr uint32_t COLS = GK * NT;  // TMEM columns: one NT-wide accumulator per group
  constexpr uint32_t A_BYTES = GEMM_ROWS * GEMM_K, B_BYTES = NT * GEMM_K;
  // instruction descriptor: D s32, A and B s8, both K-major, N = NT, M = 128
  constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(GEMM_ROWS >> 4) << 24);
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sA = smem;
  uint8_t* sB = smem + A_BYTES;
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t s_tmem;
  __shared__ float s_as[NT * GK];
  __shared__ int s_fail;
  __shared__ bool s_live[NT];  // output column n is stored (a live token of the pass)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, m0 = blockIdx.y * NT, mcount = min(NT, M - m0);
  const uint32_t bar_load = smem_u32(&bars[0]), bar_mma = smem_u32(&bars[1]);
  const size_t rows_cap = ((size_t)W.rows + GEMM_ROWS - 1) / GEMM_ROWS * GEMM_ROWS;
  constexpr uint32_t PIECE = 16384;
  auto copy = [&](uint8_t* dst, const uint8_t* src, uint32_t bytes) {
    for (uint32_t off = 0; off < bytes; off += PIECE)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst + off)),
                   "l"(src + off), "r"(min(PIECE, bytes - off)), "r"(bar_load)
                   : "memory");
  };
  auto weights = [&](int c) { return reinterpret_cast<const uint8_t*>(W.codes) + (size_t)c * rows_cap * GEMM_K + (size_t)tile * A_BYTES; };
  auto tokens = [&](int c) {
    return reinterpret_cast<const uint8_t*>(act) + (size_t)c * act_rows * GEMM_K + (size_t)(m0 / 8) * (8 * GEMM_K);
  };

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)), "r"(COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    s_fail = 0;
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar_load), "r"(1) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar_mma), "r"(1) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    // the weight tile is constant: its copy starts before the previous kernel has finished
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_load), "r"(A_BYTES + B_BYTES) : "memory");
    copy(sA, weights(0), A_BYTES);
  }
  // this thread's output row and its per-group weight scales (constant)
  const int quad = warp & 3, slice = warp >> 2;
  const int row = tile * GEMM_ROWS + quad * 32 + lane;
  const bool valid = row < (int)W.rows;
  float ws[GK];
#pragma unroll
  for (int g = 0; g < GK; ++g) ws[g] = valid ? W.scales[(size_t)row * GK + g] : 0.0f;
  // the pass's token meta comes from launches before the predecessor
  if (tid < NT) s_live[tid] = tid < mcount && !(meta && __ldcg(&meta[m0 + tid].slot) < 0);
  pdl_wait();
  if (tid == 0) copy(sB, tokens(0), B_BYTES);
  for (int i = tid; i < NT * GK; i += blockDim.x) s_as[i] = i / GK < mcount ? act_scale[(size_t)m0 * GK + i] : 0.0f;
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;

  bool ok = true;
#pragma unroll 1
  for (int c = 0; c < KCH; ++c) {
    if (c > 0 && tid == 0) {
      // chunk c - 1's MMAs have completed (every thread waited for them): its smem is free
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_load), "r"(A_BYTES + B_BYTES) : "memory");
      copy(sA, weights(c), A_BYTES);
      copy(sB, tokens(c), B_BYTES);
    }
    if (ok) ok = mbar_wait(bar_load, c & 1);
    if (ok && warp == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (lane == 0) {
        const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
#pragma unroll
        for (int g = 0; g < GEMM_K / GROUP; ++g)
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const int step = g * 4 + s;  // K bytes 32·step .. 32·step+31 = chunks 2·step, 2·step+1
            const uint64_t da = umma_desc(a0 + step * 256, 128, GEMM_KC * 128);
            const uint64_t db = umma_desc(b0 + step * 256, 128, GEMM_KC * 128);
            const uint32_t d_tmem = tmem + (c * (GEMM_K / GROUP) + g) * NT, accumulate = s > 0 ? 1u : 0u;
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "setp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
                "l"(da), "l"(db), "r"(IDESC), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
                : "memory");
          }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_mma) : "memory");
      }
      __syncwarp();
    }
    if (ok) ok = mbar_wait(bar_mma, c & 1);
  }
  if (!ok) s_fail = 1;
  pdl_trigger();  // the epilogue overlaps the next kernel's prologue
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  __syncthreads();
  if (!s_fail) {
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const int c0 = slice * 8;
    float total[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) total[j] = 0.0f;
    // four groups' accumulators per batch, loaded together and waited for once
#pragma unroll
    for (int g0 = 0; g0 < GK; g0 += 4) {
      uint32_t a[4][8];
#pragma unroll
      for (int gi = 0; gi < 4; ++gi)
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                     : "=r"(a[gi][0]), "=r"(a[gi][1]), "=r"(a[gi][2]), "=r"(a[gi][3]), "=r"(a[gi][4]), "=r"(a[gi][5]), "=r"(a[gi][6]),
                       "=r"(a[gi][7])
                     : "r"(lane_base + (g0 + gi) * NT + c0));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int gi = 0; gi < 4; ++gi) {
        const int g = g0 + gi;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float acc = group_sum_to_float(a[gi][j]);
          const float as = s_as[(c0 + j) * GK + g];
          total[j] =
              W.fused ? __fmaf_rn(acc, fmul(ws[g], as), total[j]) : fadd(total[j], fmul(fmul(fmul(acc, ws[g]), W.level_scale), as));
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = c0 + j;
      if (valid && s_live[n]) out[(size_t)(m0 + n) * out_stride + row] = total[j];
    }
  } else if (tid == 0) {
    atomicExch(error, 1);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(COLS) : "memory");
}

// ------------------------------------------- tensor-core product, large passes
// For passes of at least WIDE_MIN_TOKENS tokens through a K = 512 matrix: a
// persistent CTA per SM keeps one 128-row weight tile resident in shared
// memory and walks 64-token tiles (CTA (r, p) takes token tiles p, p + P, ...
// of row tile r), warp-specialised:
//   warp 0 (one lane)   streams each tile's token codes through a ring of
//                       32 KB stages (freed when the tile's MMAs complete) and
//                       its act scales through a ring freed by the epilogue,
//                       bulk copies onto mbarriers
//   warp 1 (one lane)   issues the tile's 16 tcgen05.mma kind::i8 (M = 128,
//                       N = 64, K = 32) into one of two TMEM accumulator sets
//                       (columns 0..255 and 256..511, [4 groups][64 tokens]),
//                       so the MMAs of one tile run while the epilogue drains
//                       the previous one
//   warp 2              transposes each tile's act scales to [group][token],
//                       so a pair of tokens' scales of one group is one 8-byte
//                       shared-memory load
//   warps 4..19         thread = weight row (warp w reads TMEM lane quadrant
//                       w % 4) for tokens 16·((w - 4) / 4) .. +15, in chunks
//                       of 8 tokens: the four groups' accumulators in order,
//                       exactly k_gemm's combine, two tokens per packed f32x2
//                       instruction; each finished chunk leaves by a TMA
//                       tensor store
// The accumulators start from the bias 0x4B400000 (written into TMEM by the
// epilogue when it hands a set back, and once before the first tile), so an
// int32 group sum s arrives as the bits of the float 1.5·2^23 + s and its
// exact f32 value is one subtraction (|s| ≤ 2^21; group_sum_to_float).
// Every wait is bounded; a wait that gives up sets the error flag, the other
// roles stop at their next wait, and the copy and MMA threads wait (bounded)
// for what they issued before the CTA frees its TMEM and exits.
constexpr int WIDE_NT = 64;
constexpr int WIDE_CODE_STAGES = 3;
constexpr int WIDE_SCALE_STAGES = 4;
constexpr int WIDE_MIN_TOKENS = 256;
constexpr int WIDE_EPI_WARPS = 16;
constexpr int WIDE_EPI_TOKENS = WIDE_NT / (WIDE_EPI_WARPS / 4);  // 16 tokens per epilogue warp
constexpr int WIDE_THREADS = (4 + WIDE_EPI_WARPS) * 32;
constexpr uint32_t WIDE_A_BYTES = GEMM_ROWS * GEMM_K, WIDE_B_BYTES = WIDE_NT * GEMM_K;
constexpr uint32_t WIDE_S_BYTES = WIDE_NT * (GEMM_K / GROUP) * 4;  // a token tile's act scales
constexpr uint32_t WIDE_O_BYTES = 8 * 32 * 4;  // an epilogue warp's output staging: [8 tokens][32 rows] f32
constexpr uint32_t WIDE_BIAS = 0x4B400000u;    // the float 1.5·2^23 as an int32
constexpr size_t wide_smem() {
  return (size_t)WIDE_A_BYTES + (size_t)WIDE_CODE_STAGES * WIDE_B_BYTES + 2 * (size_t)WIDE_SCALE_STAGES * WIDE_S_BYTES +
         (size_t)WIDE_EPI_WARPS * WIDE_O_BYTES;
}

__global__ void __launch_bounds__(WIDE_THREADS, 1) k_gemm_wide(QMat W, const int8_t* __restrict__ act, const float* __restrict__ act_scale,
                                                              float* __restrict__ out, int M, int out_stride,
                                                              const TokenMeta* __restrict__ meta, int* __restrict__ error,
                                                              const __grid_constant__ CUtensorMap out_map, int tma_out) {
  constexpr int GK = GEMM_K / GROUP;            // 4 groups
  constexpr uint32_t SET = GK * WIDE_NT;        // TMEM columns of one accumulator set: group g at g·64
  constexpr uint32_t COLS = 2 * SET;            // 512
  constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(WIDE_NT >> 3) << 17) | ((uint32_t)(GEMM_ROWS >> 4) << 24);
  constexpr uint32_t PIECE = 16384;
  constexpr int CS = WIDE_CODE_STAGES, SS = WIDE_SCALE_STAGES;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sA = smem;
  uint8_t* sB = smem + WIDE_A_BYTES;
  float* sS = reinterpret_cast<float*>(sB + (size_t)CS * WIDE_B_BYTES);  // [stage][64 tokens][4 groups], as copied
  float* sT = sS + (size_t)SS * WIDE_NT * GK;                             // [stage][4 groups][64 tokens]
  float* sO = sT + (size_t)SS * WIDE_NT * GK;                             // [epilogue warp][8 tokens][32 rows]
  __shared__ __align__(8) uint64_t bars[1 + 2 * CS + 3 * SS + 4];
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_fail;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, P = gridDim.y, p = blockIdx.y;
  const int token_tiles = (M + WIDE_NT - 1) / WIDE_NT;
  const int my_tiles = p < token_tiles ? (token_tiles - p + P - 1) / P : 0;
  const uint32_t bar_a = smem_u32(&bars[0]);
  auto cfull = [&](int s) { return smem_u32(&bars[1 + s]); };
  auto cempty = [&](int s) { return smem_u32(&bars[1 + CS + s]); };
  auto sfull = [&](int s) { return smem_u32(&bars[1 + 2 * CS + s]); };
  auto sempty = [&](int s) { return smem_u32(&bars[1 + 2 * CS + SS + s]); };
  auto tfull = [&](int s) { return smem_u32(&bars[1 + 2 * CS + 2 * SS + s]); };
  auto afull = [&](int b) { return smem_u32(&bars[1 + 2 * CS + 3 * SS + b]); };
  auto aempty = [&](int b) { return smem_u32(&bars[3 + 2 * CS + 3 * SS + b]); };
  auto copy = [&](uint8_t* dst, const uint8_t* src, uint32_t bytes, uint32_t bar) {
    for (uint32_t off = 0; off < bytes; off += PIECE)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst + off)),
                   "l"(src + off), "r"(min(PIECE, bytes - off)), "r"(bar)
                   : "memory");
  };
  auto expect = [&](uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
  };
  auto init = [&](uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
  };
  auto arrive = [&](uint32_t bar) { asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory"); };
  // the bias into 8 TMEM columns of this thread's lane
  auto bias8 = [&](uint32_t taddr) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr), "r"(WIDE_BIAS) : "memory");
  };

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)), "r"(COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    s_fail = 0;
    init(bar_a, 1);
    for (int s = 0; s < CS; ++s) {
      init(cfull(s), 1);
      init(cempty(s), 1);  // the tile's commit
    }
    for (int s = 0; s < SS; ++s) {
      init(sfull(s), 1);
      init(sempty(s), WIDE_EPI_WARPS);  // every epilogue warp has combined the tile
      init(tfull(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      init(afull(b), 1);
      init(aempty(b), WIDE_EPI_WARPS);  // completes once with the initial bias, then once per tile drained
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    // the weight tile is constant: its copy starts before the previous kernel has finished
    if (my_tiles > 0) {
      expect(bar_a, WIDE_A_BYTES);
      copy(sA, reinterpret_cast<const uint8_t*>(W.codes) + (size_t)tile * WIDE_A_BYTES, WIDE_A_BYTES, bar_a);
    }
  }
  // an epilogue thread's weight row and its per-group scales (constant)
  const int ew = warp - 4, quad = warp & 3;
  const int row = tile * GEMM_ROWS + quad * 32 + lane;
  const bool valid = ew >= 0 && row < (int)W.rows;
  float ws[GK];
#pragma unroll
  for (int g = 0; g < GK; ++g) ws[g] = valid ? W.scales[(size_t)row * GK + g] : 0.0f;
  pdl_wait();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();  // barriers initialised, TMEM allocated
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;
  const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
  const int c0 = (ew >> 2) * WIDE_EPI_TOKENS;
  int issued = 0;     // token tiles whose copies warp 0 has issued
  int committed = 0;  // token tiles whose MMAs warp 1 has issued

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < my_tiles && !s_fail; ++i) {
      const int c = i % CS, sc = i % SS;
      if ((i >= CS && !mbar_wait(cempty(c), ((i / CS) - 1) & 1)) || (i >= SS && !mbar_wait(sempty(sc), ((i / SS) - 1) & 1))) {
        s_fail = 1;
        break;
      }
      const int m0 = (p + i * P) * WIDE_NT;
      // the token tile (the activation rows are allocated in whole 128-token
      // tiles) and its act scales (only the pass's tokens: the scale rows end at M)
      const uint32_t sbytes = (uint32_t)min(WIDE_NT, M - m0) * GK * 4;
      expect(cfull(c), WIDE_B_BYTES);
      copy(sB + (size_t)c * WIDE_B_BYTES, reinterpret_cast<const uint8_t*>(act) + (size_t)(m0 / 8) * (8 * GEMM_K), WIDE_B_BYTES, cfull(c));
      expect(sfull(sc), sbytes);
      copy(reinterpret_cast<uint8_t*>(sS + (size_t)sc * WIDE_NT * GK), reinterpret_cast<const uint8_t*>(act_scale + (size_t)m0 * GK), sbytes,
           sfull(sc));
      ++issued;
    }
  } else if (warp == 1 && lane == 0) {
    if (my_tiles > 0 && !mbar_wait(bar_a, 0)) s_fail = 1;
    for (int i = 0; i < my_tiles && !s_fail; ++i) {
      const int c = i % CS, b = i & 1;
      // the code stage has landed; the epilogue has drained this set and reset it to the bias
      if (!mbar_wait(cfull(c), (i / CS) & 1) || !mbar_wait(aempty(b), (i >> 1) & 1)) {
        s_fail = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB + (size_t)c * WIDE_B_BYTES);
#pragma unroll
      for (int g = 0; g < GK; ++g)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int step = g * 4 + k;  // K bytes 32·step .. 32·step+31
          const uint64_t da = umma_desc(a0 + step * 256, 128, GEMM_KC * 128);
          const uint64_t db = umma_desc(b0 + step * 256, 128, GEMM_KC * 128);
          asm volatile("tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, 1;" ::"r"(tmem + b * SET + g * WIDE_NT), "l"(da), "l"(db),
                       "r"(IDESC)
                       : "memory");
        }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(afull(b)) : "memory");
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cempty(c)) : "memory");
      ++committed;
    }
  } else if (warp == 2) {
    for (int i = 0; i < my_tiles; ++i) {
      const int sc = i % SS;
      bool ok = !s_fail;
      if (ok && lane == 0) ok = mbar_wait(sfull(sc), (i / SS) & 1);
      if (!__shfl_sync(FULL, ok ? 1 : 0, 0)) {
        s_fail = 1;
        break;
      }
      // (a token past M transposes a stale entry; its output is not stored)
      const float* src = sS + (size_t)sc * WIDE_NT * GK;
      float* dst = sT + (size_t)sc * WIDE_NT * GK;
#pragma unroll 4
      for (int e = lane; e < WIDE_NT * GK; e += 32) dst[e] = src[(e % WIDE_NT) * GK + e / WIDE_NT];
      __syncwarp();
      if (lane == 0) arrive(tfull(sc));
    }
  } else if (ew >= 0) {
    // the bias into this warp's columns of both sets before the first tiles' MMAs
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int g = 0; g < GK; ++g)
#pragma unroll
        for (int q = 0; q < WIDE_EPI_TOKENS / 8; ++q) bias8(lane_base + b * SET + g * WIDE_NT + c0 + q * 8);
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
      arrive(aempty(0));
      arrive(aempty(1));
    }
    const float2 nz = g_negzero;
    float* stage = sO + (size_t)ew * (WIDE_O_BYTES / 4);
    // the combine per tile, with the product form (fused panels or the 4-bit
    // chain) fixed outside the loops
    auto drain = [&](auto fused_tag) {
      constexpr bool FUSED = decltype(fused_tag)::value;
      const float level = W.level_scale;
      for (int i = 0; i < my_tiles; ++i) {
        const int sc = i % SS, b = i & 1;
        bool ok = !s_fail;
        if (ok && lane == 0) ok = mbar_wait(tfull(sc), (i / SS) & 1) && mbar_wait(afull(b), (i >> 1) & 1);
        ok = __shfl_sync(FULL, ok ? 1 : 0, 0) != 0;
        if (!ok) {
          s_fail = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int m0 = (p + i * P) * WIDE_NT;
        // which of this warp's 16 tokens are stored: bit j for token m0 + c0 + j
        const int m = m0 + c0 + lane;
        const uint32_t store = __ballot_sync(FULL, lane < WIDE_EPI_TOKENS && m < M && !(meta && __ldcg(&meta[m].slot) < 0));
        // every token of this warp's 16 is stored: each finished chunk of 8
        // leaves through the warp's staging buffer as a TMA tensor store
        const bool tma = tma_out && store == (1u << WIDE_EPI_TOKENS) - 1;
        const float* tscale = sT + (size_t)sc * WIDE_NT * GK + c0;  // [group][token]
#pragma unroll
        for (int q = 0; q < WIDE_EPI_TOKENS / 8; ++q) {
          uint32_t a[GK][8];
#pragma unroll
          for (int g = 0; g < GK; ++g)
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                         : "=r"(a[g][0]), "=r"(a[g][1]), "=r"(a[g][2]), "=r"(a[g][3]), "=r"(a[g][4]), "=r"(a[g][5]), "=r"(a[g][6]),
                           "=r"(a[g][7])
                         : "r"(lane_base + b * SET + g * WIDE_NT + c0 + q * 8));
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          // the columns are read: back to the bias for the MMAs two tiles on
#pragma unroll
          for (int g = 0; g < GK; ++g) bias8(lane_base + b * SET + g * WIDE_NT + c0 + q * 8);
          float2 total[4];  // the chunk's token pairs
#pragma unroll
          for (int pp = 0; pp < 4; ++pp) {
            float2 t = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int g = 0; g < GK; ++g) {
              const float2 acc = add2(make_float2(__int_as_float((int)a[g][2 * pp]), __int_as_float((int)a[g][2 * pp + 1])),
                                      make_float2(-12582912.0f, -12582912.0f));
              const float2 as = *reinterpret_cast<const float2*>(tscale + g * WIDE_NT + q * 8 + 2 * pp);
              const float2 w = make_float2(ws[g], ws[g]);
              if (FUSED)
                t = fma2(acc, fma2(w, as, nz), t);
              else
                t = add2(t, fma2(fma2(fma2(acc, w, nz), make_float2(level, level), nz), as, nz));
            }
            total[pp] = t;
          }
          // the finished chunk through the warp's staging buffer: a TMA
          // tensor store, or (a warp with a token not to store) plain stores
          // of the live tokens
          // (an earlier tile's tensor store may still be reading the buffer)
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
          __syncwarp();
#pragma unroll
          for (int pp = 0; pp < 4; ++pp) {
            stage[(2 * pp) * 32 + lane] = total[pp].x;
            stage[(2 * pp + 1) * 32 + lane] = total[pp].y;
          }
          if (tma) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
              asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                               reinterpret_cast<uint64_t>(&out_map)),
                           "r"(tile * GEMM_ROWS + quad * 32), "r"(m0 + c0 + q * 8), "r"(smem_u32(stage))
                           : "memory");
              asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            }
          } else if (valid) {
#pragma unroll 1
            for (int j = 0; j < 8; ++j)
              if ((store >> (q * 8 + j)) & 1) out[(size_t)(m0 + c0 + q * 8 + j) * out_stride + row] = stage[j * 32 + lane];
          }
        }
        // the set's columns are read and reset to the bias; the stage's scales are read
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          arrive(aempty(b));
          arrive(sempty(sc));
        }
      }
      // the tensor stores have completed before the CTA leaves
      if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    };
    if (W.fused)
      drain(std::true_type{});
    else
      drain(std::false_type{});
  }
  pdl_trigger();
  // nothing asynchronous outlives the CTA: warp 0 waits (bounded) for every
  // copy it issued, warp 1 for every MMA it issued (the epilogue has already
  // seen them complete unless a wait gave up)
  if (warp == 0 && lane == 0) {
    for (int i = max(0, issued - CS); i < issued; ++i) mbar_wait(cfull(i % CS), (i / CS) & 1);
    for (int i = max(0, issued - SS); i < issued; ++i) mbar_wait(sfull(i % SS), (i / SS) & 1);
    if (my_tiles > 0) mbar_wait(bar_a, 0);
  } else if (warp == 1 && lane == 0) {
    if (committed > 0) mbar_wait(cempty((committed - 1) % CS), ((committed - 1) / CS) & 1);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (s_fail && tid == 0) atomicExch(error, 1);
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(COLS) : "memory");
  }
}

// -------------------------------------------------------------------- gemv
// The same product for a few tokens (decode at small batch) as a memory-bound
// int8 GEMV on the CUDA cores. A warp owns one 8-row block of the
// core-matrix layout (4 KB contiguous per 512-column chunk: eight coalesced
// 16-byte loads per lane). Lane l serves row l%8 and the 16-byte chunks
// c = 4j + l/8, so the exact int32 sum of each 128-column group (chunks
// 8g..8g+7) is two dp4a chains per lane, reduced over the row's four lanes.
// Every token's activations sit in shared memory; the output is the ordered
// per-group combine of k_gemm's epilogue (carried across chunks in shared
// memory when K > 512).
constexpr int GEMV_WARPS = 2;
constexpr int GEMV_MAX_TOKENS = 8;

template <int KCH>
__global__ void __launch_bounds__(GEMV_WARPS * 32) k_gemv(QMat W, const int8_t* __restrict__ act, const float* __restrict__ act_scale,
                                                        float* __restrict__ out, int M, int out_stride,
                                                        const TokenMeta* __restrict__ meta, int act_rows) {
  constexpr int GC = GEMM_K / GROUP;  // groups per chunk
  constexpr int GK = KCH * GC;
  __shared__ __align__(16) uint8_t s_act[GEMV_MAX_TOKENS][KCH * GEMM_K];
  __shared__ float s_as[GEMV_MAX_TOKENS][GK];
  __shared__ float s_tot[KCH > 1 ? GEMV_MAX_TOKENS : 1][GEMV_WARPS * 8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int block = blockIdx.x * GEMV_WARPS + warp;
  const int row = block * 8 + (lane & 7), q = lane >> 3;
  const bool live = block * 8 < (int)W.rows;  // storage rows are padded to 128, so a live block is whole
  const size_t rows_cap = ((size_t)W.rows + GEMM_ROWS - 1) / GEMM_ROWS * GEMM_ROWS;
  uint4 wv[8];
  float ws[GK];
  if (live) {
    const uint4* src = reinterpret_cast<const uint4*>(W.codes + (size_t)block * 8 * GEMM_K);
#pragma unroll
    for (int j = 0; j < 8; ++j) wv[j] = src[j * 32 + lane];
  }
#pragma unroll
  for (int g = 0; g < GK; ++g) ws[g] = row < (int)W.rows ? W.scales[(size_t)row * GK + g] : 0.0f;
  pdl_wait();
  for (int i = threadIdx.x; i < M * KCH * GEMM_KC; i += blockDim.x) {
    const int t = i / (KCH * GEMM_KC), k = (i % (KCH * GEMM_KC)) * 16;
    *reinterpret_cast<uint4*>(&s_act[t][k]) = *reinterpret_cast<const uint4*>(act + chunked_offset(t, k, act_rows));
  }
  for (int i = threadIdx.x; i < M * GK; i += blockDim.x) s_as[i / GK][i % GK] = act_scale[i];
  __syncthreads();
  if (!live) return;
#pragma unroll 1
  for (int c = 0; c < KCH; ++c) {
    if (c > 0) {
      const uint4* src = reinterpret_cast<const uint4*>(W.codes + (size_t)c * rows_cap * GEMM_K + (size_t)block * 8 * GEMM_K);
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[j] = src[j * 32 + lane];
    }
    for (int t = 0; t < M; ++t) {
      int acc[GC];
#pragma unroll
      for (int g = 0; g < GC; ++g) acc[g] = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 a = *reinterpret_cast<const uint4*>(&s_act[t][c * GEMM_K + (4 * j + q) * 16]);
        const int g = j >> 1;
        acc[g] = dp4a(wv[j].x, a.x, acc[g]);
        acc[g] = dp4a(wv[j].y, a.y, acc[g]);
        acc[g] = dp4a(wv[j].z, a.z, acc[g]);
        acc[g] = dp4a(wv[j].w, a.w, acc[g]);
      }
#pragma unroll
      for (int g = 0; g < GC; ++g) {
        acc[g] += __shfl_xor_sync(FULL, acc[g], 8);
        acc[g] += __shfl_xor_sync(FULL, acc[g], 16);
      }
      if (q == 0 && row < (int)W.rows) {
        float total = KCH > 1 && c > 0 ? s_tot[KCH > 1 ? t : 0][warp * 8 + lane] : 0.0f;
#pragma unroll
        for (int g = 0; g < GC; ++g) {
          const float a = group_sum_to_float((uint32_t)acc[g]), as = s_as[t][c * GC + g], w = ws[c * GC + g];
          total = W.fused ? __fmaf_rn(a, fmul(w, as), total) : fadd(total, fmul(fmul(fmul(a, w), W.level_scale), as));
        }
        if (c + 1 < KCH)
          s_tot[KCH > 1 ? t : 0][warp * 8 + lane] = total;
        else if (!(meta && meta[t].slot < 0))
          out[(size_t)t * out_stride + row] = total;
      }
    }
  }
}

template <int NT>
constexpr size_t gemm_smem() {
  return (size_t)GEMM_ROWS * GEMM_K + (size_t)NT * GEMM_K;
}

// ------------------------------------------------------------------- heads
// grid M, block 32·(heads + 2·kv_heads). One warp per q, k or v head; lane l
// holds elements l and l+32, the two halves rotary pairs (ops.rs:131-141).
// One head of one token, one warp (attention.rs:118-143): zero-centred norm
// and rotary for query and key heads, then quantise_int8 (ops.rs:112-118).
// kind 0 = query head `head`: its 64 codes go to q_out and the scale is
// returned; 1 = key head, 2 = value head: codes and scale go into the token's
// slot of its KV page.
// The head step's operands that do not come from the projection (the norm
// gains and rotary row are constants, the page slot comes from the host's
// page table): they may be loaded before pdl_wait.
struct HeadPre {
  float g0, g1;
  float2 sc;
  uint8_t* page;
  const float* taps;  // the layer's convolution gains (null without taps)
  int layer;
};
__device__ __forceinline__ HeadPre head_prefetch(const ModelDev& md, const LayerDev& L, const KvDev& kv, const TokenMeta& meta, int layer,
                                                 int kind) {
  const int lane = threadIdx.x & 31;
  const float* gain = kind == 0 ? L.q_norm : L.k_norm;
  HeadPre p;
  p.g0 = gain[lane];
  p.g1 = gain[lane + 32];
  p.sc = md.rotary[(size_t)meta.position * (HEAD_DIM / 2) + lane];
  p.page = kind == 0 ? nullptr : page_base(kv, md.page, meta.slot, layer, meta.position);
  p.taps = L.taps;
  p.layer = layer;
  return p;
}

// QKV causal convolution of one projection column (model/src/attention.rs:83-93
// for a single token, 243-276 for a chunk): Σ over tap < min(taps, position + 1)
// of gain[tap] · raw[position - tap], from +0.0 in tap order. The raw value of
// an earlier position is this pass's row `tap` places up when that row holds
// the same sequence (a pass keeps each sequence's tokens contiguous and in
// order), else the ring row an earlier pass left.
__device__ __forceinline__ float conv_column(const ModelDev& md, const Work& w, const float* taps, int layer, int t,
                                             const TokenMeta& meta, int col) {
  const int qkvg = (2 * md.heads + 2 * md.kv_heads) * HEAD_DIM, width = (int)md.qkv_width, R = (int)md.conv_taps - 1;
  const int n = min((int)md.conv_taps, meta.position + 1);
  float acc = 0.0f;
  for (int tap = 0; tap < n; ++tap) {
    const int p = meta.position - tap;
    bool here = tap == 0;
    if (!here && t - tap >= 0) {
      const TokenMeta o = load_meta(w.meta, t - tap);
      here = o.slot == meta.slot && o.position == p;
    }
    const float x = here ? __ldcg(w.proj + (size_t)(t - tap) * qkvg + col)
                         : __ldcg(md.conv_ring + (((size_t)meta.slot * md.num_layers + layer) * R + p % R) * width + col);
    acc = fadd(acc, fmul(__ldg(taps + (size_t)tap * width + col), x));
  }
  return acc;
}

__device__ __forceinline__ float head_codes(const ModelDev& md, const Work& w, int t, const TokenMeta& meta, int kind, int head,
                                            const HeadPre& pre, int8_t* q_out) {
  const int lane = threadIdx.x & 31;
  const int H = md.heads, KV = md.kv_heads;
  // proj rows: q [H*64] | k [KV*64] | v [KV*64] | gate [H*64]
  const int col = (kind == 0 ? 0 : (kind == 1 ? H * HEAD_DIM : (H + KV) * HEAD_DIM)) + head * HEAD_DIM + lane;
  const float* src = w.proj + (size_t)t * (2 * H + 2 * KV) * HEAD_DIM + col;
  float e0, e1;
  if (pre.taps) {
    e0 = conv_column(md, w, pre.taps, pre.layer, t, meta, col);
    e1 = conv_column(md, w, pre.taps, pre.layer, t, meta, col + 32);
  } else {
    e0 = src[0];
    e1 = src[32];
  }
  const float g0 = pre.g0, g1 = pre.g1;
  const float2 sc = pre.sc;
  uint8_t* page = pre.page;
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
    e0 = fmul(fmul(fadd(1.0f, g0), e0), inv);
    e1 = fmul(fmul(fadd(1.0f, g1), e1), inv);
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
    q_out[lane] = c0;
    q_out[lane + 32] = c1;
    return scale;
  }
  const PageGeometry& pg = md.page;
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
  return scale;
}

// grid M, block 32·(H + 2·KV): one warp per query, key and value head.
__global__ void k_heads(ModelDev md, LayerDev L, Work w, KvDev kv, int M, int layer) {
  pdl_wait();
  int t = blockIdx.x;
  if (t >= M) return;
  const TokenMeta meta = w.meta[t];
  if (meta.slot < 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = md.heads, KV = md.kv_heads;
  const int kind = warp < H ? 0 : (warp < H + KV ? 1 : 2);
  const int head = kind == 0 ? warp : (kind == 1 ? warp - H : warp - H - KV);
  const float scale = head_codes(md, w, t, meta, kind, head, head_prefetch(md, L, kv, meta, layer, kind),
                                 w.qcodes + ((size_t)t * H + head) * HEAD_DIM);
  if (kind == 0 && lane == 0) w.qscale[(size_t)t * H + head] = scale;
}

// ------------------------------------------------------ int8 activation prep
// in (K values, optionally times sigmoid(gate)) → fake_quantise_int8 (when
// `fake`) → per-group rotation and int8 codes of row t, by the whole block;
// s_v holds K floats, s_red one float per warp. Used for out_proj
// (attention.rs:145-150) and the logits (session.rs:170-175). The inputs are
// read from L2 (another CTA of the same kernel may have written them).
constexpr int PREP_MAX_K = 2048;

__device__ __forceinline__ void prep_token(const float* src, const float* gate, int K, int8_t* act, float* act_scale, int t,
                                           float inv_sqrt_group, int fake, int act_rows, float* s_v, float* s_red) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float peak = 0.0f;
  for (int i4 = tid; i4 < K / 4; i4 += blockDim.x) {
    float4 v = __ldcg(reinterpret_cast<const float4*>(src) + i4);
    if (gate) {
      const float4 gv = __ldcg(reinterpret_cast<const float4*>(gate) + i4);
      v = make_float4(fmul(v.x, sigmoid(gv.x)), fmul(v.y, sigmoid(gv.y)), fmul(v.z, sigmoid(gv.z)), fmul(v.w, sigmoid(gv.w)));
    }
    reinterpret_cast<float4*>(s_v)[i4] = v;
    peak = fmaxf(peak, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  const float scale = int8_scale_of(block_max(peak, s_red));
  const int groups = K / GROUP;
  for (int g = warp; g < groups; g += blockDim.x >> 5) {
    float v[4];
    *reinterpret_cast<float4*>(v) = reinterpret_cast<const float4*>(s_v + g * GROUP)[lane];
    if (fake)
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = fake_quant(v[j], scale);
    fwht128(v, inv_sqrt_group);
    uint32_t packed;
    const float sc = quantise_group(v, packed);
    *reinterpret_cast<uint32_t*>(act + chunked_offset(t, g * GROUP + 4 * lane, act_rows)) = packed;
    if (lane == 0) act_scale[(size_t)t * groups + g] = sc;
  }
}

// ---------------------------------------------------------------- attention
// grid (M, kv_heads), block W + 32: the W worker threads score, weight and
// accumulate the values of the kv head's query heads; the last warp forms the
// softmax totals in the reference's order (four running lanes,
// (l0+l1)+(l2+l3), then the tail; neon.rs:277-307) while the workers
// accumulate. Every KV byte is read once. W = 256 runs three CTAs per SM;
// W = 128 (at most two query heads per kv head: the epilogue gives each of
// the G·64 outputs a thread) runs five, for large prefill passes; W = 512
// runs one, for passes of a few tokens.
constexpr int ATT_WORKERS = 256;
constexpr int ATT_WORKERS_NARROW = 128;
constexpr int ATT_WORKERS_WIDE = 512;
constexpr int MAX_GROUP = 4;
constexpr int ATT_UNROLL = 8;
constexpr int ATT_MAX_KV = 8;

__host__ __device__ constexpr int att_min_blocks(int workers) { return workers == ATT_WORKERS ? 3 : (workers == ATT_WORKERS_NARROW ? 5 : 1); }

__host__ __device__ constexpr int att_wstride(int t_cap) { return t_cap / 4 + 2; }

// The epilogue (EPI) either writes the output rows (ATT_ROWS; k_prep then
// prepares the output projection's activations), or does k_prep's work
// itself: with ATT_CLUSTER (G * 64 values per CTA, whole 128-value groups)
// the CTAs of one token form a cluster over the kv heads, exchange the peak
// of their gated outputs in distributed shared memory and each quantises its
// own groups; with ATT_LAST every CTA writes its rows and counts itself in
// w.arrivals[t], and the token's last CTA prepares the whole row.
// With HEADS (a pass whose tokens all belong to different sequences) the CTA
// first does k_heads' work for its kv head: its query heads' codes go
// straight to shared memory, the key and value into the token's page slot,
// which only this CTA reads in this pass.
constexpr int ATT_ROWS = 0, ATT_CLUSTER = 1, ATT_LAST = 2;
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

template <int G, int EPI, bool HEADS, int W>
__global__ void __launch_bounds__(W + 32, att_min_blocks(W)) k_attend(ModelDev md, LayerDev L, Work w, KvDev kv, int M, int layer, int t_cap) {
  constexpr bool PREP = EPI == ATT_CLUSTER;
  const int global = L.global;
  extern __shared__ float sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // the token's meta, its page pointers and (HEADS) the head step's constant
  // operands come from launches before the predecessor: they load while the
  // predecessor finishes
  const int kvh = blockIdx.y;
  int t = 0;
  TokenMeta meta{-1, 0, 0, 0};
  if ((int)blockIdx.x < M) {
    t = w.order ? __ldcg(w.order + blockIdx.x) : (int)blockIdx.x;
    meta = load_meta(w.meta, t);
  }
  __shared__ const uint8_t* s_page[128];
  if (meta.slot >= 0) {
    const int* table = kv.page_table + ((size_t)meta.slot * kv.num_layers + layer) * kv.max_pages;
    const int npages = meta.position / PAGE_POSITIONS + 1;
    for (int i = tid; i < npages; i += blockDim.x) s_page[i] = kv.pool + (size_t)__ldcg(table + i) * md.page.page_bytes;
  }
  HeadPre hpre{};
  const int hkind = warp < G ? 0 : warp - G + 1;  // HEADS: warps 0..G-1 query heads, G key, G+1 value
  if (HEADS && meta.slot >= 0 && warp < G + 2) hpre = head_prefetch(md, L, kv, meta, layer, hkind);
  pdl_wait();
  if (meta.slot < 0) return;  // also past the last token; the whole cluster shares the token
  if (PREP) cluster_arrive_relaxed();  // paired with the wait before the first remote access
  const int total = meta.position + 1;
  int first = 0;
  if (md.sliding_window > 0 && !global) first = total > (int)md.sliding_window ? total - (int)md.sliding_window : 0;
  const int count = total - first;
  const int b0 = first / 4, nblk = (total - 1) / 4 - b0 + 1;
  const int ws = att_wstride(t_cap);
  float* s_e = sm;                                              // [G][t_cap] coefficients, then exponentials
  float* s_vs = sm + G * t_cap;                                 // [t_cap] value scales
  uint32_t* s_whi = reinterpret_cast<uint32_t*>(s_vs + t_cap);  // [G][ws]
  uint32_t* s_wlo = s_whi + G * ws;                             // [G][ws]
  int* s_pv = reinterpret_cast<int*>(s_wlo + G * ws);           // [(W / 16)][G][64]
  __shared__ __align__(16) uint32_t s_q[MAX_GROUP][16];
  __shared__ float s_qs[MAX_GROUP], s_peak[MAX_GROUP], s_scale2[MAX_GROUP], s_total[MAX_GROUP];
  __shared__ float s_red[MAX_GROUP][W / 32];
  __shared__ float s_gsig[EPI == ATT_ROWS ? 1 : MAX_GROUP * HEAD_DIM];  // sigmoid of this CTA's gate values
  const PageGeometry& pg = md.page;
  if (HEADS) {
    if (warp < G + 2) {
      const float sc = head_codes(md, w, t, meta, hkind, hkind == 0 ? kvh * G + warp : kvh, hpre,
                                  reinterpret_cast<int8_t*>(s_q[hkind == 0 ? warp : 0]));
      if (hkind == 0 && lane == 0) s_qs[warp] = fmul(sc, md.inv_root_qk);
    }
  } else {
    if (tid < G * 16) {
      int h = tid / 16, k = tid % 16;
      s_q[h][k] = reinterpret_cast<const uint32_t*>(w.qcodes + ((size_t)t * md.heads + kvh * G + h) * HEAD_DIM)[k];
    }
    if (tid < G) s_qs[tid] = fmul(w.qscale[(size_t)t * md.heads + kvh * G + tid], md.inv_root_qk);
  }
  if (EPI != ATT_ROWS) {
    // the output gate sigmoid(gate) of this CTA's G·64 values (attention.rs:145-150),
    // by the warps the head step leaves idle
    const int H = md.heads, KV = md.kv_heads, first_thread = HEADS ? (G + 2) * 32 : 0;
    const float* gsrc = w.proj + (size_t)t * (2 * H + 2 * KV) * HEAD_DIM + (H + 2 * KV) * HEAD_DIM + kvh * G * HEAD_DIM;
    for (int i = tid - first_thread; i >= 0 && i < G * HEAD_DIM; i += (W + 32) - first_thread) s_gsig[i] = sigmoid(gsrc[i]);
  }
  __syncthreads();  // the query codes, and with HEADS this position's key and value, are in place

  if (tid < W) {
    // pass 1: integer scores q·k, coefficients (s · key_scale) · query_scale, their
    // peak; the value scales are staged for pass 2. Two positions per thread
    // per round, both positions' loads in flight together.
    float lmax[G];
#pragma unroll
    for (int h = 0; h < G; ++h) lmax[h] = -INFINITY;
    for (int i0 = tid; i0 < count; i0 += 2 * W) {
      uint4 key[2][4];
      float ks[2], vs[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = min(i0 + u * W, count - 1);
        const int p = first + i, within = p % PAGE_POSITIONS;
        const uint8_t* page = s_page[p / PAGE_POSITIONS];
        const uint4* kp = reinterpret_cast<const uint4*>(page + ((size_t)kvh * PAGE_POSITIONS + within) * HEAD_DIM);
#pragma unroll
        for (int k = 0; k < 4; ++k) key[u][k] = kp[k];
        ks[u] = reinterpret_cast<const float*>(page + pg.kscale_offset)[kvh * PAGE_POSITIONS + within];
        vs[u] = reinterpret_cast<const float*>(page + pg.vscale_offset)[kvh * PAGE_POSITIONS + within];
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = i0 + u * W;
        if (i < count) {
          s_vs[i] = vs[u];
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const uint4* q = reinterpret_cast<const uint4*>(s_q[h]);
            int part[4] = {0, 0, 0, 0};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint4 qv = q[k];
              part[0] = dp4a(key[u][k].x, qv.x, part[0]);
              part[1] = dp4a(key[u][k].y, qv.y, part[1]);
              part[2] = dp4a(key[u][k].z, qv.z, part[2]);
              part[3] = dp4a(key[u][k].w, qv.w, part[3]);
            }
            const int s = (part[0] + part[1]) + (part[2] + part[3]);
            float c = fmul(fmul((float)s, ks[u]), s_qs[h]);
            s_e[h * t_cap + i] = c;
            lmax[h] = fmaxf(lmax[h], c);
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float m = warp_max(lmax[h]);
      if (lane == 0) s_red[h][warp] = m;
    }
  }
  __syncthreads();
  if (tid < G) {
    float m = s_red[tid][0];
    for (int k = 1; k < W / 32; ++k) m = fmaxf(m, s_red[tid][k]);
    s_peak[tid] = m;
  }
  __syncthreads();
  if (tid < W) {
    // pass 2: e = fast_exp(c - peak) and the peak of the weights e · value_scale
    float lmax[G];
#pragma unroll
    for (int h = 0; h < G; ++h) lmax[h] = 0.0f;
    for (int i = tid; i < count; i += W) {
      const float vs = s_vs[i];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float e = fast_exp(fsub(s_e[h * t_cap + i], s_peak[h]));
        s_e[h * t_cap + i] = e;
        lmax[h] = fmaxf(lmax[h], fabsf(fmul(e, vs)));
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float m = warp_max(lmax[h]);
      if (lane == 0) s_red[h][warp] = m;
    }
  }
  __syncthreads();
  if (tid < G) {
    float pk = s_red[tid][0];
    for (int k = 1; k < W / 32; ++k) pk = fmaxf(pk, s_red[tid][k]);
    s_peak[tid] = pk;
    s_scale2[tid] = fdiv(pk, 2047.0f);
  }
  __syncthreads();
  if (warp == W / 32) {
    // softmax totals in the order of neon.rs:294-305
    const int h = lane >> 2, j = lane & 3;
    const int vc = count - count % 4;
    float acc = 0.0f;
    if (h < G) {
      const float* e = s_e + h * t_cap;
      int i = j;
      // sixteen loads in flight per batch; the running sum stays one ordered chain per lane
      for (; i + 4 * 15 < vc; i += 4 * 16) {
        float v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = e[i + 4 * k];
#pragma unroll
        for (int k = 0; k < 16; ++k) acc = fadd(acc, v[k]);
      }
      for (; i < vc; i += 4) acc = fadd(acc, e[i]);
    }
    float l0 = __shfl_sync(FULL, acc, (lane & ~3) + 0), l1 = __shfl_sync(FULL, acc, (lane & ~3) + 1);
    float l2 = __shfl_sync(FULL, acc, (lane & ~3) + 2), l3 = __shfl_sync(FULL, acc, (lane & ~3) + 3);
    if (h < G && j == 0) {
      float tot = fadd(fadd(l0, l1), fadd(l2, l3));
      for (int i = vc; i < count; ++i) tot = fadd(tot, s_e[h * t_cap + i]);
      s_total[h] = tot;
    }
  } else {
    // pass 3: 12-bit weights round(c / (peak / 2047)) (half away from zero) of
    // c = e · value_scale, split into 6-bit halves per absolute 4-position
    // block (attention.rs:294-310, neon.rs:348-365)
    for (int b = tid; b < nblk; b += W) {
      const int pbase = (b0 + b) * 4;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        uint32_t hi = 0, lo = 0;
        const float sc = s_scale2[h];
        const bool live = s_peak[h] > 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int p = pbase + j;
          int wgt = 0;
          if (live && p >= first && p < total) {
            const int i = p - first;
            wgt = (int)roundf(fdiv(fmul(s_e[h * t_cap + i], s_vs[i]), sc));
          }
          hi |= (uint32_t)((wgt >> 6) & 0xff) << (8 * j);
          lo |= (uint32_t)((wgt & 63) & 0xff) << (8 * j);
        }
        s_whi[h * ws + b] = hi;
        s_wlo[h * ws + b] = lo;
      }
    }
    named_barrier(1, W);
    // pass 4: exact integer sums over the value panels; thread (dq, slice) owns
    // four dimensions and every (W / 16)-th block, ATT_UNROLL blocks per round
    const int dq = tid & 15, slice = tid >> 4;
    int hi_acc[G][4], lo_acc[G][4];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int k = 0; k < 4; ++k) hi_acc[h][k] = lo_acc[h][k] = 0;
    const size_t vbase = pg.value_offset + (size_t)kvh * PAGE_POSITIONS * HEAD_DIM + dq * 16;
    for (int bb = slice; bb < nblk; bb += ATT_UNROLL * (W / 16)) {
      uint4 v[ATT_UNROLL];
#pragma unroll
      for (int u = 0; u < ATT_UNROLL; ++u) {
        const int b = min(bb + u * (W / 16), nblk - 1);
        const int p = (b0 + b) * 4;
        v[u] = *reinterpret_cast<const uint4*>(s_page[p / PAGE_POSITIONS] + vbase + ((p % PAGE_POSITIONS) / 4) * (HEAD_DIM * 4));
      }
#pragma unroll
      for (int u = 0; u < ATT_UNROLL; ++u) {
        const int b = bb + u * (W / 16);
        if (b < nblk) {
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const uint32_t whi = s_whi[h * ws + b], wlo = s_wlo[h * ws + b];
            hi_acc[h][0] = dp4a(v[u].x, whi, hi_acc[h][0]);
            hi_acc[h][1] = dp4a(v[u].y, whi, hi_acc[h][1]);
            hi_acc[h][2] = dp4a(v[u].z, whi, hi_acc[h][2]);
            hi_acc[h][3] = dp4a(v[u].w, whi, hi_acc[h][3]);
            lo_acc[h][0] = dp4a(v[u].x, wlo, lo_acc[h][0]);
            lo_acc[h][1] = dp4a(v[u].y, wlo, lo_acc[h][1]);
            lo_acc[h][2] = dp4a(v[u].z, wlo, lo_acc[h][2]);
            lo_acc[h][3] = dp4a(v[u].w, wlo, lo_acc[h][3]);
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int k = 0; k < 4; ++k) s_pv[(slice * G + h) * HEAD_DIM + dq * 4 + k] = (hi_acc[h][k] << 6) + lo_acc[h][k];
  }
  __syncthreads();
  pdl_trigger();  // the output rows overlap the next kernel's prologue
  float out = 0.0f;
  if (tid < G * HEAD_DIM) {
    const int h = tid / HEAD_DIM, dim = tid % HEAD_DIM;
    int sum = 0;
#pragma unroll
    for (int s = 0; s < (W / 16); ++s) sum += s_pv[(s * G + h) * HEAD_DIM + dim];
    const float value = s_peak[h] > 0.0f ? fmul((float)sum, s_scale2[h]) : 0.0f;
    const float inverse = fdiv(1.0f, s_total[h]);
    out = fmul(value, inverse);
    // with ATT_LAST the rows are stored gated, ready for the last CTA's prep
    if (!PREP) w.attn[(size_t)t * md.heads * HEAD_DIM + (kvh * G + h) * HEAD_DIM + dim] = EPI == ATT_LAST ? fmul(out, s_gsig[tid]) : out;
  }
  if (EPI == ATT_LAST) {
    // the last of the token's kv-head CTAs prepares the output projection's
    // activations for the whole row (the fence orders every CTA's rows
    // before its count; the reader fences again before reading them)
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&w.arrivals[t], 1) == (int)gridDim.y - 1;
    __syncthreads();
    if (s_last) {
      __threadfence();
      const int K = md.heads * HEAD_DIM;
      prep_token(w.attn + (size_t)t * K, nullptr, K, w.act, w.act_scale, t, md.inv_sqrt_group, 1, 0, s_e, &s_red[0][0]);
      if (tid == 0) w.arrivals[t] = 0;  // ready for the next layer's attention
    }
  }
  if (PREP) {
    // k_prep (attention.rs:145-150): the output gated by sigmoid(gate), the
    // peak over the token's whole vector (all kv heads of the cluster), the
    // fake quantisation, then per 128-group rotation and int8 codes
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ __align__(16) float s_o[MAX_GROUP * HEAD_DIM];
    __shared__ float s_cpeak[ATT_MAX_KV];
    const int H = md.heads, KV = md.kv_heads;
    float mag = 0.0f;
    if (tid < G * HEAD_DIM) {
      const float v = fmul(out, s_gsig[tid]);
      s_o[tid] = v;
      mag = fabsf(v);
    }
    mag = warp_max(mag);
    if (lane == 0 && warp < G * 2) s_red[0][warp] = mag;
    __syncthreads();
    cluster_wait();  // every CTA of the cluster runs: distributed shared memory is usable
    if (tid == 0) {
      float pk = s_red[0][0];
      for (int i = 1; i < G * 2; ++i) pk = fmaxf(pk, s_red[0][i]);
      for (int r = 0; r < KV; ++r) *cluster.map_shared_rank(&s_cpeak[kvh], r) = pk;
    }
    cluster.sync();
    float peak = s_cpeak[0];
    for (int r = 1; r < KV; ++r) peak = fmaxf(peak, s_cpeak[r]);
    const float scale = int8_scale_of(peak);
    if (warp < G / 2) {
      const float4 x = reinterpret_cast<const float4*>(s_o + warp * GROUP)[lane];
      float v[4] = {fake_quant(x.x, scale), fake_quant(x.y, scale), fake_quant(x.z, scale), fake_quant(x.w, scale)};
      fwht128(v, md.inv_sqrt_group);
      uint32_t packed;
      const float sc = quantise_group(v, packed);
      const int K = H * HEAD_DIM, group = kvh * (G / 2) + warp;
      *reinterpret_cast<uint32_t*>(w.act + core_offset(t, group * GROUP + 4 * lane, K / 16)) = packed;
      if (lane == 0) w.act_scale[(size_t)t * (K / GROUP) + group] = sc;
    }
  }
}

// ------------------------------------------------------ int8 activation prep
// prep_token for M rows (row rows[m] of `in` when rows is given). grid M, block 128.
__global__ void __launch_bounds__(128) k_prep(const float* __restrict__ in, int in_stride, const int32_t* __restrict__ rows,
                                              const float* __restrict__ gate, int gate_stride, int K, int8_t* __restrict__ act,
                                              float* __restrict__ act_scale, int M, const TokenMeta* __restrict__ meta,
                                              float inv_sqrt_group, int fake, int act_rows) {
  pdl_wait();
  __shared__ __align__(16) float s_v[PREP_MAX_K];
  __shared__ float s_red[4];
  const int t = blockIdx.x;
  if (t >= M || (meta && meta[t].slot < 0)) return;
  prep_token(in + (size_t)(rows ? rows[t] : t) * in_stride, gate ? gate + (size_t)t * gate_stride : nullptr, K, act, act_scale, t,
             inv_sqrt_group, fake, act_rows, s_v, s_red);
}

// ------------------------------------------------------------ block finish
// grid M, block 256. Post norm, gated residual (session.rs:121-125), the
// Hadamard MLP (hadamard.rs:260-304) and the lane combine (lanes.rs:183-204).
//
// Each Kronecker factor application K(x) = Lᵀ·(X·R) (ops.rs:143-164) runs as
// two products C[r][c] = Σ_s A[s][r]·B[s][c] with s ascending, the reference's
// summation order for every output. A thread owns a 4×2 output tile: each
// step reads one float4 of A and one float2 of B from shared memory for 8
// multiply-adds, two columns per packed instruction. The stage-A operand X
// enters transposed (XT[j][i]). Operands arrive by cp.async, the next factor
// pair while the current stage's elementwise pass runs.

template <int S, int R, bool FUSED32>
__device__ __forceinline__ void tn_stage(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, float2 nz,
                                         int rows = R) {
  // A thread owns a 4-row × 2-column tile: per step one float4 of A, one
  // float2 of B, and the two columns of a row share one packed f32x2 product.
  // Only the first `rows` output rows (a multiple of 4) are formed.
  const int tiles = (rows / 4) * (HADA_RIGHT / 2);
  const int tid = threadIdx.x;
  if (tid < tiles) {
    const int r0 = (tid / (HADA_RIGHT / 2)) * 4, c0 = (tid % (HADA_RIGHT / 2)) * 2;
    float2 acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.0f, 0.0f);
#pragma unroll 8
    for (int s = 0; s < S; ++s) {
      const float4 a = *reinterpret_cast<const float4*>(A + s * R + r0);
      const float2 b = *reinterpret_cast<const float2*>(B + s * HADA_RIGHT + c0);
      const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 ai = make_float2(av[i], av[i]);
        if (FUSED32)
          acc[i] = fma2(ai, b, acc[i]);
        else
          acc[i] = add2(acc[i], fma2(ai, b, nz));  // product rounded, then the sum rounded
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) *reinterpret_cast<float2*>(C + (r0 + i) * HADA_RIGHT + c0) = acc[i];
  }
  __syncthreads();
}

// One Kronecker factor application; out_rows limits the second product to
// the output rows that are read afterwards.
template <int LEFT, bool FUSED32>
__device__ __forceinline__ void kronecker(float* xt, float* tmp, const float* left, const float* right, float* out, float2 nz,
                                          int out_rows = LEFT) {
  tn_stage<HADA_RIGHT, LEFT, FUSED32>(xt, right, tmp, nz);
  tn_stage<LEFT, LEFT, FUSED32>(left, tmp, out, nz, out_rows);
}

constexpr int BLOCK_THREADS = 256;

// The stage-A operand position of element e of a LEFT×32 matrix.
template <int LEFT>
__device__ __forceinline__ int transposed(int e) { return (e % HADA_RIGHT) * LEFT + e / HADA_RIGHT; }

// Rows of the last application's result that hold the d outputs (the rest
// is padding the reference drops): ceil(d / 32), rounded up to whole 4-row tiles.
template <int LEFT>
__device__ __forceinline__ int output_rows(int d) {
  return min(LEFT, (d / HADA_RIGHT + 3) / 4 * 4);
}

// The front of the Hadamard MLP (hadamard.rs:260-283) on the pre-normed
// input s_pre (d values): the rank-8 condition softmax, the modulation
// 1 + Σ_r w_r·cond_u[r] into s_mod and X = pad(x) ⊙ d1, transposed, into xt.
// cond_v must already be staged in s_condv (it is overwritten).
template <int LEFT>
__device__ __forceinline__ void hada_prepare(const HadamardDev& Hd, const int d, const float* s_pre, float* xt, float* s_mod,
                                             float* s_condv) {
  constexpr int N = LEFT * HADA_RIGHT;
  constexpr int PER = N / (4 * BLOCK_THREADS);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __shared__ float s_w[COND_RANK];
  // condition weights: four chains of rank-8 partial sums (hadamard.rs:263-276).
  // Chain (j, r) adds x[4g+j]·cond_v[4g+j][r] over g in order; the products
  // are formed in place by the whole block (element 32g + 8j + r of cond_v
  // meets x[4g + j]), then lane 8j + r of warp 0 runs the ordered sum.
  for (int i = tid; i < d * COND_RANK; i += BLOCK_THREADS) s_condv[i] = fmul(s_pre[i >> 3], s_condv[i]);
  __syncthreads();
  if (warp == 0) {
    float acc = 0.0f;
    const int G = d / 4;
    int g = 0;
    for (; g + 15 < G; g += 16) {
      float p[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) p[k] = s_condv[32 * (g + k) + lane];
#pragma unroll
      for (int k = 0; k < 16; ++k) acc = fadd(acc, p[k]);
    }
    for (; g < G; ++g) acc = fadd(acc, s_condv[32 * g + lane]);
    // lane r < 8: weight r = the four chains j = 0..3 in order from +0.0,
    // then the softmax: peak over the eight lanes, each lane's exponential,
    // the total in r order from +0.0, one division
    const float c1 = __shfl_down_sync(FULL, acc, COND_RANK), c2 = __shfl_down_sync(FULL, acc, 2 * COND_RANK),
                c3 = __shfl_down_sync(FULL, acc, 3 * COND_RANK);
    const float wv = fadd(fadd(fadd(fadd(0.0f, acc), c1), c2), c3);
    float peak = wv;
#pragma unroll
    for (int s = 1; s < COND_RANK; s <<= 1) peak = fmaxf(peak, __shfl_xor_sync(FULL, peak, s));
    const float ev = fast_exp(fsub(wv, peak));
    float total = 0.0f;
#pragma unroll
    for (int r = 0; r < COND_RANK; ++r) total = fadd(total, __shfl_sync(FULL, ev, r));
    const float inverse = fdiv(1.0f, total);
    if (lane < COND_RANK) s_w[lane] = fmul(ev, inverse);
  }
  __syncthreads();
  // modulation = 1 + Σ_r w_r·cond_u[r] (sequential over r) and X = pad(x) ⊙ d1
#pragma unroll 2
  for (int q = 0; q < PER; ++q) {
    const int i4 = tid + q * BLOCK_THREADS;
    float4 u[COND_RANK];
#pragma unroll
    for (int r = 0; r < COND_RANK; ++r) u[r] = reinterpret_cast<const float4*>(Hd.cond_u + (size_t)r * N)[i4];
    const float4 d1 = reinterpret_cast<const float4*>(Hd.d1)[i4];
    float m[4] = {1.0f, 1.0f, 1.0f, 1.0f};
#pragma unroll
    for (int r = 0; r < COND_RANK; ++r) {
      m[0] = fadd(m[0], fmul(s_w[r], u[r].x));
      m[1] = fadd(m[1], fmul(s_w[r], u[r].y));
      m[2] = fadd(m[2], fmul(s_w[r], u[r].z));
      m[3] = fadd(m[3], fmul(s_w[r], u[r].w));
    }
    *reinterpret_cast<float4*>(s_mod + 4 * i4) = make_float4(m[0], m[1], m[2], m[3]);
    const float dv[4] = {d1.x, d1.y, d1.z, d1.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int i = 4 * i4 + e;
      xt[transposed<LEFT>(i)] = fmul(i < d ? s_pre[i] : 0.0f, dv[e]);
    }
  }
  __syncthreads();
}

// The operands of the two elementwise passes, loaded into registers ahead of
// the Kronecker application they follow so their latency hides behind it.
template <int LEFT>
struct HadaPass1 {
  static constexpr int PER = LEFT * HADA_RIGHT / (4 * BLOCK_THREADS);
  int4 p1[PER];
  float4 d2v[PER], b2v[PER];
  __device__ __forceinline__ void load(const ModelDev& md, const HadamardDev& Hd) {
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int i4 = threadIdx.x + q * BLOCK_THREADS;
      p1[q] = reinterpret_cast<const int4*>(md.perm1)[i4];
      d2v[q] = reinterpret_cast<const float4*>(Hd.d2)[i4];
      b2v[q] = reinterpret_cast<const float4*>(Hd.b2)[i4];
    }
  }
  // xt[transposed(i)] = silu(d2 ⊙ modulation ⊙ in[perm1[i]] + b2)  (hadamard.rs:288-294)
  __device__ __forceinline__ void run(const float* s_mod, const float* in, float* xt) const {
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int i4 = threadIdx.x + q * BLOCK_THREADS;
      const float4 mo = *reinterpret_cast<const float4*>(s_mod + 4 * i4);
      const int pv[4] = {p1[q].x, p1[q].y, p1[q].z, p1[q].w};
      const float dv[4] = {d2v[q].x, d2v[q].y, d2v[q].z, d2v[q].w}, bv[4] = {b2v[q].x, b2v[q].y, b2v[q].z, b2v[q].w},
                  mv[4] = {mo.x, mo.y, mo.z, mo.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) xt[transposed<LEFT>(4 * i4 + e)] = silu(fadd(fmul(fmul(dv[e], mv[e]), in[pv[e]]), bv[e]));
    }
  }
};

template <int LEFT>
struct HadaPass2 {
  static constexpr int PER = LEFT * HADA_RIGHT / (4 * BLOCK_THREADS);
  int4 p2[PER];
  float4 d3v[PER];
  __device__ __forceinline__ void load(const ModelDev& md, const HadamardDev& Hd) {
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int i4 = threadIdx.x + q * BLOCK_THREADS;
      p2[q] = reinterpret_cast<const int4*>(md.perm2)[i4];
      d3v[q] = reinterpret_cast<const float4*>(Hd.d3)[i4];
    }
  }
  // xt[transposed(i)] = in[perm2[i]] ⊙ d3  (hadamard.rs:296-300)
  __device__ __forceinline__ void run(const float* in, float* xt) const {
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int i4 = threadIdx.x + q * BLOCK_THREADS;
      const int pv[4] = {p2[q].x, p2[q].y, p2[q].z, p2[q].w};
      const float dv[4] = {d3v[q].x, d3v[q].y, d3v[q].z, d3v[q].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) xt[transposed<LEFT>(4 * i4 + e)] = fmul(in[pv[e]], dv[e]);
    }
  }
};

// The Hadamard MLP of hadamard.rs:260-304 on the pre-normed input s_pre (d
// values): rank-8 condition softmax, modulation, three Kronecker factor
// applications with the two permutations and the SiLU gate. The result (before
// the final d4 scale) is left in buf0[0..d). cond_v, left[0] and right[0] must
// already be staged in s_condv, s_left and s_right; with RESIDENT all three
// factor pairs are (factor k at s_left + k·LEFT², s_right + k·32²), else the
// next pair is staged into the same place while an elementwise pass runs.
template <int LEFT, bool RESIDENT>
__device__ __forceinline__ void hadamard_core(const ModelDev& md, const HadamardDev& Hd, const int d, const float* s_pre, float* buf0,
                                              float* buf1, float* s_mod, float* s_left, float* s_right, float* s_condv) {
  constexpr bool FUSED32 = LEFT == 32;
  constexpr int LS = RESIDENT ? LEFT * LEFT : 0, RS = RESIDENT ? HADA_RIGHT * HADA_RIGHT : 0;
  const float2 nz = g_negzero;
  hada_prepare<LEFT>(Hd, d, s_pre, buf0, s_mod, s_condv);
  HadaPass1<LEFT> pass1;
  pass1.load(md, Hd);
  kronecker<LEFT, FUSED32>(buf0, buf1, s_left, s_right, buf0, nz);  // first = K1(d1 ⊙ x)
  if (!RESIDENT) {
    stage_async(s_left, Hd.left[1], LEFT * LEFT);
    stage_async(s_right, Hd.right[1], HADA_RIGHT * HADA_RIGHT);
  }
  pass1.run(s_mod, buf0, buf1);
  HadaPass2<LEFT> pass2;
  pass2.load(md, Hd);
  if (!RESIDENT) cp_async_wait_all();
  __syncthreads();
  kronecker<LEFT, FUSED32>(buf1, buf0, s_left + LS, s_right + RS, buf1, nz);  // second
  if (!RESIDENT) {
    stage_async(s_left, Hd.left[2], LEFT * LEFT);
    stage_async(s_right, Hd.right[2], HADA_RIGHT * HADA_RIGHT);
  }
  pass2.run(buf1, buf0);
  if (!RESIDENT) cp_async_wait_all();
  __syncthreads();
  kronecker<LEFT, FUSED32>(buf0, buf1, s_left + 2 * LS, s_right + 2 * RS, buf0, nz, output_rows<LEFT>(d));  // third
}

// The front of the block finish (session.rs:121-137): the layer's constant
// operands (cond_v, the first Kronecker factors, the two norm gains) by bulk
// copy, then (once the previous kernel is done) the token's rows, the post
// norm and gated residual into s_a, and the pre-Hadamard norm into s_pre.
// False when the token is not live: the CTA has then waited for its copies
// and returns. FACTORS Kronecker factor pairs are copied (k-th at
// s_left + k·LEFT², s_right + k·32²).
// With QKV convolution taps, the block finish also keeps the ring (the
// attention's head step, launches earlier, has read it): each of the last
// taps - 1 tokens of a sequence in this pass stores its raw q | k | v row at
// ring row position % (taps - 1). `part` of `parts` CTAs of the token copies
// its share.
__device__ __forceinline__ void conv_ring_store(const ModelDev& md, const LayerDev& L, const Work& w, int M, int t, int part, int parts) {
  const int R = (int)md.conv_taps - 1, width = (int)md.qkv_width;
  const TokenMeta meta = load_meta(w.meta, t);
  if (t + R < M) {
    const TokenMeta o = load_meta(w.meta, t + R);
    if (o.slot == meta.slot && o.position == meta.position + R) return;  // a later token of the pass holds this ring row
  }
  const float* src = w.proj + (size_t)t * (2 * md.heads + 2 * md.kv_heads) * HEAD_DIM;
  float* dst = md.conv_ring + (((size_t)meta.slot * md.num_layers + L.index) * R + meta.position % R) * width;
  const int share = width / parts;
  for (int i = part * share + (int)threadIdx.x; i < (part + 1) * share; i += blockDim.x) dst[i] = __ldcg(src + i);
}

// At an engram site layer the last (taps - 1) · dilation tokens of a sequence
// in this pass store their raw values in the site's ring (k_route, launches
// earlier, has read it).
__device__ __forceinline__ void engram_ring_store(const ModelDev& md, const EngramDev& E, const Work& w, int M, int t, int part, int parts) {
  const int R = (int)E.cfg.ring_rows, d = (int)md.d_model;
  const TokenMeta meta = load_meta(w.meta, t);
  if (t + R < M) {
    const TokenMeta o = load_meta(w.meta, t + R);
    if (o.slot == meta.slot && o.position == meta.position + R) return;
  }
  const float* src = w.engram_kv + (size_t)t * 2 * d + d;
  float* dst = E.ring + ((size_t)meta.slot * R + meta.position % R) * d;
  const int share = d / parts;
  for (int i = part * share + (int)threadIdx.x; i < (part + 1) * share; i += blockDim.x) dst[i] = __ldcg(src + i);
}

// No fused out product: the block finish stages the attention's out product row.
struct StagedOut {
  __device__ bool fused() const { return false; }
  __device__ void operator()() const {}
};

template <int LEFT, int FACTORS, typename OutProduct = StagedOut>
__device__ __forceinline__ bool block_front(const ModelDev& md, const LayerDev& L, const Work& w, int M, int t, int d, int* error,
                                            float* s_a, float* s_x, float* s_pre, float* s_condv, float* s_left, float* s_right,
                                            float* s_gpost, float* s_gpre, int part, int parts, const OutProduct& out_product = {}) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __shared__ float s_inv, s_gate;
  __shared__ __align__(8) uint64_t s_bar;
  const uint32_t bar = smem_u32(&s_bar);
  const HadamardDev& Hd = L.hada;
  if (tid == 0) {  // one thread arms the barrier and issues every copy
    bulk_start(bar, (d * COND_RANK + FACTORS * (LEFT * LEFT + HADA_RIGHT * HADA_RIGHT) + 2 * d) * 4);
    bulk_copy(s_condv, Hd.cond_v, d * COND_RANK * 4, bar);
    for (int k = 0; k < FACTORS; ++k) {
      bulk_copy(s_left + k * LEFT * LEFT, Hd.left[k], LEFT * LEFT * 4, bar);
      bulk_copy(s_right + k * HADA_RIGHT * HADA_RIGHT, Hd.right[k], HADA_RIGHT * HADA_RIGHT * 4, bar);
    }
    bulk_copy(s_gpost, L.post_norm, d * 4, bar);
    bulk_copy(s_gpre, L.pre_hada, d * 4, bar);
  }
  if (tid == 32) s_gate = sigmoid(L.attn_gate);
  // the routing input (k_route, launches earlier) and the token's meta load
  // while the predecessor finishes
  const bool live = t < M && load_meta(w.meta, t).slot >= 0;
  if (live) stage_async(s_x, w.x + (size_t)t * d, d);
  pdl_wait();
  if (!live) {
    if (tid == 0 && !mbar_wait(bar, 0)) atomicExch(error, 1);  // no copy outlives the CTA
    return false;
  }
  // with Whistle cross attention, k_cross_q has formed x after the residual (w.xr)
  // and, for sessions with a memory, the cross out product sits in w.outp
  if (!out_product.fused()) stage_async(s_a, (md.cross ? w.xr : w.outp) + (size_t)t * d, d);
  const bool cross_live = md.cross && md.slot_cross[load_meta(w.meta, t).slot];
  if (cross_live) stage_async(s_pre, w.outp + (size_t)t * d, d);
  if (md.conv_ring) conv_ring_store(md, L, w, M, t, part, parts);
  if (L.engram && L.engram->ring) engram_ring_store(md, *L.engram, w, M, t, part, parts);
  cp_async_wait_all();
  // the staged rows, the gate and the barrier's initialisation are visible to
  // every thread past this point; then each thread waits for the bulk copies
  __syncthreads();
  if (!mbar_wait(bar, 0) && tid == 0) atomicExch(error, 1);
  out_product();  // with the out product fused: s_a formed here, in every CTA of the cluster
  if (!md.cross) {
    if (warp == 0) {
      float ss = sum_of_squares_warp(s_a, d);
      if (lane == 0) s_inv = inverse_rms(ss, d);
    }
    __syncthreads();
    for (int i = tid; i < d; i += BLOCK_THREADS) {
      float a = fmul(fmul(fadd(1.0f, s_gpost[i]), s_a[i]), s_inv);
      s_a[i] = fadd(s_x[i], fmul(s_gate, a));
    }
    __syncthreads();
  } else if (cross_live) {
    // CrossState::apply's last step (cross.rs:176-181): the out product normed
    // with the cross post norm, then x += sigmoid(gate) · attended
    const CrossLayerDev& C = md.cross[L.index];
    if (warp == 0) {
      float ss = sum_of_squares_warp(s_pre, d);
      if (lane == 0) s_inv = inverse_rms(ss, d);
    }
    __syncthreads();
    for (int i = tid; i < d; i += BLOCK_THREADS) {
      const float a = fmul(fmul(fadd(1.0f, C.post_norm[i]), s_pre[i]), s_inv);
      s_a[i] = fadd(s_a[i], fmul(C.gain, a));
    }
    __syncthreads();
  }
  if (warp == 0) {
    float ss = sum_of_squares_warp(s_a, d);
    if (lane == 0) s_inv = inverse_rms(ss, d);
  }
  __syncthreads();
  for (int i = tid; i < d; i += BLOCK_THREADS) s_pre[i] = fmul(fmul(fadd(1.0f, s_gpre[i]), s_a[i]), s_inv);
  return true;
}

// x += mlp · d4; delta = x - input; next lane l = Σ_s res[l][s]·lane_s + post[l]·delta
// (lanes.rs:183-204) for element i.
__device__ __forceinline__ float lane_out(const float* rw, const float* sv, int l, float delta) {
  float acc = 0.0f;
#pragma unroll
  for (int s = 0; s < LANES; ++s) acc = fadd(acc, fmul(rw[LANES + l * LANES + s], sv[s]));
  return fadd(acc, fmul(rw[l], delta));
}

// grid M, block 256. Post norm, gated residual (session.rs:121-125), the
// Hadamard MLP (hadamard.rs:260-304) and the lane combine (lanes.rs:183-204).
// RES keeps all three Kronecker factor pairs resident and the lane combine's
// operands in registers from the start (two CTAs per SM); without RES one
// factor pair is staged per application and the operands load after the
// Hadamard MLP (three CTAs per SM).
template <int LEFT, bool RES>
__device__ __forceinline__ void block_finish(const ModelDev& md, const LayerDev& L, const Work& w, int M, int* error) {
  constexpr int F = RES ? 3 : 1;
  extern __shared__ float sm[];
  constexpr int N = LEFT * HADA_RIGHT;
  const int t = blockIdx.x;
  const int d = md.d_model, tid = threadIdx.x;
  float* s_a = sm;                        // d: attention output, then the running block value
  float* s_x = sm + MAX_D;                // d: the routing input
  float* s_pre = sm + 2 * MAX_D;          // d: pre-Hadamard norm
  float* buf0 = sm + 3 * MAX_D;           // N
  float* buf1 = buf0 + N;                 // N
  float* s_mod = buf1 + N;                // N
  float* s_left = s_mod + N;                  // F × LEFT*LEFT: the left factors
  float* s_right = s_left + F * LEFT * LEFT;  // F × 32*32: the right factors
  // d*8 condition values, consumed before the first Kronecker stage: they
  // borrow buf1 and s_mod when they fit there
  float* s_condv = d * COND_RANK <= 2 * N ? buf1 : s_right + F * HADA_RIGHT * HADA_RIGHT;
  float* s_gpost = s_right + F * HADA_RIGHT * HADA_RIGHT + (d * COND_RANK <= 2 * N ? 0 : d * COND_RANK);  // d post_norm gains
  float* s_gpre = s_gpost + MAX_D;                                                                         // d pre_hada gains
  const HadamardDev& Hd = L.hada;

  // the lane combine's operands (routing weights and this token's lanes, from
  // launches before the predecessor; d4) load first, and stay in registers
  // through the Hadamard MLP; one float4 column per thread (d <= 4 · 256)
  const float* route = w.route + (size_t)t * (LANES + LANES * LANES);
  float rw[LANES + LANES * LANES];
  const float* stream = w.stream + (size_t)t * LANES * d;
  float* next = w.next_stream + (size_t)t * LANES * d;
  const int i4 = tid;
  float4 sv[LANES], d4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (RES) {
#pragma unroll
    for (int k = 0; k < LANES + LANES * LANES; ++k) rw[k] = __ldcg(route + k);
    if (i4 < d / 4) {
      d4 = reinterpret_cast<const float4*>(Hd.d4)[i4];
#pragma unroll
      for (int s = 0; s < LANES; ++s) sv[s] = __ldcg(reinterpret_cast<const float4*>(stream + s * d) + i4);
    }
  }
  if (!block_front<LEFT, F>(md, L, w, M, t, d, error, s_a, s_x, s_pre, s_condv, s_left, s_right, s_gpost, s_gpre, 0, 1)) return;
  __syncthreads();
  hadamard_core<LEFT, RES>(md, Hd, d, s_pre, buf0, buf1, s_mod, s_left, s_right, s_condv);
  if (!RES) {
#pragma unroll
    for (int k = 0; k < LANES + LANES * LANES; ++k) rw[k] = __ldcg(route + k);
    if (i4 < d / 4) {
      d4 = reinterpret_cast<const float4*>(Hd.d4)[i4];
#pragma unroll
      for (int s = 0; s < LANES; ++s) sv[s] = __ldcg(reinterpret_cast<const float4*>(stream + s * d) + i4);
    }
  }
  pdl_trigger();  // the lane combine overlaps the next kernel's prologue
  if (i4 < d / 4) {
    const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
    // delta = x - routing input (lanes.rs:100-104); at an engram site x started from input + engram term
    const float* xin = L.engram_site >= 0 ? w.xin + (size_t)t * d : nullptr;
    float delta[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int i = 4 * i4 + e;
      delta[e] = fsub(fadd(s_a[i], fmul(buf0[i], dv[e])), xin ? __ldcg(xin + i) : s_x[i]);
    }
#pragma unroll
    for (int l = 0; l < LANES; ++l) {
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lanes_e[LANES] = {(&sv[0].x)[e], (&sv[1].x)[e], (&sv[2].x)[e], (&sv[3].x)[e]};
        o[e] = lane_out(rw, lanes_e, l, delta[e]);
      }
      reinterpret_cast<float4*>(next + l * d)[i4] = make_float4(o[0], o[1], o[2], o[3]);
    }
  }
}

template <int LEFT>
__global__ void __launch_bounds__(BLOCK_THREADS) k_block(ModelDev md, LayerDev L, Work w, int M, int* error) {
  block_finish<LEFT, true>(md, L, w, M, error);
}
template <int LEFT>
__global__ void __launch_bounds__(BLOCK_THREADS, 3) k_block_lean(ModelDev md, LayerDev L, Work w, int M, int* error) {
  block_finish<LEFT, false>(md, L, w, M, error);
}

// ------------------------------------------------ block finish over a cluster
// For small passes the three Kronecker applications are split over a cluster
// of CL CTAs by output column: column c of K(x) = Lᵀ·(X·R) depends only on
// column c of R, so CTA q forms columns [q·W, (q+1)·W) of both products of
// every application (one row and two columns per thread, the same ordered
// sums), then stores its slice into every CTA's copy of the result through
// distributed shared memory, since the elementwise pass after an application
// permutes the whole vector. The norms, condition softmax, modulation and
// elementwise passes run in every CTA of the cluster; the last application
// and the lane combine stay split by column.
template <int LEFT>
struct BlockSplit {
  static constexpr int W = 2 * BLOCK_THREADS / LEFT;  // columns per CTA: LEFT rows × W/2 column pairs = 256 threads
  static constexpr int CL = HADA_RIGHT / W;           // CTAs per token: 4 (LEFT 64) or 2 (LEFT 32)
};

// Σ_s A[s][r]·B[s][c..c+1] over s ascending, from +0.0 (as tn_stage).
template <int S, int R, bool FUSED32>
__device__ __forceinline__ float2 col_pair(const float* __restrict__ A, const float* __restrict__ B, int bstride, int r, int c,
                                           float2 nz) {
  float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll 8
  for (int s = 0; s < S; ++s) {
    const float a = A[s * R + r];
    const float2 b = *reinterpret_cast<const float2*>(B + s * bstride + c);
    const float2 ai = make_float2(a, a);
    acc = FUSED32 ? fma2(ai, b, acc) : add2(acc, fma2(ai, b, nz));
  }
  return acc;
}

// The out product fused into the split block finish (a pass of at most
// GEMV_MAX_TOKENS tokens, d = 512, four CTAs per token): CTA q forms rows
// q·128 .. q·128+127 of the token's out product from the attention's int8
// activations, with k_gemv's lane layout and ordered per-group combine, and
// stores them into every CTA's s_a through distributed shared memory. Its
// weight slice (64 KB of codes, 2 KB of scales) is bulk-copied before the
// predecessor finishes.
constexpr int FUSED_OUT_ROWS = 128;
constexpr uint32_t FUSED_OUT_CODES = FUSED_OUT_ROWS * GEMM_K, FUSED_OUT_SCALES = FUSED_OUT_ROWS * (GEMM_K / GROUP) * 4;
template <typename F>
struct FusedOut {
  bool on;
  F f;
  __device__ bool fused() const { return on; }
  __device__ void operator()() const {
    if (on) f();
  }
};
__host__ __device__ constexpr size_t block_split_out_offset(size_t split_floats) { return (split_floats * 4 + 127) / 128 * 128; }

template <int LEFT>
__global__ void __launch_bounds__(BLOCK_THREADS) k_block_split(ModelDev md, LayerDev L, Work w, int M, int* error, int fuse_out,
                                                               int split_floats) {
  namespace cg = cooperative_groups;
  extern __shared__ float sm[];
  constexpr int N = LEFT * HADA_RIGHT, W = BlockSplit<LEFT>::W, CL = BlockSplit<LEFT>::CL;
  constexpr bool FUSED32 = LEFT == 32;
  cg::cluster_group cluster = cg::this_cluster();
  const int q = (int)cluster.block_rank(), t = blockIdx.x / CL;
  const int d = md.d_model, tid = threadIdx.x;
  const int cq = q * W;                                           // this CTA's first column
  const int r = tid / (W / 2), cl = 2 * (tid % (W / 2));          // this thread's row and column pair (within the slice)
  float* s_a = sm;                                                // d
  float* s_x = sm + MAX_D;                                        // d
  float* s_pre = sm + 2 * MAX_D;                                  // d
  float* xa = sm + 3 * MAX_D;                                     // N: first and third applications' input (transposed)
  float* xb = xa + N;                                             // N: the second's; then the third's slice of results
  float* f1 = xb + N;                                             // N: the first application's result, all columns
  float* f2 = f1 + N;                                             // N: the second's
  float* s_mod = f2 + N;                                          // N
  float* s_t = s_mod + N;                                         // LEFT × W: this CTA's columns of X·R
  float* s_left = s_t + LEFT * W;                                 // LEFT*LEFT
  float* s_right = s_left + LEFT * LEFT;                          // 32*32
  // cond_v borrows f2 and s_mod: both stay untouched until the condition
  // weights are formed (f2 is written by the cluster only after the first
  // application, which every CTA reaches after its own condition softmax)
  float* s_condv = d * COND_RANK <= 2 * N ? f2 : s_right + HADA_RIGHT * HADA_RIGHT;
  float* s_gpost = s_right + HADA_RIGHT * HADA_RIGHT + (d * COND_RANK <= 2 * N ? 0 : d * COND_RANK);
  float* s_gpre = s_gpost + MAX_D;
  const HadamardDev& Hd = L.hada;
  const float2 nz = g_negzero;

  // this CTA's elements of the lane combine: rows 0..d/32-1 of its columns;
  // their operands (from launches before the predecessor; d4) load first
  const int rows_d = d / HADA_RIGHT, own = rows_d * W;
  const int ei = (tid / W) * HADA_RIGHT + cq + tid % W;
  const float* route = w.route + (size_t)t * (LANES + LANES * LANES);
  float rw[LANES + LANES * LANES], sv[LANES], d4 = 0.0f;
#pragma unroll
  for (int k = 0; k < LANES + LANES * LANES; ++k) rw[k] = __ldcg(route + k);
  if (tid < own) {
    d4 = Hd.d4[ei];
#pragma unroll
    for (int s = 0; s < LANES; ++s) sv[s] = __ldcg(w.stream + ((size_t)t * LANES + s) * d + ei);
  }
  // the fused out product: this CTA's weight slice, copied while the predecessor runs
  uint8_t* s_wout = reinterpret_cast<uint8_t*>(sm) + block_split_out_offset((size_t)split_floats);
  const float* s_wsc = reinterpret_cast<const float*>(s_wout + FUSED_OUT_CODES);
  __shared__ __align__(8) uint64_t s_obar;
  __shared__ __align__(16) uint4 s_act4[GEMM_KC];
  __shared__ float s_as4[GEMM_K / GROUP];
  const uint32_t obar = smem_u32(&s_obar);
  const QMat& Wout = L.out;
  if (fuse_out && tid == 0) {
    bulk_start(obar, FUSED_OUT_CODES + FUSED_OUT_SCALES);
    const uint8_t* codes = reinterpret_cast<const uint8_t*>(Wout.codes) + (size_t)q * FUSED_OUT_CODES;
    for (uint32_t off = 0; off < FUSED_OUT_CODES; off += 16384) bulk_copy(s_wout + off, codes + off, 16384, obar);
    bulk_copy(s_wout + FUSED_OUT_CODES, Wout.scales + (size_t)q * FUSED_OUT_ROWS * (GEMM_K / GROUP), FUSED_OUT_SCALES, obar);
  }
  auto out_product = [&] {
    if (!mbar_wait(obar, 0) && tid == 0) atomicExch(error, 1);
    // the token's activations (the attention, this kernel's predecessor, wrote them)
    if (tid < GEMM_KC) s_act4[tid] = __ldcg(reinterpret_cast<const uint4*>(w.act + core_offset(t, tid * 16, GEMM_KC)));
    if (tid < GEMM_K / GROUP) s_as4[tid] = __ldcg(w.act_scale + (size_t)t * (GEMM_K / GROUP) + tid);
    cluster.sync();  // every CTA of the cluster runs (remote stores below); the row is visible to the block
    const int lane = tid & 31, warp = tid >> 5, r8 = lane & 7, qd = lane >> 3;
    for (int rb = warp; rb < FUSED_OUT_ROWS / 8; rb += BLOCK_THREADS / 32) {
      // lane: row r8 of the 8-row block, 16-byte chunks 4j + qd (k_gemv's layout)
      const uint4* blk = reinterpret_cast<const uint4*>(s_wout + (size_t)rb * 8 * GEMM_K);
      int acc[GEMM_K / GROUP] = {0, 0, 0, 0};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 wv = blk[j * 32 + lane], av = s_act4[4 * j + qd];
        const int g = j >> 1;
        acc[g] = dp4a(wv.x, av.x, acc[g]);
        acc[g] = dp4a(wv.y, av.y, acc[g]);
        acc[g] = dp4a(wv.z, av.z, acc[g]);
        acc[g] = dp4a(wv.w, av.w, acc[g]);
      }
#pragma unroll
      for (int g = 0; g < GEMM_K / GROUP; ++g) {
        acc[g] += __shfl_xor_sync(FULL, acc[g], 8);
        acc[g] += __shfl_xor_sync(FULL, acc[g], 16);
      }
      if (qd == 0) {
        const int row = rb * 8 + r8;
        float total = 0.0f;
#pragma unroll
        for (int g = 0; g < GEMM_K / GROUP; ++g) {
          const float a = group_sum_to_float((uint32_t)acc[g]), as = s_as4[g], wsc = s_wsc[row * (GEMM_K / GROUP) + g];
          total = Wout.fused ? __fmaf_rn(a, fmul(wsc, as), total) : fadd(total, fmul(fmul(fmul(a, wsc), Wout.level_scale), as));
        }
#pragma unroll
        for (int p = 0; p < CL; ++p) *cluster.map_shared_rank(s_a + q * FUSED_OUT_ROWS + row, p) = total;
      }
    }
    cluster.sync();  // s_a is whole in every CTA
  };
  const FusedOut<decltype(out_product)> fused{fuse_out != 0, out_product};
  if (!block_front<LEFT, 1>(md, L, w, M, t, d, error, s_a, s_x, s_pre, s_condv, s_left, s_right, s_gpost, s_gpre, q, CL, fused)) {
    if (fuse_out && tid == 0 && !mbar_wait(obar, 0)) atomicExch(error, 1);  // no copy outlives the CTA
    return;
  }
  cluster_arrive_relaxed();  // paired with the wait before the first remote store
  __syncthreads();
  hada_prepare<LEFT>(Hd, d, s_pre, xa, s_mod, s_condv);
  HadaPass1<LEFT> pass1;
  pass1.load(md, Hd);

  // application 1: this CTA's columns, then every CTA's copy of f1
  float2 v;
  *reinterpret_cast<float2*>(s_t + r * W + cl) = col_pair<HADA_RIGHT, LEFT, FUSED32>(xa, s_right + cq, HADA_RIGHT, r, cl, nz);
  __syncthreads();
  v = col_pair<LEFT, LEFT, FUSED32>(s_left, s_t, W, r, cl, nz);
  cluster_wait();  // every CTA of the cluster runs: distributed shared memory is usable
#pragma unroll
  for (int p = 0; p < CL; ++p) *reinterpret_cast<float2*>(cluster.map_shared_rank(f1 + r * HADA_RIGHT + cq + cl, p)) = v;
  cluster.sync();  // f1 is whole in every CTA; every local read of s_left and s_right is done
  stage_async(s_left, Hd.left[1], LEFT * LEFT);
  stage_async(s_right, Hd.right[1], HADA_RIGHT * HADA_RIGHT);
  pass1.run(s_mod, f1, xb);
  HadaPass2<LEFT> pass2;
  pass2.load(md, Hd);
  cp_async_wait_all();
  __syncthreads();

  // application 2
  *reinterpret_cast<float2*>(s_t + r * W + cl) = col_pair<HADA_RIGHT, LEFT, FUSED32>(xb, s_right + cq, HADA_RIGHT, r, cl, nz);
  __syncthreads();
  v = col_pair<LEFT, LEFT, FUSED32>(s_left, s_t, W, r, cl, nz);
#pragma unroll
  for (int p = 0; p < CL; ++p) *reinterpret_cast<float2*>(cluster.map_shared_rank(f2 + r * HADA_RIGHT + cq + cl, p)) = v;
  cluster.sync();  // f2 is whole; no remote access follows, so CTAs may leave independently
  stage_async(s_left, Hd.left[2], LEFT * LEFT);
  stage_async(s_right, Hd.right[2], HADA_RIGHT * HADA_RIGHT);
  pass2.run(f2, xa);
  cp_async_wait_all();
  __syncthreads();

  // application 3: only the rows that hold the d outputs, kept in this CTA
  *reinterpret_cast<float2*>(s_t + r * W + cl) = col_pair<HADA_RIGHT, LEFT, FUSED32>(xa, s_right + cq, HADA_RIGHT, r, cl, nz);
  __syncthreads();
  if (r < rows_d) *reinterpret_cast<float2*>(xb + r * HADA_RIGHT + cq + cl) = col_pair<LEFT, LEFT, FUSED32>(s_left, s_t, W, r, cl, nz);
  __syncthreads();
  pdl_trigger();  // the lane combine overlaps the next kernel's prologue
  if (tid < own) {
    const float input = L.engram_site >= 0 ? __ldcg(w.xin + (size_t)t * d + ei) : s_x[ei];
    const float delta = fsub(fadd(s_a[ei], fmul(xb[ei], d4)), input);
    float* next = w.next_stream + (size_t)t * LANES * d;
#pragma unroll
    for (int l = 0; l < LANES; ++l) next[l * d + ei] = lane_out(rw, sv, l, delta);
  }
}

// ------------------------------------------------------------------- final
// lane_mean (session.rs:192-200) and the final zero-centred norm into the
// sequence's hidden state, for the last token of each sequence. grid M, block 128.
__global__ void __launch_bounds__(128) k_final(ModelDev md, Work w, float* __restrict__ hidden, int M) {
  pdl_wait();
  __shared__ __align__(16) float s_mean[MAX_D];
  __shared__ float s_inv;
  const int t = blockIdx.x;
  if (t >= M) return;
  const TokenMeta meta = w.meta[t];
  if (meta.slot < 0) return;
  if (md.token_ring && threadIdx.x == 0) {
    // the last token_rows token ids of each sequence in the pass join its token ring
    const int R = (int)md.token_rows;
    bool newest = true;
    if (t + R < M) {
      const TokenMeta o = w.meta[t + R];
      newest = !(o.slot == meta.slot && o.position == meta.position + R);
    }
    if (newest) md.token_ring[(size_t)meta.slot * R + meta.position % R] = w.tokens[t];
  }
  if (!meta.last) return;
  const int d = md.d_model, tid = threadIdx.x;
  const float* stream = w.stream + (size_t)t * LANES * d;
  for (int i4 = tid; i4 < d / 4; i4 += blockDim.x) {
    float4 s[LANES];
#pragma unroll
    for (int l = 0; l < LANES; ++l) s[l] = reinterpret_cast<const float4*>(stream + l * d)[i4];
    float m[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float acc = 0.0f;
#pragma unroll
      for (int l = 0; l < LANES; ++l) acc = fadd(acc, fdiv((&s[l].x)[e], (float)LANES));
      m[e] = acc;
    }
    reinterpret_cast<float4*>(s_mean)[i4] = make_float4(m[0], m[1], m[2], m[3]);
  }
  __syncthreads();
  if (tid < 32) {
    float ss = sum_of_squares_warp(s_mean, d);
    if (tid == 0) s_inv = inverse_rms(ss, d);
  }
  __syncthreads();
  for (int i = tid; i < d; i += blockDim.x) hidden[(size_t)meta.slot * d + i] = fmul(fmul(fadd(1.0f, md.final_norm[i]), s_mean[i]), s_inv);
}

// -------------------------------------------------------------- probe heads
// ProbeHead::observe (heads.rs:127-148) of one cell row (0: the embedding,
// layer + 1: after that layer) for every token of the pass. grid M, block 128.
// Each CTA forms its token's cell (lane_mean, session.rs:192-200) and its
// scores dot(cell, direction) / sqrt(d) for every head and probe; the last
// CTA of a sequence's run to arrive (a counter per run: fence, then atomic)
// then runs the online softmax over the run's tokens in position order:
// peak' = max(peak, score), rescale = exp(peak - peak') (0 while peak is
// -inf), weight = exp(score - peak'), total = total·rescale + weight,
// weighted = weighted·rescale + weight·cell, each product separately
// rounded, exp the libm one.
__global__ void __launch_bounds__(128) k_observe(ModelDev md, Work w, const float* __restrict__ stream, int M, int row) {
  __shared__ __align__(16) float s_cell[MAX_D];
  __shared__ int s_final;
  pdl_wait();
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, d = (int)md.d_model;
  if (t >= M) return;
  const TokenMeta meta = load_meta(w.meta, t);
  if (meta.slot < 0) return;
  const float* lanes_t = stream + (size_t)t * LANES * d;
  for (int i = tid; i < d; i += blockDim.x) {
    float acc = 0.0f;
#pragma unroll
    for (int l = 0; l < LANES; ++l) acc = fadd(acc, fdiv(__ldcg(lanes_t + l * d + i), (float)LANES));
    s_cell[i] = acc;
    w.cells[(size_t)t * d + i] = acc;
  }
  __syncthreads();
  int pairs = 0;
  for (uint32_t h = 0; h < md.num_probe_heads; ++h) pairs += (int)md.probe_heads[h].probes;
  const float root = md.sqrt_d;
  for (int p = warp; p < pairs; p += blockDim.x >> 5) {
    int h = 0, k = p;
    while (k >= (int)md.probe_heads[h].probes) k -= (int)md.probe_heads[h++].probes;
    const HeadDev& H = md.probe_heads[h];
    const float dot = dot_product_warp(s_cell, H.directions + ((size_t)row * H.probes + k) * d, d);
    if (lane == 0) w.scores[(size_t)t * pairs + p] = fdiv(dot, root);
  }
  const int run = meta.run & 0xffff, len = meta.run >> 16, first = t - run;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_final = atomicAdd(&w.arrivals[first], 1) == len - 1;
  __syncthreads();
  if (!s_final) return;
  __threadfence();
  // the scalar recurrence per (head, probe), token by token
  for (int p = tid; p < pairs; p += blockDim.x) {
    int h = 0, k = p;
    while (k >= (int)md.probe_heads[h].probes) k -= (int)md.probe_heads[h++].probes;
    const HeadDev& H = md.probe_heads[h];
    const size_t slot = (size_t)meta.slot * (md.num_layers + 1) * H.probes + (size_t)row * H.probes + k;
    float peak = H.peak[slot], total = H.total[slot];
    for (int r = 0; r < len; ++r) {
      const float score = __ldcg(w.scores + (size_t)(first + r) * pairs + p);
      const float next = fmaxf(peak, score);
      const float rescale = peak == -INFINITY ? 0.0f : expf_libm(fsub(peak, next));
      const float weight = expf_libm(fsub(score, next));
      total = fadd(fmul(total, rescale), weight);
      w.scan[((size_t)(first + r) * pairs + p) * 2] = rescale;
      w.scan[((size_t)(first + r) * pairs + p) * 2 + 1] = weight;
      peak = next;
    }
    H.peak[slot] = peak;
    H.total[slot] = total;
  }
  __syncthreads();
  // the weighted cells, element by element, token by token
  for (int e = tid; e < pairs * d; e += blockDim.x) {
    const int p = e / d, i = e % d;
    int h = 0, k = p;
    while (k >= (int)md.probe_heads[h].probes) k -= (int)md.probe_heads[h++].probes;
    const HeadDev& H = md.probe_heads[h];
    float* target = H.weighted + ((size_t)meta.slot * (md.num_layers + 1) * H.probes + (size_t)row * H.probes + k) * d + i;
    float v = *target;
    for (int r = 0; r < len; ++r) {
      const float* rw = w.scan + ((size_t)(first + r) * pairs + p) * 2;
      v = fadd(fmul(v, rw[0]), fmul(rw[1], __ldcg(w.cells + (size_t)(first + r) * d + i)));
    }
    *target = v;
  }
  if (tid == 0) w.arrivals[first] = 0;  // ready for the next use
}

// ProbeHead::pooled (heads.rs:85-115) of one session's head h over the model's
// rows (the embedding cell and its active layers): readouts unit_rms(weighted
// / total) · gain into `readouts`, then per query the softmax (ops.rs:92-101)
// of dot(readout, query) / sqrt(d) + row bias over the slots, and the
// weighted sum of the readouts in slot order into `pooled`. One CTA of 256.
__global__ void __launch_bounds__(256) k_head_pool(ModelDev md, int h, int slot, const int32_t* __restrict__ rows, int nrows,
                                                   float* __restrict__ readouts, float* __restrict__ weights, float* __restrict__ pooled) {
  const HeadDev& H = md.probe_heads[h];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, d = (int)md.d_model, P = (int)H.probes, slots = nrows * P;
  const int all = (int)(md.num_layers + 1) * P;
  const size_t base = (size_t)slot * all;
  // readouts: averaged = weighted · (1 / total), then unit_rms and the gain
  for (int s = warp; s < slots; s += 8) {
    const int a = rows[s / P] * P + s % P;
    const float inverse = fdiv(1.0f, H.total[base + a]);
    float* out = readouts + (size_t)s * d;
    for (int i = lane; i < d; i += 32) out[i] = fmul(H.weighted[(base + a) * d + i], inverse);
    __syncwarp();
    const float inv = inverse_rms(sum_of_squares_warp(out, d), d);
    const float gain = H.gain[a];
    for (int i = lane; i < d; i += 32) out[i] = fmul(fmul(out[i], inv), gain);
  }
  __syncthreads();
  for (int q = 0; q < (int)H.queries; ++q) {
    for (int s = warp; s < slots; s += 8) {
      const float dot = dot_product_warp(readouts + (size_t)s * d, H.query + (size_t)q * d, d);
      if (lane == 0) weights[s] = fadd(fdiv(dot, md.sqrt_d), H.row_bias[(size_t)q * all + rows[s / P] * P + s % P]);
    }
    __syncthreads();
    if (tid == 0) {  // softmax_in_place: peak, fast_exp and the total in order, then 1 / total
      float peak = -INFINITY;
      for (int s = 0; s < slots; ++s) peak = fmaxf(peak, weights[s]);
      float total = 0.0f;
      for (int s = 0; s < slots; ++s) {
        weights[s] = fast_exp(fsub(weights[s], peak));
        total = fadd(total, weights[s]);
      }
      const float inverse = fdiv(1.0f, total);
      for (int s = 0; s < slots; ++s) weights[s] = fmul(weights[s], inverse);
    }
    __syncthreads();
    for (int i = tid; i < d; i += blockDim.x) {
      float acc = 0.0f;
      for (int s = 0; s < slots; ++s) acc = fadd(acc, fmul(weights[s], readouts[(size_t)s * d + i]));
      pooled[(size_t)q * d + i] = acc;
    }
    __syncthreads();
  }
}

// out[i] += bias[i] (heads.rs:121-123). One CTA.
__global__ void k_add_bias(float* __restrict__ out, const float* __restrict__ bias, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = fadd(out[i], bias[i]);
}

// dense() (heads.rs:20-28): rows of a codebook matrix dequantised to f32 like
// QuantisedMatrix::dequantise_row (matrix.rs:140-153). grid rows, block 128.
__global__ void __launch_bounds__(128) k_dense_rows(const uint8_t* __restrict__ packed, uint32_t row_bytes, uint32_t bits,
                                                    const float* __restrict__ levels, const float* __restrict__ norms, int cols,
                                                    float inv_sqrt_group, float* __restrict__ out) {
  const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, groups = cols / GROUP;
  const uint8_t* row = packed + (size_t)r * row_bytes;
  for (int g = warp; g < groups; g += 4) {
    const float norm = norms[(size_t)r * groups + g];
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = fmul(levels[code_at(row, g * GROUP + 4 * lane + j, bits)], norm);
    fwht128(v, inv_sqrt_group);
    *reinterpret_cast<float4*>(out + (size_t)r * cols + g * GROUP + 4 * lane) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

__global__ void k_fill(float* __restrict__ p, size_t n, float value) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = value;
}

// ------------------------------------------------- Whistle cross attention
// A 64-value head held by a warp (lane: elements lane, lane + 32):
// zero_centred_norm_in_place (ops.rs:52-58; the square sum in the reference's
// eight-lane order), then quantise_int8 (ops.rs:112-118) into c0, c1; returns
// the scale.
__device__ __forceinline__ float norm_quant_head64(float e0, float e1, const float* gain, bool norm, int8_t& c0, int8_t& c1) {
  const int lane = threadIdx.x & 31;
  if (norm) {
    float acc = 0.0f;
    const int chain = lane & 7;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float v = __shfl_sync(FULL, e0, chain + 8 * c);
      acc = fadd(acc, fmul(v, v));
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float v = __shfl_sync(FULL, e1, chain + 8 * c);
      acc = fadd(acc, fmul(v, v));
    }
    float s = SUM_START;
#pragma unroll
    for (int l = 0; l < 8; ++l) s = fadd(s, __shfl_sync(FULL, acc, l));
    const float inv = inverse_rms(s, HEAD_DIM);
    e0 = fmul(fmul(fadd(1.0f, gain[lane]), e0), inv);
    e1 = fmul(fmul(fadd(1.0f, gain[lane + 32]), e1), inv);
  }
  const float peak = warp_max(fmaxf(fabsf(e0), fabsf(e1)));
  const float scale = int8_scale_of(peak);
  c0 = (int8_t)clampf(rintf(fdiv(e0, scale)), -128.0f, 127.0f);
  c1 = (int8_t)clampf(rintf(fdiv(e1, scale)), -128.0f, 127.0f);
  return scale;
}

// An int8 as f32, exactly, on the FP32 pipe: 2^23 + (v + 128) is an f32 whose
// low mantissa bits hold v + 128, and subtracting 2^23 + 128 is exact.
__device__ __forceinline__ float int8_to_float(int8_t v) {
  return fsub(__int_as_float(0x4B000000 | (int)(v + 128)), 8388736.0f);
}

// CrossWeights::memory, first step (cross.rs:64-74): row t of the encoder
// output plus the gated positional signal (sin in the first half, cos in the
// second; the angles' sin and cos come as tables). grid frames, block 128.
__global__ void __launch_bounds__(128) k_cross_memory_in(const float* __restrict__ encoded, const float* __restrict__ sin_tab,
                                                         const float* __restrict__ cos_tab, float gate, int d, float* __restrict__ out) {
  const int t = blockIdx.x, half = d / 2;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    out[(size_t)t * d + j] = fadd(encoded[(size_t)t * d + j], fmul(gate, sin_tab[(size_t)t * half + j]));
    out[(size_t)t * d + half + j] = fadd(encoded[(size_t)t * d + half + j], fmul(gate, cos_tab[(size_t)t * half + j]));
  }
}

// CrossWeights::memory, last step (cross.rs:83-96): per (frame, head) the key
// normed with k_norm and quantised, the value quantised. kv: [frames][2d]
// (keys, then values). Stored head-major, [head][frame][64] and [head][frame],
// so that one head's rows are one contiguous block. grid frames, block
// 64 · heads (a warp per head and side).
__global__ void k_cross_memory_heads(const float* __restrict__ kv, int d, int frames, const float* __restrict__ k_norm,
                                     int8_t* __restrict__ keys, float* __restrict__ kscale, int8_t* __restrict__ values,
                                     float* __restrict__ vscale) {
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, heads = d / HEAD_DIM;
  const bool key = warp < heads;
  const int h = key ? warp : warp - heads;
  const float* src = kv + (size_t)t * 2 * d + (key ? 0 : d) + h * HEAD_DIM;
  int8_t c0, c1;
  const float scale = norm_quant_head64(src[lane], src[lane + 32], k_norm, key, c0, c1);
  int8_t* codes = (key ? keys : values) + ((size_t)h * frames + t) * HEAD_DIM;
  codes[lane] = c0;
  codes[lane + 32] = c1;
  if (lane == 0) (key ? kscale : vscale)[(size_t)h * frames + t] = scale;
}

// x after the layer's attention residual (session.rs:121-125, as the block
// finish forms it) into w.xr for every token, then for the tokens of sessions
// with a cross memory CrossState::apply's first step (cross.rs:121-130):
// zero_centred_norm with the layer's cross norm, fake_quantise_int8 and the
// q|gate product's activation step. grid M, block 128.
__global__ void __launch_bounds__(128) k_cross_q(ModelDev md, LayerDev L, int layer, Work w, int M) {
  __shared__ __align__(16) float s_v[PREP_MAX_K];
  __shared__ float s_red[4];
  __shared__ float s_inv;
  pdl_wait();
  const int t = blockIdx.x, d = (int)md.d_model;
  if (t >= M) return;
  const TokenMeta meta = load_meta(w.meta, t);
  if (meta.slot < 0) return;
  for (int i = threadIdx.x; i < d; i += blockDim.x) s_v[i] = __ldcg(w.outp + (size_t)t * d + i);
  __syncthreads();
  if (threadIdx.x < 32) {
    const float ss = sum_of_squares_warp(s_v, d);
    if (threadIdx.x == 0) s_inv = inverse_rms(ss, d);
  }
  __syncthreads();
  const float gate = sigmoid(L.attn_gate), inv_a = s_inv;
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float a = fmul(fmul(fadd(1.0f, L.post_norm[i]), s_v[i]), inv_a);
    const float x = fadd(__ldcg(w.x + (size_t)t * d + i), fmul(gate, a));
    s_v[i] = x;
    w.xr[(size_t)t * d + i] = x;
  }
  if (!md.slot_cross[meta.slot]) return;  // no cross attention for this session (the whole block agrees)
  const CrossLayerDev& C = md.cross[layer];
  __syncthreads();
  if (threadIdx.x < 32) {
    const float ss = sum_of_squares_warp(s_v, d);
    if (threadIdx.x == 0) s_inv = inverse_rms(ss, d);
  }
  __syncthreads();
  float* normed = w.attn + (size_t)t * md.heads * HEAD_DIM;  // free here: the attention rows are consumed
  for (int i = threadIdx.x; i < d; i += blockDim.x) normed[i] = fmul(fmul(fadd(1.0f, C.norm[i]), s_v[i]), s_inv);
  __syncthreads();
  prep_token(normed, nullptr, d, w.act, w.act_scale, t, md.inv_sqrt_group, 1, 0, s_v, s_red);
}

// CrossState::apply, per head (cross.rs:131-163): the query normed with q_norm
// and quantised; int8 scores over the memory's frames, dot · key_scale ·
// query_scale; softmax_in_place (peak, fast_exp, one ordered total from +0.0,
// times 1 / total); the context Σ_frame (value_scale · weight) · code in frame
// order per dimension; times sigmoid(gate) (cross.rs:164-166) into the rows of
// w.attn. grid (M, heads), block 256.
constexpr int CROSS_THREADS = 256;
constexpr int CROSS_CHUNK = 128;   // frames per staged value tile (8 KB)
constexpr int CROSS_BUFFERS = 4;   // value tiles in shared memory (three in flight)
__global__ void __launch_bounds__(CROSS_THREADS) k_cross_attend(ModelDev md, int layer, Work w, int M) {
  extern __shared__ float s_sc[];  // [MAX_CROSS_FRAMES] scores, then weights; [MAX_CROSS_FRAMES] value scale · weight
  float* s_vw = s_sc + MAX_CROSS_FRAMES;
  __shared__ __align__(16) int8_t s_q[HEAD_DIM];
  __shared__ float s_qs, s_red[CROSS_THREADS / 32], s_peak, s_inverse;
  pdl_wait();
  const int t = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (t >= M) return;
  const TokenMeta meta = load_meta(w.meta, t);
  if (meta.slot < 0) return;
  const CrossMemDev* mem = md.slot_cross[meta.slot];
  if (!mem) return;
  const CrossLayerDev& C = md.cross[layer];
  const int d = (int)md.d_model, heads = (int)md.heads, frames = mem->frames;
  const int8_t* keys = mem->keys + (size_t)layer * frames * heads * HEAD_DIM;
  const float* kscale = mem->kscale + (size_t)layer * frames * heads;
  const int8_t* values = mem->values + (size_t)layer * frames * heads * HEAD_DIM;
  const float* vscale = mem->vscale + (size_t)layer * frames * heads;
  // the value rows of this head pass through CROSS_BUFFERS shared tiles of
  // CROSS_CHUNK frames (16-byte copies by every thread), CROSS_BUFFERS - 1
  // ahead: they do not depend on the softmax, so the first ones load now
  __shared__ __align__(16) int8_t s_val[CROSS_BUFFERS][CROSS_CHUNK * HEAD_DIM];
  const int8_t* vbase = values + (size_t)h * frames * HEAD_DIM;  // this head's rows, contiguous
  const size_t vstride = HEAD_DIM;
  auto stage = [&](int chunk) {  // commits one group, empty past the last chunk
    const int f0 = chunk * CROSS_CHUNK, n = min(CROSS_CHUNK, frames - f0);
    for (int i = tid; i < n * (HEAD_DIM / 16); i += CROSS_THREADS) {
      const int f = i / (HEAD_DIM / 16), part = i % (HEAD_DIM / 16);
      cp_async16(&s_val[chunk % CROSS_BUFFERS][f * HEAD_DIM + part * 16], vbase + (size_t)(f0 + f) * vstride + part * 16);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
#pragma unroll
  for (int c = 0; c < CROSS_BUFFERS - 1; ++c) stage(c);
  if (warp == 0) {
    const float* q = w.cq + (size_t)t * 2 * d + h * HEAD_DIM;
    int8_t c0, c1;
    const float scale = norm_quant_head64(__ldcg(q + lane), __ldcg(q + lane + 32), C.q_norm, true, c0, c1);
    s_q[lane] = c0;
    s_q[lane + 32] = c1;
    if (lane == 0) s_qs = fmul(scale, md.inv_root_qk);
  }
  __syncthreads();
  // the scores: four lanes per frame, each with 16 bytes of the key row (a
  // warp reads eight whole rows per load), the exact int32 dot summed over
  // the quad; each warp takes 8 frames per round, eight rounds in flight
  float peak = -INFINITY;
  const int quarter = lane & 3;
  const uint4 qq = reinterpret_cast<const uint4*>(s_q)[quarter];
  constexpr int ROUND = CROSS_THREADS / 4, DEPTH = 8;
  for (int base = warp * 8; base < frames; base += ROUND * DEPTH) {  // uniform per warp
    uint4 kk[DEPTH];
#pragma unroll
    for (int u = 0; u < DEPTH; ++u) {
      const int f = min(base + u * ROUND + (lane >> 2), frames - 1);
      kk[u] = reinterpret_cast<const uint4*>(keys + ((size_t)h * frames + f) * HEAD_DIM)[quarter];
    }
#pragma unroll
    for (int u = 0; u < DEPTH; ++u) {
      int dot = dp4a(kk[u].x, qq.x, 0);
      dot = dp4a(kk[u].y, qq.y, dot);
      dot = dp4a(kk[u].z, qq.z, dot);
      dot = dp4a(kk[u].w, qq.w, dot);
      dot += __shfl_xor_sync(FULL, dot, 1);
      dot += __shfl_xor_sync(FULL, dot, 2);
      const int f = base + u * ROUND + (lane >> 2);
      if (quarter == 0 && f < frames) {
        const float sc = fmul(fmul((float)dot, kscale[(size_t)h * frames + f]), s_qs);
        s_sc[f] = sc;
        peak = fmaxf(peak, sc);
      }
    }
  }
  peak = warp_max(peak);
  if (lane == 0) s_red[warp] = peak;
  __syncthreads();
  if (tid == 0) {
    float m = s_red[0];
    for (int k = 1; k < CROSS_THREADS / 32; ++k) m = fmaxf(m, s_red[k]);
    s_peak = m;
  }
  __syncthreads();
  for (int f = tid; f < frames; f += CROSS_THREADS) s_sc[f] = fast_exp(fsub(s_sc[f], s_peak));
  __syncthreads();
  if (warp == 0) {  // the total, one chain in frame order from +0.0 (ops.rs:92-101)
    float total = 0.0f;
    if (lane == 0) {
      int f = 0;
      for (; f + 16 <= frames; f += 16) {
        float v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = s_sc[f + k];
#pragma unroll
        for (int k = 0; k < 16; ++k) total = fadd(total, v[k]);
      }
      for (; f < frames; ++f) total = fadd(total, s_sc[f]);
      s_inverse = fdiv(1.0f, total);
    }
  }
  __syncthreads();
  for (int f = tid; f < frames; f += CROSS_THREADS) s_vw[f] = fmul(vscale[(size_t)h * frames + f], fmul(s_sc[f], s_inverse));
  pdl_trigger();
  // thread d < 64 runs dimension d's ordered sum over the frames
  const int chunks = (frames + CROSS_CHUNK - 1) / CROSS_CHUNK;
  float acc = 0.0f;
  for (int c = 0; c < chunks; ++c) {
    stage(c + CROSS_BUFFERS - 1);  // into the buffer chunk c - 1 has freed
    asm volatile("cp.async.wait_group %0;" ::"n"(CROSS_BUFFERS - 1) : "memory");
    __syncthreads();  // chunk c is in place (and, at c = 0, every s_vw entry)
    if (tid < HEAD_DIM) {
      const int f0 = c * CROSS_CHUNK, n = min(CROSS_CHUNK, frames - f0);
      const int8_t* col = &s_val[c % CROSS_BUFFERS][tid];
#pragma unroll 8
      for (int f = 0; f < n; ++f) acc = fadd(acc, fmul(s_vw[f0 + f], int8_to_float(col[f * HEAD_DIM])));
    }
    __syncthreads();  // buffer c % CROSS_BUFFERS is free for chunk c + CROSS_BUFFERS
  }
  if (tid < HEAD_DIM) {
    const float g = __ldcg(w.cq + (size_t)t * 2 * d + d + h * HEAD_DIM + tid);
    w.attn[(size_t)t * heads * HEAD_DIM + h * HEAD_DIM + tid] = fmul(acc, sigmoid(g));
  }
}

// ------------------------------------------------------------------ select
// argmax / argmax_allowed (generator.rs:147-165): the first index holding the
// maximum over the allowed ids, or over all ids when none is allowed.
// grid B, block 256; each thread keeps its 32 logits (8 float4) in registers.
constexpr int SELECT_CHUNKS = 8;

__global__ void __launch_bounds__(256) k_select(const float* __restrict__ logits, int V, const uint32_t* __restrict__ mask,
                                                const int32_t* __restrict__ active, uint32_t* __restrict__ next,
                                                float* __restrict__ peaks) {
  pdl_wait();
  __shared__ float s_red[8];
  __shared__ int s_idx[8];
  __shared__ int s_any[8];
  const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (active && active[b] == 0) {
    if (tid == 0) next[b] = 0xffffffffu;
    return;
  }
  const float4* v4 = reinterpret_cast<const float4*>(logits + (size_t)b * V);
  const uint32_t* m = mask ? mask + (size_t)b * (V / 32) : nullptr;
  float4 val[SELECT_CHUNKS];
  uint32_t bits[SELECT_CHUNKS];
#pragma unroll
  for (int c = 0; c < SELECT_CHUNKS; ++c) {
    const int i4 = c * blockDim.x + tid;
    const bool in = i4 < V / 4;
    val[c] = in ? v4[i4] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    bits[c] = in ? (m ? (m[i4 >> 3] >> ((i4 & 7) * 4)) & 15u : 15u) : 0u;
  }
  float pk_all = -INFINITY, pk_allowed = -INFINITY;
  int any = 0;
#pragma unroll
  for (int c = 0; c < SELECT_CHUNKS; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x = (&val[c].x)[e];
      pk_all = fmaxf(pk_all, x);
      if ((bits[c] >> e) & 1u) {
        pk_allowed = fmaxf(pk_allowed, x);
        any = 1;
      }
    }
  any = __any_sync(FULL, any);
  if (lane == 0) s_any[warp] = any;
  const float all = block_max(pk_all, s_red);
  const float allowed = block_max(pk_allowed, s_red);
  int anyb = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) anyb |= s_any[i];
  const bool restricted = m && anyb;
  const float target = restricted ? allowed : all;
  int best = 0x7fffffff;
#pragma unroll
  for (int c = 0; c < SELECT_CHUNKS; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * (c * (int)blockDim.x + tid) + e;
      const bool ok = restricted ? ((bits[c] >> e) & 1u) : (i < V);
      if (ok && (&val[c].x)[e] == target) best = min(best, i);
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
  pdl_wait();
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
  pdl_wait();
  int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B || meta[b].slot < 0) return;
  meta[b].position += 1;
}

// -------------------------------------------------------------------- host
void set_exp_constants(const nbx::ExpConstants& constants, const nbx::ExceptionSet& exceptions, cudaStream_t stream) {
  cudaMemcpyToSymbolAsync(c_exp, &constants, sizeof constants, 0, cudaMemcpyHostToDevice, stream);
  cudaMemcpyToSymbolAsync(g_exp_table, constants.table, sizeof constants.table, 0, cudaMemcpyHostToDevice, stream);
  cudaMemcpyToSymbolAsync(c_exceptions, &exceptions, sizeof exceptions, 0, cudaMemcpyHostToDevice, stream);
}

size_t route_smem(const ModelDev& md, bool lean = false) { return route_floats((int)md.d_model, lean) * 4; }
size_t attend_smem(const ModelDev& md, int t_cap, int workers = ATT_WORKERS) {
  int G = md.heads / md.kv_heads;
  return (size_t)(G + 1) * t_cap * 4 + 2 * (size_t)G * att_wstride(t_cap) * 4 + (size_t)(workers / 16) * G * HEAD_DIM * 4;
}
size_t block_smem(const ModelDev& md, int factors = 3) {
  int N = md.hada_left * HADA_RIGHT;
  size_t floats = 3 * MAX_D + 3 * N + factors * (md.hada_left * md.hada_left + HADA_RIGHT * HADA_RIGHT) + 2 * MAX_D;
  if ((int)md.d_model * COND_RANK > 2 * N) floats += (size_t)md.d_model * COND_RANK;
  return floats * 4;
}
size_t block_split_smem(const ModelDev& md) {
  const int left = md.hada_left, N = left * HADA_RIGHT, W = 2 * BLOCK_THREADS / left;
  size_t floats = 3 * MAX_D + 5 * N + left * W + left * left + HADA_RIGHT * HADA_RIGHT + 2 * MAX_D;
  if ((int)md.d_model * COND_RANK > 2 * N) floats += (size_t)md.d_model * COND_RANK;
  return floats * 4;
}

// The dynamic shared memory a kernel may take is an attribute of the
// function in the device's context, shared by every model open in the
// process; a model that needs less (a shorter max_seq_len, a narrower d) must
// not lower what an earlier one set. So the attribute only grows, per device
// and kernel, to the most any open model needs.
static std::mutex g_smem_mutex;
static std::map<std::pair<int, const void*>, int> g_smem_allowed;

template <typename K>
static cudaError_t allow_smem(K* kernel, int bytes) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_smem_mutex);
  int& allowed = g_smem_allowed[{device, reinterpret_cast<const void*>(kernel)}];
  if (bytes <= allowed) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) allowed = bytes;
  return e;
}

template <int G, int EPI>
static cudaError_t attend_attributes(int smem) {
  cudaError_t e = allow_smem(k_attend<G, EPI, false, ATT_WORKERS>, smem);
  if (!e) e = allow_smem(k_attend<G, EPI, true, ATT_WORKERS>, smem);
  if constexpr (G <= 2) {
    if (!e) e = allow_smem(k_attend<G, EPI, false, ATT_WORKERS_NARROW>, smem);
    if (!e) e = allow_smem(k_attend<G, EPI, true, ATT_WORKERS_NARROW>, smem);
    const int wide = smem - (ATT_WORKERS / 16) * G * HEAD_DIM * 4 + (ATT_WORKERS_WIDE / 16) * G * HEAD_DIM * 4;
    if (!e) e = allow_smem(k_attend<G, EPI, false, ATT_WORKERS_WIDE>, wide);
    if (!e) e = allow_smem(k_attend<G, EPI, true, ATT_WORKERS_WIDE>, wide);
  }
  return e;
}

cudaError_t configure(const ModelDev& md, int t_cap) {
  cudaError_t e;
  if ((e = allow_smem(k_route<false>, (int)route_smem(md)))) return e;
  if ((e = allow_smem(k_route<true>, (int)route_smem(md, true)))) return e;
  const int att_smem = (int)attend_smem(md, t_cap);
  if ((e = attend_attributes<1, ATT_ROWS>(att_smem)) || (e = attend_attributes<1, ATT_LAST>(att_smem)) ||
      (e = attend_attributes<2, ATT_ROWS>(att_smem)) || (e = attend_attributes<2, ATT_CLUSTER>(att_smem)) ||
      (e = attend_attributes<2, ATT_LAST>(att_smem)) || (e = attend_attributes<4, ATT_ROWS>(att_smem)) ||
      (e = attend_attributes<4, ATT_CLUSTER>(att_smem)) || (e = attend_attributes<4, ATT_LAST>(att_smem)))
    return e;
  if ((e = allow_smem(k_block<64>, (int)block_smem(md)))) return e;
  if ((e = allow_smem(k_block<32>, (int)block_smem(md)))) return e;
  if ((e = allow_smem(k_block_lean<64>, (int)block_smem(md, 1)))) return e;
  if ((e = allow_smem(k_block_lean<32>, (int)block_smem(md, 1)))) return e;
  const int split_max = (int)(block_split_out_offset(block_split_smem(md) / 4) + FUSED_OUT_CODES + FUSED_OUT_SCALES);
  if ((e = allow_smem(k_block_split<64>, split_max))) return e;
  if ((e = allow_smem(k_block_split<32>, split_max))) return e;
  if ((e = allow_smem(k_stats, 2 * 8192 * 4))) return e;
  if ((e = allow_smem(k_cross_attend, 2 * MAX_CROSS_FRAMES * 4))) return e;
  if ((e = allow_smem(k_gemm<16, 1>, (int)gemm_smem<16>()))) return e;
  if ((e = allow_smem(k_gemm<32, 1>, (int)gemm_smem<32>()))) return e;
  if ((e = allow_smem(k_gemm<16, 4>, (int)gemm_smem<16>()))) return e;
  if ((e = allow_smem(k_gemm<32, 4>, (int)gemm_smem<32>()))) return e;
  if ((e = allow_smem(k_gemm_wide, (int)wide_smem()))) return e;

  return cudaSuccess;
}


// Every kernel of a pass launches with programmatic stream serialisation:
// its prologue (constant weight loads, tensor-memory allocation) overlaps the
// tail of its predecessor; see pdl_wait in device.cuh. On B200 this pays at
// every pass size (decode batches of 1..256, prefill passes of 1024 tokens).
// $NEEDLE_B200_PDL=0 turns the overlap off; $NEEDLE_B200_PDL_TOKENS=N keeps it
// to passes of at most N tokens.
constexpr int PDL_MAX_TOKENS = 1 << 30;
static thread_local int t_pass_tokens = 0;

static bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("NEEDLE_B200_PDL");
    return !(e && e[0] == '0');
  }();
  static const int max_tokens = [] {
    const char* e = std::getenv("NEEDLE_B200_PDL_TOKENS");
    return e ? std::atoi(e) : PDL_MAX_TOKENS;
  }();
  return on && t_pass_tokens <= max_tokens;
}

static thread_local long t_launches = 0;  // kernels this thread has launched (or recorded into a graph)
long launch_counter() { return t_launches; }
void note_launch() { ++t_launches; }

template <typename... P, typename... A>
static void launch_clustered(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, dim3 cluster, A&&... args) {
  ++t_launches;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cluster.x * cluster.y * cluster.z > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster.x;
    attr[1].val.clusterDim.y = cluster.y;
    attr[1].val.clusterDim.z = cluster.z;
    cfg.numAttrs = 2;
  }
  cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
}

template <typename... P, typename... A>
static void launch(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A&&... args) {
  launch_clustered(kernel, grid, block, smem, st, dim3(1, 1, 1), std::forward<A>(args)...);
}

// The output of a wide product as a 2-D tensor map (rows innermost, one
// token per outer index) for TMA stores of [8 tokens][32 rows] boxes; rows
// past `rows` and tokens past M are clipped by the copy. False (plain stores
// then) when the driver entry point is missing or the base or the token
// stride is not 16-byte aligned.
static bool wide_out_map(CUtensorMap* map, const float* out, int rows, int M, int out_stride) {
  static const PFN_cuTensorMapEncodeTiled encode = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult found = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &found) != cudaSuccess ||
        found != cudaDriverEntryPointSuccess)
      return (PFN_cuTensorMapEncodeTiled) nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
  }();
  std::memset(map, 0, sizeof *map);
  if (!encode || (reinterpret_cast<uintptr_t>(out) & 15) || ((size_t)out_stride * 4) % 16) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)rows, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)out_stride * 4};
  const cuuint32_t box[2] = {32, 8}, elements[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(out), dims, strides, box, elements, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Passes of at least this many tokens take the persistent product
// ($NEEDLE_B200_WIDE_TOKENS overrides WIDE_MIN_TOKENS).
static int wide_min_tokens() {
  static const int n = [] {
    const char* e = std::getenv("NEEDLE_B200_WIDE_TOKENS");
    return e ? std::max(1, std::atoi(e)) : WIDE_MIN_TOKENS;
  }();
  return n;
}

// One codebook product of M tokens through W (K = W.cols: 512, or 2048 in the
// product benchmark): the CUDA-core GEMV for a few tokens, the pipelined
// persistent tcgen05 kernel for passes of at least WIDE_MIN_TOKENS tokens at
// K = 512, else tcgen05 tiles of 16 or 32 tokens. act_rows is the row
// capacity of the activation buffer (it places the chunks of K > 512).
static void project(const QMat& W, const int8_t* act, const float* act_scale, float* out, int M, int out_stride,
                    const TokenMeta* meta, cudaStream_t st, int* error, int act_rows = 0) {
  const int tiles = (W.rows + GEMM_ROWS - 1) / GEMM_ROWS;
  const bool wide = W.cols == 4 * GEMM_K;
  if (M <= GEMV_MAX_TOKENS) {
    const int ctas = ((W.rows + 7) / 8 + GEMV_WARPS - 1) / GEMV_WARPS;
    if (wide)
      launch(k_gemv<4>, ctas, GEMV_WARPS * 32, 0, st, W, act, act_scale, out, M, out_stride, meta, act_rows);
    else
      launch(k_gemv<1>, ctas, GEMV_WARPS * 32, 0, st, W, act, act_scale, out, M, out_stride, meta, act_rows);
  } else if (!wide && M >= wide_min_tokens()) {
    // persistent CTAs, one per SM: P of them share each row tile's token tiles
    static const int sms = [] {
      int device = 0, n = 0;
      cudaGetDevice(&device);
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
      return n > 0 ? n : 148;
    }();
    const int token_tiles = (M + WIDE_NT - 1) / WIDE_NT;
    const int P = std::max(1, std::min(token_tiles, sms / tiles));
    CUtensorMap map;
    const int tma = wide_out_map(&map, out, (int)W.rows, M, out_stride) ? 1 : 0;
    launch(k_gemm_wide, dim3(tiles, P), WIDE_THREADS, wide_smem(), st, W, act, act_scale, out, M, out_stride, meta, error, map, tma);
  } else if (M <= 16) {
    auto k = wide ? k_gemm<16, 4> : k_gemm<16, 1>;
    launch(k, dim3(tiles, 1), GEMM_THREADS_PER_TOKEN * 16, gemm_smem<16>(), st, W, act, act_scale, out, M, out_stride, meta, error, act_rows);
  } else {
    auto k = wide ? k_gemm<32, 4> : k_gemm<32, 1>;
    launch(k, dim3(tiles, (M + 31) / 32), GEMM_THREADS_PER_TOKEN * 32, gemm_smem<32>(), st, W, act, act_scale, out, M, out_stride, meta, error,
           act_rows);
  }
}

void launch_embed(const ModelDev& md, const Work& w, int M, cudaStream_t st) {
  t_pass_tokens = M;
  launch(k_embed, M, 128, 0, st, md, w, M);
}

// The block finish: split over a cluster by Kronecker output column for
// passes of at most BLOCK_SPLIT_MAX_TOKENS tokens, where one CTA per token
// leaves most SMs idle and the FP32 products set the latency; one CTA per
// token above, where the whole GPU is busy and the split's repeated front
// (norms, softmax, elementwise passes in every CTA of a cluster) would cost
// throughput. $NEEDLE_B200_BLOCK_SPLIT=N sets the threshold (0: never).
constexpr int BLOCK_SPLIT_MAX_TOKENS = 64;
static bool block_split_path(const ModelDev& md, int M) {
  static const int max_tokens = [] {
    const char* e = std::getenv("NEEDLE_B200_BLOCK_SPLIT");
    return e ? std::atoi(e) : BLOCK_SPLIT_MAX_TOKENS;
  }();
  const int W = 2 * BLOCK_THREADS / (int)md.hada_left;
  // every thread of a CTA takes at most one element of the lane combine
  return M <= max_tokens && ((int)md.d_model / HADA_RIGHT) * W <= BLOCK_THREADS;
}

// Whether the pass's out product runs inside the split block finish: a few
// tokens (the product would be k_gemv's), d = 512 on four CTAs per token, no
// cross attention (whose step reads the out product itself).
// $NEEDLE_B200_FUSE_OUT=0 keeps the separate product.
static bool fuse_out_product(const ModelDev& md, const LayerDev& L, int M, bool cross) {
  static const bool off = [] {
    const char* e = std::getenv("NEEDLE_B200_FUSE_OUT");
    return e && e[0] == '0';
  }();
  const int CL = HADA_RIGHT / (2 * BLOCK_THREADS / (int)md.hada_left);
  return !off && !cross && M <= GEMV_MAX_TOKENS && block_split_path(md, M) && CL * FUSED_OUT_ROWS == (int)md.d_model &&
         L.out.rows == md.d_model && L.out.cols == (uint32_t)GEMM_K;
}

// the lean block finish from this many tokens on (prefill passes; the
// 128-token decode chains keep two resident-factor CTAs per SM)
constexpr int BLOCK_LEAN_MIN_TOKENS = 256;

static void launch_block(const ModelDev& md, const LayerDev& L, const Work& w, int M, cudaStream_t st, bool fuse_out = false) {
  const int left = md.hada_left, W = 2 * BLOCK_THREADS / left, CL = HADA_RIGHT / W;
  if (block_split_path(md, M)) {
    auto k = left == 64 ? k_block_split<64> : k_block_split<32>;
    const int split_floats = (int)(block_split_smem(md) / 4);
    const size_t smem = fuse_out ? block_split_out_offset(split_floats) + FUSED_OUT_CODES + FUSED_OUT_SCALES : block_split_smem(md);
    launch_clustered(k, dim3(M * CL), BLOCK_THREADS, smem, st, dim3(CL, 1, 1), md, L, w, M, md.error, fuse_out ? 1 : 0, split_floats);
  } else {
    // $NEEDLE_B200_BLOCK_LEAN=N: the lean block finish for passes of at least N tokens
    static const int lean_from = [] {
      const char* e = std::getenv("NEEDLE_B200_BLOCK_LEAN");
      return e ? std::atoi(e) : BLOCK_LEAN_MIN_TOKENS;
    }();
    if (M >= lean_from) {
      auto k = left == 64 ? k_block_lean<64> : k_block_lean<32>;
      launch(k, M, BLOCK_THREADS, block_smem(md, 1), st, md, L, w, M, md.error);
    } else {
      auto k = left == 64 ? k_block<64> : k_block<32>;
      launch(k, M, BLOCK_THREADS, block_smem(md), st, md, L, w, M, md.error);
    }
  }
}

// the lean routing from this many tokens on (prefill passes; the decode
// chains keep the phi rows in shared memory, off the token's L2 latency chain)
constexpr int ROUTE_LEAN_MIN_TOKENS = 256;

void launch_layer(const ModelDev& md, const LayerDev& L, const EngramDev* engram, const CrossLayerDev* cross, const Work& w,
                  const KvDev& kv, int M, int layer, int slot, int t_cap, bool distinct, cudaStream_t st) {
  t_pass_tokens = M;
  const int d = md.d_model, H = md.heads, KV = md.kv_heads;
  const int proj_stride = (2 * H + 2 * KV) * HEAD_DIM;
  if (engram) {  // the site's key and raw value rows (engram.rs:84-90)
    launch(k_engram_gather, M, 128, 0, st, md, *engram, w, M);
    project(engram->kv, w.act, w.act_scale, w.engram_kv, M, 2 * d, w.meta, st, md.error, (int)w.act_rows);
  }
  // $NEEDLE_B200_ROUTE_LEAN=N: the lean routing for passes of at least N tokens
  static const int route_lean_from = [] {
    const char* e = std::getenv("NEEDLE_B200_ROUTE_LEAN");
    return e ? std::atoi(e) : ROUTE_LEAN_MIN_TOKENS;
  }();
  if (M >= route_lean_from)
    launch(k_route<true>, M, 256, route_smem(md, true), st, md, L, w, M, layer, slot, md.error);
  else
    launch(k_route<false>, M, 256, route_smem(md), st, md, L, w, M, layer, slot, md.error);
  project(L.qkvg, w.act, w.act_scale, w.proj, M, proj_stride, w.meta, st, md.error);
  // the head step runs inside the attention when each token of the pass
  // belongs to a different sequence; $NEEDLE_B200_FUSE_HEADS=0 keeps k_heads
  static const bool heads_off = [] {
    const char* e = std::getenv("NEEDLE_B200_FUSE_HEADS");
    return e && e[0] == '0';
  }();
  const bool heads = distinct && !heads_off;
  if (!heads) launch(k_heads, M, 32 * (H + 2 * KV), 0, st, md, L, w, kv, M, layer);
  if (!launch_attention(md, L, w, kv, M, layer, t_cap, heads, st))
    launch(k_prep, M, 128, 0, st, (const float*)w.attn, H * HEAD_DIM, (const int32_t*)nullptr,
           (const float*)(w.proj + (H + 2 * KV) * HEAD_DIM), proj_stride, H * HEAD_DIM, w.act, w.act_scale, M, w.meta,
           md.inv_sqrt_group, 1, 0);
  const bool fuse_out = fuse_out_product(md, L, M, cross != nullptr);
  if (!fuse_out) project(L.out, w.act, w.act_scale, w.outp, M, d, w.meta, st, md.error);
  if (cross) {  // Whistle: CrossState::apply after the attention residual (session.rs:126-128)
    launch(k_cross_q, M, 128, 0, st, md, L, layer, w, M);
    project(cross->qg, w.act, w.act_scale, w.cq, M, 2 * d, w.meta, st, md.error);
    launch(k_cross_attend, dim3(M, md.heads), CROSS_THREADS, 2 * MAX_CROSS_FRAMES * sizeof(float), st, md, layer, w, M);
    launch(k_prep, M, 128, 0, st, (const float*)w.attn, H * HEAD_DIM, (const int32_t*)nullptr, (const float*)nullptr, 0, H * HEAD_DIM,
           w.act, w.act_scale, M, w.meta, md.inv_sqrt_group, 1, 0);
    project(cross->out, w.act, w.act_scale, w.outp, M, d, w.meta, st, md.error);  // the block finish adds it
  }
  launch_block(md, L, w, M, st, fuse_out);
}

cudaError_t cross_memory(const ModelDev& md, const std::vector<CrossLayerDev>& layers, const float* encoded, int frames,
                         const float* sin_tab, const float* cos_tab, float gate, float* rows, int8_t* act, float* act_scale, int act_rows,
                         float* kv, int8_t* keys, float* kscale, int8_t* values, float* vscale, cudaStream_t st) {
  const int d = (int)md.d_model, heads = (int)md.heads;
  k_cross_memory_in<<<frames, 128, 0, st>>>(encoded, sin_tab, cos_tab, gate, d, rows);
  k_prep<<<frames, 128, 0, st>>>(rows, d, (const int32_t*)nullptr, (const float*)nullptr, 0, d, act, act_scale, frames,
                                 (const TokenMeta*)nullptr, md.inv_sqrt_group, 1, act_rows);
  for (size_t l = 0; l < layers.size(); ++l) {
    project(layers[l].kv, act, act_scale, kv, frames, 2 * d, nullptr, st, md.error, act_rows);
    const size_t at = l * (size_t)frames * heads;
    k_cross_memory_heads<<<frames, 64 * heads, 0, st>>>(kv, d, frames, layers[l].k_norm, keys + at * HEAD_DIM, kscale + at,
                                                       values + at * HEAD_DIM, vscale + at);
  }
  return cudaGetLastError();
}

void launch_observe(const ModelDev& md, const Work& w, const float* stream, int M, int row, cudaStream_t st) {
  t_pass_tokens = M;
  launch(k_observe, M, 128, 0, st, md, w, stream, M, row);
}

void head_output(const ModelDev& md, const HeadDev& H, int h, int slot, const int32_t* rows, int nrows, float* readouts, float* weights,
                 float* pooled, int8_t* act, float* act_scale, int act_rows, float* out, bool project_out, cudaStream_t st) {
  k_head_pool<<<1, 256, 0, st>>>(md, h, slot, rows, nrows, readouts, weights, pooled);
  if (!project_out) return;
  // ProbeHead::project (heads.rs:117-125): rotate and quantise per group (no
  // fake quantisation), the product, then the bias
  const int K = (int)H.queries * (int)md.d_model;
  k_prep<<<1, 128, 0, st>>>(pooled, K, (const int32_t*)nullptr, (const float*)nullptr, 0, K, act, act_scale, 1, (const TokenMeta*)nullptr,
                            md.inv_sqrt_group, 0, act_rows);
  project(H.proj, act, act_scale, out, 1, (int)H.proj.rows, nullptr, st, md.error, act_rows);
  k_add_bias<<<1, 128, 0, st>>>(out, H.bias, (int)H.outputs);
}

void dense_rows(const uint8_t* packed, uint32_t row_bytes, uint32_t bits, const float* levels, const float* norms, int rows, int cols,
                float inv_sqrt_group, float* out, cudaStream_t st) {
  k_dense_rows<<<rows, 128, 0, st>>>(packed, row_bytes, bits, levels, norms, cols, inv_sqrt_group, out);
}

void fill(float* p, size_t n, float value, cudaStream_t st) {
  if (n) k_fill<<<(unsigned)std::min<size_t>((n + 255) / 256, 1184), 256, 0, st>>>(p, n, value);
}

void launch_final(const ModelDev& md, const Work& w, float* hidden, int M, cudaStream_t st) {
  t_pass_tokens = M;
  launch(k_final, M, 128, 0, st, md, w, hidden, M);
}

void launch_logits(const ModelDev& md, const float* hidden, const int32_t* slots, int B, int8_t* act, float* act_scale, float* logits,
                   cudaStream_t st) {
  t_pass_tokens = B;
  launch(k_prep, B, 128, 0, st, hidden, (int)md.d_model, slots, (const float*)nullptr, 0, (int)md.d_model, act, act_scale, B,
         (const TokenMeta*)nullptr, md.inv_sqrt_group, 1, 0);
  project(md.logits, act, act_scale, logits, B, md.output_vocab, nullptr, st, md.error);
}

void launch_select(const float* logits, int V, const uint32_t* mask, const int32_t* active, uint32_t* next, float* peaks, int B,
                   cudaStream_t st) {
  t_pass_tokens = B;
  launch(k_select, B, 256, 0, st, logits, V, mask, active, next, peaks);
}

void launch_stats(const float* logits, int V, const uint32_t* mask, const int32_t* active, const uint32_t* next, const float* peaks,
                  float* stats, int stats_stride, int B, cudaStream_t st) {
  t_pass_tokens = B;
  launch(k_stats, B, 256, (size_t)2 * V * 4, st, logits, V, mask, active, next, peaks, stats, stats_stride);
}

void launch_advance(TokenMeta* meta, int B, cudaStream_t st) {
  t_pass_tokens = B;
  launch(k_advance, (B + 127) / 128, 128, 0, st, meta, B);
}

// The attention of a pass with its neighbours fused in where the shapes
// allow: the head step when `heads`, and the output projection's activation
// step, by the cluster epilogue for passes of at most FUSE_PREP_MAX_TOKENS
// tokens (a launch saved on the latency path) and by the last-CTA epilogue
// above (the cluster over kv heads would cost the attention CTA scheduling
// freedom there). False when k_prep must still run.
// $NEEDLE_B200_FUSE_PREP=0 always leaves the activation step to k_prep.
constexpr int FUSE_PREP_MAX_TOKENS = 64;
// the narrow attention CTAs from this many tokens on: prefill passes, whose
// many short contexts (a CTA per query token and kv head) are bound by the
// fixed phases, which five CTAs per SM overlap better than three; the
// 128-token decode chains, longer contexts on fewer CTAs, keep the wide ones
constexpr int ATT_NARROW_MIN_TOKENS = 256;
// the wide attention CTAs up to this many tokens: at batch 1 a token's four
// kv-head CTAs are the whole launch, so each CTA's phases get a whole SM
constexpr int ATT_WIDE_MAX_TOKENS = 8;

template <int G, int EPI>
static void attend_variant(bool heads, const ModelDev& md, const LayerDev& L, const Work& w, const KvDev& kv, int M, int layer,
                           int t_cap, cudaStream_t st) {
  // $NEEDLE_B200_ATT_NARROW=N: the narrow CTAs (G <= 2) for passes of at least N tokens
  static const int narrow_from = [] {
    const char* e = std::getenv("NEEDLE_B200_ATT_NARROW");
    return e ? std::atoi(e) : ATT_NARROW_MIN_TOKENS;
  }();
  const dim3 grid(M, md.kv_heads), cluster(1, EPI == ATT_CLUSTER ? md.kv_heads : 1, 1);
  // $NEEDLE_B200_ATT_WIDE=N: the wide CTAs (G <= 2) for passes of at most N tokens
  static const int wide_to = [] {
    const char* e = std::getenv("NEEDLE_B200_ATT_WIDE");
    return e ? std::atoi(e) : ATT_WIDE_MAX_TOKENS;
  }();
  if constexpr (G <= 2) {
    if (M <= wide_to) {
      constexpr int W = ATT_WORKERS_WIDE;
      const size_t smem = attend_smem(md, t_cap, W);
      if (heads)
        launch_clustered(k_attend<G, EPI, true, W>, grid, W + 32, smem, st, cluster, md, L, w, kv, M, layer, t_cap);
      else
        launch_clustered(k_attend<G, EPI, false, W>, grid, W + 32, smem, st, cluster, md, L, w, kv, M, layer, t_cap);
      return;
    }
    if (M >= narrow_from) {
      constexpr int W = ATT_WORKERS_NARROW;
      const size_t smem = attend_smem(md, t_cap, W);
      if (heads)
        launch_clustered(k_attend<G, EPI, true, W>, grid, W + 32, smem, st, cluster, md, L, w, kv, M, layer, t_cap);
      else
        launch_clustered(k_attend<G, EPI, false, W>, grid, W + 32, smem, st, cluster, md, L, w, kv, M, layer, t_cap);
      return;
    }
  }
  const size_t smem = attend_smem(md, t_cap);
  if (heads)
    launch_clustered(k_attend<G, EPI, true, ATT_WORKERS>, grid, ATT_WORKERS + 32, smem, st, cluster, md, L, w, kv, M, layer, t_cap);
  else
    launch_clustered(k_attend<G, EPI, false, ATT_WORKERS>, grid, ATT_WORKERS + 32, smem, st, cluster, md, L, w, kv, M, layer, t_cap);
}

bool launch_attention(const ModelDev& md, const LayerDev& L, const Work& w, const KvDev& kv, int M, int layer, int t_cap, bool heads,
                      cudaStream_t st) {
  static const bool prep_off = [] {
    const char* e = std::getenv("NEEDLE_B200_FUSE_PREP");
    return e && e[0] == '0';
  }();
  t_pass_tokens = M;
  const int G = md.heads / md.kv_heads, K = md.heads * HEAD_DIM;
  int epi = ATT_ROWS;
  if (!prep_off) {
    const bool whole_groups = (G == 2 || G == 4) && md.kv_heads <= ATT_MAX_KV && K == (int)md.d_model;
    if (M <= FUSE_PREP_MAX_TOKENS && whole_groups)
      epi = ATT_CLUSTER;
    else if (K <= PREP_MAX_K && (size_t)G * t_cap >= (size_t)K && w.arrivals)
      epi = ATT_LAST;
  }
  if (G == 1) {
    if (epi == ATT_LAST)
      attend_variant<1, ATT_LAST>(heads, md, L, w, kv, M, layer, t_cap, st);
    else
      attend_variant<1, ATT_ROWS>(heads, md, L, w, kv, M, layer, t_cap, st);
    return epi == ATT_LAST;
  }
  if (G == 2) {
    if (epi == ATT_CLUSTER) attend_variant<2, ATT_CLUSTER>(heads, md, L, w, kv, M, layer, t_cap, st);
    if (epi == ATT_LAST) attend_variant<2, ATT_LAST>(heads, md, L, w, kv, M, layer, t_cap, st);
    if (epi == ATT_ROWS) attend_variant<2, ATT_ROWS>(heads, md, L, w, kv, M, layer, t_cap, st);
  } else {
    if (epi == ATT_CLUSTER) attend_variant<4, ATT_CLUSTER>(heads, md, L, w, kv, M, layer, t_cap, st);
    if (epi == ATT_LAST) attend_variant<4, ATT_LAST>(heads, md, L, w, kv, M, layer, t_cap, st);
    if (epi == ATT_ROWS) attend_variant<4, ATT_ROWS>(heads, md, L, w, kv, M, layer, t_cap, st);
  }
  return epi != ATT_ROWS;
}

// ------------------------------------------------------------------- debug
// Element-wise device math for the kernel-level tests: 0 expf (f32::exp),
// 1 sigmoid, 2 fast_exp, 3 silu.
__global__ void k_debug_math(int op, const float* in, float* out, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float x = in[i];
  const float MIN_POSITIVE = 1.17549435e-38f;
  out[i] = op == 0   ? expf_libm(x)
           : op == 1 ? sigmoid(x)
           : op == 2 ? fast_exp(x)
           : op == 3 ? silu(x)
                     : rcp_positive(fmaxf(x, MIN_POSITIVE));  // x <= 4, as the Sinkhorn's totals
}

void launch_debug_math(int op, const float* in, float* out, int n, cudaStream_t st) {
  k_debug_math<<<(n + 255) / 256, 256, 0, st>>>(op, in, out, n);
}

// HadamardWeights::apply (hadamard.rs:260-304) of one layer on `M` inputs.
template <int LEFT>
__global__ void __launch_bounds__(BLOCK_THREADS) k_debug_hadamard(ModelDev md, HadamardDev Hd, const float* in, float* out, int M) {
  extern __shared__ float sm[];
  constexpr int N = LEFT * HADA_RIGHT;
  const int t = blockIdx.x, d = md.d_model;
  float* s_pre = sm + 2 * MAX_D;
  float* buf0 = sm + 3 * MAX_D;
  float* buf1 = buf0 + N;
  float* s_mod = buf1 + N;
  float* s_left = s_mod + N;
  float* s_right = s_left + LEFT * LEFT;
  float* s_condv = d * COND_RANK <= 2 * N ? buf1 : s_right + HADA_RIGHT * HADA_RIGHT;
  stage_async(s_condv, Hd.cond_v, d * COND_RANK);
  stage_async(s_left, Hd.left[0], LEFT * LEFT);
  stage_async(s_right, Hd.right[0], HADA_RIGHT * HADA_RIGHT);
  stage_async(s_pre, in + (size_t)t * d, d);
  cp_async_wait_all();
  __syncthreads();
  hadamard_core<LEFT, false>(md, Hd, d, s_pre, buf0, buf1, s_mod, s_left, s_right, s_condv);
  for (int i = threadIdx.x; i < d; i += BLOCK_THREADS) out[(size_t)t * d + i] = fmul(buf0[i], Hd.d4[i]);
}

void launch_debug_hadamard(const ModelDev& md, const LayerDev& L, const float* in, float* out, int M, cudaStream_t st) {
  if (md.hada_left == 64) {
    cudaFuncSetAttribute(k_debug_hadamard<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)block_smem(md));
    k_debug_hadamard<64><<<M, BLOCK_THREADS, block_smem(md), st>>>(md, L.hada, in, out, M);
  } else {
    cudaFuncSetAttribute(k_debug_hadamard<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)block_smem(md));
    k_debug_hadamard<32><<<M, BLOCK_THREADS, block_smem(md), st>>>(md, L.hada, in, out, M);
  }
}

// One codebook product of K-wide inputs (rotated and quantised per group,
// without the whole-vector fake quantisation) — QuantisedMatrix::prepare +
// multiply_vector (matrix.rs:123-165).
void launch_debug_project(const ModelDev& md, const QMat& W, const float* in, int K, int M, int8_t* act, float* act_scale,
                          float* out, int out_stride, cudaStream_t st) {
  k_prep<<<M, 128, 0, st>>>(in, K, nullptr, nullptr, 0, K, act, act_scale, M, nullptr, md.inv_sqrt_group, 0, 0);
  project(W, act, act_scale, out, M, out_stride, nullptr, st, md.error);
}

// The product benchmark of the test hooks: k_prep (rotation and per-group
// int8 activations, no fake quantisation) then the product; with reps > 0
// the product alone is replayed reps times between CUDA events.
cudaError_t launch_product_bench(const QMat& W, const float* in, int M, int8_t* act, float* act_scale, int act_rows, float* out,
                                 int* error, int reps, float* ms, cudaStream_t st) {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(k_gemm<16, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem<16>()))) return e;
  if ((e = cudaFuncSetAttribute(k_gemm<32, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem<32>()))) return e;
  if ((e = cudaFuncSetAttribute(k_gemm<16, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem<16>()))) return e;
  if ((e = cudaFuncSetAttribute(k_gemm<32, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem<32>()))) return e;
  if ((e = cudaFuncSetAttribute(k_gemm_wide, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wide_smem()))) return e;
  t_pass_tokens = M;
  const int K = (int)W.cols;
  k_prep<<<M, 128, 0, st>>>(in, K, nullptr, nullptr, 0, K, act, act_scale, M, nullptr, 1.0f / std::sqrt((float)GROUP), 0, act_rows);
  project(W, act, act_scale, out, M, (int)W.rows, nullptr, st, error, act_rows);
  if ((e = cudaGetLastError())) return e;
  *ms = 0.0f;
  if (reps <= 0) return cudaSuccess;
  cudaEvent_t start, stop;
  if ((e = cudaEventCreate(&start))) return e;
  if ((e = cudaEventCreate(&stop))) return e;
  cudaEventRecord(start, st);
  for (int r = 0; r < reps; ++r) project(W, act, act_scale, out, M, (int)W.rows, nullptr, st, error, act_rows);
  cudaEventRecord(stop, st);
  e = cudaEventSynchronize(stop);
  float total = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&total, start, stop);
  cudaEventDestroy(start);
  cudaEventDestroy(stop);
  *ms = total / (float)reps;
  return e;
}

cudaError_t set_expire_route(int count, cudaStream_t st) {
  return cudaMemcpyToSymbolAsync(g_expire_route, &count, sizeof(int), 0, cudaMemcpyHostToDevice, st);
}

// ------------------------------------------------------- read bandwidth
// A plain streaming read of `n16` 16-byte words through L2 (ld.global.cg, no
// L1 allocation), `passes` times over in one launch so the launch and the ramp
// are a small part of the time: every thread keeps four loads in flight and
// folds them into one word, which is stored only when it equals a value no
// input produces (the sink keeps the loads live). Timed over a buffer smaller
// than L2 it is the L2 read peak the batch-1 roofline is quoted against; over
// a buffer several times larger than L2, the HBM read bandwidth.
__global__ void __launch_bounds__(512) k_read_stream(const uint4* __restrict__ data, size_t n16, int passes, uint32_t* sink) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  uint32_t acc = 0;
  for (int pass = 0; pass < passes; ++pass) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n16; i += 4 * stride) {
      const uint4 a = __ldcg(data + i), b = __ldcg(data + i + stride), c = __ldcg(data + i + 2 * stride),
                  d = __ldcg(data + i + 3 * stride);
      acc ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w ^ c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
    }
    for (; i < n16; i += stride) {
      const uint4 a = __ldcg(data + i);
      acc ^= a.x ^ a.y ^ a.z ^ a.w;
    }
    acc = acc * 0x01000193u + (uint32_t)pass;  // each pass's loads feed the word
  }
  if (acc == 0x9E3779B9u) sink[0] = acc;
}

cudaError_t launch_read_bench(const void* data, size_t bytes, int passes, uint32_t* sink, int reps, float* ms, cudaStream_t st) {
  int device = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return e;
  const size_t n16 = bytes / 16;
  const int blocks = sms * 4;  // four 512-thread CTAs per SM
  const uint4* p = static_cast<const uint4*>(data);
  for (int w = 0; w < 3; ++w) k_read_stream<<<blocks, 512, 0, st>>>(p, n16, passes, sink);
  if ((e = cudaGetLastError())) return e;
  cudaEvent_t start, stop;
  if ((e = cudaEventCreate(&start))) return e;
  if ((e = cudaEventCreate(&stop))) {
    cudaEventDestroy(start);
    return e;
  }
  cudaEventRecord(start, st);
  for (int r = 0; r < reps; ++r) k_read_stream<<<blocks, 512, 0, st>>>(p, n16, passes, sink);
  cudaEventRecord(stop, st);
  e = cudaEventSynchronize(stop);
  float total = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&total, start, stop);
  cudaEventDestroy(start);
  cudaEventDestroy(stop);
  *ms = total / (float)reps;
  return e;
}

// ------------------------------------------------ allocation-free product
// The one codebook product above for callers that may not allocate device
// memory: a host that has handed all of the GPU's memory to its own pool, or
// a thread that must not take the implicit device-wide synchronisation of
// cudaMalloc/cudaFree. Its scratch — the int8 activations in the
// core-matrix layout, their per-group scales and the flag of a bounded wait
// that gave up — is this file-scope array, one per device, shared by every
// call: two calls that overlap in time (on any streams or threads) race on it.
// Nothing in it has to start at zero except the flag, which each call clears;
// the product reads the unused token rows of its last tile but stores none of
// their columns.
constexpr size_t STATIC_ACT_BYTES = (size_t)STATIC_MAX_TOKENS * GEMM_K;
constexpr size_t STATIC_SCALE_BYTES = (size_t)STATIC_MAX_TOKENS * (GEMM_K / GROUP) * sizeof(float);
constexpr size_t STATIC_SCRATCH_BYTES = STATIC_ACT_BYTES + STATIC_SCALE_BYTES + 256;
static_assert(STATIC_MAX_TOKENS % 32 == 0, "the scratch must hold whole 32-token tiles");
static __device__ __align__(256) uint8_t g_static_scratch[STATIC_SCRATCH_BYTES];

constexpr int STATIC_MAX_DEVICES = 64;
static uint8_t* g_static_address[STATIC_MAX_DEVICES];
static std::mutex g_static_mutex;

cudaError_t static_scratch_setup(int device) {
  if (device < 0 || device >= STATIC_MAX_DEVICES) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_static_mutex);
  if (g_static_address[device]) return cudaSuccess;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return e;
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess) return e;
  g_static_address[device] = static_cast<uint8_t*>(p);
  return cudaSuccess;
}

cudaError_t launch_static_project(int device, const ModelDev& md, const QMat& W, const float* in, int M, float* out,
                                  cudaStream_t st, int* wait_failed) {
  uint8_t* base = g_static_address[device];
  int8_t* act = reinterpret_cast<int8_t*>(base);
  float* act_scale = reinterpret_cast<float*>(base + STATIC_ACT_BYTES);
  int* flag = reinterpret_cast<int*>(base + STATIC_ACT_BYTES + STATIC_SCALE_BYTES);
  cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int), st);
  if (e != cudaSuccess) return e;
  const int K = GEMM_K, tiles = (W.rows + GEMM_ROWS - 1) / GEMM_ROWS;
  k_prep<<<M, 128, 0, st>>>(in, K, nullptr, nullptr, 0, K, act, act_scale, M, nullptr, md.inv_sqrt_group, 0, 0);
  if (M <= 16)
    k_gemm<16, 1><<<dim3(tiles, 1), GEMM_THREADS_PER_TOKEN * 16, gemm_smem<16>(), st>>>(W, act, act_scale, out, M, (int)W.rows, nullptr, flag, 0);
  else
    k_gemm<32, 1><<<dim3(tiles, (M + 31) / 32), GEMM_THREADS_PER_TOKEN * 32, gemm_smem<32>(), st>>>(W, act, act_scale, out, M, (int)W.rows, nullptr, flag, 0);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  *wait_failed = 0;
  if ((e = cudaMemcpyAsync(wait_failed, flag, sizeof(int), cudaMemcpyDeviceToHost, st)) != cudaSuccess) return e;
  return cudaStreamSynchronize(st);
}

}  // namespace nbk
