// device.cuh — device-side building blocks shared by the Needle-3 kernels.
//
// Every float operation is written with an explicitly rounded intrinsic so the
// association order of the reference survives compilation (the library is also
// built with -fmad=false). Reductions whose order the reference fixes (the
// 8-lane sum of squares of crates/kernels/src/ops.rs:7-17, sequential sums) are
// evaluated in that order; max and integer reductions, which are exact in any
// order, use warp shuffles.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "exactmath.h"
#include "layout.h"

namespace nbk {

constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float frcp(float a) { return __frcp_rn(a); }
__device__ __forceinline__ float fsqrt(float a) { return __fsqrt_rn(a); }

// Exact int32 → f32 of a 128-column group sum of int8 × int8 products
// (|x| ≤ 128·128·128 = 2^21 < 2^22), by the magic-number method: the bits
// 0x4B400000 + x are the float 1.5·2^23 + x (unit spacing in [2^23, 2^24), the
// exponent unchanged for |x| < 2^22), and subtracting 1.5·2^23 is exact. Two
// full-rate instructions in place of a conversion-unit I2F.
__device__ __forceinline__ float group_sum_to_float(uint32_t x) {
  return fsub(__int_as_float((int)(0x4B400000u + x)), 12582912.0f);
}

// Packed two-lane f32 arithmetic (PTX add/fma .rn.f32x2): each component
// rounded to nearest exactly as the scalar .rn instruction.
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// -0.0 in both lanes, read from memory so the compiler cannot see the value:
// fma(a, b, -0.0) is a·b rounded once, exactly mul.rn, and a packed fma is
// never merged with the packed add that follows it (a visible packed multiply
// would be, into one fused multiply-add the reference never performs).
__device__ float2 g_negzero = {-0.0f, -0.0f};

// Programmatic dependent launch. Every kernel of the token loop is launched
// with programmatic stream serialisation: it may start while its predecessor
// on the stream still runs. pdl_wait() blocks until the predecessor grid has
// completed and its writes are visible; pdl_trigger() lets the successor
// start once every CTA of this grid has triggered or exited. Every CTA passes
// pdl_wait() before it triggers or exits, so when a kernel starts, every
// launch before its immediate predecessor has completed. Before pdl_wait() a
// kernel therefore writes nothing to global memory and reads only the
// model's constant weights and data that launches at least two back (or the
// host, before the pass) produced; it reads the latter through L2
// (ld.global.cg), never through a possibly stale L1 line.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Bounded mbarrier waits: a wait that gives up returns false, and its caller
// raises the device error flag and skips the work instead of hanging.
constexpr uint32_t MBAR_WAIT_LIMIT = 1u << 24;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool mbar_wait_polls(uint32_t bar, uint32_t phase, uint32_t polls) {
  for (uint32_t i = 0; i < polls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(phase)
        : "memory");
    if (done) return true;
  }
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase) {
  for (uint32_t i = 0; i < MBAR_WAIT_LIMIT; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(phase)
        : "memory");
    if (done) return true;
  }
  return false;
}

// Bulk copies (cp.async.bulk) of contiguous global ranges into shared memory,
// completing on one mbarrier: one thread initialises the barrier, announces
// the bytes and issues every copy; addresses and sizes are 16-byte multiples.
__device__ __forceinline__ void bulk_start(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(1) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)), "l"(src),
               "r"(bytes), "r"(bar)
               : "memory");
}

// Rust's float Iterator::sum starts from -0.0.
constexpr float SUM_START = -0.0f;

// Set per device by set_exp_constants (kernels.cu). The 2^(j/64) table is
// also held in global memory: lanes index it with their own j, which the
// constant cache would serve one address at a time; L1 serves a warp's reads
// of the 512-byte table in at most four wavefronts.
__constant__ nbx::ExpConstants c_exp;
__constant__ nbx::ExceptionSet c_exceptions;
__device__ double g_exp_table[64];

// f32::exp of the host libm (see exactmath.h): the same double-precision
// evaluation as nbx::exp_double_core, written out for the device. 2^m is
// applied as a multiply by an exactly built power of two (m ∈ [-159, 128], so
// y·2^m is a normal double, the same value ldexp gives), and the
// near-midpoint test uses the result's positive sign (e^x > 0).
__device__ __forceinline__ float expf_libm(float x) {
  if (isnan(x)) return x;
  if (x > 89.0f) return INFINITY;
  if (x < -110.0f) return 0.0f;
  const double xd = (double)x;
  const double kd = rint(__dmul_rn(xd, c_exp.inv_step));
  const int k = (int)kd;
  const double t = __ldg(&g_exp_table[k & 63]);
  double r = __dadd_rn(xd, -__dmul_rn(kd, c_exp.step_hi));
  r = __dadd_rn(r, -__dmul_rn(kd, c_exp.step_lo));
  double p = 1.0 / 5040.0;
  p = __fma_rn(p, r, 1.0 / 720.0);
  p = __fma_rn(p, r, 1.0 / 120.0);
  p = __fma_rn(p, r, 1.0 / 24.0);
  p = __fma_rn(p, r, 1.0 / 6.0);
  p = __fma_rn(p, r, 0.5);
  p = __fma_rn(p, r, 1.0);
  p = __fma_rn(p, r, 1.0);
  const double scale = __longlong_as_double((long long)((k >> 6) + 1023) << 52);  // 2^m, m = (k - (k & 63)) / 64
  const double y = __dmul_rn(__dmul_rn(t, p), scale);
  float f = __double2float_rn(y);
  if ((double)f != y) {
    // the other binary32 neighbour of y, and whether y lies within
    // near_relative·y of their midpoint (nbx::near_midpoint for y > 0)
    const float other = __int_as_float(__float_as_int(f) + ((double)f < y ? 1 : -1));
    const double mid = __dmul_rn(__dadd_rn((double)f, (double)other), 0.5);
    if (fabs(__dadd_rn(y, -mid)) <= __dmul_rn(y, c_exp.near_relative) && !isinf(f) &&
        nbx::exception_contains(c_exceptions, nbx::float_bits(x)))
      f = other;
  }
  return f;
}

// 1/b correctly rounded, for a positive normal b below 2^126 (so 1/b is
// normal too), by Markstein's refinement of the hardware approximation
// (P. W. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Develop. 34(1), 1990): y0 =
// rcp.approx(b) lies within an ulp of 1/b, so e = 1 - b·y0 is exact in one
// fma, and y0 + y0·e is rounded once. Straight-line code (no slow path), so
// independent reciprocals overlap. Compared bit for bit with __frcp_rn over
// every b in [2^-126, 2^126) on B200: no difference.
__device__ __forceinline__ float rcp_positive(float b) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
  const float e = __fmaf_rn(-b, y, 1.0f);
  return __fmaf_rn(e, y, y);
}

// crates/kernels/src/ops.rs:69-71
__device__ __forceinline__ float sigmoid(float v) { return fdiv(1.0f, fadd(1.0f, expf_libm(-v))); }

// crates/kernels/src/ops.rs:83-90: clamp, scale by log2(e), round half away
// from zero, degree-5 polynomial of the fraction, then the power of two.
__device__ __forceinline__ float fast_exp(float value) {
  float c = value;
  if (c < -87.0f) c = -87.0f;
  if (c > 87.0f) c = 87.0f;
  float scaled = fmul(c, 1.44269504088896341f);
  float whole = roundf(scaled);
  float f = fsub(scaled, whole);
  float p = fmul(f, 0.0013333558f);
  p = fadd(0.009618129f, p);
  p = fmul(f, p);
  p = fadd(0.05550411f, p);
  p = fmul(f, p);
  p = fadd(0.2402265f, p);
  p = fmul(f, p);
  p = fadd(0.69314718055994531f, p);
  p = fmul(f, p);
  p = fadd(1.0f, p);
  int w = isnan(whole) ? 0 : (int)whole;
  return fmul(p, __int_as_float((w + 127) << 23));
}

// crates/kernels/src/ops.rs:74-76
__device__ __forceinline__ float silu(float v) { return fdiv(v, fadd(1.0f, fast_exp(-v))); }

__device__ __forceinline__ float clampf(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, s));
  return v;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) v += __shfl_xor_sync(FULL, v, s);
  return v;
}

// Max over a block; `scratch` holds one float per warp. All threads get the result.
__device__ __forceinline__ float block_max(float v, float* scratch) {
  v = warp_max(v);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = scratch[0];
  for (int i = 1; i < warps; ++i) r = fmaxf(r, scratch[i]);
  return r;
}

// ops.rs:7-17 over n values in shared memory: eight running lanes (lane l
// takes values l, l+8, ...), the lanes summed in order from -0.0, then the tail.
// Called by one whole warp; every lane returns the sum.
__device__ __forceinline__ float sum_of_squares_warp(const float* v, int n) {
  int lane = threadIdx.x & 31;
  int whole = n / 8 * 8;
  float acc = 0.0f;
  if (lane < 8) {
    int i = lane;
    // sixteen loads in flight per batch; the running sum itself stays one ordered chain
    for (; i + 8 * 15 < whole; i += 8 * 16) {
      float sq[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float x = v[i + 8 * k];
        sq[k] = fmul(x, x);
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) acc = fadd(acc, sq[k]);
    }
    for (; i < whole; i += 8) acc = fadd(acc, fmul(v[i], v[i]));
  }
  float s = SUM_START;
#pragma unroll
  for (int l = 0; l < 8; ++l) s = fadd(s, __shfl_sync(FULL, acc, l));
  float tail = SUM_START;
  for (int i = whole; i < n; ++i) tail = fadd(tail, fmul(v[i], v[i]));
  return fadd(s, tail);
}

// dot_product (ops.rs:19-30) of two n-vectors, n a multiple of 8, the same
// lane structure as sum_of_squares_warp. Called by one whole warp; every lane
// returns the sum.
__device__ __forceinline__ float dot_product_warp(const float* a, const float* b, int n) {
  const int lane = threadIdx.x & 31;
  float acc = 0.0f;
  if (lane < 8) {
    int i = lane;
    for (; i + 8 * 15 < n; i += 8 * 16) {
      float p[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) p[k] = fmul(a[i + 8 * k], b[i + 8 * k]);
#pragma unroll
      for (int k = 0; k < 16; ++k) acc = fadd(acc, p[k]);
    }
    for (; i < n; i += 8) acc = fadd(acc, fmul(a[i], b[i]));
  }
  float s = SUM_START;
#pragma unroll
  for (int l = 0; l < 8; ++l) s = fadd(s, __shfl_sync(FULL, acc, l));
  return fadd(s, SUM_START);  // the empty tail
}

// 1 / sqrt(mean_square + 1e-6) of ops.rs:44-66.
__device__ __forceinline__ float inverse_rms(float sum_squares, int n) {
  float ms = fdiv(sum_squares, (float)n);
  return fdiv(1.0f, fsqrt(fadd(ms, 1e-6f)));
}

// The normalised Walsh–Hadamard transform of one 128-value group held by a
// warp, four consecutive values per lane (walsh.rs:41-76): the radix-4 first
// stage, then butterflies of span 4..64 (lane distance 1..16), then the scale.
__device__ __forceinline__ void fwht128(float v[4], float inv_sqrt_group) {
  int lane = threadIdx.x & 31;
  float a = v[0], b = v[1], c = v[2], d = v[3];
  float ls = fadd(a, b), ld = fsub(a, b), hs = fadd(c, d), hd = fsub(c, d);
  v[0] = fadd(ls, hs);
  v[1] = fadd(ld, hd);
  v[2] = fsub(ls, hs);
  v[3] = fsub(ld, hd);
#pragma unroll
  for (int s = 1; s < 32; s <<= 1) {
    bool upper = lane & s;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float o = __shfl_xor_sync(FULL, v[j], s);
      v[j] = upper ? fsub(o, v[j]) : fadd(v[j], o);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = fmul(v[j], inv_sqrt_group);
}

// Per-group int8 activation of neon.rs:22-46 / panel.rs:46-65 for the 128
// values a warp holds (4 per lane): scale = peak/127 (1 when the group is 0),
// codes = round-half-even(x / scale) clamped to ±127. Returns the scale and
// the lane's four codes packed little-endian.
__device__ __forceinline__ float quantise_group(const float v[4], uint32_t& packed) {
  float peak = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) peak = fmaxf(peak, fabsf(v[j]));
  peak = warp_max(peak);
  float scale = peak > 0.0f ? fdiv(peak, 127.0f) : 1.0f;
  packed = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int q = (int)clampf(rintf(fdiv(v[j], scale)), -127.0f, 127.0f);
    packed |= (uint32_t)(q & 0xff) << (8 * j);
  }
  return scale;
}

// fake_quantise_int8 element step (ops.rs:120-125) given the vector's scale.
__device__ __forceinline__ float fake_quant(float v, float scale) { return fmul(clampf(rintf(fdiv(v, scale)), -128.0f, 127.0f), scale); }
__device__ __forceinline__ float int8_scale_of(float peak) { return peak > 0.0f ? fdiv(peak, 127.0f) : 1.0f; }

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

}  // namespace nbk
