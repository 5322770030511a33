// exactmath.h — binary32 arithmetic that reproduces the reference's float
// results bit for bit, shared by host code and sm_100a kernels.
//
// rustc never fuses a multiply with an add, so device code spells every
// rounding out with __fmul_rn/__fadd_rn/__fdiv_rn/__fsqrt_rn (the library is
// also compiled with -fmad=false); the one fused step the reference performs
// (the 2-bit panel combine, crates/kernels/src/panel.rs:187) is __fmaf_rn.
//
// f32::exp is the host libm expf. exp_binary32() below evaluates e^x in
// double precision by a method of this file's own (table-driven reduction
// with 64 subintervals, a Cody–Waite split of ln2/64 and the degree-7 Taylor
// polynomial of e^r on |r| <= ln2/128) and rounds once to binary32; that is
// the correctly rounded result except within ~1e-16 of a rounding midpoint.
// glibc's expf rounds the other way on a known, finite set of inputs; those
// are listed in a table built on the host (expf_table.cpp) by comparing the
// two over every binary32 input, and the device consults it only when the
// double result lies near a midpoint.
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define NB_HD __host__ __device__ __forceinline__
#else
#define NB_HD inline
#endif

namespace nbx {

// Constants of the exponential, computed once on the host (exp2 in long
// double) and copied to the device.
struct ExpConstants {
  double table[64];     // 2^(j/64), j = 0..63
  double inv_step;      // 64 / ln 2
  double step_hi;       // ln2/64 rounded to binary32 precision (so k*step_hi is exact)
  double step_lo;       // ln2/64 - step_hi
  double near_relative; // half-width of the "near a midpoint" band, relative to |y|
};

NB_HD uint32_t float_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

NB_HD float bits_float(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

#ifdef __CUDACC__
__device__ __forceinline__ double d_mul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double d_add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double d_fma(double a, double b, double c) { return __fma_rn(a, b, c); }
__device__ __forceinline__ float to_float(double y) { return __double2float_rn(y); }
#endif
inline double h_mul(double a, double b) { return a * b; }
inline double h_add(double a, double b) { return a + b; }
inline double h_fma(double a, double b, double c) { return fma(a, b, c); }
inline float h_to_float(double y) { return (float)y; }

// e^x in double for binary32 x in [-110, 89]; the caller handles the rest.
template <typename Mul, typename Add, typename Fma>
NB_HD double exp_double_core(float xf, const ExpConstants& C, Mul mul, Add add, Fma fma3) {
  double x = (double)xf;
  double kd = rint(mul(x, C.inv_step));
  int k = (int)kd;
  double r = add(x, -mul(kd, C.step_hi));  // exact: both terms carry few bits
  r = add(r, -mul(kd, C.step_lo));
  double p = 1.0 / 5040.0;
  p = fma3(p, r, 1.0 / 720.0);
  p = fma3(p, r, 1.0 / 120.0);
  p = fma3(p, r, 1.0 / 24.0);
  p = fma3(p, r, 1.0 / 6.0);
  p = fma3(p, r, 0.5);
  p = fma3(p, r, 1.0);
  p = fma3(p, r, 1.0);
  int j = k & 63;
  int m = (k - j) / 64;
  double y = mul(C.table[j], p);
  return ldexp(y, m);
}

// The two binary32 values around y and whether y is close to their midpoint.
NB_HD bool near_midpoint(double y, float f, double near_relative) {
  if (!(fabs(y) > 0.0) || isinf(f)) return false;
  float other = ((double)f < y) ? nextafterf(f, INFINITY) : nextafterf(f, -INFINITY);
  if ((double)f == y) return false;
  double mid = ((double)f + (double)other) * 0.5;
  return fabs(y - mid) <= fabs(y) * near_relative;
}

NB_HD float other_neighbour(double y, float f) { return ((double)f < y) ? nextafterf(f, INFINITY) : nextafterf(f, -INFINITY); }

// Host reference of the device exponential before the libm correction.
inline float exp_binary32_host(float x, const ExpConstants& C, double* y_out = nullptr) {
  if (isnan(x)) return x;
  if (x > 89.0f) return INFINITY;
  if (x < -110.0f) return 0.0f;
  double y = exp_double_core(x, C, h_mul, h_add, h_fma);
  if (y_out) *y_out = y;
  return h_to_float(y);
}

inline ExpConstants make_exp_constants() {
  ExpConstants C;
  const long double ln2 = 0.693147180559945309417232121458176568L;
  for (int j = 0; j < 64; ++j) C.table[j] = (double)exp2l((long double)j / 64.0L);
  C.inv_step = (double)(64.0L / ln2);
  C.step_hi = (double)(float)(ln2 / 64.0L);
  C.step_lo = (double)(ln2 / 64.0L - (long double)C.step_hi);
  C.near_relative = ldexp(1.0, -31);
  return C;
}

// Hash set of binary32 input bit patterns (open addressing, linear probing;
// 0 marks an empty slot — e^0 and e^-0 are exact and never listed).
struct ExceptionSet {
  const uint32_t* slots;
  uint32_t mask;
};

NB_HD uint32_t exception_hash(uint32_t key) { return key * 0x9E3779B1u; }

NB_HD bool exception_contains(const ExceptionSet& s, uint32_t key) {
  if (!s.slots) return false;
  uint32_t i = exception_hash(key) & s.mask;
  for (uint32_t probe = 0; probe <= s.mask; ++probe) {
    uint32_t v = s.slots[i];
    if (v == key) return true;
    if (v == 0) return false;
    i = (i + 1) & s.mask;
  }
  return false;
}

}  // namespace nbx
