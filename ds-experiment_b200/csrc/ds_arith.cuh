// Double-single (DS) arithmetic on the device.
//
// Every operation is an explicit round-to-nearest intrinsic (__fadd_rn,
// __fsub_rn, __fmul_rn, __dsub_rn, __dadd_rn), which nvcc never contracts into
// an FMA.  The library is additionally built with --fmad=false.  With the
// same IEEE operations in the same order as the reference's CPU handlers
// (x86-64, SSE, no FMA), results are bit-identical to them, subnormals
// included (no flush-to-zero: the library is built without fast-math).
//
// Operation order follows the reference helpers in
// cpp/ds_fused_add_mul_to_f64.cpp:8-66 (two_sum, split, two_prod,
// ds_from_double, ds_add_pair, ds_mul_pair, ds_to_double) and the subtract
// body of cpp/ds_sub.cpp:51-61.
#pragma once

#include <cuda_runtime.h>

namespace dsb {

struct ds2 {
  float hi, lo;
};

// Knuth's error-free sum: s = fl(a + b), e = (a + b) - s exactly.
__device__ __forceinline__ void two_sum(float a, float b, float& s, float& e) {
  s = __fadd_rn(a, b);
  const float bb = __fsub_rn(s, a);
  e = __fadd_rn(__fsub_rn(a, __fsub_rn(s, bb)), __fsub_rn(b, bb));
}

// Veltkamp split with C = 2^12 + 1 into two 12-bit halves.
__device__ __forceinline__ void split(float a, float& hi, float& lo) {
  const float t = __fmul_rn(4097.0f, a);
  hi = __fsub_rn(t, __fsub_rn(t, a));
  lo = __fsub_rn(a, hi);
}

// Dekker's error-free product with the Veltkamp split:
// e = ((ah*bh - p) + ah*bl + al*bh) + al*bl, evaluated left to right.
__device__ __forceinline__ void two_prod(float a, float b, float& p, float& e) {
  p = __fmul_rn(a, b);
  float ah, al, bh, bl;
  split(a, ah, al);
  split(b, bh, bl);
  float t = __fsub_rn(__fmul_rn(ah, bh), p);
  t = __fadd_rn(t, __fmul_rn(ah, bl));
  t = __fadd_rn(t, __fmul_rn(al, bh));
  e = __fadd_rn(t, __fmul_rn(al, bl));
}

// The same product when b's split (bh, bl) is already known (loop-invariant
// operands of the recurrences).  Bit-identical to two_prod(a, b).
__device__ __forceinline__ void two_prod_bsplit(float a, float b, float bh,
                                                float bl, float& p, float& e) {
  p = __fmul_rn(a, b);
  float ah, al;
  split(a, ah, al);
  float t = __fsub_rn(__fmul_rn(ah, bh), p);
  t = __fadd_rn(t, __fmul_rn(ah, bl));
  t = __fadd_rn(t, __fmul_rn(al, bh));
  e = __fadd_rn(t, __fmul_rn(al, bl));
}

// Dekker's error term of p = a * b with b's split (bh, bl) known: the error
// half of two_prod_bsplit.
__device__ __forceinline__ float dekker_err_bsplit(float a, float bh, float bl, float p) {
  float ah, al;
  split(a, ah, al);
  float t = __fsub_rn(__fmul_rn(ah, bh), p);
  t = __fadd_rn(t, __fmul_rn(ah, bl));
  t = __fadd_rn(t, __fmul_rn(al, bh));
  return __fadd_rn(t, __fmul_rn(al, bl));
}

// Where an FMA gives Dekker's bits.  For |a|, |b| < 2^115 and
// 2^-90 <= |p| <= 2^120 neither split overflows and every partial product
// of Dekker's algorithm is exact (their lowest bits lie at or above 2^-138,
// on the subnormal grid), so Dekker's e is the exact error a*b - p, which
// is what __fmaf_rn(a, b, -p) returns.  With |b| in [2^-5, 2^115) (checked
// once per loop-invariant b), |p| in [2^-90, 2^110] implies |a| < 2^115.
__device__ __forceinline__ bool fma_b_range(float b) {
  const float ab = fabsf(b);
  return ab >= 0x1p-5f && ab < 0x1p115f;
}
__device__ __forceinline__ bool fma_p_range(float p) {
  const float ap = fabsf(p);
  return ap >= 0x1p-90f && ap <= 0x1p110f;
}

// f64 -> DS: hi = f32(x), lo = f32(x - f64(hi)).
__device__ __forceinline__ ds2 from_f64(double x) {
  ds2 r;
  r.hi = __double2float_rn(x);
  r.lo = __double2float_rn(__dsub_rn(x, static_cast<double>(r.hi)));
  return r;
}

// DS -> f64: f64(hi) + f64(lo).
__device__ __forceinline__ double to_f64(ds2 a) {
  return __dadd_rn(static_cast<double>(a.hi), static_cast<double>(a.lo));
}

// ds_add: no final renormalisation, exactly as the reference.
__device__ __forceinline__ ds2 add(ds2 a, ds2 b) {
  float s1, e1, s2, e2, t1, t2;
  two_sum(a.hi, b.hi, s1, e1);
  two_sum(a.lo, b.lo, s2, e2);
  two_sum(s1, __fadd_rn(s2, e1), t1, t2);
  return ds2{t1, __fadd_rn(t2, e2)};
}

// ds_sub: ds_add with the negation inside two_sum's operands.
__device__ __forceinline__ ds2 sub(ds2 a, ds2 b) {
  float s1, e1, s2, e2, t1, t2;
  two_sum(a.hi, -b.hi, s1, e1);
  two_sum(a.lo, -b.lo, s2, e2);
  two_sum(s1, __fadd_rn(s2, e1), t1, t2);
  return ds2{t1, __fadd_rn(t2, e2)};
}

// ds_mul: out_lo = (e1 + e2) + al*bl.
__device__ __forceinline__ ds2 mul(ds2 a, ds2 b) {
  float p1, e1, s, e2;
  two_prod(a.hi, b.hi, p1, e1);
  const float cross = __fadd_rn(__fmul_rn(a.hi, b.lo), __fmul_rn(a.lo, b.hi));
  two_sum(p1, cross, s, e2);
  return ds2{s, __fadd_rn(__fadd_rn(e1, e2), __fmul_rn(a.lo, b.lo))};
}

// ds_mul with b's Veltkamp split of b.hi precomputed (bh, bl).
__device__ __forceinline__ ds2 mul_bsplit(ds2 a, ds2 b, float bh, float bl) {
  float p1, e1, s, e2;
  two_prod_bsplit(a.hi, b.hi, bh, bl, p1, e1);
  const float cross = __fadd_rn(__fmul_rn(a.hi, b.lo), __fmul_rn(a.lo, b.hi));
  two_sum(p1, cross, s, e2);
  return ds2{s, __fadd_rn(__fadd_rn(e1, e2), __fmul_rn(a.lo, b.lo))};
}

// ds_mul after its head product: p1 = a.hi * b.hi and its exact error e1
// given, the rest of mul() in the same order (the same bits).
__device__ __forceinline__ ds2 mul_finish(ds2 a, ds2 b, float p1, float e1) {
  float s, e2;
  const float cross = __fadd_rn(__fmul_rn(a.hi, b.lo), __fmul_rn(a.lo, b.hi));
  two_sum(p1, cross, s, e2);
  return ds2{s, __fadd_rn(__fadd_rn(e1, e2), __fmul_rn(a.lo, b.lo))};
}

// Apply a reduction body (0 add, 1 subtract, 2 multiply).
__device__ __forceinline__ ds2 apply_body(int body, ds2 acc, ds2 x) {
  return body == 2 ? mul(acc, x) : (body == 1 ? sub(acc, x) : add(acc, x));
}

}  // namespace dsb
