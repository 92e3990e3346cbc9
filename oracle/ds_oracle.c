/*
 * CPU oracle for the double-single (DS) hot path.  TEST INFRASTRUCTURE ONLY:
 * the parity tests, the smoke check and the CPU-baseline leg of bench.py call
 * it to check results against.  The product path never links or calls it.
 *
 * Each function restates, operation for operation, a CPU handler of the
 * reference (rcast915/ds-experiment, cpp/).  The reference sources need the
 * XLA-FFI headers, which are absent here, so they cannot be compiled; this
 * restatement keeps their arithmetic and loop order exactly and drops only the
 * XLA-FFI buffer plumbing.  Build with -O2 -ffp-contract=off (see Makefile):
 * the reference is built for plain x86-64 without -mfma, so no product is ever
 * fused into an add, and this file must not be either.
 *
 * Packed DS layout: element i of an [N,2] f32 array holds hi at 2i and lo at
 * 2i+1 (cpp/ds_add.cpp:46-49,60-61).
 *
 * Every elementwise loop takes a thread count; nthreads <= 1 runs the plain
 * single-threaded loop of the reference, larger values split the index range
 * with OpenMP (elements are independent, so results are identical).
 */
#include "ds_oracle.h"

#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- scalar primitives (cpp/ds_fused_add_mul_to_f64.cpp:8-62) ---------- */

/* Knuth two_sum: cpp/ds_add.cpp:15-19. */
static inline void two_sum(float a, float b, float* s, float* e) {
  float ss = a + b;
  float bb = ss - a;
  *s = ss;
  *e = (a - (ss - bb)) + (b - bb);
}

/* Veltkamp split with C = 4097: cpp/ds_mul.cpp:15-20. */
static inline void split(float a, float* hi, float* lo) {
  const float c = 4097.0f;
  float t = c * a;
  float h = t - (t - a);
  *hi = h;
  *lo = a - h;
}

/* Dekker two_prod: cpp/ds_mul.cpp:28-34. */
static inline void two_prod(float a, float b, float* p, float* e) {
  float pp = a * b;
  float ah, al, bh, bl;
  split(a, &ah, &al);
  split(b, &bh, &bl);
  *p = pp;
  *e = ((ah * bh - pp) + ah * bl + al * bh) + al * bl;
}

/* f64 -> DS: cpp/ds_fused_add_mul_to_f64.cpp:29-32 (and ds_from_f64.cpp:35-36). */
static inline void from_double(double x, float* hi, float* lo) {
  float h = (float)x;
  *hi = h;
  *lo = (float)(x - (double)h);
}

/* DS -> f64: cpp/ds_fused_add_mul_to_f64.cpp:64-66 (and ds_to_f64.cpp:36). */
static inline double to_double(float hi, float lo) {
  return (double)hi + (double)lo;
}

/* ds_add_pair: cpp/ds_fused_add_mul_to_f64.cpp:34-48 (== cpp/ds_add.cpp:51-61). */
static inline void add_pair(float ah, float al, float bh, float bl,
                            float* oh, float* ol) {
  float s1, e1, s2, e2, t1, t2;
  two_sum(ah, bh, &s1, &e1);
  two_sum(al, bl, &s2, &e2);
  two_sum(s1, s2 + e1, &t1, &t2);
  *oh = t1;
  *ol = t2 + e2;
}

/* ds_sub body: cpp/ds_sub.cpp:51-61 (negation applied inside two_sum's operand). */
static inline void sub_pair(float ah, float al, float bh, float bl,
                            float* oh, float* ol) {
  float s1, e1, s2, e2, t1, t2;
  two_sum(ah, -bh, &s1, &e1);
  two_sum(al, -bl, &s2, &e2);
  two_sum(s1, s2 + e1, &t1, &t2);
  *oh = t1;
  *ol = t2 + e2;
}

/* ds_mul_pair: cpp/ds_fused_add_mul_to_f64.cpp:50-62 (== cpp/ds_mul.cpp:66-74).
 * out_lo = (e1 + e2) + al*bl, left to right as C evaluates it. */
static inline void mul_pair(float ah, float al, float bh, float bl,
                            float* oh, float* ol) {
  float p1, e1, s, e2;
  two_prod(ah, bh, &p1, &e1);
  float cross = ah * bl + al * bh;
  two_sum(p1, cross, &s, &e2);
  *oh = s;
  *ol = e1 + e2 + al * bl;
}

#ifdef _OPENMP
#define DSO_PARALLEL_FOR _Pragma("omp parallel for schedule(static) num_threads(nthreads) if(nthreads > 1)")
#else
#define DSO_PARALLEL_FOR
#endif

/* ---- packed [N,2] ops ---------------------------------------------------- */

/* DsAddImpl hot loop: cpp/ds_add.cpp:45-62. */
void dso_add(const float* a, const float* b, float* y, int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) {
    float h, l;
    add_pair(a[2 * i], a[2 * i + 1], b[2 * i], b[2 * i + 1], &h, &l);
    y[2 * i] = h;
    y[2 * i + 1] = l;
  }
}

/* DsSubImpl hot loop: cpp/ds_sub.cpp:45-62. */
void dso_sub(const float* a, const float* b, float* y, int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) {
    float h, l;
    sub_pair(a[2 * i], a[2 * i + 1], b[2 * i], b[2 * i + 1], &h, &l);
    y[2 * i] = h;
    y[2 * i + 1] = l;
  }
}

/* DsMulImpl hot loop: cpp/ds_mul.cpp:60-75. */
void dso_mul(const float* a, const float* b, float* y, int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) {
    float h, l;
    mul_pair(a[2 * i], a[2 * i + 1], b[2 * i], b[2 * i + 1], &h, &l);
    y[2 * i] = h;
    y[2 * i + 1] = l;
  }
}

/* ---- split / recombine --------------------------------------------------- */

/* DsFromF64Impl: cpp/ds_from_f64.cpp:34-39. */
void dso_from_f64(const double* x, float* y, int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) {
    float h, l;
    from_double(x[i], &h, &l);
    y[2 * i] = h;
    y[2 * i + 1] = l;
  }
}

/* DsToF64Impl: cpp/ds_to_f64.cpp:33-37. */
void dso_to_f64(const float* x, double* y, int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) y[i] = to_double(x[2 * i], x[2 * i + 1]);
}

/* DsFromF32Impl: cpp/ds_from_f32.cpp:29-32. */
void dso_from_f32(const float* x, float* y, int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) {
    y[2 * i] = x[i];
    y[2 * i + 1] = 0.0f;
  }
}

/* DsToF32Impl: cpp/ds_to_f32.cpp:29-30 (an f32 add of hi and lo). */
void dso_to_f32(const float* x, float* y, int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) y[i] = x[2 * i] + x[2 * i + 1];
}

/* ---- fused f64 chains ---------------------------------------------------- */

/* DsFusedAddMulImpl: cpp/ds_fused_add_mul.cpp:88-101, (x+y)*y, packed out. */
void dso_fused_add_mul(const double* x, const double* y, float* out, int64_t n,
                       int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) {
    float xh, xl, yh, yl, sh, sl, ph, pl;
    from_double(x[i], &xh, &xl);
    from_double(y[i], &yh, &yl);
    add_pair(xh, xl, yh, yl, &sh, &sl);
    mul_pair(sh, sl, yh, yl, &ph, &pl);
    out[2 * i] = ph;
    out[2 * i + 1] = pl;
  }
}

/* DsFusedAddMulToF64Impl: cpp/ds_fused_add_mul_to_f64.cpp:81-93, (x+y)*y.
 * DsFusedAxpyImpl (cpp/ds_fused_axpy.cpp:96-108) and the CUDA kernel
 * DsFusedAddMulToF64Kernel (cpp/ds_fused_add_mul_to_f64_cuda.cu:65-83) compute
 * the same chain. */
void dso_fused_add_mul_to_f64(const double* x, const double* y, double* out,
                              int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) {
    float xh, xl, yh, yl, sh, sl, ph, pl;
    from_double(x[i], &xh, &xl);
    from_double(y[i], &yh, &yl);
    add_pair(xh, xl, yh, yl, &sh, &sl);
    mul_pair(sh, sl, yh, yl, &ph, &pl);
    out[i] = to_double(ph, pl);
  }
}

/* Three-input (a+b)*c: the same helpers as DsFusedAddMulToF64Impl
 * (cpp/ds_fused_add_mul_to_f64.cpp:81-93) with the multiplier split from a
 * third input instead of reusing y. */
void dso_fused_add_mul3_to_f64(const double* a, const double* b, const double* c,
                               double* out, int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) {
    float ah, al, bh, bl, ch, cl, sh, sl, ph, pl;
    from_double(a[i], &ah, &al);
    from_double(b[i], &bh, &bl);
    from_double(c[i], &ch, &cl);
    add_pair(ah, al, bh, bl, &sh, &sl);
    mul_pair(sh, sl, ch, cl, &ph, &pl);
    out[i] = to_double(ph, pl);
  }
}

/* DsFusedAddSubToF64Kernel: cpp/ds_fused_add_sub_to_f64_cuda.cu:52-70, (x+y)-x. */
void dso_fused_add_sub_to_f64(const double* x, const double* y, double* out,
                              int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) {
    float xh, xl, yh, yl, sh, sl, rh, rl;
    from_double(x[i], &xh, &xl);
    from_double(y[i], &yh, &yl);
    add_pair(xh, xl, yh, yl, &sh, &sl);
    sub_pair(sh, sl, xh, xl, &rh, &rl);
    out[i] = to_double(rh, rl);
  }
}

/* DsRecurrenceAddMulToF64Kernel: cpp/ds_recurrence_add_mul_to_f64_cuda.cu:69-93,
 * z <- split(x); k times z = (z + y) * y; out = f64(z). */
void dso_recurrence_add_mul_to_f64(const double* x, const double* y, int32_t k,
                                   double* out, int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) {
    float zh, zl, yh, yl;
    from_double(x[i], &zh, &zl);
    from_double(y[i], &yh, &yl);
    for (int32_t it = 0; it < k; ++it) {
      float sh, sl, ph, pl;
      add_pair(zh, zl, yh, yl, &sh, &sl);
      mul_pair(sh, sl, yh, yl, &ph, &pl);
      zh = ph;
      zl = pl;
    }
    out[i] = to_double(zh, zl);
  }
}

/* x <- x*a + b, k times: ds_add(ds_mul(X, A), B) composed from the reference
 * helpers (cpp/ds_recurrence_add_mul_to_f64_cuda.cu:35-63), same loop shape
 * as DsRecurrenceAddMulToF64Kernel. */
void dso_recurrence_mul_add_to_f64(const double* x, const double* a,
                                   const double* b, int32_t k, double* out,
                                   int64_t n, int nthreads) {
  (void)nthreads;
  DSO_PARALLEL_FOR
  for (int64_t i = 0; i < n; ++i) {
    float zh, zl, ah, al, bh, bl;
    from_double(x[i], &zh, &zl);
    from_double(a[i], &ah, &al);
    from_double(b[i], &bh, &bl);
    for (int32_t it = 0; it < k; ++it) {
      float ph, pl, sh, sl;
      mul_pair(zh, zl, ah, al, &ph, &pl);
      add_pair(ph, pl, bh, bl, &sh, &sl);
      zh = sh;
      zl = sl;
    }
    out[i] = to_double(zh, zl);
  }
}

/* ---- reduce -------------------------------------------------------------- */

/* Sequential DS fold over f64 inputs split with from_double, starting from
 * (init_hi, init_lo): the reduce body of the DS pass (DsTransformPass.cpp:
 * 413-441) applied in index order, as tests/ds_ref.py:89-96 and
 * tests/test_f64_ds.py:116-120 do.  body: 0 add, 1 subtract, 2 multiply. */
void dso_reduce_f64_seq(const double* x, int64_t n, int body, float init_hi,
                        float init_lo, float* out_hi, float* out_lo) {
  float ah = init_hi, al = init_lo;
  for (int64_t i = 0; i < n; ++i) {
    float xh, xl, h, l;
    from_double(x[i], &xh, &xl);
    if (body == 0)
      add_pair(ah, al, xh, xl, &h, &l);
    else if (body == 1)
      sub_pair(ah, al, xh, xl, &h, &l);
    else
      mul_pair(ah, al, xh, xl, &h, &l);
    ah = h;
    al = l;
  }
  *out_hi = ah;
  *out_lo = al;
}

/* The same fold over SoA (hi, lo) f32 inputs. */
void dso_reduce_ds_seq(const float* hi, const float* lo, int64_t n, int body,
                       float init_hi, float init_lo, float* out_hi,
                       float* out_lo) {
  float ah = init_hi, al = init_lo;
  for (int64_t i = 0; i < n; ++i) {
    float h, l;
    if (body == 0)
      add_pair(ah, al, hi[i], lo[i], &h, &l);
    else if (body == 1)
      sub_pair(ah, al, hi[i], lo[i], &h, &l);
    else
      mul_pair(ah, al, hi[i], lo[i], &h, &l);
    ah = h;
    al = l;
  }
  *out_hi = ah;
  *out_lo = al;
}

/* Sequential DS dot product with exact products, tests/ds_ref.py:69-86:
 * acc = ds_add(acc, two_prod(a_i, b_i)) over f32 inputs. */
void dso_dot_f32_seq(const float* a, const float* b, int64_t n, float* out_hi,
                     float* out_lo) {
  float ah = 0.0f, al = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    float ph, pl, h, l;
    two_prod(a[i], b[i], &ph, &pl);
    add_pair(ah, al, ph, pl, &h, &l);
    ah = h;
    al = l;
  }
  *out_hi = ah;
  *out_lo = al;
}

/* Scalar primitives exposed for the golden-vector pins. */
void dso_two_sum(const float* a, const float* b, float* s, float* e, int64_t n) {
  for (int64_t i = 0; i < n; ++i) two_sum(a[i], b[i], &s[i], &e[i]);
}

void dso_two_prod(const float* a, const float* b, float* p, float* e, int64_t n) {
  for (int64_t i = 0; i < n; ++i) two_prod(a[i], b[i], &p[i], &e[i]);
}

void dso_split(const float* a, float* hi, float* lo, int64_t n) {
  for (int64_t i = 0; i < n; ++i) split(a[i], &hi[i], &lo[i]);
}

int dso_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
