/* CPU oracle for the DS hot path (test infrastructure only; see ds_oracle.c). */
#ifndef DS_ORACLE_H
#define DS_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void dso_add(const float* a, const float* b, float* y, int64_t n, int nthreads);
void dso_sub(const float* a, const float* b, float* y, int64_t n, int nthreads);
void dso_mul(const float* a, const float* b, float* y, int64_t n, int nthreads);
void dso_from_f64(const double* x, float* y, int64_t n, int nthreads);
void dso_to_f64(const float* x, double* y, int64_t n, int nthreads);
void dso_from_f32(const float* x, float* y, int64_t n, int nthreads);
void dso_to_f32(const float* x, float* y, int64_t n, int nthreads);
void dso_fused_add_mul(const double* x, const double* y, float* out, int64_t n,
                       int nthreads);
void dso_fused_add_mul_to_f64(const double* x, const double* y, double* out,
                              int64_t n, int nthreads);
void dso_fused_add_mul3_to_f64(const double* a, const double* b, const double* c,
                               double* out, int64_t n, int nthreads);
void dso_fused_add_sub_to_f64(const double* x, const double* y, double* out,
                              int64_t n, int nthreads);
void dso_recurrence_add_mul_to_f64(const double* x, const double* y, int32_t k,
                                   double* out, int64_t n, int nthreads);
void dso_recurrence_mul_add_to_f64(const double* x, const double* a,
                                   const double* b, int32_t k, double* out,
                                   int64_t n, int nthreads);
void dso_reduce_f64_seq(const double* x, int64_t n, int body, float init_hi,
                        float init_lo, float* out_hi, float* out_lo);
void dso_reduce_ds_seq(const float* hi, const float* lo, int64_t n, int body,
                       float init_hi, float init_lo, float* out_hi,
                       float* out_lo);
void dso_dot_f32_seq(const float* a, const float* b, int64_t n, float* out_hi,
                     float* out_lo);
void dso_two_sum(const float* a, const float* b, float* s, float* e, int64_t n);
void dso_two_prod(const float* a, const float* b, float* p, float* e, int64_t n);
void dso_split(const float* a, float* hi, float* lo, int64_t n);
int dso_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
