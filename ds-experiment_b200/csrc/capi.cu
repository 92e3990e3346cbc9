// The C ABI of libds_b200 (declared in include/ds_b200.h): shape checks with
// the reference handlers' messages, then the launchers in kernels.h.
#include <cstring>
#include <mutex>
#include <algorithm>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace dsb {

namespace {
thread_local std::string g_last_error;
}

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int ok() { return DS_OK; }

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= static_cast<int>(cache.size())) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

namespace {

int invalid(const std::string& msg) { return set_error(DS_INVALID_ARGUMENT, msg); }

bool valid_buffer(const ds_buffer* b) {
  return b != nullptr && b->rank >= 0 && b->rank <= 16 && (b->rank == 0 || b->dims != nullptr);
}

// Product of all dims but the last (cpp/ds_add.cpp:8-13); 1 for rank <= 1.
int64_t batch_size(const ds_buffer* b) {
  int64_t n = 1;
  for (int64_t i = 0; i + 1 < b->rank; ++i) n *= b->dims[i];
  return n;
}

int64_t last_dim(const ds_buffer* b) { return b->rank > 0 ? b->dims[b->rank - 1] : 1; }

int64_t total(const ds_buffer* b) {
  int64_t n = 1;
  for (int64_t i = 0; i < b->rank; ++i) n *= b->dims[i];
  return n;
}

bool bad_dims(const ds_buffer* b) {
  for (int64_t i = 0; i < b->rank; ++i)
    if (b->dims[i] < 0) return true;
  return false;
}

int check_buffers(std::initializer_list<const ds_buffer*> bufs, const char* op) {
  for (const ds_buffer* b : bufs) {
    if (!valid_buffer(b) || bad_dims(b)) return invalid(std::string(op) + ": invalid buffer descriptor");
  }
  for (const ds_buffer* b : bufs) {
    if (total(b) > 0 && b->data == nullptr) return invalid(std::string(op) + ": null data pointer");
  }
  return DS_OK;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Shape checks of DsAdd / DsSub / DsMul (cpp/ds_add.cpp:30-38).
int packed_binary(const char* op, int which, const ds_buffer* a, const ds_buffer* b,
                  const ds_buffer* y, void* stream) {
  if (int st = check_buffers({a, b, y}, op)) return st;
  const std::string name(op);
  if (a->rank == 0 || b->rank == 0 || last_dim(a) != 2 || last_dim(b) != 2)
    return invalid(name + " expects last dim == 2");
  if (a->rank != b->rank || batch_size(a) != batch_size(b))
    return invalid(name + " input shapes must match");
  if (y->rank == 0 || last_dim(y) != 2 || batch_size(y) != batch_size(a))
    return invalid(name + " output shape mismatch");
  return ew_packed(which, static_cast<const float*>(a->data), static_cast<const float*>(b->data),
                   static_cast<float*>(y->data), batch_size(a), as_stream(stream));
}

// Shape checks of the rank-1 fused handlers (cpp/ds_fused_add_mul_to_f64.cpp:
// 77-86): rank-1 inputs of equal length, output [N] (or [N,2] when packed).
int fused_checks(const char* op, std::initializer_list<const ds_buffer*> ins,
                 const ds_buffer* out, bool packed_out) {
  std::vector<const ds_buffer*> all(ins);
  all.push_back(out);
  for (const ds_buffer* b : all)
    if (!valid_buffer(b) || bad_dims(b)) return invalid(std::string(op) + ": invalid buffer descriptor");
  for (const ds_buffer* b : ins)
    if (b->rank != 1) return invalid(std::string(op) + " expects rank-1 inputs");
  const int64_t n = (*ins.begin())->dims[0];
  for (const ds_buffer* b : ins)
    if (b->dims[0] != n) return invalid("input lengths must match");
  if (packed_out) {
    if (out->rank != 2 || out->dims[0] != n || out->dims[1] != 2)
      return invalid("output shape must be [N,2]");
  } else if (out->rank != 1 || out->dims[0] != n) {
    return invalid("output shape must be [N]");
  }
  for (const ds_buffer* b : all)
    if (n > 0 && b->data == nullptr) return invalid(std::string(op) + ": null data pointer");
  return DS_OK;
}

const double* f64p(const ds_buffer* b) { return static_cast<const double*>(b->data); }

// [outer, red, inner] view of a reduce over contiguous ascending dims.
int reduce_geometry(const char* op, const ds_buffer* in, const int64_t* dims, int64_t nd,
                    const ds_buffer* out, int64_t& outer, int64_t& red, int64_t& inner) {
  if (nd < 0 || (nd > 0 && dims == nullptr)) return invalid(std::string(op) + ": invalid dimensions");
  for (int64_t i = 0; i < nd; ++i) {
    if (dims[i] < 0 || dims[i] >= in->rank)
      return invalid(std::string(op) + ": reduce dimension out of range");
    if (i > 0 && dims[i] != dims[i - 1] + 1)
      return invalid(std::string(op) +
                     ": reduce dimensions must be contiguous and ascending");
  }
  outer = 1;
  red = 1;
  inner = 1;
  const int64_t d0 = nd > 0 ? dims[0] : in->rank;
  for (int64_t i = 0; i < in->rank; ++i) {
    if (i < d0)
      outer *= in->dims[i];
    else if (i < d0 + nd)
      red *= in->dims[i];
    else
      inner *= in->dims[i];
  }
  // Output shape: the input shape without the reduced dims.
  if (out->rank != in->rank - nd) return invalid(std::string(op) + ": output shape mismatch");
  for (int64_t i = 0, o = 0; i < in->rank; ++i) {
    if (i >= d0 && i < d0 + nd) continue;
    if (out->dims[o++] != in->dims[i]) return invalid(std::string(op) + ": output shape mismatch");
  }
  return DS_OK;
}

// One operand of dot_general as the products read it: its dimensions
// grouped into batch (in the order of the batching list), free (ascending:
// the result's order) and contracting (in the order of the contracting
// list, which pairs them with the other operand's).  Each group is one
// index, (batch, rows, K), with one element stride when the group's
// dimensions nest (each outer stride = inner stride x inner size, unit
// dimensions ignored); otherwise the operand is first copied to a
// contiguous [batch][rows][K] buffer in the workspace.
struct DotSide {
  int64_t batch = 1, rows = 1, K = 1;
  int64_t s_b = 0, s_r = 0, s_k = 0;
  bool nested = true;
  int nd = 0;                       // the copy: dimensions in group order ...
  int64_t size[DS_DOT_MAX_DIMS];    // ... their sizes
  int64_t stride[DS_DOT_MAX_DIMS];  // ... and strides in the operand
};

struct DotGeom {
  int64_t batch = 1, M = 1, N = 1, K = 1;
  DotSide a, b;
};

// Sizes and strides of `idx` (n dimensions of x) nested into one index.
bool nest(const int64_t* dims, const int64_t* strides, const int64_t* idx, int64_t n,
          int64_t& size, int64_t& stride) {
  size = 1;
  stride = 0;
  bool ok = true;
  for (int64_t t = n - 1; t >= 0; --t) {
    const int64_t len = dims[idx[t]];
    if (len == 1) continue;
    if (size == 1) {
      stride = strides[idx[t]];
    } else if (strides[idx[t]] != stride * size) {
      ok = false;
    }
    size *= len;
  }
  return ok;
}

int dot_side(const ds_buffer* x, const int64_t* batch, int64_t nb, const int64_t* contracting,
             int64_t nc, DotSide& d, std::vector<int64_t>& free_dims) {
  const int64_t r = x->rank;
  if (r > DS_DOT_MAX_DIMS)
    return invalid("dot_general: operands of rank above " + std::to_string(DS_DOT_MAX_DIMS) +
                   " are not supported");
  int64_t strides[DS_DOT_MAX_DIMS];
  for (int64_t i = r - 1, s = 1; i >= 0; --i) {
    strides[i] = s;
    s *= x->dims[i];
  }
  int role[DS_DOT_MAX_DIMS] = {0};  // 0 free, 1 batch, 2 contracting
  for (int64_t i = 0; i < nb; ++i) {
    if (batch[i] < 0 || batch[i] >= r || role[batch[i]])
      return invalid("dot_general: batching dimensions out of range or repeated");
    role[batch[i]] = 1;
  }
  for (int64_t i = 0; i < nc; ++i) {
    if (contracting[i] < 0 || contracting[i] >= r || role[contracting[i]])
      return invalid("dot_general: contracting dimensions out of range or repeated");
    role[contracting[i]] = 2;
  }
  free_dims.clear();
  for (int64_t i = 0; i < r; ++i)
    if (role[i] == 0) free_dims.push_back(i);
  bool ok = nest(x->dims, strides, batch, nb, d.batch, d.s_b);
  ok = nest(x->dims, strides, free_dims.data(), static_cast<int64_t>(free_dims.size()), d.rows,
            d.s_r) && ok;
  ok = nest(x->dims, strides, contracting, nc, d.K, d.s_k) && ok;
  d.nested = ok;
  d.nd = 0;
  auto add = [&](int64_t dim) {
    d.size[d.nd] = x->dims[dim];
    d.stride[d.nd] = strides[dim];
    ++d.nd;
  };
  for (int64_t i = 0; i < nb; ++i) add(batch[i]);
  for (int64_t dim : free_dims) add(dim);
  for (int64_t i = 0; i < nc; ++i) add(contracting[i]);
  return DS_OK;
}

int dot_geometry(const ds_buffer* lhs, const ds_buffer* rhs, const ds_dot_dims* dd,
                 const ds_buffer* out, DotGeom& g) {
  if (dd == nullptr) return invalid("dot_general: missing dimension numbers");
  const int64_t nb = dd->n_batch, nc = dd->n_contracting;
  if (nb < 0 || nb > DS_DOT_MAX_DIMS || nc < 0 || nc > DS_DOT_MAX_DIMS)
    return invalid("dot_general: bad count of batching or contracting dimensions");
  std::vector<int64_t> lfree, rfree;
  if (int st = dot_side(lhs, dd->lhs_batch, nb, dd->lhs_contracting, nc, g.a, lfree)) return st;
  if (int st = dot_side(rhs, dd->rhs_batch, nb, dd->rhs_contracting, nc, g.b, rfree)) return st;
  // The contracting pairs may be taken in any order (the sum does not
  // depend on it): of the given order and the pairs sorted by the lhs or the
  // rhs dimension, the one whose operands nest best (fewest copies) is used.
  if (nc > 1 && !(g.a.nested && g.b.nested)) {
    auto copies = [](const DotSide& a, const DotSide& b) {
      return (a.nested ? 0 : a.batch * a.rows * a.K) + (b.nested ? 0 : b.batch * b.rows * b.K);
    };
    int64_t best = copies(g.a, g.b);
    for (int by = 0; by < 2; ++by) {
      std::vector<int64_t> order(nc);
      for (int64_t i = 0; i < nc; ++i) order[i] = i;
      const int64_t* key = by == 0 ? dd->lhs_contracting : dd->rhs_contracting;
      std::sort(order.begin(), order.end(), [key](int64_t x, int64_t y) { return key[x] < key[y]; });
      int64_t lc[DS_DOT_MAX_DIMS], rc[DS_DOT_MAX_DIMS];
      for (int64_t i = 0; i < nc; ++i) {
        lc[i] = dd->lhs_contracting[order[i]];
        rc[i] = dd->rhs_contracting[order[i]];
      }
      DotSide a, b;
      std::vector<int64_t> f1, f2;
      dot_side(lhs, dd->lhs_batch, nb, lc, nc, a, f1);
      dot_side(rhs, dd->rhs_batch, nb, rc, nc, b, f2);
      if (copies(a, b) < best) {
        best = copies(a, b);
        g.a = a;
        g.b = b;
      }
    }
  }
  for (int64_t i = 0; i < nb; ++i)
    if (lhs->dims[dd->lhs_batch[i]] != rhs->dims[dd->rhs_batch[i]])
      return invalid("dot_general: batch dimensions must match");
  for (int64_t i = 0; i < nc; ++i)
    if (lhs->dims[dd->lhs_contracting[i]] != rhs->dims[dd->rhs_contracting[i]])
      return invalid("dot_general: contracting dimensions must match");
  g.batch = g.a.batch;
  g.M = g.a.rows;
  g.N = g.b.rows;
  g.K = g.a.K;
  // Result: [batch (lhs order)..., lhs free..., rhs free...], row-major.
  std::vector<int64_t> want;
  for (int64_t i = 0; i < nb; ++i) want.push_back(lhs->dims[dd->lhs_batch[i]]);
  for (int64_t d : lfree) want.push_back(lhs->dims[d]);
  for (int64_t d : rfree) want.push_back(rhs->dims[d]);
  if (out->rank != static_cast<int64_t>(want.size())) return invalid("dot_general: output shape mismatch");
  for (size_t i = 0; i < want.size(); ++i)
    if (out->dims[i] != want[i]) return invalid("dot_general: output shape mismatch");
  return DS_OK;
}

// Bytes of the contiguous copy of a side that does not nest (8 per element:
// one f64, or an f32 hi and an f32 lo), 256-byte aligned.
size_t side_copy_bytes(const DotSide& d, int64_t rows) {
  if (d.nested) return 0;
  const size_t n = static_cast<size_t>(d.batch) * rows * d.K;
  return (n * 8 + 255) / 256 * 256;
}

size_t dot_workspace(const DotGeom& g, int32_t algorithm) {
  const size_t copies = side_copy_bytes(g.a, g.M) + side_copy_bytes(g.b, g.N);
  if (g.M == 1 && g.N == 1) return copies + dot_vec_workspace_bytes(g.batch, g.K);
  if (algorithm == DS_DOT_TENSOR_INT8 && dot_ozaki_supported(g.M, g.N, g.K))
    return copies + dot_ozaki_workspace_bytes(g.batch, g.M, g.N, g.K);
  return copies;
}

// Copy a side that does not nest into [batch][rows][K] at `at`, and point
// the operand there.
int place_side(const DotSide& d, int64_t rows, DotOperand& o, uint8_t*& at, cudaStream_t s) {
  if (d.nested) {
    o.s_b = d.s_b;
    o.s_r = d.s_r;
    o.s_k = d.s_k;
    return DS_OK;
  }
  const size_t n = static_cast<size_t>(d.batch) * rows * d.K;
  if (o.f64) {
    double* dst = reinterpret_cast<double*>(at);
    if (int st = gather_strided(o.f64, dst, 8, d.size, d.stride, d.nd, s)) return st;
    o.f64 = dst;
  } else {
    float* hi = reinterpret_cast<float*>(at);
    float* lo = hi + n;
    if (int st = gather_strided(o.hi, hi, 4, d.size, d.stride, d.nd, s)) return st;
    if (int st = gather_strided(o.lo, lo, 4, d.size, d.stride, d.nd, s)) return st;
    o.hi = hi;
    o.lo = lo;
  }
  o.s_b = rows * d.K;
  o.s_r = d.K;
  o.s_k = 1;
  at += side_copy_bytes(d, rows);
  return DS_OK;
}

int dot_run(const DotGeom& g, DotProblem& p, int32_t algorithm, void* ws, size_t ws_bytes,
            cudaStream_t s) {
  if (algorithm != DS_DOT_TENSOR_INT8 && algorithm != DS_DOT_CUDA_CORE)
    return invalid("dot_general: unknown algorithm");
  p.batch = g.batch;
  p.M = g.M;
  p.N = g.N;
  p.K = g.K;
  if (g.batch * g.M * g.N == 0) return ok();
  const size_t copies = side_copy_bytes(g.a, g.M) + side_copy_bytes(g.b, g.N);
  if (copies > ws_bytes || (copies && !aligned(ws, 256)))
    return invalid("dot_general: workspace too small (need " +
                   std::to_string(dot_workspace(g, algorithm)) + " bytes, 256-byte aligned)");
  uint8_t* at = static_cast<uint8_t*>(ws);
  if (int st = place_side(g.a, g.M, p.a, at, s)) return st;
  if (int st = place_side(g.b, g.N, p.b, at, s)) return st;
  ws = at;
  ws_bytes -= copies;
  if (g.M == 1 && g.N == 1) return dot_batched_vec(p, ws, ws_bytes, s);
  if (algorithm == DS_DOT_TENSOR_INT8 && dot_ozaki_supported(g.M, g.N, g.K))
    return dot_ozaki(p, ws, ws_bytes, s);
  return dot_simt(p, s);
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" {

const char* ds_last_error(void) { return g_last_error.c_str(); }

const char* ds_version(void) { return "ds_b200 0.1 (sm_100a)"; }

int ds_dot_tensor_kernel_info(int32_t* cta_pairs, int32_t* query_error) {
  int p = 0, e = 0;
  const int st = dot_ozaki_kernel_info(&p, &e);
  if (cta_pairs) *cta_pairs = p;
  if (query_error) *query_error = e;
  return st;
}

int ds_dot_tensor_plan(int64_t K, int32_t* moduli, int32_t* bits) {
  if (K < 1) return invalid("ds_dot_tensor_plan: K must be positive");
  int m = 0, b = 0;
  dot_ozaki_params(K, &m, &b);
  if (moduli) *moduli = m;
  if (bits) *bits = b;
  return DS_OK;
}

int ds_from_f64(const ds_buffer* x, const ds_buffer* y, void* stream) {
  if (int st = check_buffers({x, y}, "ds_from_f64")) return st;
  if (y->rank == 0 || last_dim(y) != 2) return invalid("ds_from_f64 output last dim must be 2");
  const int64_t n = batch_size(x) * last_dim(x);
  if (batch_size(y) != n) return invalid("ds_from_f64 shape mismatch");
  return ew_from_f64(f64p(x), static_cast<float*>(y->data), n, as_stream(stream));
}

int ds_to_f64(const ds_buffer* x, const ds_buffer* y, void* stream) {
  if (int st = check_buffers({x, y}, "ds_to_f64")) return st;
  if (x->rank == 0 || last_dim(x) != 2) return invalid("ds_to_f64 input last dim must be 2");
  if (batch_size(x) != batch_size(y) * last_dim(y)) return invalid("ds_to_f64 shape mismatch");
  return ew_to_f64(static_cast<const float*>(x->data), static_cast<double*>(y->data),
                   batch_size(x), as_stream(stream));
}

int ds_from_f32(const ds_buffer* x, const ds_buffer* y, void* stream) {
  if (int st = check_buffers({x, y}, "ds_from_f32")) return st;
  if (y->rank == 0 || last_dim(y) != 2) return invalid("ds_from_f32 output last dim must be 2");
  if (total(x) * 2 != total(y)) return invalid("ds_from_f32 shape mismatch");
  return ew_from_f32(static_cast<const float*>(x->data), static_cast<float*>(y->data), total(x),
                     as_stream(stream));
}

int ds_to_f32(const ds_buffer* x, const ds_buffer* y, void* stream) {
  if (int st = check_buffers({x, y}, "ds_to_f32")) return st;
  if (x->rank == 0 || last_dim(x) != 2) return invalid("ds_to_f32 input last dim must be 2");
  if (total(x) != total(y) * 2) return invalid("ds_to_f32 shape mismatch");
  return ew_to_f32(static_cast<const float*>(x->data), static_cast<float*>(y->data), total(y),
                   as_stream(stream));
}

int ds_add(const ds_buffer* a, const ds_buffer* b, const ds_buffer* y, void* stream) {
  return packed_binary("ds.add", 0, a, b, y, stream);
}

int ds_sub(const ds_buffer* a, const ds_buffer* b, const ds_buffer* y, void* stream) {
  return packed_binary("ds.sub", 1, a, b, y, stream);
}

int ds_mul(const ds_buffer* a, const ds_buffer* b, const ds_buffer* y, void* stream) {
  return packed_binary("ds.mul", 2, a, b, y, stream);
}

int ds_fused_add_mul(const ds_buffer* x, const ds_buffer* y, const ds_buffer* out,
                     void* stream) {
  if (int st = fused_checks("ds.fused_add_mul", {x, y}, out, true)) return st;
  return ew_fused_add_mul_packed(f64p(x), f64p(y), static_cast<float*>(out->data), x->dims[0],
                                 as_stream(stream));
}

static int fused_add_mul_f64(const char* op, const ds_buffer* x, const ds_buffer* y,
                             const ds_buffer* out, void* stream) {
  if (int st = fused_checks(op, {x, y}, out, false)) return st;
  return ew_fused_add_mul_f64(f64p(x), f64p(y), static_cast<double*>(out->data), x->dims[0],
                              as_stream(stream));
}

int ds_fused_add_mul_to_f64(const ds_buffer* x, const ds_buffer* y, const ds_buffer* out,
                            void* stream) {
  return fused_add_mul_f64("ds.fused_add_mul_to_f64", x, y, out, stream);
}

int ds_fused_axpy(const ds_buffer* x, const ds_buffer* y, const ds_buffer* out, void* stream) {
  return fused_add_mul_f64("ds_fused_axpy", x, y, out, stream);
}

int ds_fused_add_mul_to_f64_cuda(const ds_buffer* x, const ds_buffer* y, const ds_buffer* out,
                                 void* stream) {
  return fused_add_mul_f64("ds_fused_add_mul_to_f64_cuda", x, y, out, stream);
}

int ds_fused_add_sub_to_f64_cuda(const ds_buffer* x, const ds_buffer* y, const ds_buffer* out,
                                 void* stream) {
  if (int st = fused_checks("ds_fused_add_sub_to_f64_cuda", {x, y}, out, false)) return st;
  return ew_fused_add_sub_f64(f64p(x), f64p(y), static_cast<double*>(out->data), x->dims[0],
                              as_stream(stream));
}

int ds_recurrence_add_mul_to_f64_cuda(const ds_buffer* x, const ds_buffer* y, int32_t k,
                                      const ds_buffer* out, void* stream) {
  if (int st = fused_checks("ds_recurrence_add_mul_to_f64_cuda", {x, y}, out, false)) return st;
  if (k < 0) return invalid("k must be nonnegative");
  return ew_recurrence_add_mul(f64p(x), f64p(y), static_cast<double*>(out->data), x->dims[0], k,
                               as_stream(stream));
}

int ds_fused_add_mul3_to_f64(const ds_buffer* a, const ds_buffer* b, const ds_buffer* c,
                             const ds_buffer* out, void* stream) {
  if (int st = fused_checks("ds_fused_add_mul3_to_f64", {a, b, c}, out, false)) return st;
  return ew_fused_add_mul3_f64(f64p(a), f64p(b), f64p(c), static_cast<double*>(out->data),
                               a->dims[0], as_stream(stream));
}

int ds_recurrence_mul_add_to_f64(const ds_buffer* x, const ds_buffer* a, const ds_buffer* b,
                                 int32_t k, const ds_buffer* out, void* stream) {
  if (int st = fused_checks("ds_recurrence_mul_add_to_f64", {x, a, b}, out, false)) return st;
  if (k < 0) return invalid("k must be nonnegative");
  return ew_recurrence_mul_add(f64p(x), f64p(a), f64p(b), static_cast<double*>(out->data),
                               x->dims[0], k, as_stream(stream));
}

size_t ds_reduce_workspace_size(const ds_buffer* in, const int64_t* dimensions,
                                int64_t n_dimensions) {
  if (!valid_buffer(in) || bad_dims(in)) return 0;
  if (n_dimensions < 0 || (n_dimensions > 0 && dimensions == nullptr)) return 0;
  for (int64_t i = 0; i < n_dimensions; ++i)
    if (dimensions[i] < 0 || dimensions[i] >= in->rank) return 0;
  const int64_t d0 = n_dimensions > 0 ? dimensions[0] : in->rank;
  int64_t outer = 1, red = 1, inner = 1;
  for (int64_t i = 0; i < in->rank; ++i) {
    if (i < d0)
      outer *= in->dims[i];
    else if (i < d0 + n_dimensions)
      red *= in->dims[i];
    else
      inner *= in->dims[i];
  }
  return reduce_workspace_bytes(outer, red, inner);
}

static int reduce_common(const char* op, const ds_buffer* in, const int64_t* dimensions,
                         int64_t n_dimensions, int32_t body, const ds_buffer* out,
                         ReduceArgs& args) {
  if (body < DS_BODY_ADD || body > DS_BODY_MUL) return invalid(std::string(op) + ": unknown body");
  return reduce_geometry(op, in, dimensions, n_dimensions, out, args.outer, args.red, args.inner);
}

int ds_reduce(const ds_buffer* in_hi, const ds_buffer* in_lo, const ds_buffer* init_hi,
              const ds_buffer* init_lo, const int64_t* dimensions, int64_t n_dimensions,
              int32_t body, const ds_buffer* out_hi, const ds_buffer* out_lo, void* workspace,
              size_t workspace_bytes, void* stream) {
  if (int st = check_buffers({in_hi, in_lo, init_hi, init_lo, out_hi, out_lo}, "ds_reduce"))
    return st;
  if (in_hi->rank != in_lo->rank || total(in_hi) != total(in_lo))
    return invalid("ds_reduce: hi and lo inputs must have the same shape");
  if (out_hi->rank != out_lo->rank || total(out_hi) != total(out_lo))
    return invalid("ds_reduce: hi and lo outputs must have the same shape");
  if (total(init_hi) != 1 || total(init_lo) != 1)
    return invalid("ds_reduce: init values must be scalars");
  ReduceArgs a;
  if (int st = reduce_common("ds_reduce", in_hi, dimensions, n_dimensions, body, out_hi, a))
    return st;
  a.in_hi = static_cast<const float*>(in_hi->data);
  a.in_lo = static_cast<const float*>(in_lo->data);
  a.init_hi = static_cast<const float*>(init_hi->data);
  a.init_lo = static_cast<const float*>(init_lo->data);
  a.out_hi = static_cast<float*>(out_hi->data);
  a.out_lo = static_cast<float*>(out_lo->data);
  a.body = body;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return reduce_launch(a, as_stream(stream));
}

int ds_reduce_f64(const ds_buffer* in, const ds_buffer* init, const int64_t* dimensions,
                  int64_t n_dimensions, int32_t body, const ds_buffer* out, void* workspace,
                  size_t workspace_bytes, void* stream) {
  if (int st = check_buffers({in, init, out}, "ds_reduce_f64")) return st;
  if (total(init) != 1) return invalid("ds_reduce_f64: init value must be a scalar");
  ReduceArgs a;
  if (int st = reduce_common("ds_reduce_f64", in, dimensions, n_dimensions, body, out, a))
    return st;
  a.in_f64 = f64p(in);
  a.init_f64 = f64p(init);
  a.out_f64 = static_cast<double*>(out->data);
  a.body = body;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return reduce_launch(a, as_stream(stream));
}

int ds_reduce_f64_multi(const ds_buffer* const* ins, const ds_buffer* const* inits,
                        const int32_t* bodies, int32_t n_inputs, const int64_t* dimensions,
                        int64_t n_dimensions, const ds_buffer* const* outs, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (n_inputs < 1 || !ins || !inits || !bodies || !outs)
    return invalid("ds_reduce_f64_multi: at least one input, init, body and output");
  for (int32_t k = 0; k < n_inputs; ++k) {
    if (int st = check_buffers({ins[k], inits[k], outs[k]}, "ds_reduce_f64_multi")) return st;
    if (ins[k]->rank != ins[0]->rank)
      return invalid("ds_reduce_f64_multi: inputs must have the same shape");
    for (int64_t d = 0; d < ins[k]->rank; ++d)
      if (ins[k]->dims[d] != ins[0]->dims[d])
        return invalid("ds_reduce_f64_multi: inputs must have the same shape");
  }
  // The reductions share the workspace one after another on the stream.
  for (int32_t k = 0; k < n_inputs; ++k) {
    if (int st = ds_reduce_f64(ins[k], inits[k], dimensions, n_dimensions, bodies[k], outs[k],
                               workspace, workspace_bytes, stream))
      return st;
  }
  return ok();
}

int ds_reduce_packed(const ds_buffer* in, const ds_buffer* init_hi, const ds_buffer* init_lo,
                     const int64_t* dimensions, int64_t n_dimensions, int32_t body,
                     const ds_buffer* out_hi, const ds_buffer* out_lo, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (int st = check_buffers({in, init_hi, init_lo, out_hi, out_lo}, "ds_reduce_packed")) return st;
  if (in->rank == 0 || last_dim(in) != 2) return invalid("ds_reduce_packed expects last dim == 2");
  if (total(init_hi) != 1 || total(init_lo) != 1)
    return invalid("ds_reduce_packed: init values must be scalars");
  if (out_hi->rank != out_lo->rank || total(out_hi) != total(out_lo))
    return invalid("ds_reduce_packed: hi and lo outputs must have the same shape");
  // the logical tensor: the packed shape without its trailing 2
  const ds_buffer logical{in->data, in->dims, in->rank - 1};
  ReduceArgs a;
  if (int st = reduce_common("ds_reduce_packed", &logical, dimensions, n_dimensions, body, out_hi,
                             a))
    return st;
  a.in_packed = static_cast<const float*>(in->data);
  a.init_hi = static_cast<const float*>(init_hi->data);
  a.init_lo = static_cast<const float*>(init_lo->data);
  a.out_hi = static_cast<float*>(out_hi->data);
  a.out_lo = static_cast<float*>(out_lo->data);
  a.body = body;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return reduce_launch(a, as_stream(stream));
}

size_t ds_exchange_bytes(void) { return kExchangeBytes; }

size_t ds_exchange_handle_bytes(void) { return peer_handle_bytes(); }

int ds_exchange_alloc(void** buffer, void* handle) {
  return peer_alloc(kExchangeBytes, buffer, handle);
}

int ds_exchange_open(const void* handle, void** buffer) { return peer_open(handle, buffer); }

int ds_exchange_close(void* buffer) { return peer_close(buffer); }

int ds_exchange_free(void* buffer) { return peer_free(buffer); }

int ds_exchange_error(const void* buffer, uint32_t* code) { return peer_read_error(buffer, code); }

size_t ds_reduce_f64_sharded_workspace_size(const ds_buffer* in) {
  if (!valid_buffer(in) || bad_dims(in)) return 0;
  return reduce_sharded_workspace_bytes(total(in));
}

int ds_reduce_f64_sharded(const ds_buffer* in, const ds_buffer* init, int32_t body,
                          const ds_buffer* out, void* const* buffers, int32_t world,
                          int32_t rank, uint64_t epoch, int32_t timeout_ms, void* workspace,
                          size_t workspace_bytes, void* stream) {
  if (int st = check_buffers({in, init, out}, "ds_reduce_f64_sharded")) return st;
  if (total(init) != 1) return invalid("ds_reduce_f64_sharded: init value must be a scalar");
  if (total(out) != 1) return invalid("ds_reduce_f64_sharded: output must have one element");
  if (body < DS_BODY_ADD || body > DS_BODY_MUL)
    return invalid("ds_reduce_f64_sharded: unknown body");
  if (buffers == nullptr) return invalid("ds_reduce_f64_sharded: null exchange buffer list");
  if (epoch == 0) return invalid("ds_reduce_f64_sharded: epochs start at 1");
  if (timeout_ms <= 0) return invalid("ds_reduce_f64_sharded: timeout_ms must be positive");
  ShardedReduceArgs a;
  a.in = f64p(in);
  a.n = total(in);
  a.init = f64p(init);
  a.out = static_cast<double*>(out->data);
  a.body = body;
  a.buffers = buffers;
  a.world = world;
  a.rank = rank;
  a.epoch = epoch;
  a.timeout_ns = static_cast<int64_t>(timeout_ms) * 1000000;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return reduce_sharded_launch(a, as_stream(stream));
}

int ds_reduce_from_f64(const ds_buffer* in, const ds_buffer* init, const int64_t* dimensions,
                       int64_t n_dimensions, int32_t body, const ds_buffer* out_hi,
                       const ds_buffer* out_lo, void* workspace, size_t workspace_bytes,
                       void* stream) {
  if (int st = check_buffers({in, init, out_hi, out_lo}, "ds_reduce_from_f64")) return st;
  if (total(init) != 1) return invalid("ds_reduce_from_f64: init value must be a scalar");
  if (out_hi->rank != out_lo->rank || total(out_hi) != total(out_lo))
    return invalid("ds_reduce_from_f64: hi and lo outputs must have the same shape");
  ReduceArgs a;
  if (int st = reduce_common("ds_reduce_from_f64", in, dimensions, n_dimensions, body, out_hi, a))
    return st;
  a.in_f64 = f64p(in);
  a.init_f64 = f64p(init);
  a.out_hi = static_cast<float*>(out_hi->data);
  a.out_lo = static_cast<float*>(out_lo->data);
  a.body = body;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return reduce_launch(a, as_stream(stream));
}

int ds_reduce_f64_noalloc(const ds_buffer* in, const ds_buffer* init,
                          const int64_t* dimensions, int64_t n_dimensions, int32_t body,
                          const ds_buffer* out, void* stream) {
  if (int st = check_buffers({in, init, out}, "ds_reduce_f64_noalloc")) return st;
  if (total(init) != 1) return invalid("ds_reduce_f64_noalloc: init value must be a scalar");
  ReduceArgs a;
  if (int st = reduce_common("ds_reduce_f64_noalloc", in, dimensions, n_dimensions, body, out, a))
    return st;
  a.in_f64 = f64p(in);
  a.init_f64 = f64p(init);
  a.out_f64 = static_cast<double*>(out->data);
  a.body = body;
  return reduce_launch_noalloc(a, as_stream(stream));
}

size_t ds_dot_general_workspace_size(const ds_buffer* lhs, const ds_buffer* rhs,
                                     const ds_dot_dims* dims, int32_t algorithm) {
  if (!valid_buffer(lhs) || !valid_buffer(rhs) || bad_dims(lhs) || bad_dims(rhs) ||
      dims == nullptr)
    return 0;
  // The output descriptor the dimension numbers imply, to reuse the checks.
  const std::string saved = g_last_error;
  DotGeom g;
  std::vector<int64_t> lfree, rfree, od;
  const int64_t nb = dims->n_batch, nc = dims->n_contracting;
  int st = (nb < 0 || nb > DS_DOT_MAX_DIMS || nc < 0 || nc > DS_DOT_MAX_DIMS) ? DS_INVALID_ARGUMENT
           : dot_side(lhs, dims->lhs_batch, nb, dims->lhs_contracting, nc, g.a, lfree);
  if (st == DS_OK) st = dot_side(rhs, dims->rhs_batch, nb, dims->rhs_contracting, nc, g.b, rfree);
  if (st == DS_OK) {
    for (int64_t i = 0; i < nb; ++i) od.push_back(lhs->dims[dims->lhs_batch[i]]);
    for (int64_t d : lfree) od.push_back(lhs->dims[d]);
    for (int64_t d : rfree) od.push_back(rhs->dims[d]);
    ds_buffer out{nullptr, od.data(), static_cast<int64_t>(od.size())};
    st = dot_geometry(lhs, rhs, dims, &out, g);
  }
  g_last_error = saved;
  if (st != DS_OK) return 0;
  return dot_workspace(g, algorithm);
}

int ds_dot_general(const ds_buffer* lhs_hi, const ds_buffer* lhs_lo, const ds_buffer* rhs_hi,
                   const ds_buffer* rhs_lo, const ds_dot_dims* dims, int32_t algorithm,
                   const ds_buffer* out_hi, const ds_buffer* out_lo, void* workspace,
                   size_t workspace_bytes, void* stream) {
  if (int st = check_buffers({lhs_hi, lhs_lo, rhs_hi, rhs_lo, out_hi, out_lo}, "ds_dot_general"))
    return st;
  if (total(lhs_hi) != total(lhs_lo) || total(rhs_hi) != total(rhs_lo) ||
      total(out_hi) != total(out_lo))
    return invalid("ds_dot_general: hi and lo tensors must have the same shape");
  DotGeom g;
  if (int st = dot_geometry(lhs_hi, rhs_hi, dims, out_hi, g)) return st;
  DotProblem p;
  p.a.hi = static_cast<const float*>(lhs_hi->data);
  p.a.lo = static_cast<const float*>(lhs_lo->data);
  p.b.hi = static_cast<const float*>(rhs_hi->data);
  p.b.lo = static_cast<const float*>(rhs_lo->data);
  p.c.hi = static_cast<float*>(out_hi->data);
  p.c.lo = static_cast<float*>(out_lo->data);
  return dot_run(g, p, algorithm, workspace, workspace_bytes, as_stream(stream));
}

int ds_dot_general_f64(const ds_buffer* lhs, const ds_buffer* rhs, const ds_dot_dims* dims,
                       int32_t algorithm, const ds_buffer* out, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (int st = check_buffers({lhs, rhs, out}, "ds_dot_general_f64")) return st;
  DotGeom g;
  if (int st = dot_geometry(lhs, rhs, dims, out, g)) return st;
  DotProblem p;
  p.a.f64 = f64p(lhs);
  p.b.f64 = f64p(rhs);
  p.c.f64 = static_cast<double*>(out->data);
  return dot_run(g, p, algorithm, workspace, workspace_bytes, as_stream(stream));
}

}  // extern "C"
