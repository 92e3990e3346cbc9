// Fused elementwise DS programs: the DS pass's lowering of an elementwise
// DAG (DsTransformPass.cpp:244-321 -- constants and f64 arguments split by
// emitFromFloat, broadcast_in_dim applied to hi and lo alike, add / subtract
// / multiply as DS operations, the result recombined at the return) emitted
// as ONE kernel instead of one custom call, or one StableHLO fusion, per op.
//
// The program is a list of SSA operations (inputs, constants, add, sub, mul,
// negate).  The host generates CUDA C++ for it -- the DS primitives of
// ds_arith.cuh, the same source the library's own kernels are built from,
// so the arithmetic is the same operation for operation -- with the
// broadcast index arithmetic of every input folded to constants, compiles it
// once with NVRTC for sm_100a (no FMA contraction) and caches the function
// per device.  NVRTC and the driver's module calls are looked up at run time
// (dlopen / cudaGetDriverEntryPoint), so the library has no link-time
// dependency on either.
#include <cuda.h>
#include <dlfcn.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "profile.h"

namespace dsb {
namespace {

// The DS primitives, as source text (generated from ds_arith.cuh at build
// time).
const char kDsArithSource[] =
#include "ds_arith_src.inc"
    ;

constexpr int kMaxFusedOps = 256;
constexpr int kMaxFusedInputs = 16;
constexpr int kMaxRank = 8;

// ---- NVRTC, loaded on first use -------------------------------------------

typedef int nvrtcResult_t;
typedef struct _nvrtcProgram* nvrtcProgram_t;
struct Nvrtc {
  void* handle = nullptr;
  nvrtcResult_t (*create)(nvrtcProgram_t*, const char*, const char*, int, const char* const*,
                          const char* const*) = nullptr;
  nvrtcResult_t (*compile)(nvrtcProgram_t, int, const char* const*) = nullptr;
  nvrtcResult_t (*log_size)(nvrtcProgram_t, size_t*) = nullptr;
  nvrtcResult_t (*log)(nvrtcProgram_t, char*) = nullptr;
  nvrtcResult_t (*cubin_size)(nvrtcProgram_t, size_t*) = nullptr;
  nvrtcResult_t (*cubin)(nvrtcProgram_t, char*) = nullptr;
  nvrtcResult_t (*destroy)(nvrtcProgram_t*) = nullptr;
  std::string error;
};

const Nvrtc& nvrtc() {
  static Nvrtc n;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[] = {"libnvrtc.so.12", "libnvrtc.so"};
    for (const char* nm : names) {
      n.handle = dlopen(nm, RTLD_NOW | RTLD_LOCAL);
      if (n.handle) break;
    }
    if (!n.handle) {
      n.error = "NVRTC (libnvrtc.so.12) could not be loaded";
      return;
    }
    auto sym = [&](const char* s) { return dlsym(n.handle, s); };
    n.create = reinterpret_cast<decltype(n.create)>(sym("nvrtcCreateProgram"));
    n.compile = reinterpret_cast<decltype(n.compile)>(sym("nvrtcCompileProgram"));
    n.log_size = reinterpret_cast<decltype(n.log_size)>(sym("nvrtcGetProgramLogSize"));
    n.log = reinterpret_cast<decltype(n.log)>(sym("nvrtcGetProgramLog"));
    n.cubin_size = reinterpret_cast<decltype(n.cubin_size)>(sym("nvrtcGetCUBINSize"));
    n.cubin = reinterpret_cast<decltype(n.cubin)>(sym("nvrtcGetCUBIN"));
    n.destroy = reinterpret_cast<decltype(n.destroy)>(sym("nvrtcDestroyProgram"));
    if (!n.create || !n.compile || !n.log_size || !n.log || !n.cubin_size || !n.cubin ||
        !n.destroy)
      n.error = "NVRTC is missing an entry point";
  });
  return n;
}

// ---- driver module calls ----------------------------------------------------

struct Driver {
  CUresult (*load)(CUmodule*, const void*) = nullptr;
  CUresult (*get)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*launch_ex)(const CUlaunchConfig*, CUfunction, void**, void**) = nullptr;
  bool ok = false;
};

const Driver& driver() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char* name) -> void* {
      void* f = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint(name, &f, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess)
        return nullptr;
      return f;
    };
    d.load = reinterpret_cast<decltype(d.load)>(get("cuModuleLoadData"));
    d.get = reinterpret_cast<decltype(d.get)>(get("cuModuleGetFunction"));
    d.launch_ex = reinterpret_cast<decltype(d.launch_ex)>(get("cuLaunchKernelEx"));
    d.ok = d.load && d.get && d.launch_ex;
  });
  return d;
}

// Launches a generated kernel as a programmatic dependent of the previous
// kernel on the stream: every generated kernel waits on griddepcontrol
// before its first memory access, so its launch overlaps that kernel's tail.
CUresult launch_generated(CUfunction fn, unsigned grid, unsigned threads, void* stream,
                          void** args) {
  CUlaunchAttribute attr[1] = {};
  attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr[0].value.programmaticStreamSerializationAllowed = 1;
  CUlaunchConfig cfg = {};
  cfg.gridDimX = grid;
  cfg.gridDimY = 1;
  cfg.gridDimZ = 1;
  cfg.blockDimX = threads;
  cfg.blockDimY = 1;
  cfg.blockDimZ = 1;
  cfg.sharedMemBytes = 0;
  cfg.hStream = static_cast<CUstream>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return driver().launch_ex(&cfg, fn, args, nullptr);
}

// ---- program description and code generation -------------------------------

struct InputView {
  int type;                 // DS_FUSED_F64, DS_FUSED_F32, DS_FUSED_PACKED
  int64_t stride[kMaxRank];  // element stride per output dimension (0: broadcast)
  bool full;                 // the input is the output's own layout
};

struct Desc {
  std::vector<ds_fused_op> ops;
  std::vector<InputView> in;
  int out_type = DS_FUSED_F64;
  int rank = 0;
  int64_t dims[kMaxRank] = {};
  int64_t n = 1;
  bool pairs = false;  // all inputs full and 16-byte aligned, output too
  int reduce_body = -1;  // DS_BODY_ADD / DS_BODY_MUL: a full reduction of the results
  int rows_reduced = 0;  // > 0: reduce only that many trailing dimensions, per row
};

const char* ctype(int type) {
  return type == DS_FUSED_F64 ? "double" : (type == DS_FUSED_F32 ? "float" : "float2");
}

std::string hex32(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  char b[16];
  std::snprintf(b, sizeof b, "0x%08xu", u);
  return b;
}

// Index of input k for output element i: sum over the output dimensions of
// ((i / out_stride_d) % dim_d) * in_stride_d, all constants.
std::string index_expr(const Desc& d, const InputView& v) {
  if (v.full) return "i";
  std::string e;
  int64_t out_stride = 1;
  std::vector<std::string> terms;
  for (int k = d.rank - 1; k >= 0; --k) {
    if (v.stride[k] != 0 && d.dims[k] > 1) {
      std::string t = "(i / " + std::to_string(out_stride) + "LL)";
      if (k > 0) t = "(" + t + " % " + std::to_string(d.dims[k]) + "LL)";
      if (v.stride[k] != 1) t += " * " + std::to_string(v.stride[k]) + "LL";
      terms.push_back(t);
    }
    out_stride *= d.dims[k];
  }
  if (terms.empty()) return "0";
  for (size_t t = 0; t < terms.size(); ++t) e += (t ? " + " : "") + terms[t];
  return e;
}

// The operations of the program for one element; `load(k)` gives the DS
// value of input k, every name gets `sfx`.
template <typename Load>
std::string program_body(const Desc& d, const std::string& sfx, Load load) {
  std::string s;
  for (size_t j = 0; j < d.ops.size(); ++j) {
    const ds_fused_op& o = d.ops[j];
    const std::string v = "v" + std::to_string(j) + sfx;
    auto ref = [&](int k) { return "v" + std::to_string(k) + sfx; };
    switch (o.code) {
      case DS_FUSED_INPUT:
        s += "    const ds2 " + v + " = " + load(o.a) + ";\n";
        break;
      case DS_FUSED_CONST: {
        // emitFromFloat of the constant, on the host: hi = (float)c,
        // lo = (float)(c - (double)hi), exact bit patterns in the source.
        const float hi = static_cast<float>(o.value);
        const float lo = static_cast<float>(o.value - static_cast<double>(hi));
        s += "    const ds2 " + v + " = ds2{__uint_as_float(" + hex32(hi) + "), __uint_as_float(" +
             hex32(lo) + ")};\n";
        break;
      }
      case DS_FUSED_ADD:
        s += "    const ds2 " + v + " = add(" + ref(o.a) + ", " + ref(o.b) + ");\n";
        break;
      case DS_FUSED_SUB:
        s += "    const ds2 " + v + " = sub(" + ref(o.a) + ", " + ref(o.b) + ");\n";
        break;
      case DS_FUSED_MUL:
        s += "    const ds2 " + v + " = mul(" + ref(o.a) + ", " + ref(o.b) + ");\n";
        break;
      default:  // DS_FUSED_NEG: exact
        s += "    const ds2 " + v + " = ds2{-" + ref(o.a) + ".hi, -" + ref(o.a) + ".lo};\n";
        break;
    }
  }
  return s;
}

std::string from_value(int type, const std::string& x) {
  if (type == DS_FUSED_F64) return "from_f64(" + x + ")";
  if (type == DS_FUSED_F32) return "ds2{" + x + ", 0.0f}";
  return "ds2{(" + x + ").x, (" + x + ").y}";
}

std::string to_value(int type, const std::string& r) {
  if (type == DS_FUSED_F64) return "to_f64(" + r + ")";
  if (type == DS_FUSED_F32) return "__fadd_rn(" + r + ".hi, " + r + ".lo)";
  return "make_float2(" + r + ".hi, " + r + ".lo)";
}

// Vector types of two consecutive elements.
const char* pair_type(int type) {
  return type == DS_FUSED_F64 ? "double2" : (type == DS_FUSED_F32 ? "float2" : "float4");
}

// The kernel for program `d`.  A map writes every element's result to
// `out`.  A reduction folds each thread's results with the body, in the
// order it visits them, into a DS accumulator.  It then combines the
// accumulators of a warp (shuffles) and of the block (shared memory), and
// writes one (hi, lo) pair per block to `out`.
std::string generate(const Desc& d) {
  const bool reduce = d.reduce_body >= 0;
  const std::string body = d.reduce_body == DS_BODY_MUL ? "mul" : "add";
  const std::string ident = d.reduce_body == DS_BODY_MUL ? "ds2{1.0f, 0.0f}" : "ds2{0.0f, 0.0f}";
  std::string s;
  s += kDsArithSource;
  s += "\nusing namespace dsb;\n";
  s += "extern \"C\" __global__ void __launch_bounds__(256) ds_fused_kernel(";
  for (size_t k = 0; k < d.in.size(); ++k)
    s += std::string("const ") + ctype(d.in[k].type) + "* __restrict__ in" + std::to_string(k) +
         ", ";
  s += std::string(reduce ? "float2" : ctype(d.out_type)) + "* __restrict__ out, long long n) {\n";
  s += "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n";
  s += "  const long long stride = (long long)gridDim.x * blockDim.x;\n";
  s += "  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;\n";
  if (reduce) s += "  ds2 acc = " + ident + ";\n";
  const std::string last = std::to_string(d.ops.size() - 1);
  // element i, one at a time
  auto scalar_loop = [&](const std::string& first) {
    std::string t = "  for (long long i = " + first + "; i < n; i += stride) {\n";
    t += program_body(d, "", [&](int k) {
      const InputView& in = d.in[k];
      return from_value(in.type, "__ldg(in" + std::to_string(k) + " + (" + index_expr(d, in) + "))");
    });
    if (reduce)
      t += "    acc = " + body + "(acc, v" + last + ");\n  }\n";
    else
      t += "    out[i] = " + to_value(d.out_type, "v" + last) + ";\n  }\n";
    return t;
  };
  if (d.pairs) {
    // every input is laid out like the output and 16-byte aligned: two
    // elements per thread per step, one vector load per input
    s += "  const long long npairs = n >> 1;\n";
    s += "  for (long long p = tid; p < npairs; p += stride) {\n";
    for (size_t k = 0; k < d.in.size(); ++k)
      s += std::string("    const ") + pair_type(d.in[k].type) + " x" + std::to_string(k) +
           " = __ldcs(reinterpret_cast<const " + pair_type(d.in[k].type) + "*>(in" +
           std::to_string(k) + ") + p);\n";
    for (int e = 0; e < 2; ++e) {
      const std::string sfx = e == 0 ? "_0" : "_1";
      s += program_body(d, sfx, [&](int k) {
        const int t = d.in[k].type;
        const std::string x = "x" + std::to_string(k);
        if (t == DS_FUSED_PACKED)
          return std::string("ds2{") + x + (e == 0 ? ".x, " : ".z, ") + x + (e == 0 ? ".y}" : ".w}");
        return from_value(t, x + (e == 0 ? ".x" : ".y"));
      });
    }
    const std::string r0 = "v" + last + "_0", r1 = "v" + last + "_1";
    if (reduce)
      s += "    acc = " + body + "(" + body + "(acc, " + r0 + "), " + r1 + ");\n";
    else if (d.out_type == DS_FUSED_F64)
      s += "    __stcs(reinterpret_cast<double2*>(out) + p, make_double2(to_f64(" + r0 +
           "), to_f64(" + r1 + ")));\n";
    else if (d.out_type == DS_FUSED_F32)
      s += "    __stcs(reinterpret_cast<float2*>(out) + p, make_float2(" + to_value(DS_FUSED_F32, r0) +
           ", " + to_value(DS_FUSED_F32, r1) + "));\n";
    else
      s += "    __stcs(reinterpret_cast<float4*>(out) + p, make_float4(" + r0 + ".hi, " + r0 +
           ".lo, " + r1 + ".hi, " + r1 + ".lo));\n";
    s += "  }\n";
    s += scalar_loop("2 * npairs + tid");  // the odd last element
  } else {
    s += scalar_loop("tid");
  }
  if (reduce) {
    // warp, then block: 8 warp totals through shared memory to warp 0
    s += "  for (int o = 16; o > 0; o >>= 1) {\n";
    s += "    const ds2 t = ds2{__shfl_xor_sync(0xffffffffu, acc.hi, o), "
         "__shfl_xor_sync(0xffffffffu, acc.lo, o)};\n";
    s += "    acc = " + body + "(acc, t);\n  }\n";
    s += "  __shared__ float2 part[8];\n";
    s += "  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = make_float2(acc.hi, acc.lo);\n";
    s += "  __syncthreads();\n";
    s += "  if (threadIdx.x < 32) {\n";
    s += "    acc = threadIdx.x < 8 ? ds2{part[threadIdx.x].x, part[threadIdx.x].y} : " + ident +
         ";\n";
    s += "    for (int o = 4; o > 0; o >>= 1) {\n";
    s += "      const ds2 t = ds2{__shfl_xor_sync(0xffffffffu, acc.hi, o), "
         "__shfl_xor_sync(0xffffffffu, acc.lo, o)};\n";
    s += "      acc = " + body + "(acc, t);\n    }\n";
    s += "    if (threadIdx.x == 0) out[blockIdx.x] = make_float2(acc.hi, acc.lo);\n";
    s += "  }\n";
  }
  s += "}\n";
  return s;
}

// The kernel for a reduction over the trailing dimensions of the program's
// shape: each block owns whole rows (grid-strided), its threads fold the
// row's elements they visit, warp and block trees combine them, and thread 0
// writes body(init, row total) -- init alone for an empty row.
// Lanes that fold one row: a whole block for rows of at least 2048 values
// (0 here), else the power of two nearest R / 8 (at least 1, at most 32),
// so a lane folds about eight values before the group's shuffle tree.
int rows_lanes(int64_t R) {
  if (R >= 2048) return 0;
  int L = 1;
  while (L < 32 && static_cast<int64_t>(L) * 8 < R) L <<= 1;
  return L;
}

int64_t rows_len(const Desc& d) {
  int64_t R = 1;
  for (int k = d.rank - d.rows_reduced; k < d.rank; ++k) R *= d.dims[k];
  return R;
}

std::string generate_rows_groups(const Desc& d, int L);

std::string generate_rows(const Desc& d) {
  if (const int L = rows_lanes(rows_len(d))) return generate_rows_groups(d, L);
  const std::string body = d.reduce_body == DS_BODY_MUL ? "mul" : "add";
  const std::string ident = d.reduce_body == DS_BODY_MUL ? "ds2{1.0f, 0.0f}" : "ds2{0.0f, 0.0f}";
  const std::string last = std::to_string(d.ops.size() - 1);
  std::string s;
  s += kDsArithSource;
  s += "\nusing namespace dsb;\n";
  s += "extern \"C\" __global__ void __launch_bounds__(256) ds_fused_kernel(";
  for (size_t k = 0; k < d.in.size(); ++k)
    s += std::string("const ") + ctype(d.in[k].type) + "* __restrict__ in" + std::to_string(k) +
         ", ";
  s += "float* __restrict__ out_hi, float* __restrict__ out_lo, const float* __restrict__ init_hi, "
       "const float* __restrict__ init_lo, long long rows, long long R) {\n";
  s += "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n";
  s += "  const ds2 init = ds2{*init_hi, *init_lo};\n";
  s += "  __shared__ float2 part[8];\n";
  s += "  for (long long row = blockIdx.x; row < rows; row += gridDim.x) {\n";
  s += "    ds2 acc = " + ident + ";\n";
  s += "    for (long long j = threadIdx.x; j < R; j += blockDim.x) {\n";
  s += "      const long long i = row * R + j;\n";
  s += program_body(d, "", [&](int k) {
    const InputView& in = d.in[k];
    return from_value(in.type, "__ldg(in" + std::to_string(k) + " + (" + index_expr(d, in) + "))");
  });
  s += "      acc = " + body + "(acc, v" + last + ");\n    }\n";
  s += "    for (int o = 16; o > 0; o >>= 1) {\n";
  s += "      const ds2 t = ds2{__shfl_xor_sync(0xffffffffu, acc.hi, o), "
       "__shfl_xor_sync(0xffffffffu, acc.lo, o)};\n";
  s += "      acc = " + body + "(acc, t);\n    }\n";
  s += "    if (blockDim.x > 32) {\n";
  s += "      if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = make_float2(acc.hi, acc.lo);\n";
  s += "      __syncthreads();\n";
  s += "      if (threadIdx.x < 32) {\n";
  s += "        acc = threadIdx.x < (blockDim.x >> 5) ? ds2{part[threadIdx.x].x, part[threadIdx.x].y} : " +
       ident + ";\n";
  s += "        for (int o = 4; o > 0; o >>= 1) {\n";
  s += "          const ds2 t = ds2{__shfl_xor_sync(0xffffffffu, acc.hi, o), "
       "__shfl_xor_sync(0xffffffffu, acc.lo, o)};\n";
  s += "          acc = " + body + "(acc, t);\n        }\n";
  s += "      }\n";
  s += "      __syncthreads();  // part is refilled by the next row\n";
  s += "    }\n";
  s += "    if (threadIdx.x == 0) {\n";
  s += "      const ds2 r = R == 0 ? init : " + body + "(init, acc);\n";
  s += "      out_hi[row] = r.hi;\n      out_lo[row] = r.lo;\n    }\n";
  s += "  }\n}\n";
  return s;
}

// Short rows: groups of L lanes (L divides 32) each fold one row.  The row
// loop advances a whole warp at a time so that every lane reaches every
// shuffle; a group past the last row folds nothing and writes nothing.
std::string generate_rows_groups(const Desc& d, int L) {
  const std::string body = d.reduce_body == DS_BODY_MUL ? "mul" : "add";
  const std::string ident = d.reduce_body == DS_BODY_MUL ? "ds2{1.0f, 0.0f}" : "ds2{0.0f, 0.0f}";
  const std::string last = std::to_string(d.ops.size() - 1);
  const std::string Ls = std::to_string(L), gpw = std::to_string(32 / L);
  std::string s;
  s += kDsArithSource;
  s += "\nusing namespace dsb;\n";
  s += "extern \"C\" __global__ void __launch_bounds__(256) ds_fused_kernel(";
  for (size_t k = 0; k < d.in.size(); ++k)
    s += std::string("const ") + ctype(d.in[k].type) + "* __restrict__ in" + std::to_string(k) +
         ", ";
  s += "float* __restrict__ out_hi, float* __restrict__ out_lo, const float* __restrict__ init_hi, "
       "const float* __restrict__ init_lo, long long rows, long long R) {\n";
  s += "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n";
  s += "  const ds2 init = ds2{*init_hi, *init_lo};\n";
  s += "  const int lane = threadIdx.x & 31, sub = lane % " + Ls + ";\n";
  s += "  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;\n";
  s += "  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;\n";
  s += "  for (long long base = wid * " + gpw + "; base < rows; base += nw * " + gpw + ") {\n";
  s += "    const long long row = base + lane / " + Ls + ";\n";
  s += "    ds2 acc = " + ident + ";\n";
  s += "    if (row < rows) {\n";
  s += "      for (long long j = sub; j < R; j += " + Ls + ") {\n";
  s += "        const long long i = row * R + j;\n";
  s += program_body(d, "", [&](int k) {
    const InputView& in = d.in[k];
    return from_value(in.type, "__ldg(in" + std::to_string(k) + " + (" + index_expr(d, in) + "))");
  });
  s += "        acc = " + body + "(acc, v" + last + ");\n      }\n    }\n";
  s += "    for (int o = " + std::to_string(L / 2) + "; o > 0; o >>= 1) {\n";
  s += "      const ds2 t = ds2{__shfl_xor_sync(0xffffffffu, acc.hi, o), "
       "__shfl_xor_sync(0xffffffffu, acc.lo, o)};\n";
  s += "      acc = " + body + "(acc, t);\n    }\n";
  s += "    if (sub == 0 && row < rows) {\n";
  s += "      const ds2 r = R == 0 ? init : " + body + "(init, acc);\n";
  s += "      out_hi[row] = r.hi;\n      out_lo[row] = r.lo;\n    }\n";
  s += "  }\n}\n";
  return s;
}

int invalid(const std::string& m) { return set_error(DS_INVALID_ARGUMENT, m); }

int64_t prod(const int64_t* d, int64_t r) {
  int64_t n = 1;
  for (int64_t i = 0; i < r; ++i) n *= d[i];
  return n;
}

// Validate the program and the buffers and fill `d` (numpy broadcasting of
// every input's logical shape to the output's).
int describe(const ds_fused_op* ops, int32_t n_ops, const int32_t* input_types,
             const ds_buffer* const* inputs, int32_t n_inputs, int32_t out_type,
             const ds_buffer* out, Desc& d) {
  if (ops == nullptr || n_ops < 1 || n_ops > kMaxFusedOps)
    return invalid("ds_fused: 1 to 256 operations expected");
  if (n_inputs < 0 || n_inputs > kMaxFusedInputs || (n_inputs > 0 && (!inputs || !input_types)))
    return invalid("ds_fused: 0 to 16 inputs expected");
  if (out_type < DS_FUSED_F64 || out_type > DS_FUSED_PACKED)
    return invalid("ds_fused: unknown output type");
  if (out == nullptr || out->rank < 0 || out->rank > kMaxRank + 1 || (out->rank && !out->dims))
    return invalid("ds_fused: invalid output buffer");
  // logical output shape
  int64_t orank = out->rank;
  if (out_type == DS_FUSED_PACKED) {
    if (orank == 0 || out->dims[orank - 1] != 2)
      return invalid("ds_fused: a packed output needs last dim == 2");
    --orank;
  }
  if (orank > kMaxRank) return invalid("ds_fused: at most 8 dimensions");
  d.rank = static_cast<int>(orank);
  for (int k = 0; k < d.rank; ++k) {
    if (out->dims[k] < 0) return invalid("ds_fused: negative dimension");
    d.dims[k] = out->dims[k];
  }
  d.n = prod(d.dims, d.rank);
  if (d.n > 0 && out->data == nullptr) return invalid("ds_fused: null output pointer");
  d.out_type = out_type;
  d.in.resize(n_inputs);
  for (int32_t k = 0; k < n_inputs; ++k) {
    const ds_buffer* b = inputs[k];
    const int t = input_types[k];
    if (t < DS_FUSED_F64 || t > DS_FUSED_PACKED) return invalid("ds_fused: unknown input type");
    if (b == nullptr || b->rank < 0 || b->rank > kMaxRank + 1 || (b->rank && !b->dims))
      return invalid("ds_fused: invalid input buffer");
    int64_t r = b->rank;
    if (t == DS_FUSED_PACKED) {
      if (r == 0 || b->dims[r - 1] != 2) return invalid("ds_fused: a packed input needs last dim == 2");
      --r;
    }
    if (r > d.rank) return invalid("ds_fused: an input has more dimensions than the output");
    InputView& v = d.in[k];
    v.type = t;
    int64_t st = 1;
    bool full = r == d.rank;
    for (int q = d.rank - 1; q >= 0; --q) {
      const int64_t src = q - (d.rank - r);  // right-aligned
      const int64_t dim = src >= 0 ? b->dims[src] : 1;
      if (dim != d.dims[q] && dim != 1)
        return invalid("ds_fused: input " + std::to_string(k) + " does not broadcast to the output");
      v.stride[q] = (dim == 1 && d.dims[q] != 1) ? 0 : st;
      if (dim != d.dims[q]) full = false;
      st *= dim;
    }
    v.full = full;
    if (prod(b->dims, r) > 0 && b->data == nullptr) return invalid("ds_fused: null input pointer");
  }
  d.pairs = aligned(out->data, 16);
  for (int32_t k = 0; k < n_inputs; ++k)
    d.pairs = d.pairs && d.in[k].full && aligned(inputs[k]->data, 16);
  d.ops.assign(ops, ops + n_ops);
  for (int32_t j = 0; j < n_ops; ++j) {
    const ds_fused_op& o = ops[j];
    switch (o.code) {
      case DS_FUSED_INPUT:
        if (o.a < 0 || o.a >= n_inputs) return invalid("ds_fused: input index out of range");
        break;
      case DS_FUSED_CONST:
        break;
      case DS_FUSED_ADD:
      case DS_FUSED_SUB:
      case DS_FUSED_MUL:
        if (o.a < 0 || o.a >= j || o.b < 0 || o.b >= j)
          return invalid("ds_fused: operands must be earlier operations");
        break;
      case DS_FUSED_NEG:
        if (o.a < 0 || o.a >= j) return invalid("ds_fused: operands must be earlier operations");
        break;
      default:
        return invalid("ds_fused: unknown operation code");
    }
  }
  return DS_OK;
}

// Compiled functions per (device, source).
std::mutex g_mu;
std::map<std::pair<int, std::string>, CUfunction> g_funcs;

// Everything the generated source depends on, as a short byte string: the
// operations, each input's type, broadcast strides and layout, the output
// type and shape, the pair path and the reduction body.  A call looks its
// function up by this key and generates the source only on a miss.
std::string key_of(const Desc& d) {
  std::string k;
  auto put = [&k](const void* p, size_t n) { k.append(static_cast<const char*>(p), n); };
  const int32_t head[5] = {static_cast<int32_t>(d.ops.size()), static_cast<int32_t>(d.in.size()),
                           d.out_type, d.rank,
                           (d.pairs ? 1 : 0) | ((d.reduce_body + 1) << 1) | (d.rows_reduced << 4)};
  put(head, sizeof head);
  put(d.dims, sizeof(int64_t) * d.rank);
  for (const ds_fused_op& o : d.ops) {
    const int32_t c[3] = {o.code, o.a, o.b};
    put(c, sizeof c);
    put(&o.value, sizeof o.value);
  }
  for (const InputView& v : d.in) {
    const int32_t t[2] = {v.type, v.full ? 1 : 0};
    put(t, sizeof t);
    put(v.stride, sizeof(int64_t) * d.rank);
  }
  return k;
}
std::map<std::pair<int, std::string>, CUfunction> g_by_key;

int compile(const std::string& src, CUfunction* fn);

int compile_desc(const Desc& d, CUfunction* fn) {
  int dev = 0;
  DSB_CUDA_TRY(cudaGetDevice(&dev));
  const std::string key = key_of(d);
  {
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_by_key.find({dev, key});
    if (it != g_by_key.end()) {
      *fn = it->second;
      return DS_OK;
    }
  }
  if (int st = compile(d.rows_reduced > 0 ? generate_rows(d) : generate(d), fn)) return st;
  std::lock_guard<std::mutex> lock(g_mu);
  g_by_key[{dev, key}] = *fn;
  return DS_OK;
}

int compile(const std::string& src, CUfunction* fn) {
  int dev = 0;
  DSB_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_funcs.find({dev, src});
  if (it != g_funcs.end()) {
    *fn = it->second;
    return DS_OK;
  }
  const Nvrtc& nv = nvrtc();
  if (!nv.error.empty()) return set_error(DS_INTERNAL, "ds_fused: " + nv.error);
  const Driver& drv = driver();
  if (!drv.ok) return set_error(DS_INTERNAL, "ds_fused: driver module calls unavailable");
  nvrtcProgram_t prog = nullptr;
  if (nv.create(&prog, src.c_str(), "ds_fused.cu", 0, nullptr, nullptr) != 0)
    return set_error(DS_INTERNAL, "ds_fused: nvrtcCreateProgram failed");
  const char* opts[] = {"-arch=sm_100a", "--fmad=false", "-std=c++17", "-default-device"};
  const int rc = nv.compile(prog, 4, opts);
  if (rc != 0) {
    size_t n = 0;
    nv.log_size(prog, &n);
    std::string log(n, '\0');
    if (n) nv.log(prog, &log[0]);
    nv.destroy(&prog);
    return set_error(DS_INTERNAL, "ds_fused: NVRTC compilation failed: " + log);
  }
  size_t n = 0;
  nv.cubin_size(prog, &n);
  std::vector<char> cubin(n);
  nv.cubin(prog, cubin.data());
  nv.destroy(&prog);
  CUmodule mod = nullptr;
  if (drv.load(&mod, cubin.data()) != CUDA_SUCCESS)
    return set_error(DS_INTERNAL, "ds_fused: cuModuleLoadData failed");
  CUfunction f = nullptr;
  if (drv.get(&f, mod, "ds_fused_kernel") != CUDA_SUCCESS)
    return set_error(DS_INTERNAL, "ds_fused: cuModuleGetFunction failed");
  g_funcs[{dev, src}] = f;
  *fn = f;
  return DS_OK;
}

// Compile without loading (no GPU needed): the NVRTC log on failure.
int nvrtc_check(const std::string& src) {
  const Nvrtc& nv = nvrtc();
  if (!nv.error.empty()) return set_error(DS_INTERNAL, "ds_fused: " + nv.error);
  nvrtcProgram_t prog = nullptr;
  if (nv.create(&prog, src.c_str(), "ds_fused.cu", 0, nullptr, nullptr) != 0)
    return set_error(DS_INTERNAL, "ds_fused: nvrtcCreateProgram failed");
  const char* opts[] = {"-arch=sm_100a", "--fmad=false", "-std=c++17", "-default-device"};
  const int rc = nv.compile(prog, 4, opts);
  std::string log;
  if (rc != 0) {
    size_t n = 0;
    nv.log_size(prog, &n);
    log.assign(n, '\0');
    if (n) nv.log(prog, &log[0]);
  }
  nv.destroy(&prog);
  if (rc != 0) return set_error(DS_INTERNAL, "ds_fused: NVRTC compilation failed: " + log);
  return ok();
}

}  // namespace
}  // namespace dsb

using namespace dsb;

extern "C" {

int ds_fused_source(const ds_fused_op* ops, int32_t n_ops, const int32_t* input_types,
                    const ds_buffer* const* inputs, int32_t n_inputs, int32_t out_type,
                    const ds_buffer* out, char* buf, size_t cap, size_t* len) {
  Desc d;
  if (int st = describe(ops, n_ops, input_types, inputs, n_inputs, out_type, out, d)) return st;
  const std::string src = generate(d);
  if (len) *len = src.size() + 1;
  if (buf && cap) {
    const size_t k = src.size() < cap - 1 ? src.size() : cap - 1;
    std::memcpy(buf, src.data(), k);
    buf[k] = '\0';
  }
  return ok();
}

int ds_fused_compile_check(const ds_fused_op* ops, int32_t n_ops, const int32_t* input_types,
                           const ds_buffer* const* inputs, int32_t n_inputs, int32_t out_type,
                           const ds_buffer* out) {
  Desc d;
  if (int st = describe(ops, n_ops, input_types, inputs, n_inputs, out_type, out, d)) return st;
  return nvrtc_check(generate(d));
}

int ds_fused_run(const ds_fused_op* ops, int32_t n_ops, const int32_t* input_types,
                 const ds_buffer* const* inputs, int32_t n_inputs, int32_t out_type,
                 const ds_buffer* out, void* stream) {
  Desc d;
  if (int st = describe(ops, n_ops, input_types, inputs, n_inputs, out_type, out, d)) return st;
  if (d.n == 0) return ok();
  CUfunction fn = nullptr;
  if (int st = compile_desc(d, &fn)) return st;
  std::vector<void*> ptrs(n_inputs + 1);
  std::vector<void*> args(n_inputs + 2);
  for (int32_t k = 0; k < n_inputs; ++k) {
    ptrs[k] = inputs[k]->data;
    args[k] = &ptrs[k];
  }
  ptrs[n_inputs] = out->data;
  args[n_inputs] = &ptrs[n_inputs];
  long long n = d.n;
  args[n_inputs + 1] = &n;
  const unsigned grid = grid_for(d.pairs ? (d.n + 1) / 2 : d.n, 256, 8);
  ProfileScope prof("fused", static_cast<cudaStream_t>(stream));
  if (launch_generated(fn, grid, 256, stream, args.data()) != CUDA_SUCCESS)
    return set_error(DS_INTERNAL, "ds_fused: cuLaunchKernelEx failed");
  return ok();
}

// A fused program reduced to one DS value: stage 1 is the generated kernel
// with its reduction sink (one partial pair per block into the workspace),
// stage 2 the library's packed reduce over those partials with the init.
static int64_t fused_reduce_max_blocks() { return static_cast<int64_t>(sm_count()) * 8; }

static size_t fused_reduce_partial_bytes() {
  return static_cast<size_t>((fused_reduce_max_blocks() * 8 + 255) / 256 * 256);
}

size_t ds_fused_reduce_workspace_size(const int64_t* dims, int32_t rank) {
  if (rank < 0 || rank > kMaxRank || (rank > 0 && dims == nullptr)) return 0;
  const int64_t blocks = fused_reduce_max_blocks();
  const int64_t pdims[1] = {blocks};
  alignas(16) static char stand_in[16];
  const ds_buffer logical{stand_in, pdims, 1};
  const int64_t dim0 = 0;
  return fused_reduce_partial_bytes() + ds_reduce_workspace_size(&logical, &dim0, 1) + 256;
}

int ds_fused_reduce(const ds_fused_op* ops, int32_t n_ops, const int32_t* input_types,
                    const ds_buffer* const* inputs, int32_t n_inputs, const int64_t* dims,
                    int32_t rank, int32_t body, const ds_buffer* init_hi,
                    const ds_buffer* init_lo, const ds_buffer* out_hi, const ds_buffer* out_lo,
                    void* workspace, size_t workspace_bytes, void* stream) {
  if (body != DS_BODY_ADD && body != DS_BODY_MUL)
    return invalid("ds_fused_reduce: the body is DS_BODY_ADD or DS_BODY_MUL");
  if (rank < 0 || rank > kMaxRank || (rank > 0 && dims == nullptr))
    return invalid("ds_fused_reduce: at most 8 dimensions");
  if (!init_hi || !init_lo || !out_hi || !out_lo || !init_hi->data || !init_lo->data ||
      !out_hi->data || !out_lo->data)
    return invalid("ds_fused_reduce: null init or output buffer");
  const size_t need = ds_fused_reduce_workspace_size(dims, rank);
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 256))
    return invalid("ds_fused_reduce: workspace too small or not 256-byte aligned (need " +
                   std::to_string(need) + " bytes)");
  // the map's logical shape, written by no one: the partials stand in for
  // its data pointer (16-byte aligned, so the pair path is decided by the inputs)
  const ds_buffer shape{workspace, dims, rank};
  Desc d;
  if (int st = describe(ops, n_ops, input_types, inputs, n_inputs, DS_FUSED_F64, &shape, d))
    return st;
  d.reduce_body = body;
  float2* partials = static_cast<float2*>(workspace);
  unsigned grid = 0;
  if (d.n > 0) {
    CUfunction fn = nullptr;
    if (int st = compile_desc(d, &fn)) return st;
    std::vector<void*> ptrs(n_inputs + 1);
    std::vector<void*> args(n_inputs + 2);
    for (int32_t k = 0; k < n_inputs; ++k) {
      ptrs[k] = inputs[k]->data;
      args[k] = &ptrs[k];
    }
    ptrs[n_inputs] = partials;
    args[n_inputs] = &ptrs[n_inputs];
    long long n = d.n;
    args[n_inputs + 1] = &n;
    grid = grid_for(d.pairs ? (d.n + 1) / 2 : d.n, 256, 8);
    ProfileScope prof("fused_reduce", static_cast<cudaStream_t>(stream));
    if (launch_generated(fn, grid, 256, stream, args.data()) != CUDA_SUCCESS)
      return set_error(DS_INTERNAL, "ds_fused_reduce: cuLaunchKernelEx failed");
  }
  const int64_t pdims[2] = {static_cast<int64_t>(grid), 2};
  const ds_buffer pbuf{partials, pdims, 2};
  const int64_t dim0 = 0;
  const size_t off = fused_reduce_partial_bytes();
  return ds_reduce_packed(&pbuf, init_hi, init_lo, &dim0, 1, body, out_hi, out_lo,
                          static_cast<char*>(workspace) + off, workspace_bytes - off, stream);
}

// The per-row reduction: checks shared by the entry point and its compile
// check; fills `d` and the row count and length.
static int describe_rows(const ds_fused_op* ops, int32_t n_ops, const int32_t* input_types,
                         const ds_buffer* const* inputs, int32_t n_inputs, const int64_t* dims,
                         int32_t rank, int32_t n_reduced, int32_t body, void* stand_in,
                         Desc& d, int64_t& rows, int64_t& row_len) {
  if (body != DS_BODY_ADD && body != DS_BODY_MUL)
    return invalid("ds_fused_reduce_rows: the body is DS_BODY_ADD or DS_BODY_MUL");
  if (rank < 1 || rank > kMaxRank || dims == nullptr)
    return invalid("ds_fused_reduce_rows: 1 to 8 dimensions");
  if (n_reduced < 1 || n_reduced > rank)
    return invalid("ds_fused_reduce_rows: 1 to rank trailing dimensions are reduced");
  const ds_buffer shape{stand_in, dims, rank};
  if (int st = describe(ops, n_ops, input_types, inputs, n_inputs, DS_FUSED_F64, &shape, d))
    return st;
  d.reduce_body = body;
  d.rows_reduced = n_reduced;
  rows = prod(dims, rank - n_reduced);
  row_len = prod(dims + (rank - n_reduced), n_reduced);
  return DS_OK;
}

int ds_fused_reduce_rows(const ds_fused_op* ops, int32_t n_ops, const int32_t* input_types,
                         const ds_buffer* const* inputs, int32_t n_inputs, const int64_t* dims,
                         int32_t rank, int32_t n_reduced, int32_t body, const ds_buffer* init_hi,
                         const ds_buffer* init_lo, const ds_buffer* out_hi,
                         const ds_buffer* out_lo, void* stream) {
  if (!init_hi || !init_lo || !out_hi || !out_lo || !init_hi->data || !init_lo->data ||
      !out_hi->data || !out_lo->data)
    return invalid("ds_fused_reduce_rows: null init or output buffer");
  Desc d;
  int64_t rows = 0, row_len = 0;
  if (int st = describe_rows(ops, n_ops, input_types, inputs, n_inputs, dims, rank, n_reduced,
                             body, out_hi->data, d, rows, row_len))
    return st;
  auto total = [](const ds_buffer* b) {
    int64_t n = 1;
    for (int64_t i = 0; i < b->rank; ++i) n *= b->dims[i];
    return n;
  };
  if ((out_hi->rank && !out_hi->dims) || (out_lo->rank && !out_lo->dims) ||
      total(out_hi) != rows || total(out_lo) != rows)
    return invalid("ds_fused_reduce_rows: outputs must hold one value per row (" +
                   std::to_string(rows) + ")");
  if ((init_hi->rank && !init_hi->dims) || (init_lo->rank && !init_lo->dims) ||
      total(init_hi) != 1 || total(init_lo) != 1)
    return invalid("ds_fused_reduce_rows: init values must be scalars");
  if (rows == 0) return ok();
  CUfunction fn = nullptr;
  if (int st = compile_desc(d, &fn)) return st;
  std::vector<void*> ptrs(n_inputs + 4);
  std::vector<void*> args(n_inputs + 6);
  for (int32_t k = 0; k < n_inputs; ++k) {
    ptrs[k] = inputs[k]->data;
    args[k] = &ptrs[k];
  }
  ptrs[n_inputs] = out_hi->data;
  ptrs[n_inputs + 1] = out_lo->data;
  ptrs[n_inputs + 2] = init_hi->data;
  ptrs[n_inputs + 3] = init_lo->data;
  for (int q = 0; q < 4; ++q) args[n_inputs + q] = &ptrs[n_inputs + q];
  long long nrows = rows, len = row_len;
  args[n_inputs + 4] = &nrows;
  args[n_inputs + 5] = &len;
  // long rows: a block of 256 per row; short ones: groups of L lanes per
  // row, 256 / L rows per block
  const int L = rows_lanes(row_len);
  const unsigned threads = 256u;
  const int64_t per_block = L ? 256 / L : 1;
  const int64_t need = (rows + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  const unsigned grid = static_cast<unsigned>(need < cap ? need : cap);
  ProfileScope prof("fused_reduce", static_cast<cudaStream_t>(stream));
  if (launch_generated(fn, grid, threads, stream, args.data()) != CUDA_SUCCESS)
    return set_error(DS_INTERNAL, "ds_fused_reduce_rows: cuLaunchKernelEx failed");
  return ok();
}

int ds_fused_reduce_rows_compile_check(const ds_fused_op* ops, int32_t n_ops,
                                       const int32_t* input_types,
                                       const ds_buffer* const* inputs, int32_t n_inputs,
                                       const int64_t* dims, int32_t rank, int32_t n_reduced,
                                       int32_t body) {
  alignas(16) static char stand_in[16];
  Desc d;
  int64_t rows = 0, row_len = 0;
  if (int st = describe_rows(ops, n_ops, input_types, inputs, n_inputs, dims, rank, n_reduced,
                             body, stand_in, d, rows, row_len))
    return st;
  return nvrtc_check(generate_rows(d));
}

int ds_fused_reduce_compile_check(const ds_fused_op* ops, int32_t n_ops,
                                  const int32_t* input_types, const ds_buffer* const* inputs,
                                  int32_t n_inputs, const int64_t* dims, int32_t rank,
                                  int32_t body) {
  if (body != DS_BODY_ADD && body != DS_BODY_MUL)
    return invalid("ds_fused_reduce: the body is DS_BODY_ADD or DS_BODY_MUL");
  if (rank < 0 || rank > kMaxRank || (rank > 0 && dims == nullptr))
    return invalid("ds_fused_reduce: at most 8 dimensions");
  alignas(16) static char stand_in[16];
  const ds_buffer shape{stand_in, dims, rank};
  Desc d;
  if (int st = describe(ops, n_ops, input_types, inputs, n_inputs, DS_FUSED_F64, &shape, d))
    return st;
  d.reduce_body = body;
  return nvrtc_check(generate(d));
}

}  // extern "C"
