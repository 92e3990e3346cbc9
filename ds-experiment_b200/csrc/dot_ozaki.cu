// Tensor-core DS dot_general: exact integer-residue GEMM (Ozaki scheme II)
// on the int8 tcgen05 tensor cores of sm_100a.
//
// The DS value of every operand element (hi + lo, i.e. the f64 input after
// the DS split) is scaled by a power of two per row of A and per column of B,
//     a_int = rint(a * 2^sa_i),  |a_int| <= 2^P,
// so the product of the integer matrices is an integer matrix with
// |C_int| <= K 2^(2P).  C_int is computed exactly through its residues modulo
// L = 14 pairwise-coprime moduli m_l <= 256 (product Mprod ~ 2^110.2):
//   1. split:  residues (a_int mod m_l) as int8 planes [L][batch][rows][K]
//              (K-major, rows padded to the tile, K padded to 128), plus the
//              per-row scale exponents;
//   2. gemm:   for every modulus, one int8 x int8 -> int32 GEMM on the
//              tensor cores (exact: |sum| <= K * 128^2 < 2^31 for K <= 2^17);
//              the epilogue stores (P mod m_l) as one byte;
//   3. crt:    C_int from its L residues by the Chinese remainder theorem,
//              evaluated exactly in three 40-bit f64 limbs, then
//              C = C_int * 2^-(sa_i + sb_j) in f64.
// P = min(50, floor((log2 Mprod - 2 - log2 K) / 2)) keeps |C_int| <= Mprod/4,
// so the quotient in step 3 is exact.  For K = 4096, P = 48: every input is
// quantised to 49 bits relative to its row (column) maximum, i.e. at least
// the precision of the DS input itself; the products and sums add no error.
//
// GEMM kernel (step 2): persistent, one CTA per SM, warp-specialised.
//   warp 0      TMA producer: 128x128 (A) and 256x128 (B) int8 tiles, 128B
//               swizzle, 4-stage mbarrier ring (48 KB per stage);
//   warp 1      TMEM allocator and MMA issuer: one thread issues
//               tcgen05.mma.cta_group::1.kind::i8 M=128 N=256 K=32 (4 per
//               stage) into one of two 256-column int32 TMEM accumulators;
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time, mod m_l, byte
//               stores; overlaps the MMAs of the next tile.
// Work units are (modulus, batch, tile_m, tile_n), modulus outermost, so the
// planes of one modulus (2 x 16 MB at 4096^2) stay in L2 while all CTAs use
// them.  Every mbarrier wait is bounded (~2 s of clock64); on timeout the
// kernel records an error code, unwinds and the CRT step writes NaN.  No TMA
// multicast is used anywhere.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <climits>
#include <cmath>
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "ds_arith.cuh"
#include "kernels.h"
#include "profile.h"

namespace dsb {
namespace {

constexpr int kL = 14;
constexpr int kTileM = 128, kTileN = 256, kTileK = 128;  // int8: 128 bytes of K
constexpr int kStages = 4;
constexpr int kStageA = kTileM * kTileK;  // 16 KB
constexpr int kStageB = kTileN * kTileK;  // 32 KB
constexpr int kGemmThreads = 192;
// u8 x u8 products summed in int32: K * 255^2 < 2^31 needs K <= 33025.
constexpr int kMaxK = 1 << 15;
constexpr int kShiftNonFinite = INT_MIN;
// Shift code of a row (column) whose values are all zero: its products are
// exactly zero, so its outputs need no error certificate.
constexpr int kShiftZero = INT_MIN + 1;
constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 1.9 GHz

__host__ __device__ constexpr int mod_of(int l) {
  return l == 0 ? 256 : l == 1 ? 255 : l == 2 ? 253 : l == 3 ? 251 : l == 4 ? 247
       : l == 5 ? 241 : l == 6 ? 239 : l == 7 ? 233 : l == 8 ? 229 : l == 9 ? 227
       : l == 10 ? 223 : l == 11 ? 217 : l == 12 ? 211 : 199;
}

// Moduli whose split residue is taken from the FP64 pipe (one FMA and one
// integer multiply-add) rather than the integer pipes (two byte dot
// products and a multiply-high reduction).  Ten of the thirteen were
// fastest: with all thirteen the row split spills (its group loop keeps
// every 1 / m in a register), with seven both splits are 4 to 6% slower.
__host__ __device__ constexpr bool residue_fp64(int l) { return l >= 1 && l <= 10; }

// ---------------------------------------------------------------------------
// Host-side constants: P from K, and the CRT weights in 40-bit limbs.

// The weights and the modulus product split at bit kCrtSplit: W = W_hi 2^70 +
// W_lo.  W_hi < 2^40.2, so the 14 products r W_hi (r < 2^8) sum exactly in
// f64 (< 2^53); W_lo < 2^70 is rounded to 53 bits.
constexpr int kCrtSplit = 70;

struct CrtConsts {
  double w[kL][2];  // W_l = (Mprod/m_l) * ((Mprod/m_l)^-1 mod m_l): {W_hi, W_lo}
  double mlimb[2];  // Mprod: {hi, lo}
  double inv_m;     // 1 / Mprod
  double log2_m;
};

using u128 = unsigned __int128;

const CrtConsts& crt_consts() {
  static CrtConsts c;
  static std::once_flag once;
  std::call_once(once, [] {
    u128 M = 1;
    for (int l = 0; l < kL; ++l) M *= static_cast<u128>(mod_of(l));
    const u128 lo_mask = (static_cast<u128>(1) << kCrtSplit) - 1;
    auto to_double = [](u128 v) { return static_cast<double>(v); };  // rounded to nearest
    for (int l = 0; l < kL; ++l) {
      const int m = mod_of(l);
      const u128 Ml = M / m;
      const int r = static_cast<int>(Ml % m);
      int inv = 1;
      while ((r * inv) % m != 1) ++inv;  // m <= 256: trivial search
      const u128 W = Ml * static_cast<u128>(inv);  // < M
      c.w[l][0] = static_cast<double>(static_cast<uint64_t>(W >> kCrtSplit));
      c.w[l][1] = to_double(W & lo_mask);
    }
    c.mlimb[0] = static_cast<double>(static_cast<uint64_t>(M >> kCrtSplit));
    c.mlimb[1] = to_double(M & lo_mask);
    const double Md = to_double(M);
    c.inv_m = 1.0 / Md;
    c.log2_m = std::log2(Md);
  });
  return c;
}

int bits_for_k(int64_t K) {
  const double lk = std::log2(static_cast<double>(K < 1 ? 1 : K));
  int P = static_cast<int>(std::floor((crt_consts().log2_m - 2.0 - lk) / 2.0));
  return P > 50 ? 50 : P;
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// Uncertified outputs (see the CRT step) are listed, up to kFixListMax of
// them, for a warp each; with more, every output is recomputed.
constexpr int64_t kFixListMax = 1 << 20;
constexpr int kFixTile = 64;

struct Layout {
  int64_t batch, M, N, K, Mp, Np, Kp;
  size_t off_a, off_b, off_c, off_sa, off_sb, off_ca, off_cb, off_err, off_fix_list, total;
  int64_t fix_cap;
};

Layout layout_of(int64_t batch, int64_t M, int64_t N, int64_t K) {
  Layout g{};
  g.batch = batch;
  g.M = M;
  g.N = N;
  g.K = K;
  g.Mp = round_up(M, 2 * kTileM);  // 256: one tile of a CTA pair
  g.Np = round_up(N, kTileN);
  g.Kp = round_up(K < 1 ? 1 : K, kTileK);
  size_t off = 0;
  auto take = [&off](size_t bytes) {
    const size_t at = off;
    off = static_cast<size_t>(round_up(static_cast<int64_t>(off + bytes), 1024));
    return at;
  };
  g.off_a = take(static_cast<size_t>(kL) * batch * g.Mp * g.Kp);
  g.off_b = take(static_cast<size_t>(kL) * batch * g.Np * g.Kp);
  g.off_c = take(static_cast<size_t>(kL) * batch * g.Mp * g.Np);
  g.off_sa = take(sizeof(int) * batch * g.Mp);
  g.off_sb = take(sizeof(int) * batch * g.Np);
  g.off_ca = take(sizeof(int) * batch * g.Mp);
  g.off_cb = take(sizeof(int) * batch * g.Np);
  // error word ([0]) and the count of uncertified outputs ([1])
  g.off_err = take(sizeof(int) * 4);
  g.fix_cap = batch * M * N < kFixListMax ? batch * M * N : kFixListMax;
  g.off_fix_list = take(sizeof(uint64_t) * static_cast<size_t>(g.fix_cap));
  g.total = off;
  return g;
}

// ---------------------------------------------------------------------------
// Step 1: split.

// The value an operand element contributes: an f64 input as it is (it is at
// least as precise as its DS split), a SoA DS input as hi + lo.
__device__ __forceinline__ double op_value(const DotOperand& o, int64_t idx) {
  return o.f64 ? o.f64[idx]
               : __dadd_rn(static_cast<double>(o.hi[idx]), static_cast<double>(o.lo[idx]));
}

// v * 2^s for any int s (exact unless the result under/overflows).
__device__ __forceinline__ double scale2(double v, int s) {
  if (s >= -1000 && s <= 1000) return v * __longlong_as_double(static_cast<long long>(1023 + s) << 52);
  return ldexp(v, s);
}

constexpr double kMagic = 6755399441055744.0;  // 1.5 * 2^52

// The biased integer t = rint(v * 2^shift) + 2^51, for |v * 2^shift| <= 2^50:
// adding 1.5 * 2^52 rounds to an integer (to nearest even) and leaves t in
// the low 52 bits of the sum, so no conversion instruction is needed.
__device__ __forceinline__ uint64_t quantise(double v, int shift) {
  const double y = (shift >= -1000 && shift <= 1000)
                       ? __fma_rn(v, __longlong_as_double(static_cast<long long>(1023 + shift) << 52), kMagic)
                       : __dadd_rn(ldexp(v, shift), kMagic);
  return static_cast<uint64_t>(__double_as_longlong(y)) & ((1ull << 52) - 1);
}

// t = hi * 2^32 + lo (hi < 2^20): the seven bytes of t in two words, and
// x - 128 as an f64 for the unbiased integer x = t - 2^51 (exact:
// |x| <= 2^50).
struct Limbs {
  uint32_t lo, hi;
  double xs;
};

__device__ __forceinline__ Limbs limbs_of(uint64_t t) {
  // t is the mantissa of 1.5 * 2^52 + x_int, a double in [2^52, 2^53)
  const double y = __longlong_as_double(static_cast<long long>(0x4330000000000000ull | t));
  return Limbs{static_cast<uint32_t>(t), static_cast<uint32_t>(t >> 32),
               __dsub_rn(y, kMagic + 128.0)};
}

// 2^e mod m, for the byte weights below.
__host__ __device__ constexpr uint32_t pow2_mod(int e, uint32_t m) {
  uint32_t r = 1 % m;
  for (int i = 0; i < e; ++i) r = (r * 2u) % m;
  return r;
}

// Four byte weights packed for __dp4a: byte j of the word is 2^(8 (j + j0)) mod m.
__host__ __device__ constexpr uint32_t byte_weights(int j0, int count, uint32_t m) {
  uint32_t w = 0;
  for (int j = 0; j < count; ++j) w |= pow2_mod(8 * (j0 + j), m) << (8 * j);
  return w;
}

// Residue in [0, m) of the unbiased integer t - 2^51 modulo m = mod_of(l).
// The bytes of t dotted with the weights 2^(8j) mod m (two byte dot
// products), plus the constant that cancels the bias, give s < 2^19 with
// s = t - 2^51 (mod m); then s mod m = s - m * umulhi(s, ceil(2^32 / m)),
// exact because s * (ceil(2^32 / m) * m - 2^32) < 2^19 * 2^8 < 2^32.
// m = 256 is the low byte of t (2^51 = 0 mod 256).
// Per modulus: {byte weights of the low word, of the high word, the bias
// correction, ceil(2^32 / m)}.  In the constant bank, so the instructions
// read them as operands instead of materialising 52 immediates per element.
struct SplitConsts {
  uint32_t w_lo, w_hi, unbias, magic;
};

__host__ __device__ constexpr SplitConsts split_consts(uint32_t m) {
  return SplitConsts{byte_weights(0, 4, m), byte_weights(4, 3, m), (m - pow2_mod(51, m)) % m,
                     m == 256u ? 0u : 0xFFFFFFFFu / m + 1u};
}

__constant__ SplitConsts c_split[kL] = {
    split_consts(mod_of(0)),  split_consts(mod_of(1)),  split_consts(mod_of(2)),
    split_consts(mod_of(3)),  split_consts(mod_of(4)),  split_consts(mod_of(5)),
    split_consts(mod_of(6)),  split_consts(mod_of(7)),  split_consts(mod_of(8)),
    split_consts(mod_of(9)),  split_consts(mod_of(10)), split_consts(mod_of(11)),
    split_consts(mod_of(12)), split_consts(mod_of(13))};

// 1 / m rounded, for the residue from the FP64 pipe: (x - 128) / m to
// 2^-10 for |x| <= 2^50.
__constant__ double c_inv_m[kL] = {
    1.0 / mod_of(0),  1.0 / mod_of(1),  1.0 / mod_of(2),  1.0 / mod_of(3),  1.0 / mod_of(4),
    1.0 / mod_of(5),  1.0 / mod_of(6),  1.0 / mod_of(7),  1.0 / mod_of(8),  1.0 / mod_of(9),
    1.0 / mod_of(10), 1.0 / mod_of(11), 1.0 / mod_of(12), 1.0 / mod_of(13)};

// With kMixed, the moduli of residue_fp64 take the FP64 path and the others
// the integer one; otherwise all take the integer path.  0 (256) is a mask.
template <bool kMixed>
constexpr bool residue_on_fp64(int l) { return kMixed && residue_fp64(l); }

// Residue from the FP64 pipe, two instructions: one FMA gives
// 1.5 * 2^52 + q with q = rint((x - 128) / m) (x.xs = x - 128; the rounded
// 1 / m puts q within one of the nearest integer), so r = x - q m =
// 128 + ((x - 128) - q m) lies in [128 - m / 2 - m 2^-10,
// 128 + m / 2 + m 2^-10], inside [0, 255] for m <= 255.  r is then exact in
// 32-bit integer arithmetic from the low words: x mod 2^32 is x.lo (2^51 is
// 0 mod 2^32) and q mod 2^32 is the low word of the FMA's result, so one
// multiply-add x.lo - q m gives r.  r is a residue of x in [0, 256) but not
// always below m; the GEMM only needs an unsigned byte of the right class.
__device__ __forceinline__ uint32_t residue_fp64_path(const Limbs& x, double inv, uint32_t m) {
  const double qd = __fma_rn(x.xs, inv, kMagic);
  return x.lo - static_cast<uint32_t>(__double2loint(qd)) * m;
}

// Residue in [0, m) on the integer pipes.
__device__ __forceinline__ uint32_t residue_int(const Limbs& x, const SplitConsts& c, uint32_t m) {
  const uint32_t s = __dp4a(x.lo, c.w_lo, __dp4a(x.hi, c.w_hi, c.unbias));
  return s - __umulhi(s, c.magic) * m;
}

template <int l, bool kMixed>
__device__ __forceinline__ uint32_t residue(const Limbs& x) {
  constexpr uint32_t m = mod_of(l);
  if constexpr (m == 256u) {
    return x.lo & 0xFFu;
  } else if constexpr (residue_on_fp64<kMixed>(l)) {
    return residue_fp64_path(x, c_inv_m[l], m);
  } else {
    return residue_int(x, c_split[l], m);
  }
}

// Four residues (each < 256) as the bytes of one word: three byte permutes.
__device__ __forceinline__ uint32_t pack4(uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  return __byte_perm(__byte_perm(r0, r1, 0x0040), __byte_perm(r2, r3, 0x0040), 0x5410);
}

// Residues of N = 4, 8 or 16 consecutive values -> one 4-, 8- or 16-byte
// store per modulus plane.
template <int N, bool kMixed, int l = 0>
__device__ __forceinline__ void store_planes_n(const Limbs (&x)[N], uint8_t* base,
                                               size_t plane_stride) {
  if constexpr (l < kL) {
    uint32_t w[N / 4];
#pragma unroll
    for (int q = 0; q < N / 4; ++q)
      w[q] = pack4(residue<l, kMixed>(x[q * 4]), residue<l, kMixed>(x[q * 4 + 1]),
                   residue<l, kMixed>(x[q * 4 + 2]), residue<l, kMixed>(x[q * 4 + 3]));
    uint8_t* dst = base + l * plane_stride;
    if constexpr (N == 4) {
      *reinterpret_cast<uint32_t*>(dst) = w[0];
    } else if constexpr (N == 8) {
      *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    store_planes_n<N, kMixed, l + 1>(x, base, plane_stride);
  }
}

// The residue with the modulus picked at run time: the same arithmetic as
// residue<l, true>, its constants read from the constant bank by index
// (m = 256 works on the integer path too: its weights select byte 0 and its
// magic is 0).  A loop over the moduli built from it is a fourteenth of the
// unrolled code, which keeps the column split's instruction stream in cache.
__constant__ uint32_t c_mod_rt[kL] = {mod_of(0), mod_of(1), mod_of(2),  mod_of(3),  mod_of(4),
                                      mod_of(5), mod_of(6), mod_of(7),  mod_of(8),  mod_of(9),
                                      mod_of(10), mod_of(11), mod_of(12), mod_of(13)};

__device__ __forceinline__ uint32_t residue_rt(const Limbs& x, int l) {
  if (residue_fp64(l)) return residue_fp64_path(x, c_inv_m[l], c_mod_rt[l]);
  return residue_int(x, c_split[l], c_mod_rt[l]);
}

// Residues of 16 consecutive values -> one 16-byte store per modulus plane,
// the moduli looped at run time.
__device__ __forceinline__ void store_planes_16_rt(const Limbs (&x)[16], uint8_t* base,
                                                   size_t plane_stride) {
#pragma unroll 1
  for (int l = 0; l < kL; ++l) {
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      w[q] = pack4(residue_rt(x[q * 4], l), residue_rt(x[q * 4 + 1], l),
                   residue_rt(x[q * 4 + 2], l), residue_rt(x[q * 4 + 3], l));
    *reinterpret_cast<uint4*>(base + l * plane_stride) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__device__ __forceinline__ int shift_for(double mx, bool nonfinite, int P) {
  if (nonfinite) return kShiftNonFinite;
  if (mx == 0.0) return kShiftZero;
  return P - (ilogb(mx) + 1);  // |v| <= mx < 2^(ilogb+1)
}

// Encoded row exponent for atomicMax across blocks: 0 = all zero,
// kExpNonFinite = a NaN/Inf seen, else ilogb(max) + 1 + kExpBias.
constexpr int kExpBias = 2048;
constexpr int kExpNonFinite = 0x7FFFFFFF;

__device__ __forceinline__ int shift_from_code(int code, int P) {
  if (code == kExpNonFinite) return kShiftNonFinite;
  if (code == 0) return kShiftZero;
  return P - (code - kExpBias);
}

// Operand rows contiguous in K (s_k == 1): one block per (row, batch), of
// 256 threads, or 512 for rows longer than 4096.  An f64 row of at most 16
// values per thread at a 16-byte aligned address is read into registers
// (four groups of four consecutive k, 4 * blockDim.x apart, so every load
// is coalesced) and reduced to the row maximum; the groups are then read
// again one at a time (L1 hits) and quantised.  Other rows take the same two
// passes with the second mostly from L2.  Four residues per thread per
// modulus make one coalesced 4-byte store.
constexpr int kSplitRowsMaxThreads = 512;

__host__ __device__ constexpr int split_rows_threads(int64_t K) {
  return K > 4096 && K <= 16 * kSplitRowsMaxThreads ? kSplitRowsMaxThreads : 256;
}

__device__ __forceinline__ void split_rows_body(const DotOperand& o, int64_t rows, int64_t K,
                                                int64_t rows_pad, int64_t Kp, int64_t batch,
                                                int P, uint8_t* __restrict__ planes,
                                                int* __restrict__ shifts, int64_t r, int64_t b) {
  __shared__ double s_max[kSplitRowsMaxThreads / 32];
  __shared__ int s_bad[kSplitRowsMaxThreads / 32];
  const bool live = r < rows;
  const int64_t base = b * o.s_b + r * o.s_r;
  const bool vec = o.f64 && o.s_k == 1 && (reinterpret_cast<uintptr_t>(o.f64 + base) & 15) == 0;
  const int64_t group = 4 * static_cast<int64_t>(blockDim.x);  // k covered by one group
  const bool in_regs = vec && K <= 4 * group;
  double v[16];
  double mx = 0.0;
  bool bad = false;
  if (in_regs) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int64_t k0 = g * group + threadIdx.x * 4;
      if (live && k0 + 4 <= K) {
        const double2* p = reinterpret_cast<const double2*>(o.f64 + base + k0);
        const double2 v01 = __ldg(p), v23 = __ldg(p + 1);
        v[g * 4 + 0] = v01.x;
        v[g * 4 + 1] = v01.y;
        v[g * 4 + 2] = v23.x;
        v[g * 4 + 3] = v23.y;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[g * 4 + j] = (live && k0 + j < K) ? o.f64[base + k0 + j] : 0.0;
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      bad |= !isfinite(v[j]);
      mx = fmax(mx, fabs(v[j]));
    }
  } else if (live) {
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
      const double x = op_value(o, base + k * o.s_k);
      bad |= !isfinite(x);
      mx = fmax(mx, fabs(x));
    }
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, d));
    bad |= __shfl_xor_sync(0xffffffffu, static_cast<int>(bad), d) != 0;
  }
  if ((threadIdx.x & 31) == 0) {
    s_max[threadIdx.x >> 5] = mx;
    s_bad[threadIdx.x >> 5] = bad;
  }
  __syncthreads();
  mx = 0.0;
  bad = false;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
    mx = fmax(mx, s_max[w]);
    bad |= s_bad[w] != 0;
  }
  const int shift = live ? shift_for(mx, bad, P) : 0;
  if (threadIdx.x == 0) shifts[b * rows_pad + r] = shift;
  const bool zero = !live || shift == kShiftNonFinite || shift == kShiftZero;
  const int sh = zero ? 0 : shift;
  const size_t plane_stride = static_cast<size_t>(batch) * rows_pad * Kp;
  uint8_t* row_out = planes + (static_cast<size_t>(b) * rows_pad + r) * Kp;
  if (in_regs) {
    // the groups again, one at a time from L1 (the first pass read them
    // through it): the residue code appears once rather than four times
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      const int64_t k0 = g * group + threadIdx.x * 4;
      if (k0 < Kp) {
        double w[4];
        if (!zero && k0 + 4 <= K) {
          const double2* p = reinterpret_cast<const double2*>(o.f64 + base + k0);
          const double2 v01 = __ldg(p), v23 = __ldg(p + 1);
          w[0] = v01.x;
          w[1] = v01.y;
          w[2] = v23.x;
          w[3] = v23.y;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) w[j] = (zero || k0 + j >= K) ? 0.0 : o.f64[base + k0 + j];
        }
        Limbs x[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = limbs_of(quantise(w[j], sh));
        store_planes_n<4, true>(x, row_out + k0, plane_stride);
      }
    }
    return;
  }
  for (int64_t k0 = static_cast<int64_t>(threadIdx.x) * 4; k0 < Kp; k0 += 4 * blockDim.x) {
    double w[4];
    if (!zero && vec && k0 + 4 <= K) {
      const double2* p = reinterpret_cast<const double2*>(o.f64 + base + k0);
      const double2 v01 = p[0], v23 = p[1];
      w[0] = v01.x;
      w[1] = v01.y;
      w[2] = v23.x;
      w[3] = v23.y;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t k = k0 + j;
        w[j] = (zero || k >= K) ? 0.0 : op_value(o, base + k * o.s_k);
      }
    }
    Limbs x[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = limbs_of(quantise(w[j], sh));
    store_planes_n<4, true>(x, row_out + k0, plane_stride);
  }
}

__global__ void __launch_bounds__(kSplitRowsMaxThreads, 2)
split_kmajor_kernel(DotOperand o, int64_t rows, int64_t K, int64_t rows_pad, int64_t Kp,
                    int64_t batch, int P, uint8_t* __restrict__ planes, int* __restrict__ shifts,
                    int64_t row0) {
  split_rows_body(o, rows, K, rows_pad, Kp, batch, P, planes, shifts, row0 + blockIdx.x,
                  blockIdx.y);
}

// Operand rows contiguous across rows (s_r == 1, e.g. B[K, N] row-major):
// blocks of 64 rows x 256 K.  Pairs of adjacent rows load as one 16-byte
// value when the layout allows it (paired_rows).
constexpr int kColTileR = 64;

__device__ __forceinline__ bool paired_rows(const DotOperand& o) {
  return o.f64 && o.s_r == 1 && (reinterpret_cast<uintptr_t>(o.f64) & 15) == 0 &&
         (o.s_k & 1) == 0 && (o.s_b & 1) == 0;
}

// Values of rows (row, row + 1) at k; zero outside the operand.
__device__ __forceinline__ void load_row_pair(const DotOperand& o, bool paired, int64_t b,
                                              int64_t row, int64_t k, int64_t rows, int64_t K,
                                              double& x0, double& x1) {
  x0 = x1 = 0.0;
  if (k >= K) return;
  const int64_t off = b * o.s_b + row * o.s_r + k * o.s_k;
  if (paired && row + 2 <= rows) {
    const double2 d = __ldcs(reinterpret_cast<const double2*>(o.f64 + off));
    x0 = d.x;
    x1 = d.y;
  } else {
    if (row < rows) x0 = op_value(o, off);
    if (row + 1 < rows) x1 = op_value(o, off + o.s_r);
  }
}

// Pass 1: per-row maximum over a kColmaxSlab-deep slab of K per block, merged
// across blocks with atomicMax on an encoded exponent (codes start at 0).
constexpr int kColmaxSlab = 128;

__device__ __forceinline__ void colmax_body(const DotOperand& o, int64_t rows, int64_t K,
                                            int64_t rows_pad, int* __restrict__ codes,
                                            int64_t bx, int64_t by, int64_t b) {
  __shared__ double s_max[8][kColTileR];
  __shared__ int s_bad[8][kColTileR];
  const int lane = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t r0 = bx * kColTileR;
  const int64_t row = r0 + 2 * lane;
  const int64_t k0 = by * kColmaxSlab;
  double m0 = 0.0, m1 = 0.0;
  bool bad = false, bad1 = false;
  const int64_t k1 = k0 + kColmaxSlab < K ? k0 + kColmaxSlab : K;
  if (paired_rows(o) && row + 2 <= rows) {
    const double* p = o.f64 + b * o.s_b + row;
#pragma unroll 4
    for (int64_t k = k0 + ty; k < k1; k += 8) {
      const double2 d = __ldcs(reinterpret_cast<const double2*>(p + k * o.s_k));
      bad |= !isfinite(d.x);
      bad1 |= !isfinite(d.y);
      m0 = fmax(m0, fabs(d.x));
      m1 = fmax(m1, fabs(d.y));
    }
  } else {
    for (int64_t k = k0 + ty; k < k1; k += 8) {
      double x0, x1;
      load_row_pair(o, false, b, row, k, rows, K, x0, x1);
      bad |= !isfinite(x0);
      bad1 |= !isfinite(x1);
      m0 = fmax(m0, fabs(x0));
      m1 = fmax(m1, fabs(x1));
    }
  }
  s_max[ty][2 * lane] = m0;
  s_max[ty][2 * lane + 1] = m1;
  s_bad[ty][2 * lane] = bad;
  s_bad[ty][2 * lane + 1] = bad1;
  __syncthreads();
  if (threadIdx.x < kColTileR) {
    const int64_t r = r0 + threadIdx.x;
    double mx = 0.0;
    bool nf = false;
    for (int w = 0; w < 8; ++w) {
      mx = fmax(mx, s_max[w][threadIdx.x]);
      nf |= s_bad[w][threadIdx.x] != 0;
    }
    const int code = nf ? kExpNonFinite : (mx == 0.0 ? 0 : ilogb(mx) + 1 + kExpBias);
    if (r < rows && code != 0) atomicMax(&codes[b * rows_pad + r], code);
  }
}

__global__ void __launch_bounds__(256, 6)
colmax_kernel(DotOperand o, int64_t rows, int64_t K, int64_t rows_pad,
              int* __restrict__ codes) {
  colmax_body(o, rows, K, rows_pad, codes, blockIdx.x, blockIdx.y, blockIdx.z);
}

// One launch for the row split of A (compute-bound) and the column maxima of
// B (memory-bound), their blocks interleaved evenly so the two overlap on
// every SM: block t is a column-maximum block when floor((t + 1) nc / total)
// steps up.  256 threads (rows of at most 4096 values).
__global__ void __launch_bounds__(256, 4)
split_rows_colmax_kernel(DotOperand a, int64_t rows_a, int64_t rows_a_pad, DotOperand bop,
                         int64_t rows_b, int64_t rows_b_pad, int64_t K, int64_t Kp, int P,
                         uint8_t* __restrict__ planes_a, int* __restrict__ shifts_a,
                         int* __restrict__ codes_b, int64_t nc, int64_t cgx, int64_t cgy) {
  const int64_t t = blockIdx.x, total = rows_a_pad + nc;
  const int64_t c0 = t * nc / total, c1 = (t + 1) * nc / total;
  if (c1 > c0) {
    colmax_body(bop, rows_b, K, rows_b_pad, codes_b, c0 % cgx, c0 / cgx % cgy, c0 / (cgx * cgy));
  } else {
    split_rows_body(a, rows_a, K, rows_a_pad, Kp, 1, P, planes_a, shifts_a, t - c0, 0);
  }
}

// Pass 2: one block per (64 rows, 64 K) tile.  Values are loaded along rows
// (coalesced), quantised into a shared-memory tile, and written transposed
// (K-major): each thread turns 16 consecutive k of one row into one 16-byte
// store per modulus.  Warps read the tile along rows (conflict-free).
constexpr int kColTileK = 64;
constexpr int kColTilePitch = kColTileR + 2;  // 16-byte aligned rows of the tile

__global__ void __launch_bounds__(256)
split_cols_kernel(DotOperand o, int64_t rows, int64_t K, int64_t rows_pad, int64_t Kp,
                  int64_t batch, int P, const int* __restrict__ codes,
                  uint8_t* __restrict__ planes, int* __restrict__ shifts) {
  __shared__ __align__(16) uint64_t tile[kColTileK][kColTilePitch];
  __shared__ int s_shift[kColTileR];
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kColTileR, b = blockIdx.z;
  const int64_t kc = static_cast<int64_t>(blockIdx.y) * kColTileK;
  if (threadIdx.x < kColTileR) {
    const int64_t r = r0 + threadIdx.x;
    const int sh = r < rows ? shift_from_code(codes[b * rows_pad + r], P) : 0;
    s_shift[threadIdx.x] = sh;
    if (blockIdx.y == 0) shifts[b * rows_pad + r] = sh;
  }
  __syncthreads();
  const bool paired = paired_rows(o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double x[8][2];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    load_row_pair(o, paired, b, r0 + 2 * lane, kc + warp + 8 * i, rows, K, x[i][0], x[i][1]);
  const int sh0 = s_shift[2 * lane], sh1 = s_shift[2 * lane + 1];
  const bool z0 = sh0 == kShiftNonFinite || sh0 == kShiftZero;
  const bool z1 = sh1 == kShiftNonFinite || sh1 == kShiftZero;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint64_t t0 = quantise(z0 ? 0.0 : x[i][0], z0 ? 0 : sh0);
    const uint64_t t1 = quantise(z1 ? 0.0 : x[i][1], z1 ? 0 : sh1);
    *reinterpret_cast<ulonglong2*>(&tile[warp + 8 * i][2 * lane]) = make_ulonglong2(t0, t1);
  }
  __syncthreads();
  const int my_row = lane + 32 * (warp & 1), my_grp = warp >> 1;
  Limbs q[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) q[j] = limbs_of(tile[my_grp * 16 + j][my_row]);
  const size_t plane_stride = static_cast<size_t>(batch) * rows_pad * Kp;
  store_planes_16_rt(q, planes + (static_cast<size_t>(b) * rows_pad + r0 + my_row) * Kp +
                            kc + my_grp * 16,
                     plane_stride);
}

// Pass 2 for an operand whose rows are contiguous (s_r == 1) into
// row-contiguous planes [l][batch][Kp][rows_pad] (the GEMM reads them as an
// MN-major operand, so nothing is transposed): one block per (kMnRows rows,
// kMnSlab k), each thread kMnCols consecutive rows over the slab.  A warp
// reads 32 * kMnCols values of one k and writes 32 * kMnCols contiguous
// bytes per modulus.  The slab is unrolled: a loop would keep the moduli's
// constants in registers across iterations and spill.  (Two rows per thread,
// 40 registers and half again as many warps, was 15% slower.)
constexpr int kMnCols = 4, kMnRows = 256 * kMnCols, kMnSlab = 2;

__global__ void __launch_bounds__(256, 4)
split_mn_kernel(DotOperand o, int64_t rows, int64_t K, int64_t rows_pad, int64_t Kp,
                int64_t batch, int P, const int* __restrict__ codes,
                uint8_t* __restrict__ planes, int* __restrict__ shifts) {
  const int64_t b = blockIdx.z;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kMnRows + threadIdx.x * kMnCols;
  if (r0 >= rows_pad) return;  // rows_pad is a multiple of kMnCols
  int sh[kMnCols];
  bool z[kMnCols];
#pragma unroll
  for (int j = 0; j < kMnCols; ++j) {
    const int64_t r = r0 + j;
    const int s = r < rows ? shift_from_code(codes[b * rows_pad + r], P) : 0;
    if (blockIdx.y == 0) shifts[b * rows_pad + r] = s;
    z[j] = r >= rows || s == kShiftNonFinite || s == kShiftZero;
    sh[j] = z[j] ? 0 : s;
  }
  const bool vec = o.f64 && o.s_r == 1 && r0 + kMnCols <= rows && (o.s_k & 1) == 0 &&
                   (o.s_b & 1) == 0 && (reinterpret_cast<uintptr_t>(o.f64) & 15) == 0;
  const size_t plane_stride = static_cast<size_t>(batch) * Kp * rows_pad;
  const int64_t k0 = static_cast<int64_t>(blockIdx.y) * kMnSlab;
#pragma unroll
  for (int64_t k = k0; k < k0 + kMnSlab && k < Kp; ++k) {
    double w[kMnCols];
#pragma unroll
    for (int j = 0; j < kMnCols; ++j) w[j] = 0.0;
    if (k < K) {
      const int64_t off = b * o.s_b + r0 * o.s_r + k * o.s_k;
      if (vec) {
        const double2* p = reinterpret_cast<const double2*>(o.f64 + off);
#pragma unroll
        for (int h = 0; h < kMnCols / 2; ++h) {
          const double2 v = __ldcs(p + h);
          w[2 * h] = v.x;
          w[2 * h + 1] = v.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < kMnCols; ++j)
          if (r0 + j < rows) w[j] = op_value(o, off + j * o.s_r);
      }
    }
    Limbs x[kMnCols];
#pragma unroll
    for (int j = 0; j < kMnCols; ++j) x[j] = limbs_of(quantise(z[j] ? 0.0 : w[j], sh[j]));
    store_planes_n<kMnCols, true>(x, planes + (static_cast<size_t>(b) * Kp + k) * rows_pad + r0,
                                  plane_stride);
  }
}

// The same split for an f64 operand, with its loads made asynchronous:
// block (c, g) of gridDim.x = chunks of kMnRows rows takes chunk c at
// k = g, g + gridDim.y, ...; each thread copies its four values of the next
// kMnStages - 1 k into its own shared-memory slots with cp.async (zero fill
// past K or the rows) while it quantises the current ones, so no register
// holds a load in flight and the column shifts are loaded once per block.
// Two blocks per SM: with four (64 registers) the k loop keeps every 1 / m
// in a register and spills, and runs at half the speed; six stages were no
// faster than four.  (The same pipeline for A's rows, with B's column
// maxima in a kernel of their own, was slower than split_rows_colmax_kernel:
// 0.095 + 0.030 ms against 0.102 ms for both.)
constexpr int kMnStages = 4;

__device__ __forceinline__ void cp_async8(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src),
               "r"(valid ? 8 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(256, 2)
split_mn_async_kernel(DotOperand o, int64_t rows, int64_t K, int64_t rows_pad, int64_t Kp,
                      int64_t batch, int P, const int* __restrict__ codes,
                      uint8_t* __restrict__ planes, int* __restrict__ shifts) {
  __shared__ __align__(16) double stage[kMnStages][256][kMnCols];
  wait_previous_grid();  // the column maxima
  const int64_t b = blockIdx.z;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kMnRows + threadIdx.x * kMnCols;
  if (r0 >= rows_pad) return;  // rows_pad is a multiple of kMnCols
  int sh[kMnCols];
  bool z[kMnCols];
#pragma unroll
  for (int j = 0; j < kMnCols; ++j) {
    const int64_t r = r0 + j;
    const int sv = r < rows ? shift_from_code(codes[b * rows_pad + r], P) : 0;
    if (blockIdx.y == 0) shifts[b * rows_pad + r] = sv;
    z[j] = r >= rows || sv == kShiftNonFinite || sv == kShiftZero;
    sh[j] = z[j] ? 0 : sv;
  }
  const bool vec = r0 + kMnCols <= rows && (o.s_k & 1) == 0 && (o.s_b & 1) == 0 &&
                   (reinterpret_cast<uintptr_t>(o.f64) & 15) == 0;
  // addresses of copies that read nothing (zero fill) still point inside
  // the operand
  const double* base = o.f64 + b * o.s_b + (r0 < rows ? r0 : 0);
  const size_t plane_stride = static_cast<size_t>(batch) * Kp * rows_pad;
  const int64_t kstep = gridDim.y;
  auto issue = [&](int64_t k, int slot) {
    double* dst = stage[slot][threadIdx.x];
    const bool in = k < K;
    const double* src = base + (in ? k : 0) * o.s_k;
    if (vec) {
      cp_async16(dst, src, in);
      cp_async16(dst + 2, src + 2, in);
    } else {
#pragma unroll
      for (int j = 0; j < kMnCols; ++j) {
        const bool valid = in && r0 + j < rows;
        cp_async8(dst + j, valid ? src + j : base, valid);
      }
    }
  };
  // prologue: the first kMnStages - 1 k of this block (empty groups past Kp)
  int64_t kn = blockIdx.y;
#pragma unroll
  for (int st = 0; st < kMnStages - 1; ++st, kn += kstep) {
    if (kn < Kp) issue(kn, st);
    cp_async_commit();
  }
  int slot = 0;
#pragma unroll 1
  for (int64_t k = blockIdx.y; k < Kp; k += kstep) {
    if (kn < Kp) issue(kn, (slot + kMnStages - 1) % kMnStages);
    cp_async_commit();
    kn += kstep;
    cp_async_wait<kMnStages - 1>();  // this thread's copies of k have landed
    const double* w = stage[slot][threadIdx.x];
    Limbs x[kMnCols];
#pragma unroll
    for (int j = 0; j < kMnCols; ++j) x[j] = limbs_of(quantise(z[j] ? 0.0 : w[j], sh[j]));
    store_planes_n<kMnCols, true>(x, planes + (static_cast<size_t>(b) * Kp + k) * rows_pad + r0,
                                  plane_stride);
    slot = slot + 1 == kMnStages ? 0 : slot + 1;
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// Step 2: tcgen05 int8 GEMM.

struct GemmParams {
  int batch, tiles_m, tiles_n, kblocks;
  int tm0;  // first tile row of this launch (a band of tiles_m tile rows)
  int64_t Mp, Np;
  int64_t units;
  uint8_t* cres;
  int* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false (and an error code recorded) after ~2 s, or at once if
// another role of any CTA has already given up.  The first try is inlined
// into the pipeline loops; only a wait that has to spin makes the call (a
// call per K-block cost the GEMM 9% of its time).
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, int* err, int code) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*reinterpret_cast<volatile int*>(err) != 0) return false;
    if (clock64() - t0 > kTimeoutCycles) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity, err, code);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// K-major operand tile with 128-byte swizzle: rows of 128 B, 8-row atoms of
// 1024 B (stride byte offset), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(1) << 16;          // leading byte offset (unused here): 16 B
  d |= static_cast<uint64_t>(1024 >> 4) << 32;  // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;          // version
  d |= static_cast<uint64_t>(2) << 61;          // SWIZZLE_128B
  return d;
}

// MN-major operand tile with 128-byte swizzle, 128 bytes (one swizzle atom)
// of M or N per CTA: rows of 128 B along MN, one per k; 8-k atoms of 1024 B
// (stride byte offset).  The leading byte offset steps between 128-byte MN
// atoms, of which a CTA's tile has one, so it is never applied.
__device__ __forceinline__ uint64_t sdesc_mn(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(1) << 16;          // leading byte offset (unused here): 16 B
  d |= static_cast<uint64_t>(1024 >> 4) << 32;  // stride byte offset: 8 k of 128 B
  d |= static_cast<uint64_t>(1) << 46;          // version
  d |= static_cast<uint64_t>(2) << 61;          // SWIZZLE_128B
  return d;
}

// kind::i8, D = s32, A = B = unsigned 8-bit (residues in [0, m)), both
// K-major, N = 256, M = 128.
constexpr uint32_t kIdesc = (2u << 4) | (0u << 7) | (0u << 10) |
                            (static_cast<uint32_t>(kTileN >> 3) << 17) |
                            (static_cast<uint32_t>(kTileM >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
        "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
        "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct Unit {
  int l, b, tm, tn;
};

__device__ __forceinline__ Unit unit_of(int64_t u, const GemmParams& p) {
  const int64_t per_l = static_cast<int64_t>(p.batch) * p.tiles_m * p.tiles_n;
  Unit x;
  x.l = static_cast<int>(u / per_l);
  int64_t rem = u - x.l * per_l;
  const int64_t per_b = static_cast<int64_t>(p.tiles_m) * p.tiles_n;
  x.b = static_cast<int>(rem / per_b);
  rem -= x.b * per_b;
  const int tm = static_cast<int>(rem / p.tiles_n);
  x.tn = static_cast<int>(rem - static_cast<int64_t>(tm) * p.tiles_n);
  x.tm = p.tm0 + tm;
  return x;
}

// v mod m for 0 <= v < 2^31 (a u8 x u8 -> s32 accumulator, K <= 32768):
// floor(v / m) = umulhi(v, ceil(2^39 / m)) >> 7 exactly, because
// v * (ceil(2^39 / m) * m - 2^39) < 2^31 * 2^8 = 2^39.  Integer pipes only.
__host__ __device__ constexpr uint32_t epilogue_magic(uint32_t m) {
  return static_cast<uint32_t>(((1ull << 39) + m - 1) / m);
}

__device__ __forceinline__ uint32_t mod_u8(uint32_t v, uint32_t m, uint32_t magic) {
  return v - (__umulhi(v, magic) >> 7) * m;
}

// Four accumulators -> their residues as the bytes of one word.
__device__ __forceinline__ uint32_t mod_pack4(const uint32_t* v, uint32_t m, uint32_t magic) {
  return __byte_perm(__byte_perm(mod_u8(v[0], m, magic), mod_u8(v[1], m, magic), 0x0040),
                     __byte_perm(mod_u8(v[2], m, magic), mod_u8(v[3], m, magic), 0x0040), 0x5410);
}

__global__ void __launch_bounds__(kGemmThreads, 1)
ozaki_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                  const __grid_constant__ CUtensorMap tmap_b, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + kStages * kStageA;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * (kStageA + kStageB));
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drained = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drained, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer ----
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
        const Unit w = unit_of(u, p);
        const int ya = static_cast<int>((static_cast<int64_t>(w.l) * p.batch + w.b) * p.Mp +
                                        static_cast<int64_t>(w.tm) * kTileM);
        const int yb = static_cast<int>((static_cast<int64_t>(w.l) * p.batch + w.b) * p.Np +
                                        static_cast<int64_t>(w.tn) * kTileN);
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], kStageA + kStageB);
          tma_load_2d(smem_a + stage * kStageA, &tmap_a, kb * kTileK, ya, &full[stage]);
          tma_load_2d(smem_b + stage * kStageB, &tmap_b, kb * kTileK, yb, &full[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // After an abort, give copies already issued time to land (a few
      // microseconds suffice) before the CTA can exit.  On the normal path
      // the MMA warp has consumed every filled stage.
      if (!ok) {
        const long long t0 = clock64();
        while (clock64() - t0 < 200000) {
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * kTileN);
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem_a + stage * kStageA);
          const uint32_t b0 = smem_u32(smem_b + stage * kStageB);
#pragma unroll
          for (int k = 0; k < kTileK / 32; ++k) {
            mma_i8(d, sdesc(a0 + k * 32), sdesc(b0 + k * 32), kIdesc, (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // All issued MMAs complete before TMEM is released.
      mma_commit(drained);
      const long long t0 = clock64();
      while (!mbar_try_wait(drained, 0) && clock64() - t0 < kTimeoutCycles) {
      }
    }
  } else {
    // ---- epilogue (warps 2..5; TMEM lanes 32*(warp%4) ..) ----
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int64_t u = blockIdx.x; u < p.units; u += gridDim.x) {
      if (!mbar_wait(&tfull[acc], acc_phase, p.err, 4)) break;
      tc_fence_after();
      const Unit w = unit_of(u, p);
      const uint32_t m = static_cast<uint32_t>(mod_of(w.l));
      const uint32_t magic = epilogue_magic(m);
      const int64_t row = (static_cast<int64_t>(w.l) * p.batch + w.b) * p.Mp +
                          static_cast<int64_t>(w.tm) * kTileM + row_in_tile;
      uint8_t* out = p.cres + row * p.Np + static_cast<int64_t>(w.tn) * kTileN;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * kTileN);
#pragma unroll 1
      for (int c0 = 0; c0 < kTileN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tbase + c0, v);
        uint32_t packed[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) packed[q] = mod_pack4(v + q * 4, m, magic);
        uint4* dst = reinterpret_cast<uint4*>(out + c0);
        dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// ---- CTA-pair variant (tcgen05 cta_group::2) ---------------------------------
//
// A cluster of two CTAs computes 256x256 tiles.  Each CTA stages its own 128
// rows of A and its 128-row half of the B tile (16 + 16 KB per 128-byte
// K sub-tile instead of 16 + 32 KB; a pipeline stage holds two sub-tiles,
// so the barrier round trip, the commit and the TMA issues are paid once
// per 256 bytes of K), the even CTA issues tcgen05.mma.cta_group::2
// M=256 N=256 K=32 over both CTAs' shared memory, and each CTA drains its
// own 128 rows from its own TMEM.  Both CTAs' TMA loads complete on the even
// CTA's "full" barrier (addressed with mapa); the MMA commits arrive on both
// CTAs' "empty" / "tmem full" barriers (commit multicast); every epilogue warp
// of the pair arrives on the even CTA's "tmem empty" barrier.  No load uses
// multicast.

constexpr int kStages2 = 3;
constexpr int kSub2 = 2;  // 128-byte K sub-tiles per stage
constexpr int kStage2 = kTileM * kTileK;  // 16 KB: A rows, or half of the B tile
constexpr uint32_t kIdesc2 = (2u << 4) | (0u << 7) | (0u << 10) | ((256u >> 3) << 17) |
                             ((256u >> 4) << 24);
constexpr uint32_t kIdescBMajorMN = 1u << 16;  // B MN-major

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Shared::cluster address of the same variable in CTA rank 0 of the cluster.
__device__ __forceinline__ uint32_t in_rank0(const void* p) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(smem_u32(p)));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __noinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (*reinterpret_cast<volatile int*>(err) != 0) return false;
    if (clock64() - t0 > kTimeoutCycles) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t mbar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar_cluster)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, int x, int y,
                                                 int z, uint32_t mbar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(mbar_cluster)
      : "memory");
}

__device__ __forceinline__ void mma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive (when the prior MMAs complete) on the barrier at this address in
// both CTAs of the pair.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(mask)
      : "memory");
}

__device__ __forceinline__ void mma_commit_pair_self(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// kBMn: B's planes are [l][batch][Kp][Np] (N contiguous, from split_mn_kernel)
// and load as MN-major tiles through a 3-D tensor map {Np, Kp, planes};
// otherwise [l][batch][Np][Kp] like A's.
template <bool kBMn>
__global__ void __launch_bounds__(kGemmThreads, 1)
ozaki_gemm2_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + kStages2 * kSub2 * kStage2;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kStages2 * kSub2 * kStage2);
  uint64_t* empty = full + kStages2;
  uint64_t* tfull = empty + kStages2;
  uint64_t* tempty = tfull + 2;
  uint64_t* drained = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // 4 epilogue warps in each of the 2 CTAs
    }
    mbar_init(drained, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int64_t cid = cluster_id_x(), ncl = nclusters_x();

  if (warp == 0) {
    // ---- TMA producer (both CTAs) ----
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int64_t u = cid; u < p.units && ok; u += ncl) {
        const Unit w = unit_of(u, p);
        const int ya = static_cast<int>((static_cast<int64_t>(w.l) * p.batch + w.b) * p.Mp +
                                        static_cast<int64_t>(w.tm) * 256 + rank * 128);
        const int yb = static_cast<int>((static_cast<int64_t>(w.l) * p.batch + w.b) * p.Np +
                                        static_cast<int64_t>(w.tn) * 256 + rank * 128);
        const int xb = w.tn * 256 + static_cast<int>(rank) * 128;
        const int zb = w.l * p.batch + w.b;
        for (int kb = 0; kb < (p.kblocks + kSub2 - 1) / kSub2; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, 11)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&full[stage], 4 * kSub2 * kStage2);
          const uint32_t full0 = in_rank0(&full[stage]);
#pragma unroll
          for (int sub = 0; sub < kSub2; ++sub) {
            const int x = (kb * kSub2 + sub) * kTileK;
            tma_load_2d_pair(smem_a + (stage * kSub2 + sub) * kStage2, &tmap_a, x, ya, full0);
            if constexpr (kBMn)
              tma_load_3d_pair(smem_b + (stage * kSub2 + sub) * kStage2, &tmap_b, xb, x, zb, full0);
            else
              tma_load_2d_pair(smem_b + (stage * kSub2 + sub) * kStage2, &tmap_b, x, yb, full0);
          }
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        const long long t0 = clock64();
        while (clock64() - t0 < 200000) {
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (even CTA only) ----
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int64_t u = cid; u < p.units && ok; u += ncl) {
        if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1, p.err, 12)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * 256);
        constexpr uint32_t idesc = kBMn ? kIdesc2 | kIdescBMajorMN : kIdesc2;
        for (int kb = 0; kb < (p.kblocks + kSub2 - 1) / kSub2; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, 13)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int sub = 0; sub < kSub2; ++sub) {
            const uint32_t a0 = smem_u32(smem_a + (stage * kSub2 + sub) * kStage2);
            const uint32_t b0 = smem_u32(smem_b + (stage * kSub2 + sub) * kStage2);
#pragma unroll
            for (int k = 0; k < kTileK / 32; ++k) {
              // 32 k per instruction: 32 bytes along a K-major row, or 32
              // rows of 128 bytes of an MN-major tile
              const uint64_t bdesc = kBMn ? sdesc_mn(b0 + k * 32 * 128) : sdesc(b0 + k * 32);
              mma_i8_pair(d, sdesc(a0 + k * 32), bdesc, idesc, (kb | sub | k) != 0 ? 1u : 0u);
            }
          }
          mma_commit_pair(&empty[stage]);
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      mma_commit_pair_self(drained);
      const long long t0 = clock64();
      while (!mbar_try_wait(drained, 0) && clock64() - t0 < kTimeoutCycles) {
      }
    }
  } else {
    // ---- epilogue (both CTAs; warps 2..5, TMEM lanes 32*(warp%4) ..) ----
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t tempty0[2] = {in_rank0(&tempty[0]), in_rank0(&tempty[1])};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int64_t u = cid; u < p.units; u += ncl) {
      if (!mbar_wait(&tfull[acc], acc_phase, p.err, 14)) break;
      tc_fence_after();
      const Unit w = unit_of(u, p);
      const uint32_t m = static_cast<uint32_t>(mod_of(w.l));
      const uint32_t magic = epilogue_magic(m);
      const int64_t row = (static_cast<int64_t>(w.l) * p.batch + w.b) * p.Mp +
                          static_cast<int64_t>(w.tm) * 256 + rank * 128 + row_in_tile;
      uint8_t* out = p.cres + row * p.Np + static_cast<int64_t>(w.tn) * 256;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * 256);
#pragma unroll 1
      for (int c0 = 0; c0 < 256; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tbase + c0, v);
        uint32_t packed[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) packed[q] = mod_pack4(v + q * 4, m, magic);
        uint4* dst = reinterpret_cast<uint4*>(out + c0);
        dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty0[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// ---------------------------------------------------------------------------
// Step 3: CRT reconstruction and scaling.

struct CrtParams {
  double w[kL][2];
  double mlimb[2];
  double inv_m;
  // Outputs whose rebuilt integer |C_int| lies below this bound are not
  // certified by the quantisation error bound and are recomputed (below).
  double certify_below;
  int P;
  int* fix_count;      // err[1]
  uint64_t* fix_list;  // [fix_cap] flat output indices
  int64_t fix_cap;
  int64_t batch, M, N, Mp, Np, K;
  int64_t row_begin, row_end;  // rows of the flattened [batch * M] output this launch covers
  const uint8_t* cres;
  const int* sa;  // [batch][Mp]
  const int* sb;  // [batch][Np]
  const int* err;
  DotOperand a, b;
  DotResult c;
};

__device__ __forceinline__ void put_result(const DotResult& c, int64_t idx, double v) {
  if (c.f64) {
    c.f64[idx] = v;
  } else {
    const ds2 d = from_f64(v);
    c.hi[idx] = d.hi;
    c.lo[idx] = d.lo;
  }
}

constexpr int kCrtThreads = 128;
constexpr int kCrtCols = 4;  // consecutive outputs per thread: one residue word per plane

// Byte q of `word` as an f64: the bits of 2^52 + byte, minus 2^52 -- one
// add on the FP64 pipe instead of a quarter-rate integer conversion.
__device__ __forceinline__ double byte_to_f64(uint32_t word, int q) {
  const uint32_t byte = __byte_perm(word, 0u, 0x4440u + static_cast<uint32_t>(q));
  return __dsub_rn(__hiloint2double(0x43300000, static_cast<int>(byte)), 0x1p52);
}

// 2^e as an f64 for a normal exponent.
__device__ __forceinline__ double pow2_normal(int e) {
  return __longlong_as_double(static_cast<long long>(1023 + e) << 52);
}

// Error certificate.  A row of A enters the GEMM as a_int = rint(a 2^sa)
// with |a_int| <= 2^P, so |a 2^sa - a_int| <= 1/2; likewise for B.  In units
// of C_int the quantisation error of an output is at most
//     (||b_int||_1 + ||a_int||_1) / 2 + K / 4 <= K 2^P (+ K / 4),
// and the CRT's low limb adds below 2^34.  An output is certified when
// |C_int| >= 2^24 (K 2^P + 2^35): its error is then at most 2^-24 |C| (in
// practice far less: the quantisation errors are not aligned).  This bound
// is relative to the row maximum of A and the column maximum of B, so it
// fails exactly where those maxima do not take part in the output: a large
// entry facing zeros, values spread over many binades, or cancellation.
// Such outputs are recomputed with a compensated dot product (fix_kernel).
constexpr int kCertifyBits = 24;

__device__ __forceinline__ bool shift_ordinary(int s) {
  return s != kShiftNonFinite && s != kShiftZero;
}

// One output of the CRT from its two limbs: non-finite operands, zero rows
// and columns, and uncertified outputs (listed for fix_kernel) included.
__device__ __forceinline__ void crt_finish(const CrtParams& p, bool failed, int64_t row,
                                           int64_t b, int64_t i, int64_t j, int sa, int sb,
                                           double s_hi, double s_lo) {
  double out;
  if (failed) {
    out = __longlong_as_double(0x7ff8000000000000LL);
  } else if (sa == kShiftNonFinite || sb == kShiftNonFinite) {
    // A non-finite operand: the IEEE sum of the products carries NaN/Inf
    // as a float GEMM would.
    double s = 0.0;
    for (int64_t k = 0; k < p.K; ++k)
      s += op_value(p.a, b * p.a.s_b + i * p.a.s_r + k * p.a.s_k) *
           op_value(p.b, b * p.b.s_b + j * p.b.s_r + k * p.b.s_k);
    out = s;
  } else if (sa == kShiftZero || sb == kShiftZero) {
    out = 0.0;  // a row or column of zeros
  } else {
    // C = S - round(S / Mprod) * Mprod: the quotient is exact (S / Mprod
    // lies within 0.22 of an integer), the high limb difference is an
    // exact integer below 2^53, and the low limb carries the only
    // rounding (below 2^34 units of C_int).
    const double approx = __fma_rn(s_hi, 0x1p70, s_lo);
    const double qt = rint(approx * p.inv_m);
    const double t_hi = __fma_rn(-qt, p.mlimb[0], s_hi);
    const double t_lo = __fma_rn(-qt, p.mlimb[1], s_lo);
    const double c = __fma_rn(t_hi, 0x1p70, t_lo);
    if (!(fabs(c) >= p.certify_below)) {
      // uncertified: listed for fix_kernel, which writes this output
      const int slot = atomicAdd(p.fix_count, 1);
      if (slot < p.fix_cap) p.fix_list[slot] = static_cast<uint64_t>(row * p.N + j);
      return;
    }
    // scale by 2^-(sa + sb): one exact multiply when 2^-(sa+sb) is normal
    const int e = -(sa + sb);
    out = (e >= -1022 && e <= 1023) ? c * pow2_normal(e) : scale2(scale2(c, -sa), -sb);
  }
  put_result(p.c, row * p.N + j, out);
}

// The 14 residue words (4 outputs each) of one row of a thread.
__device__ __forceinline__ void crt_load(uint32_t (&w)[kL], const uint8_t* src, size_t plane) {
#pragma unroll
  for (int l = 0; l < kL; ++l) w[l] = __ldcs(reinterpret_cast<const unsigned int*>(src + l * plane));
}

// blockIdx.x * kCrtThreads * kCrtCols is the first column of the block;
// blockIdx.y strides over the batch*M output rows, so each thread rebuilds
// kCrtCols consecutive outputs of several rows (one 4-byte load per residue
// plane and row) with its columns' scale exponents loaded once per batch
// entry.  Rows and columns with ordinary shifts (the common case) take a
// path without per-output tests of the special codes, and store their four
// outputs as two 16-byte words when all four are certified.  Occupancy
// decides its speed: issuing the next row's loads before this row's
// arithmetic (80 registers) or capping the registers at 48 or 40 (spills)
// were 7 to 10% slower than 64 registers and 8 blocks per SM.
__global__ void __launch_bounds__(kCrtThreads, 8)
crt_kernel(CrtParams p) {
  constexpr int kCols = kCrtCols;
  wait_previous_grid();  // the GEMM's residues
  const size_t plane = static_cast<size_t>(p.batch) * p.Mp * p.Np;
  const bool failed = *p.err != 0;
  const int64_t j0 = (static_cast<int64_t>(blockIdx.x) * kCrtThreads + threadIdx.x) * kCols;
  int64_t row = p.row_begin + blockIdx.y;
  if (j0 >= p.N || row >= p.row_end) return;
  int64_t cur_b = -1;
  int sbv[kCols];
  bool cols_ordinary = false;  // all kCols columns exist and have ordinary shifts
  // (b, i) of the flattened row, advanced without a 64-bit division per row
  int64_t b = row / p.M;
  int64_t i = row - b * p.M;
  auto src_of = [&](int64_t bb, int64_t ii) {
    return p.cres + (static_cast<size_t>(bb) * p.Mp + ii) * p.Np + j0;
  };
  uint32_t cur[kL];
  crt_load(cur, src_of(b, i), plane);
  for (;;) {
    const int64_t next = row + gridDim.y;
    int64_t nb = b, ni = i + gridDim.y;
    while (ni >= p.M) {
      ni -= p.M;
      ++nb;
    }
    const bool more = next < p.row_end;
    if (b != cur_b) {
      cur_b = b;
      cols_ordinary = !failed && j0 + kCols <= p.N;
#pragma unroll
      for (int q = 0; q < kCols; ++q) {
        sbv[q] = j0 + q < p.N ? p.sb[b * p.Np + j0 + q] : 0;
        cols_ordinary &= shift_ordinary(sbv[q]);
      }
    }
    const int sa = p.sa[b * p.Mp + i];
    double s_hi[kCols], s_lo[kCols];
#pragma unroll
    for (int q = 0; q < kCols; ++q) s_hi[q] = s_lo[q] = 0.0;
#pragma unroll
    for (int l = 0; l < kL; ++l) {
      const double w_hi = p.w[l][0], w_lo = p.w[l][1];
#pragma unroll
      for (int q = 0; q < kCols; ++q) {
        const double r = byte_to_f64(cur[l], q);
        s_hi[q] = __fma_rn(r, w_hi, s_hi[q]);  // exact
        s_lo[q] = __fma_rn(r, w_lo, s_lo[q]);
      }
    }
    if (cols_ordinary && shift_ordinary(sa)) {
      double out[kCols];
      bool cert[kCols];
      bool all = true;
#pragma unroll
      for (int q = 0; q < kCols; ++q) {
        const double approx = __fma_rn(s_hi[q], 0x1p70, s_lo[q]);
        const double qt = rint(approx * p.inv_m);
        const double t_hi = __fma_rn(-qt, p.mlimb[0], s_hi[q]);
        const double t_lo = __fma_rn(-qt, p.mlimb[1], s_lo[q]);
        const double c = __fma_rn(t_hi, 0x1p70, t_lo);
        cert[q] = fabs(c) >= p.certify_below;
        all &= cert[q];
        if (!cert[q]) {
          // uncertified: listed for fix_kernel, which writes this output
          const int slot = atomicAdd(p.fix_count, 1);
          if (slot < p.fix_cap) p.fix_list[slot] = static_cast<uint64_t>(row * p.N + j0 + q);
        }
        const int e = -(sa + sbv[q]);
        out[q] = (e >= -1022 && e <= 1023) ? c * pow2_normal(e) : scale2(scale2(c, -sa), -sbv[q]);
      }
      double* dst = p.c.f64 ? p.c.f64 + row * p.N + j0 : nullptr;
      if (all && dst && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        reinterpret_cast<double2*>(dst)[0] = make_double2(out[0], out[1]);
        reinterpret_cast<double2*>(dst)[1] = make_double2(out[2], out[3]);
      } else {
#pragma unroll
        for (int q = 0; q < kCols; ++q)
          if (cert[q]) put_result(p.c, row * p.N + j0 + q, out[q]);
      }
    } else {
#pragma unroll
      for (int q = 0; q < kCols; ++q) {
        if (j0 + q >= p.N) break;
        crt_finish(p, failed, row, b, i, j0 + q, sa, sbv[q], s_hi[q], s_lo[q]);
      }
    }
    if (!more) break;
    row = next;
    b = nb;
    i = ni;
    crt_load(cur, src_of(b, i), plane);
  }
}

// ---- recomputation of uncertified outputs ----------------------------------
//
// sum_k a_ik b_kj by Ogita, Rump and Oishi's Dot2: each product split exactly
// by an FMA, the products summed with two_sum and the error terms summed
// aside, which is as accurate as the dot product evaluated in twice the
// working precision and then rounded.  Operands are scaled by 2^(sa - P) and
// 2^(sb - P) (below 1 in magnitude, so no product overflows); the scaling is
// undone at the end.

struct Dot2 {
  double p = 0.0, s = 0.0;
};

__device__ __forceinline__ void two_sum64(double a, double b, double& s, double& e) {
  s = __dadd_rn(a, b);
  const double bb = __dsub_rn(s, a);
  e = __dadd_rn(__dsub_rn(a, __dsub_rn(s, bb)), __dsub_rn(b, bb));
}

__device__ __forceinline__ void dot2_add(Dot2& d, double x, double y) {
  const double h = __dmul_rn(x, y);
  const double r = __fma_rn(x, y, -h);
  double q;
  two_sum64(d.p, h, d.p, q);
  d.s = __dadd_rn(d.s, __dadd_rn(q, r));
}

__device__ __forceinline__ void dot2_merge(Dot2& d, const Dot2& o) {
  double q;
  two_sum64(d.p, o.p, d.p, q);
  d.s = __dadd_rn(__dadd_rn(d.s, o.s), q);
}

struct FixParams {
  DotOperand a, b;
  DotResult c;
  int64_t batch, M, N, Mp, Np, K;
  int P;
  const int* sa;
  const int* sb;
  const int* err;  // [0] error word, [1] uncertified outputs
  const uint64_t* list;
  int64_t cap;
};

constexpr int kFixThreads = 256;
constexpr int kFixChains = 8;

// One output by one block: thread t owns k = t + 256 (8 n + u) in chain u
// (eight chains keep sixteen loads in flight), the chains are merged in a
// fixed tree, then the lanes of each warp, then the warps in order, so the
// result is deterministic.  Returns it on thread 0.
__device__ double dot2_block(const FixParams& p, int64_t b, int64_t i, int64_t j, int da, int db) {
  __shared__ Dot2 s_warp[kFixThreads / 32];
  const int64_t abase = b * p.a.s_b + i * p.a.s_r, bbase = b * p.b.s_b + j * p.b.s_r;
  constexpr int64_t kStep = static_cast<int64_t>(kFixThreads) * kFixChains;
  Dot2 ch[kFixChains];
  int64_t k = threadIdx.x;
  for (; k + (kFixChains - 1) * kFixThreads < p.K; k += kStep) {
    double x[kFixChains], y[kFixChains];
#pragma unroll
    for (int u = 0; u < kFixChains; ++u) {
      x[u] = op_value(p.a, abase + (k + kFixThreads * u) * p.a.s_k);
      y[u] = op_value(p.b, bbase + (k + kFixThreads * u) * p.b.s_k);
    }
#pragma unroll
    for (int u = 0; u < kFixChains; ++u) dot2_add(ch[u], scale2(x[u], da), scale2(y[u], db));
  }
  for (; k < p.K; k += kFixThreads)
    dot2_add(ch[0], scale2(op_value(p.a, abase + k * p.a.s_k), da),
             scale2(op_value(p.b, bbase + k * p.b.s_k), db));
#pragma unroll
  for (int w = 1; w < kFixChains; w <<= 1)
#pragma unroll
    for (int u = 0; u + w < kFixChains; u += 2 * w) dot2_merge(ch[u], ch[u + w]);
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    Dot2 o;
    o.p = __shfl_down_sync(0xffffffffu, ch[0].p, off);
    o.s = __shfl_down_sync(0xffffffffu, ch[0].s, off);
    if (lane + off < 32) dot2_merge(ch[0], o);
  }
  if (lane == 0) s_warp[threadIdx.x >> 5] = ch[0];
  __syncthreads();
  double v = 0.0;
  if (threadIdx.x == 0) {
    Dot2 d = s_warp[0];
    for (int w = 1; w < kFixThreads / 32; ++w) dot2_merge(d, s_warp[w]);
    v = scale2(scale2(__dadd_rn(d.p, d.s), -da), -db);
  }
  __syncthreads();  // s_warp is reused by the next output
  return v;
}


// A 64 x 64 output tile by one block: 16 x 16 threads, each with 4 x 4
// outputs (rows ty + 16 u, columns tx + 16 v), k in slabs of 16 staged in
// shared memory with the scaling applied.  Outputs of non-finite or zero
// rows and columns keep what the CRT wrote.
__device__ void dot2_tile(const FixParams& p, int64_t b, int64_t tm, int64_t tn) {
  __shared__ double sA[kFixTile][17];
  __shared__ double sB[16][kFixTile + 1];
  __shared__ int sShA[kFixTile], sShB[kFixTile];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t i0 = tm * kFixTile, j0 = tn * kFixTile;
  if (threadIdx.x < kFixTile) {
    const int64_t i = i0 + threadIdx.x, j = j0 + threadIdx.x;
    sShA[threadIdx.x] = i < p.M ? p.sa[b * p.Mp + i] : kShiftZero;
    sShB[threadIdx.x] = j < p.N ? p.sb[b * p.Np + j] : kShiftZero;
  }
  __syncthreads();
  auto usable = [](int sh) { return sh != kShiftNonFinite && sh != kShiftZero; };
  Dot2 acc[4][4];
  for (int64_t k0 = 0; k0 < p.K; k0 += 16) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int e = threadIdx.x + t * kFixThreads;  // 0 .. 1023
      {  // A: 64 rows x 16 k
        const int r = e >> 4, kk = e & 15;
        const int64_t i = i0 + r, k = k0 + kk;
        const int sh = sShA[r];
        double v = 0.0;
        if (k < p.K && usable(sh))
          v = scale2(op_value(p.a, b * p.a.s_b + i * p.a.s_r + k * p.a.s_k), sh - p.P);
        sA[r][kk] = v;
      }
      {  // B: 16 k x 64 columns
        const int kk = e >> 6, c = e & 63;
        const int64_t j = j0 + c, k = k0 + kk;
        const int sh = sShB[c];
        double v = 0.0;
        if (k < p.K && usable(sh))
          v = scale2(op_value(p.b, b * p.b.s_b + j * p.b.s_r + k * p.b.s_k), sh - p.P);
        sB[kk][c] = v;
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < 16; ++kk) {
      double x[4], y[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) x[u] = sA[ty + 16 * u][kk];
#pragma unroll
      for (int v = 0; v < 4; ++v) y[v] = sB[kk][tx + 16 * v];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) dot2_add(acc[u][v], x[u], y[v]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int64_t i = i0 + ty + 16 * u;
    const int sha = sShA[ty + 16 * u];
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int64_t j = j0 + tx + 16 * v;
      const int shb = sShB[tx + 16 * v];
      if (i < p.M && j < p.N && usable(sha) && usable(shb)) {
        const double r = __dadd_rn(acc[u][v].p, acc[u][v].s);
        put_result(p.c, (b * p.M + i) * p.N + j, scale2(scale2(r, p.P - sha), p.P - shb));
      }
    }
  }
}

// Writes every uncertified output: with at most `cap` of them, one block per
// listed output; with more (inputs whose rows or columns mostly defeat the
// certificate), every output is recomputed by the tiled Dot2 product, at
// CUDA-core FP64 speed.  Which of the two runs depends only on the count, so
// the result is deterministic.  Nothing to do costs one read.
__global__ void __launch_bounds__(kFixThreads, 2)
fix_kernel(FixParams p) {
  wait_previous_grid();  // the CRT's list
  const int count = p.err[1];
  if (count == 0 || p.err[0] != 0) return;
  if (count <= p.cap) {
    for (int64_t e = blockIdx.x; e < count; e += gridDim.x) {
      const uint64_t flat = p.list[e];
      const int64_t row = static_cast<int64_t>(flat / static_cast<uint64_t>(p.N));
      const int64_t j = static_cast<int64_t>(flat) - row * p.N;
      const int64_t b = row / p.M, i = row - b * p.M;
      const int sa = p.sa[b * p.Mp + i], sb = p.sb[b * p.Np + j];
      const double v = dot2_block(p, b, i, j, sa - p.P, sb - p.P);
      if (threadIdx.x == 0) put_result(p.c, static_cast<int64_t>(flat), v);
    }
    return;
  }
  const int64_t tm = (p.M + kFixTile - 1) / kFixTile, tn = (p.N + kFixTile - 1) / kFixTile;
  const int64_t tiles = p.batch * tm * tn;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t b = t / (tm * tn);
    const int64_t r = t - b * tm * tn;
    dot2_tile(p, b, r / tn, r % tn);
  }
}

// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

int make_tmap(CUtensorMap* map, const void* base, int64_t Kp, int64_t rows, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(DS_INTERNAL, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(Kp), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(Kp)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DS_INTERNAL, "cuTensorMapEncodeTiled failed");
  return DS_OK;
}

// Row-contiguous planes [planes][Kp][Np] (MN-major B): boxes of 128 rows
// (128 bytes) x 128 k of one plane.  k past Kp reads as zero.
int make_tmap_mn(CUtensorMap* map, const void* base, int64_t Np, int64_t Kp, int64_t planes) {
  auto fn = encode_fn();
  if (!fn) return set_error(DS_INTERNAL, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(Np), static_cast<cuuint64_t>(Kp),
                              static_cast<cuuint64_t>(planes)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(Np), static_cast<cuuint64_t>(Np * Kp)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kTileN / 2), static_cast<cuuint32_t>(kTileK),
                             1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DS_INTERNAL, "cuTensorMapEncodeTiled failed");
  return DS_OK;
}

size_t gemm_smem_bytes() {
  return 1024 + kStages * (kStageA + kStageB) + (2 * kStages + 5) * sizeof(uint64_t) + 16;
}

size_t gemm2_smem_bytes() {
  return 1024 + 2 * kStages2 * kSub2 * kStage2 + (2 * kStages2 + 5) * sizeof(uint64_t) + 16;
}

// Kernel choice and per-device launch limits, set up once per device.
struct GemmSetup {
  cudaError_t err = cudaSuccess;
  int pair_clusters = 0;  // co-resident CTA pairs (0: use the one-CTA kernel)
  int query_error = 0;    // cudaError_t of the cluster occupancy query
};

const GemmSetup& gemm_setup() {
  static std::mutex mu;
  static std::vector<GemmSetup> by_device;
  static std::vector<bool> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= static_cast<int>(by_device.size())) {
    by_device.resize(dev + 1);
    done.resize(dev + 1, false);
  }
  if (!done[dev]) {
    GemmSetup g;
    g.err = cudaFuncSetAttribute(ozaki_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(gemm_smem_bytes()));
    if (g.err == cudaSuccess)
      g.err = cudaFuncSetAttribute(ozaki_gemm2_kernel<false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(gemm2_smem_bytes()));
    if (g.err == cudaSuccess)
      g.err = cudaFuncSetAttribute(ozaki_gemm2_kernel<true>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(gemm2_smem_bytes()));
    const char* one = std::getenv("DS_B200_GEMM_1CTA");
    if (g.err == cudaSuccess && !(one && one[0] == '1')) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(2 * 74);
      cfg.blockDim = dim3(kGemmThreads);
      cfg.dynamicSmemBytes = gemm2_smem_bytes();
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      // both instantiations have the same resources
      const cudaError_t qe = cudaOccupancyMaxActiveClusters(&n, ozaki_gemm2_kernel<false>, &cfg);
      if (qe == cudaSuccess) {
        g.pair_clusters = n;
      } else {
        g.query_error = static_cast<int>(qe);
        cudaGetLastError();  // fall back to the one-CTA kernel
      }
    }
    by_device[dev] = g;
    done[dev] = true;
  }
  return by_device[dev];
}

// Split of one operand.  Rows contiguous in K take split_kmajor_kernel over
// rows [row0, row1) of the padded row range; other layouts take the column
// max and the tiled column split over all rows.
bool split_by_rows(const DotOperand& o, int64_t rows) { return o.s_k == 1 || rows == 1; }

// Pass 2 of a column split: K-major planes (split_cols_kernel), or with mn
// row-contiguous ones (split_mn_kernel).
cudaError_t launch_split_cols(const DotOperand& o, int64_t batch, int64_t rows, int64_t rows_pad,
                              int64_t K, int64_t Kp, int P, const int* codes, uint8_t* planes,
                              int* shifts, bool mn, cudaStream_t s) {
  ProfileScope prof("ozaki_split_cols", s);
  if (mn && o.f64) {
    // two blocks per SM in one wave, each over many k of one chunk
    const int64_t chunks = (rows_pad + kMnRows - 1) / kMnRows;
    int64_t ky = (2 * static_cast<int64_t>(sm_count()) + chunks * batch - 1) / (chunks * batch);
    if (ky > Kp) ky = Kp;
    if (ky > 65535) ky = 65535;
    dim3 g(static_cast<unsigned>(chunks), static_cast<unsigned>(ky < 1 ? 1 : ky),
           static_cast<unsigned>(batch));
    return launch_dependent(split_mn_async_kernel, g, dim3(256), s, o, rows, K, rows_pad, Kp,
                            batch, P, codes, planes, shifts);
  } else if (mn) {
    dim3 g(static_cast<unsigned>((rows_pad + kMnRows - 1) / kMnRows),
           static_cast<unsigned>((Kp + kMnSlab - 1) / kMnSlab), static_cast<unsigned>(batch));
    split_mn_kernel<<<g, 256, 0, s>>>(o, rows, K, rows_pad, Kp, batch, P, codes, planes, shifts);
  } else {
    dim3 g(static_cast<unsigned>(rows_pad / kColTileR), static_cast<unsigned>(Kp / kColTileK),
           static_cast<unsigned>(batch));
    split_cols_kernel<<<g, 256, 0, s>>>(o, rows, K, rows_pad, Kp, batch, P, codes, planes, shifts);
  }
  return cudaGetLastError();
}

int launch_split(const DotOperand& o, int64_t batch, int64_t rows, int64_t rows_pad, int64_t K,
                 int64_t Kp, int P, uint8_t* planes, int* shifts, int* codes, cudaStream_t s,
                 bool mn = false, int64_t row0 = 0, int64_t row1 = -1) {
  if (split_by_rows(o, rows)) {
    if (row1 < 0) row1 = rows_pad;
    ProfileScope prof("ozaki_split_rows", s);
    dim3 grid(static_cast<unsigned>(row1 - row0), static_cast<unsigned>(batch));
    split_kmajor_kernel<<<grid, split_rows_threads(K), 0, s>>>(o, rows, K, rows_pad, Kp, batch,
                                                               P, planes, shifts, row0);
  } else {
    DSB_CUDA_TRY(cudaMemsetAsync(codes, 0, sizeof(int) * batch * rows_pad, s));
    dim3 g1(static_cast<unsigned>(rows_pad / kColTileR),
            static_cast<unsigned>((K + kColmaxSlab - 1) / kColmaxSlab),
            static_cast<unsigned>(batch));
    {
      ProfileScope prof("ozaki_colmax", s);
      colmax_kernel<<<g1, 256, 0, s>>>(o, rows, K, rows_pad, codes);
    }
    DSB_CUDA_TRY(launch_split_cols(o, batch, rows, rows_pad, K, Kp, P, codes, planes, shifts, mn, s));
  }
  return launch_status();
}

}  // namespace

// Contractions longer than kMaxK run as chunks of kMaxK: each chunk is one
// exact integer product, rebuilt and rounded to f64, and the chunk results
// are added in f64 (one more rounding per chunk, far below the DS level).
bool dot_ozaki_supported(int64_t M, int64_t N, int64_t K) { return M >= 2 && N >= 2 && K >= 1; }

namespace {

int64_t k_chunks(int64_t K) { return (K + kMaxK - 1) / kMaxK; }

size_t chunk_result_bytes(int64_t batch, int64_t M, int64_t N) {
  return static_cast<size_t>(round_up(batch * M * N * static_cast<int64_t>(sizeof(double)), 1024));
}

__global__ void add_f64_kernel(double* __restrict__ acc, const double* __restrict__ part, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    acc[i] = __dadd_rn(acc[i], part[i]);
}

__global__ void store_result_kernel(DotResult c, const double* __restrict__ v, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    put_result(c, i, v[i]);
}

}  // namespace

size_t dot_ozaki_workspace_bytes(int64_t batch, int64_t M, int64_t N, int64_t K) {
  if (K <= kMaxK) return layout_of(batch, M, N, K).total;
  return layout_of(batch, M, N, kMaxK).total + 2 * chunk_result_bytes(batch, M, N);
}

int dot_ozaki_params(int64_t K, int* moduli, int* bits) {
  if (moduli) *moduli = kL;
  if (bits) *bits = bits_for_k(K);
  return DS_OK;
}

int dot_ozaki_kernel_info(int* cta_pairs, int* query_error) {
  const GemmSetup& g = gemm_setup();
  if (cta_pairs) *cta_pairs = g.pair_clusters;
  if (query_error) *query_error = g.query_error;
  return g.err == cudaSuccess ? DS_OK : cuda_status(g.err);
}

namespace {
int dot_ozaki_one(const DotProblem& p, void* workspace, size_t workspace_bytes, cudaStream_t s);
}

int dot_ozaki(const DotProblem& p, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  if (p.K <= kMaxK || p.batch == 0 || p.M == 0 || p.N == 0)
    return dot_ozaki_one(p, workspace, workspace_bytes, s);
  const size_t need = dot_ozaki_workspace_bytes(p.batch, p.M, p.N, p.K);
  if (workspace_bytes < need || !aligned(workspace, 256))
    return set_error(DS_INVALID_ARGUMENT, "dot_general: workspace too small (need " +
                                              std::to_string(need) + " bytes, 256-byte aligned)");
  const size_t one = layout_of(p.batch, p.M, p.N, kMaxK).total;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  double* acc = reinterpret_cast<double*>(ws + one);
  double* part = reinterpret_cast<double*>(ws + one + chunk_result_bytes(p.batch, p.M, p.N));
  const int64_t n = p.batch * p.M * p.N;
  const unsigned grid = grid_for(n, 256, 8);
  for (int64_t c = 0; c < k_chunks(p.K); ++c) {
    const int64_t k0 = c * kMaxK;
    DotProblem q = p;
    q.K = p.K - k0 < kMaxK ? p.K - k0 : kMaxK;
    auto shift = [k0](DotOperand& o) {
      const int64_t off = k0 * o.s_k;
      if (o.f64) o.f64 += off;
      if (o.hi) o.hi += off;
      if (o.lo) o.lo += off;
    };
    shift(q.a);
    shift(q.b);
    q.c = DotResult{c == 0 ? acc : part, nullptr, nullptr};
    if (int st = dot_ozaki_one(q, ws, one, s)) return st;
    if (c > 0) add_f64_kernel<<<grid, 256, 0, s>>>(acc, part, n);
  }
  store_result_kernel<<<grid, 256, 0, s>>>(p.c, acc, n);
  return launch_status();
}

namespace {

int dot_ozaki_one(const DotProblem& p, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  if (p.batch == 0 || p.M == 0 || p.N == 0) return ok();
  const Layout g = layout_of(p.batch, p.M, p.N, p.K);
  if (workspace_bytes < g.total || !aligned(workspace, 256))
    return set_error(DS_INVALID_ARGUMENT,
                     "dot_general: workspace too small (need " + std::to_string(g.total) +
                         " bytes, 256-byte aligned)");
  const int64_t max_rows = (1LL << 31) - 1;  // TMA y coordinates are int32
  if (p.batch > 65535 || kL * p.batch * g.Mp > max_rows || kL * p.batch * g.Np > max_rows ||
      g.Kp > max_rows)
    return set_error(DS_INVALID_ARGUMENT, "dot_general: problem too large for the tensor-core path");
  const GemmSetup& setup = gemm_setup();
  if (setup.err != cudaSuccess) return cuda_status(setup.err);
  const bool pair = setup.pair_clusters > 0;

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* planes_a = ws + g.off_a;
  uint8_t* planes_b = ws + g.off_b;
  uint8_t* cres = ws + g.off_c;
  int* sa = reinterpret_cast<int*>(ws + g.off_sa);
  int* sb = reinterpret_cast<int*>(ws + g.off_sb);
  int* ca = reinterpret_cast<int*>(ws + g.off_ca);
  int* cb = reinterpret_cast<int*>(ws + g.off_cb);
  int* err = reinterpret_cast<int*>(ws + g.off_err);
  const int P = bits_for_k(p.K);

  // B split by columns with its rows contiguous (a row-major [K, N] B) is
  // written N-contiguous and read by the pair kernel as an MN-major operand.
  const bool b_mn = pair && !split_by_rows(p.b, p.N) && p.b.s_r == 1;
  CUtensorMap ta, tb;
  if (int st = make_tmap(&ta, planes_a, g.Kp, kL * p.batch * g.Mp, kTileM)) return st;
  // The pair kernel loads half of each 256-row B tile per CTA.
  if (b_mn) {
    if (int st = make_tmap_mn(&tb, planes_b, g.Np, g.Kp, kL * p.batch)) return st;
  } else if (int st = make_tmap(&tb, planes_b, g.Kp, kL * p.batch * g.Np,
                                pair ? kTileN / 2 : kTileN)) {
    return st;
  }
  const int tile_rows = pair ? 2 * kTileM : kTileM;
  GemmParams gp{};
  gp.batch = static_cast<int>(p.batch);
  gp.tiles_n = static_cast<int>(g.Np / kTileN);
  gp.kblocks = static_cast<int>(g.Kp / kTileK);
  gp.Mp = g.Mp;
  gp.Np = g.Np;
  gp.cres = cres;
  gp.err = err;

  const CrtConsts& cc = crt_consts();
  CrtParams cp{};
  std::memcpy(cp.w, cc.w, sizeof(cp.w));
  std::memcpy(cp.mlimb, cc.mlimb, sizeof(cp.mlimb));
  cp.inv_m = cc.inv_m;
  cp.P = P;
  cp.certify_below =
      std::ldexp(static_cast<double>(p.K) * std::ldexp(1.0, P) + 0x1p35, kCertifyBits);
  cp.fix_count = err + 1;
  cp.fix_list = reinterpret_cast<uint64_t*>(ws + g.off_fix_list);
  cp.fix_cap = g.fix_cap;
  cp.batch = p.batch;
  cp.M = p.M;
  cp.N = p.N;
  cp.Mp = g.Mp;
  cp.Np = g.Np;
  cp.K = p.K;
  cp.cres = cres;
  cp.sa = sa;
  cp.sb = sb;
  cp.err = err;
  cp.a = p.a;
  cp.b = p.b;
  cp.c = p.c;

  // GEMM over tile rows [tm0, tm0 + tiles) on stream `st`.
  auto launch_gemm = [&](int tm0, int tiles, cudaStream_t st) -> int {
    GemmParams q = gp;
    q.tm0 = tm0;
    q.tiles_m = tiles;
    q.units = static_cast<int64_t>(kL) * p.batch * tiles * q.tiles_n;
    ProfileScope prof("ozaki_gemm", st);
    if (pair) {
      const int64_t clusters = q.units < setup.pair_clusters ? q.units : setup.pair_clusters;
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters));
      cfg.blockDim = dim3(kGemmThreads);
      cfg.dynamicSmemBytes = gemm2_smem_bytes();
      cfg.stream = st;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (b_mn)
        DSB_CUDA_TRY(cudaLaunchKernelEx(&cfg, ozaki_gemm2_kernel<true>, ta, tb, q));
      else
        DSB_CUDA_TRY(cudaLaunchKernelEx(&cfg, ozaki_gemm2_kernel<false>, ta, tb, q));
    } else {
      const int grid = static_cast<int>(q.units < sm_count() ? q.units : sm_count());
      ozaki_gemm_kernel<<<grid, kGemmThreads, gemm_smem_bytes(), st>>>(ta, tb, q);
    }
    return launch_status();
  };
  // CRT of output rows [r0, r1) of the flattened [batch * M] result.
  auto launch_crt = [&](int64_t r0, int64_t r1, cudaStream_t st) -> int {
    if (r1 <= r0) return ok();
    CrtParams q = cp;
    q.row_begin = r0;
    q.row_end = r1;
    ProfileScope prof("ozaki_crt", st);
    // about 16 blocks of 128 threads per SM in one wave, each thread taking
    // several rows
    const int64_t n = r1 - r0;
    const int64_t gx = (p.N + kCrtThreads * kCrtCols - 1) / (kCrtThreads * kCrtCols);
    int64_t gy = (static_cast<int64_t>(sm_count()) * 16 + gx - 1) / gx;
    if (gy > n) gy = n;
    if (gy > 65535) gy = 65535;
    dim3 cg(static_cast<unsigned>(gx), static_cast<unsigned>(gy < 1 ? 1 : gy));
    DSB_CUDA_TRY(launch_dependent(crt_kernel, cg, dim3(kCrtThreads), st, q));
    return launch_status();
  };

  // One stream, one launch per step: nothing else runs beside the GEMM.  An
  // overlapped schedule (bands of A's rows, the GEMM of band i on a second
  // stream beside the split of band i + 1 and the CRT of band i - 1) left
  // CTA pairs of the GEMM blocked in tcgen05.alloc on some SMs; it is not
  // used.
  // A split by rows and B by columns (the usual row-major A and B): the
  // column maxima of B are taken in the same launch as A's row split.
  uint8_t* const clear_end = reinterpret_cast<uint8_t*>(err + 2);
  const bool merged = p.batch == 1 && split_by_rows(p.a, p.M) && !split_by_rows(p.b, p.N) &&
                      split_rows_threads(p.K) == 256;
  if (merged) {
    ProfileScope prof("ozaki_split", s);
    // B's column-maximum codes, the error word and the uncertified-output
    // count are neighbours in the workspace (in that order): one memset
    // clears them all
    DSB_CUDA_TRY(cudaMemsetAsync(cb, 0, clear_end - reinterpret_cast<uint8_t*>(cb), s));
    const int64_t cgx = g.Np / kColTileR, cgy = (p.K + kColmaxSlab - 1) / kColmaxSlab;
    const int64_t nc = cgx * cgy;
    {
      ProfileScope prof2("ozaki_split_rows_colmax", s);
      split_rows_colmax_kernel<<<static_cast<unsigned>(g.Mp + nc), 256, 0, s>>>(
          p.a, p.M, g.Mp, p.b, p.N, g.Np, p.K, g.Kp, P, planes_a, sa, cb, nc, cgx, cgy);
      if (int st = launch_status()) return st;
    }
    DSB_CUDA_TRY(launch_split_cols(p.b, 1, p.N, g.Np, p.K, g.Kp, P, cb, planes_b, sb, b_mn, s));
    if (int st = launch_status()) return st;
  } else {
    DSB_CUDA_TRY(cudaMemsetAsync(err, 0, clear_end - reinterpret_cast<uint8_t*>(err), s));
    ProfileScope prof("ozaki_split", s);
    if (int st = launch_split(p.a, p.batch, p.M, g.Mp, p.K, g.Kp, P, planes_a, sa, ca, s))
      return st;
    if (int st = launch_split(p.b, p.batch, p.N, g.Np, p.K, g.Kp, P, planes_b, sb, cb, s, b_mn))
      return st;
  }
  if (int st = launch_gemm(0, static_cast<int>(g.Mp / tile_rows), s)) return st;
  if (int st = launch_crt(0, p.batch * p.M, s)) return st;
  FixParams fp{};
  fp.a = p.a;
  fp.b = p.b;
  fp.c = p.c;
  fp.batch = p.batch;
  fp.M = p.M;
  fp.N = p.N;
  fp.Mp = g.Mp;
  fp.Np = g.Np;
  fp.K = p.K;
  fp.P = P;
  fp.sa = sa;
  fp.sb = sb;
  fp.err = err;
  fp.list = cp.fix_list;
  fp.cap = g.fix_cap;
  ProfileScope prof("ozaki_fix", s);
  DSB_CUDA_TRY(launch_dependent(fix_kernel, dim3(static_cast<unsigned>(2 * sm_count())),
                                dim3(kFixThreads), s, fp));
  return launch_status();
}

}  // namespace

}  // namespace dsb
