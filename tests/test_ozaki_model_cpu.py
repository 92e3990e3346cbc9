"""CPU model of the tensor-core dot_general's integer arithmetic.

The GPU kernel (ds-experiment_b200/csrc/dot_ozaki.cu) quantises each operand
row to a P-bit integer, multiplies residues modulo 14 coprime moduli exactly,
and rebuilds the product by the Chinese remainder theorem in two f64 limbs
(the weights split at bit 70).  This restates those steps in NumPy/Python
integers at small sizes: the byte-dot-product residues of the biased
quantised integers (in [0, m)), the FP64-pipe residues of half of the
moduli (in [0, 255], not always below m), the unsigned residue GEMM with the
epilogue's reduction, and the two-limb reconstruction, whose only rounding
is far below the quantisation error.
"""
import math
from fractions import Fraction

import numpy as np

from oracle import exact

MODULI = [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199]
FP64_PATH = set(range(1, 11))  # indices of the moduli split on the FP64 pipe
SPLIT = 70  # W = W_hi * 2^70 + W_lo
MAGIC = 1.5 * 2.0 ** 52


def consts():
    M = math.prod(MODULI)
    W = []
    for m in MODULI:
        Ml = M // m
        inv = pow(Ml % m, -1, m)
        W.append(Ml * inv)
    return M, W


def bits_for_k(K):
    M, _ = consts()
    P = math.floor((math.log2(M) - 2.0 - math.log2(max(K, 1))) / 2.0)
    return min(P, 50)


def test_moduli_pairwise_coprime():
    for i, a in enumerate(MODULI):
        for b in MODULI[i + 1:]:
            assert math.gcd(a, b) == 1
    M, _ = consts()
    assert 110 < math.log2(M) < 111


def quantise(X, P):
    """Row-wise: shift = P - (ilogb(max|x|) + 1); x_int = rint(x * 2^shift)."""
    shifts = []
    ints = []
    for row in X:
        mx = np.max(np.abs(row))
        e = 0 if mx == 0 else math.frexp(mx)[1]  # mx < 2^e
        sh = P - e
        q = np.rint(np.ldexp(row, sh))
        assert np.max(np.abs(q)) <= 2.0 ** P
        shifts.append(sh)
        ints.append([int(v) for v in q])
    return ints, shifts


def byte_residue(x_int, m):
    """The split kernel's residue: t = x_int + 2^51 as seven bytes, dotted
    with the weights 2^(8j) mod m (two 4-byte dot products), plus the
    constant that cancels the bias, then s - m * umulhi(s, ceil(2^32 / m))."""
    t = x_int + 2 ** 51
    assert 0 <= t < 2 ** 52
    if m == 256:
        return t & 255
    w = [pow(2, 8 * j, m) for j in range(7)]
    unbias = (m - pow(2, 51, m)) % m
    s = sum(((t >> (8 * j)) & 255) * w[j] for j in range(7)) + unbias
    assert s < 2 ** 19
    magic = (2 ** 32 - 1) // m + 1
    return s - ((s * magic) >> 32) * m


def rint_even(f):
    """Round a Fraction to the nearest integer, ties to even."""
    fl = math.floor(f)
    d = f - fl
    if d > Fraction(1, 2) or (d == Fraction(1, 2) and fl % 2 == 1):
        return fl + 1
    return fl


def fp64_residue(x_int, m):
    """The split kernel's FP64-pipe residue: fma(x - 128, RN(1/m), 1.5 * 2^52)
    = 1.5 * 2^52 + q ((x - 128) * RN(1/m) rounded to an integer, ties to
    even), then x.lo - (low word of that) * m in 32-bit arithmetic, which is
    x - q m when x - q m lies in [0, 2^32)."""
    inv = Fraction(1.0 / m)  # the double nearest 1/m, exactly
    q = rint_even(Fraction(x_int - 128) * inv)
    qd = Fraction(MAGIC) + q  # the fma's result, exact: a double with ulp 1
    assert qd == int(qd) and 2 ** 52 <= qd < 2 ** 53
    t = x_int + 2 ** 51  # the split's biased integer; its low word is x.lo
    r32 = ((t & 0xFFFFFFFF) - (int(qd) & 0xFFFFFFFF) * m) & 0xFFFFFFFF
    assert r32 == x_int - q * m
    return r32


def residue(x_int, l):
    """The residue of modulus index l as the split writes it (a byte)."""
    m = MODULI[l]
    return fp64_residue(x_int, m) if l in FP64_PATH else byte_residue(x_int, m)


def test_fp64_residues():
    """x - q m is in [0, 255] for |x| <= 2^50, including x next to the
    points where (x - 128) / m is a half-integer and the rounded quotient
    may pick either neighbour."""
    rng = np.random.default_rng(4)
    for l in FP64_PATH:
        m = MODULI[l]
        vals = [0, 1, -1, 127, 128, 129, 2 ** 50, -(2 ** 50), 2 ** 50 - 1]
        vals += [int(v) for v in rng.integers(-(2 ** 50), 2 ** 50, 4000)]
        for k in [int(v) for v in rng.integers(-(2 ** 50) // m, 2 ** 50 // m, 400)]:
            for d in (-1, 0, 1):
                vals.append(128 + k * m + m // 2 + d)
                vals.append(128 + k * m - m // 2 + d)
        for x in vals:
            if abs(x) > 2 ** 50:
                continue
            r = fp64_residue(x, m)
            assert 0 <= r <= 255
            assert (x - r) % m == 0


def test_byte_residues():
    rng = np.random.default_rng(3)
    edges = [0, 1, -1, 2 ** 50, -(2 ** 50), 2 ** 50 - 1, 12345678901234]
    vals = edges + [int(v) for v in rng.integers(-(2 ** 50), 2 ** 50, 20000)]
    for m in MODULI:
        for x in vals:
            assert byte_residue(x, m) == x % m


def crt_limbs(residues):
    """The kernel's two-limb f64 reconstruction, step by step: s_hi exact,
    s_lo rounded, q = rint(S / M) exact, t_hi exact, one final rounding."""
    M, W = consts()
    lo_mask = (1 << SPLIT) - 1
    w_hi = [float(w >> SPLIT) for w in W]
    w_lo = [float(w & lo_mask) for w in W]
    m_hi, m_lo = float(M >> SPLIT), float(M & lo_mask)
    s_hi = s_lo = 0.0
    for r, wh, wl in zip(residues, w_hi, w_lo):
        s_hi = float(r) * wh + s_hi  # exact: < 2^53
        s_lo = float(r) * wl + s_lo  # rounded (numpy has no fma; error within the bound)
    approx = s_hi * 2.0 ** SPLIT + s_lo
    q = float(np.rint(approx * (1.0 / float(M))))
    t_hi = s_hi - q * m_hi
    t_lo = s_lo - q * m_lo
    return t_hi * 2.0 ** SPLIT + t_lo, (s_hi, q, t_hi)


# Absolute error of the reconstruction in units of C_int: the rounded low
# limb (weights rounded to 53 bits, 14 rounded accumulations, q * m_lo) stays
# below 2^34; one unit of C_int is 2^-2P of max|a_row| * max|b_col|.
CRT_ABS_ERR = 2.0 ** 34


def test_crt_limbs_accuracy():
    rng = np.random.default_rng(0)
    M, W = consts()
    assert max(w >> SPLIT for w in W) < 2 ** 41
    assert 14 * 255 * max(w >> SPLIT for w in W) < 2 ** 53
    for K in (1, 64, 4096, 8192, 32768):
        P = bits_for_k(K)
        bound = K * 2 ** (2 * P)
        assert 4 * bound <= M
        for _ in range(200):
            c = int(rng.integers(-2 ** 62, 2 ** 62)) * int(rng.integers(0, 2 ** 40)) % bound
            c = c if rng.random() < 0.5 else -c
            res = [c % m for m in MODULI]
            got, (s_hi, q, t_hi) = crt_limbs(res)
            for v in (s_hi, t_hi):
                assert abs(v) < 2.0 ** 53 and v == int(v)
            assert int(q) == (sum(r * w for r, w in zip(res, W)) - c) // M
            assert abs(got - c) <= CRT_ABS_ERR + abs(c) * 2.0 ** -52


def model_gemm(A, B):
    K = A.shape[1]
    P = bits_for_k(K)
    ai, sa = quantise(A, P)
    bi, sb = quantise(B.T, P)
    M_rows, N_cols = A.shape[0], B.shape[1]
    out = np.empty((M_rows, N_cols))
    for i in range(M_rows):
        for j in range(N_cols):
            exact_int = sum(x * y for x, y in zip(ai[i], bi[j]))
            # per-modulus GEMM on unsigned residues (u8 x u8 -> s32), as the
            # tensor cores do; the epilogue keeps the sum mod m
            res = []
            for l, m in enumerate(MODULI):
                acc = sum(residue(x, l) * residue(y, l) for x, y in zip(ai[i], bi[j]))
                assert 0 <= acc < 2 ** 31
                res.append(acc % m)
            got, _ = crt_limbs(res)
            assert abs(got - exact_int) <= CRT_ABS_ERR + abs(exact_int) * 2.0 ** -52
            out[i, j] = math.ldexp(got, -(sa[i] + sb[j]))
    return out


def test_model_gemm_accuracy():
    rng = np.random.default_rng(1)
    A = rng.uniform(-1, 1, (4, 300))
    B = rng.uniform(-1, 1, (300, 3))
    got = model_gemm(A, B)
    rows, cols = np.meshgrid(range(4), range(3), indexing="ij")
    truth = exact.exact_gemm_entries(A, B, rows.ravel(), cols.ravel()).reshape(4, 3)
    mag = np.abs(A) @ np.abs(B)
    assert np.max(np.abs(got - truth) / mag) < 2.0 ** -46


def test_epilogue_modulo():
    """The GEMM epilogue's v mod m = v - m * (umulhi(v, ceil(2^39/m)) >> 7),
    exact for every s32 accumulator value 0 <= v < 2^31."""
    rng = np.random.default_rng(9)
    vals = [0, 1, 2 ** 31 - 1, 2 ** 30, 255 * 255 * 32768] + \
        [int(v) for v in rng.integers(0, 2 ** 31, 50000)]
    for m in MODULI:
        magic = (2 ** 39 + m - 1) // m
        assert magic < 2 ** 32
        assert (2 ** 31) * (magic * m - 2 ** 39) < 2 ** 39
        for v in vals + [k * m - 1 for k in range(1, 2 ** 31 // m, 2 ** 31 // m // 1000)]:
            q = ((v * magic) >> 32) >> 7
            assert v - q * m == v % m


def _ozaki_exact(A, B):
    """C_int of the quantised operands (Python integers) and the shifts."""
    K = A.shape[1]
    P = bits_for_k(K)
    qa, sa = quantise(A, P)
    qb, sb = quantise(B.T, P)
    C = [[sum(x * y for x, y in zip(ra, rb)) for rb in qb] for ra in qa]
    return C, sa, sb, P


def test_certificate_bounds_the_quantisation_error():
    """An output with |C_int| >= 2^24 (K 2^P + 2^35) has error at most
    2^-24 |C| against the exact product; the bound is checked on inputs that
    defeat the row-maximum scaling (a large entry facing zeros, values over
    60 binades) and on plain uniform ones."""
    rng = np.random.default_rng(5)
    M, K, N = 12, 96, 10
    cases = [rng.uniform(-1, 1, (M, K)), rng.uniform(-1, 1, (M, K)) * 2.0 ** -rng.uniform(0, 60, (M, K))]
    wide = rng.uniform(-1, 1, (M, K)) * 2.0 ** -30
    wide[:, 0] = 1.0
    cases.append(wide)
    for A in cases:
        B = rng.uniform(-1, 1, (K, N)) * 2.0 ** -rng.uniform(0, 20, (K, N))
        B[0, ::2] = 0.0
        C, sa, sb, P = _ozaki_exact(A, B)
        bound = 2 ** 24 * (K * 2 ** P + 2 ** 35)
        certified = 0
        for i in range(M):
            for j in range(N):
                if abs(C[i][j]) < bound:
                    continue
                certified += 1
                got = math.ldexp(float(C[i][j]), -(sa[i] + sb[j]))
                truth = exact.exact_dot(A[i], B[:, j])
                assert abs(got - truth) <= 2.0 ** -24 * abs(got), (i, j, got, truth)
        assert certified > 0
