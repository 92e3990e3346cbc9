"""CPU model of the tensor-core dot_general's integer arithmetic.

The GPU kernel (ds-experiment_b200/csrc/dot_ozaki.cu) quantises each operand
row to a P-bit integer, multiplies residues modulo 14 coprime moduli exactly,
and rebuilds the product by the Chinese remainder theorem in three 40-bit f64
limbs.  This restates those steps in NumPy/Python integers at small sizes to
check that the chosen P keeps the CRT exact and that the limb arithmetic
reproduces the exact integer product.
"""
import math

import numpy as np

from oracle import exact

MODULI = [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199]
MASK40 = (1 << 40) - 1


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


def sym_residue(x, m):
    r = x % m
    if r > (m - 1) // 2:
        r -= m
    return r


def crt_limbs(residues):
    """The kernel's f64 three-limb reconstruction, step by step."""
    M, W = consts()
    wl = [(w & MASK40, (w >> 40) & MASK40, w >> 80) for w in W]
    ml = (M & MASK40, (M >> 40) & MASK40, M >> 80)
    s = [0.0, 0.0, 0.0]
    for r, w in zip(residues, wl):
        for j in range(3):
            s[j] = float(r) * float(w[j]) + s[j]  # exact: all < 2^53
    approx = s[2] * 2.0 ** 80 + s[1] * 2.0 ** 40
    Md = ml[2] * 2.0 ** 80 + ml[1] * 2.0 ** 40 + ml[0]
    q = float(np.rint(approx * (1.0 / Md)))
    t = [s[j] - q * float(ml[j]) for j in range(3)]
    hi = t[2] * 2.0 ** 40 + t[1]
    return hi * 2.0 ** 40 + t[0], (s, q, t)


def test_crt_limbs_exact():
    rng = np.random.default_rng(0)
    M, _ = consts()
    for K in (1, 64, 4096, 8192, 65536):
        P = bits_for_k(K)
        bound = K * 2 ** (2 * P)
        assert 4 * bound <= M
        for _ in range(200):
            c = int(rng.integers(-2 ** 62, 2 ** 62)) * int(rng.integers(0, 2 ** 40)) % bound
            c = c if rng.random() < 0.5 else -c
            res = [c % m for m in MODULI]
            got, (s, q, t) = crt_limbs(res)
            for v in s + t:
                assert abs(v) < 2.0 ** 53 and v == int(v)
            assert got == float(c) or abs(got - c) <= abs(c) * 2.0 ** -52


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
            # per-modulus GEMM on symmetric residues, as the tensor cores do
            res = []
            for m in MODULI:
                acc = sum(sym_residue(x, m) * sym_residue(y, m) for x, y in zip(ai[i], bi[j]))
                assert abs(acc) < 2 ** 31
                res.append(acc % m)
            got, _ = crt_limbs(res)
            assert got == float(exact_int) or abs(got - exact_int) <= abs(exact_int) * 2.0 ** -52
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
