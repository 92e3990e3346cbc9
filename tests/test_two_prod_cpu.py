"""Where an FMA gives Dekker's two_prod bits.

The reference computes the error of an f32 product with Dekker's algorithm
on Veltkamp's 4097 split (cpp/ds_mul.cpp:15-34).  An FMA computes the same
error exactly, e = RN(a*b - p), and the recurrence kernels use it when

    |a|, |b| < 2^115 and 2^-90 <= |p| <= 2^120   (p = RN(a*b))

(they test |b| in [2^-5, 2^115) once and |p| in [2^-90, 2^110] per product,
which implies it), falling back to Dekker elsewhere.  In that range the
split cannot overflow and no partial product drops bits below the subnormal
grid, so Dekker's e is the exact error too: the two agree bit for bit.  This
checks that on random operands over the whole exponent range, with the exact
error taken from the f64 product (a*b is exact in f64: 24 + 24 bits).
"""
import numpy as np

F32 = np.float32


def split(a):
    t = F32(4097.0) * a
    hi = t - (t - a)
    return hi, a - hi


def dekker(a, b):
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        p = a * b
        ah, al = split(a)
        bh, bl = split(b)
        e = (((ah * bh - p) + ah * bl) + al * bh) + al * bl
    return p, e


def in_fma_range(a, b, p):
    ap = np.abs(p)
    return (np.abs(a) < F32(2.0 ** 115)) & (np.abs(b) < F32(2.0 ** 115)) & \
           (ap >= F32(2.0 ** -90)) & (ap <= F32(2.0 ** 120))


def kernel_range(a, b, p):
    """The test the recurrence kernels apply (a subset of in_fma_range)."""
    ab, ap = np.abs(b), np.abs(p)
    return (ab >= F32(2.0 ** -5)) & (ab < F32(2.0 ** 115)) & (ap >= F32(2.0 ** -90)) & \
           (ap <= F32(2.0 ** 110))


def random_f32(rng, n, lo, hi):
    """Random signs, 24-bit mantissas and exponents in [lo, hi)."""
    m = rng.integers(1 << 23, 1 << 24, n).astype(np.float64)
    e = rng.integers(lo, hi, n)
    s = np.where(rng.integers(0, 2, n) == 0, 1.0, -1.0)
    return (s * np.ldexp(m, e - 23)).astype(F32)


def test_fma_error_term_equals_dekker_in_range():
    rng = np.random.default_rng(17)
    checked = 0
    for lo, hi in ((-149, 128), (-60, 60), (-75, -20), (55, 64), (-10, 10)):
        a = random_f32(rng, 400_000, lo, hi)
        b = random_f32(rng, 400_000, lo, hi)
        p, e = dekker(a, b)
        ok = in_fma_range(a, b, p)
        assert np.all(ok[kernel_range(a, b, p)])
        exact = (a.astype(np.float64) * b.astype(np.float64) - p.astype(np.float64))
        fma = exact.astype(F32)  # the FMA's RN(a*b - p); exact in range
        assert np.all(fma[ok].astype(np.float64) == exact[ok])
        assert np.array_equal(e[ok].view(np.uint32), fma[ok].view(np.uint32))
        checked += int(ok.sum())
    assert checked > 1_000_000


def test_range_edges():
    """Operands at the edges of the range, zero products and exact products."""
    edges = [F32(v) for v in (2.0 ** 114.9, 2.0 ** 60, 2.0 ** 45, 1.0, 1.5, 3.0, 2.0 ** -45,
                              2.0 ** -46, 2.0 ** -60, 1 + 2.0 ** -23, 2.0 ** -90, 2.0 ** 120)]
    vals = np.array([s * v for v in edges for s in (1, -1)], F32)
    a, b = np.meshgrid(vals, vals)
    a, b = a.ravel(), b.ravel()
    p, e = dekker(a, b)
    ok = in_fma_range(a, b, p)
    exact = (a.astype(np.float64) * b.astype(np.float64) - p.astype(np.float64)).astype(F32)
    assert ok.sum() > 100
    assert np.array_equal(e[ok].view(np.uint32), exact[ok].view(np.uint32))
