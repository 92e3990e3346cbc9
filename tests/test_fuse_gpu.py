"""Fused elementwise programs on the GPU: bit-exact against the C oracle
composing the same DS operations (the pass's per-op lowering), with
broadcasting, f32 and packed inputs, and every output type."""
import numpy as np
import pytest

from conftest import assert_bits_equal
from gpu_util import cu, host

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fuse():
    from ds_b200 import fuse as _fuse
    return _fuse


class OracleDS:
    """A DS value on the host: packed [..., 2] f32 evaluated with the oracle."""

    def __init__(self, dso, p):
        self.dso, self.p = dso, np.ascontiguousarray(p, np.float32)

    def _o(self, other):
        if isinstance(other, OracleDS):
            return other.p
        return self.dso.ds_from_f64(np.full(self.p.shape[:-1], float(other)))

    def __add__(self, o):
        return OracleDS(self.dso, self.dso.ds_add(self.p, self._o(o)))

    def __radd__(self, o):
        return OracleDS(self.dso, self.dso.ds_add(self._o(o), self.p))

    def __sub__(self, o):
        return OracleDS(self.dso, self.dso.ds_sub(self.p, self._o(o)))

    def __rsub__(self, o):
        return OracleDS(self.dso, self.dso.ds_sub(self._o(o), self.p))

    def __mul__(self, o):
        return OracleDS(self.dso, self.dso.ds_mul(self.p, self._o(o)))

    def __rmul__(self, o):
        return OracleDS(self.dso, self.dso.ds_mul(self._o(o), self.p))

    def __neg__(self):
        return OracleDS(self.dso, -self.p)


def oracle_eval(dso, fn, args, shape):
    """fn on broadcast host arrays through the oracle's DS ops."""
    vals = []
    for a in args:
        if isinstance(a, float):
            vals.append(a)
            continue
        kind, arr = a
        if kind == "packed":
            p = np.broadcast_to(arr, shape + (2,))
        else:
            b = np.broadcast_to(arr, shape)
            p = dso.ds_from_f64(b.ravel()).reshape(shape + (2,)) if kind == "f64" else \
                dso.ds_from_f32(b.ravel()).reshape(shape + (2,))
        vals.append(OracleDS(dso, p))
    return fn(*vals).p


def f3(x, y, z):
    return (x + y) * z - 0.1 * x


@pytest.mark.parametrize("n", [1, 7, 1000, (1 << 20) + 3])
def test_full_f64_bit_exact(fuse, dso, n):
    rng = np.random.default_rng(n)
    x, y, z = (rng.uniform(-1, 1, n) for _ in range(3))
    got = host(fuse.jit(f3)(cu(x), cu(y), cu(z)))
    want = dso.ds_to_f64(oracle_eval(dso, f3, [("f64", x), ("f64", y), ("f64", z)], (n,)))
    assert_bits_equal(got, want, "f3")


def test_config1_chain_matches_hand_written_kernel(fuse, dso):
    from ds_b200 import ops
    rng = np.random.default_rng(0)
    a, b, c = (rng.uniform(-1, 1, 1 << 20) for _ in range(3))
    got = host(fuse.jit(lambda a, b, c: (a + b) * c)(cu(a), cu(b), cu(c)))
    assert_bits_equal(got, host(ops.ds_fused_add_mul3_to_f64(cu(a), cu(b), cu(c))), "config 1")
    assert_bits_equal(got, dso.ds_fused_add_mul3_to_f64(a, b, c), "oracle")


def test_broadcast_f32_and_scalars(fuse, dso):
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, (37, 513))
    row = rng.uniform(-1, 1, 513)
    col = rng.uniform(-1, 1, (37, 1)).astype(np.float32)
    g = fuse.jit(f3)
    got = host(g(cu(x), cu(row), cu(col)))
    want = dso.ds_to_f64(oracle_eval(dso, f3, [("f64", x), ("f64", row), ("f32", col)],
                                     (37, 513)).reshape(-1, 2)).reshape(37, 513)
    assert_bits_equal(got, want, "broadcast")
    # a scalar argument is a constant split like an f64 argument
    h = fuse.jit(lambda v, c: v * c - c)
    got = host(h(cu(x), 1.0 / 3.0))
    want = dso.ds_to_f64(oracle_eval(dso, lambda v, c: v * c - c, [("f64", x), 1.0 / 3.0],
                                     (37, 513)).reshape(-1, 2)).reshape(37, 513)
    assert_bits_equal(got, want, "scalar")


def test_packed_io_and_f32_output(fuse, dso):
    rng = np.random.default_rng(5)
    x = rng.uniform(-1, 1, 4099)
    px = dso.ds_from_f64(x)
    import torch
    g = fuse.jit(lambda p, q: p * p - q, out_dtype="packed")
    got = host(g(fuse.Packed(cu(px)), cu(x)))
    want = oracle_eval(dso, lambda p, q: p * p - q, [("packed", px), ("f64", x)], (4099,))
    assert_bits_equal(got, want, "packed")
    x32 = x.astype(np.float32)
    got32 = host(fuse.jit(lambda a: -a * a + 2.0)(cu(x32)))
    want32 = dso.ds_to_f32(oracle_eval(dso, lambda a: -a * a + 2.0, [("f32", x32)], (4099,)))
    assert got32.dtype == np.float32
    assert_bits_equal(got32, want32, "f32 out")


def test_unrolled_recurrence_matches_oracle(fuse, dso):
    """x <- x*a + b four times in one program, against the oracle's
    recurrence (the same DS operations in the same order)."""
    rng = np.random.default_rng(3)
    n = 1 << 16
    x0 = rng.uniform(-1, 1, n)
    a = rng.uniform(0.999, 1.001, n)
    b = rng.uniform(-1e-3, 1e-3, n)

    def rec(x, a, b):
        for _ in range(4):
            x = x * a + b
        return x
    got = host(fuse.jit(rec)(cu(x0), cu(a), cu(b)))
    assert_bits_equal(got, dso.ds_recurrence_mul_add_to_f64(x0, a, b, 4), "recurrence")


def test_compile_cache_and_empty(fuse):
    import torch
    g = fuse.jit(lambda v: v + 1.0)
    e = torch.zeros(0, dtype=torch.float64, device="cuda")
    assert g(e).shape == (0,)
    v = torch.arange(10, dtype=torch.float64, device="cuda")
    assert float(host(g(v))[-1]) == 10.0
    assert float(host(g(v * 2))[-1]) == 19.0  # same signature: cached kernel
    assert len(g._cache) == 2
