"""DSTensor on the GPU: packed storage keeps the lo word between calls, and
a lazy expression gives the bits of one target call per operation (the C
oracle composing the same DS operations)."""
import numpy as np
import pytest

from conftest import assert_bits_equal
from gpu_util import cu, host

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dst():
    from ds_b200 import dstensor
    return dstensor


def test_storage_keeps_lo(dst, dso):
    x = np.random.default_rng(1).uniform(-1, 1, 10_001) * 1e8 + 1e-3
    a = dst.DSTensor.from_f64(cu(x))
    assert_bits_equal(host(a.packed), dso.ds_from_f64(x), "split")
    assert_bits_equal(host(a.to_f64()), dso.ds_to_f64(dso.ds_from_f64(x)), "recombine")


def test_lazy_chain_matches_per_op_calls(dst, dso):
    rng = np.random.default_rng(2)
    x = rng.uniform(-1, 1, 65_537)
    y = rng.uniform(-1, 1, 65_537).astype(np.float32)
    a = dst.DSTensor.from_f64(cu(x))
    b = (a + cu(y)) * a - 0.1
    X = dso.ds_from_f64(x)
    Y = dso.ds_from_f32(y)
    want = dso.ds_sub(dso.ds_mul(dso.ds_add(X, Y), X), dso.ds_from_f64(np.full(x.size, 0.1)))
    assert_bits_equal(host(b.packed), want, "packed")
    c = (a + cu(y)) * a - 0.1
    assert_bits_equal(host(c.to_f64()), dso.ds_to_f64(want), "f64 out")
    # a materialised value used again keeps its DS pairs
    d = b * b
    assert_bits_equal(host(d.packed), dso.ds_mul(want, want), "reuse")


def test_long_expression_is_split_and_still_exact(dst, dso):
    rng = np.random.default_rng(3)
    n = 4099
    x0 = rng.uniform(-1, 1, n)
    a = rng.uniform(0.999, 1.001, n)
    b = rng.uniform(-1e-3, 1e-3, n)
    X = dst.DSTensor.from_f64(cu(x0))
    ta, tb = cu(a), cu(b)
    for _ in range(150):  # 300 operations: more than one generated program
        X = X * ta + tb
    got = host(X.to_f64())
    assert_bits_equal(got, dso.ds_recurrence_mul_add_to_f64(x0, a, b, 150), "recurrence")


def test_sum_and_matmul(dst):
    import math
    from ds_b200 import ops
    from oracle import exact
    rng = np.random.default_rng(4)
    x = rng.uniform(-1, 1, 300_001)
    s = dst.DSTensor.from_f64(cu(x)).sum()
    assert s.shape == ()
    assert abs(float(host(s.to_f64())) - math.fsum(x.tolist())) < 1e-12
    A = rng.uniform(-1, 1, (96, 80))
    B = rng.uniform(-1, 1, (80, 64))
    dA, dB = dst.DSTensor.from_f64(cu(A)), dst.DSTensor.from_f64(cu(B))
    C = (dA @ dB).to_f64()
    # the product of the DS values themselves (A and B rounded to DS)
    want = ops.ds_matmul_f64(dA.to_f64(), dB.to_f64())
    assert_bits_equal(host(C), host(ops.ds_to_f64(ops.ds_from_f64(want))), "matmul")
