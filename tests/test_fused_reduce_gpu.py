"""ds_fused_reduce on the GPU: an elementwise DAG reduced in its own kernel.

The map is the fused program's, so its values equal the C oracle's DS
operations bit for bit.  The reduction order (per-thread folds, warp and
block trees, then the packed reduce of the block partials) is the kernel's
own; as for every DS reduce, parity is measured as error: against the exact
sum of the DS values the map produces, within a small multiple of the
sequential DS fold's error or the DS bound of the magnitudes
(DsTransformPass.cpp:376-448 defines the body, XLA the order).
"""
import math

import numpy as np
import pytest
import torch

from conftest import assert_bits_equal
from gpu_util import cu, host, misaligned
from oracle import exact

pytestmark = pytest.mark.gpu

I, CONST, ADD, SUB, MUL = 0, 1, 2, 3, 4


@pytest.fixture(scope="module")
def fuse():
    from ds_b200 import fuse as _fuse
    return _fuse


def ds_bound(v):
    a = np.abs(v)
    return 2.0 ** -46 * (a.max() * math.log2(max(a.size, 2)) * 64 + 1e-300)


def check_sum(got, Z, dso):
    """got: (hi, lo) tensors; Z: the map's DS values (packed, from the oracle).

    The kernel and the sequential fold add the same DS values exactly as
    given, in different orders (a tree against a running sum), so neither
    error bounds the other: the result is held to 4x the sequential error or
    the DS bound of the values, whichever is larger."""
    vals = Z[..., 0].astype(np.float64).ravel()
    los = Z[..., 1].astype(np.float64).ravel()
    truth = exact.exact_sum(np.concatenate([vals, los]))
    h, l = dso.ds_reduce_ds_seq(Z[..., 0].ravel(), Z[..., 1].ravel())
    ref_err = abs(float(h) + float(l) - truth)
    res = float(np.float64(host(got[0]))) + float(np.float64(host(got[1])))
    assert abs(res - truth) <= max(4 * ref_err, ds_bound(vals)), (res, truth, ref_err)


@pytest.mark.parametrize("n", [1, 2, 3, 257, 65_537, 1 << 20, (1 << 22) + 5])
def test_add_mul_sum(fuse, dso, n):
    """sum((a + b) * c), config 1's chain, over f64 inputs."""
    rng = np.random.default_rng(n)
    a, b, c = (rng.uniform(-1, 1, n) for _ in range(3))
    p = fuse.Prepared([(I, 0, 0, 0.0), (I, 1, 0, 0.0), (ADD, 0, 1, 0.0), (I, 2, 0, 0.0),
                       (MUL, 2, 3, 0.0)], ["f64"] * 3, "packed")
    got = p.reduce([cu(a), cu(b), cu(c)], (n,))
    Z = dso.ds_mul(dso.ds_add(dso.ds_from_f64(a), dso.ds_from_f64(b)), dso.ds_from_f64(c))
    # the map itself is the oracle's, bit for bit
    assert_bits_equal(host(p([cu(a), cu(b), cu(c)], (n,))), Z, "map")
    check_sum(got, Z, dso)


def test_cancellation_heavy(fuse, dso):
    """x_i = s_i 1e8 + u_i 1e-3 (the reduce workload's values) through x * 1."""
    n = (1 << 20) + 3
    s = np.where(np.arange(n) % 2 == 0, 1.0, -1.0)
    x = s * 1e8 + np.random.default_rng(1).uniform(0, 1, n) * 1e-3
    p = fuse.Prepared([(I, 0, 0, 0.0), (CONST, 0, 0, 1.0), (MUL, 0, 1, 0.0)], ["f64"], "packed")
    got = p.reduce([cu(x)], (n,))
    Z = dso.ds_mul(dso.ds_from_f64(x), dso.ds_from_f64(np.ones(n)))
    check_sum(got, Z, dso)


def test_broadcast_and_unaligned_inputs(fuse, dso):
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, (300, 1))
    y = rng.uniform(-1, 1, (1, 77)).astype(np.float32)
    z = rng.uniform(-1, 1, 300 * 77)
    p = fuse.Prepared([(I, 0, 0, 0.0), (I, 1, 0, 0.0), (SUB, 0, 1, 0.0), (I, 2, 0, 0.0),
                       (MUL, 2, 3, 0.0)], ["f64", "f32", "f64"], "packed")
    zz = misaligned(z).reshape(300, 77)
    got = p.reduce([cu(x), cu(y), zz], (300, 77))
    X = dso.ds_from_f64(np.broadcast_to(x, (300, 77)))
    Y = dso.ds_from_f32(np.broadcast_to(y, (300, 77)))
    Z = dso.ds_mul(dso.ds_sub(X, Y), dso.ds_from_f64(z.reshape(300, 77)))
    check_sum(got, Z, dso)


def test_product_body_and_init(fuse, dso):
    rng = np.random.default_rng(4)
    x = 1.0 + 1e-7 * rng.uniform(-1, 1, 50_001)
    p = fuse.Prepared([(I, 0, 0, 0.0)], ["f64"], "packed")
    hi, lo = p.reduce([cu(x)], (x.size,), "mul", init=(2.0, 0.0))
    h, l = dso.ds_reduce_f64_seq(x, body="mul", init=(2.0, 0.0))
    want = float(h) + float(l)
    got = float(np.float64(host(hi))) + float(np.float64(host(lo)))
    assert abs(got - want) / abs(want) < 1e-12


def test_packed_input_and_determinism(fuse, dso):
    rng = np.random.default_rng(5)
    x = rng.uniform(-1, 1, 1 << 21)
    P = np.ascontiguousarray(dso.ds_from_f64(x))
    p = fuse.Prepared([(I, 0, 0, 0.0), (I, 0, 0, 0.0), (MUL, 0, 1, 0.0)], ["packed"], "packed")
    t = cu(P)
    first = [host(v) for v in p.reduce([t], (x.size,))]
    for _ in range(3):
        again = [host(v) for v in p.reduce([t], (x.size,))]
        assert_bits_equal(again[0], first[0], "hi")
        assert_bits_equal(again[1], first[1], "lo")
    check_sum([torch.tensor(first[0]), torch.tensor(first[1])], dso.ds_mul(P, P), dso)


def test_empty_returns_init(fuse):
    p = fuse.Prepared([(I, 0, 0, 0.0)], ["f64"], "packed")
    hi, lo = p.reduce([torch.zeros(0, dtype=torch.float64, device="cuda")], (0,), "add",
                      init=(1.5, 2.0 ** -30))
    assert float(host(hi)) == 1.5 and float(host(lo)) == 2.0 ** -30


def test_dstensor_sum_uses_one_kernel(dso):
    from ds_b200 import _lib
    from ds_b200.dstensor import DSTensor
    rng = np.random.default_rng(6)
    x, y = rng.uniform(-1, 1, 100_001), rng.uniform(-1, 1, 100_001)
    a = DSTensor.from_f64(cu(x))
    expr = (a + cu(y)) * a
    _lib.profile_reset()
    _lib.profile_enable(True)
    s = expr.sum()
    torch.cuda.synchronize()
    _lib.profile_enable(False)
    assert _lib.profile_read("fused_reduce")[1] == 1
    assert _lib.profile_read("fused")[1] == 0
    X = dso.ds_from_f64(x)
    Z = dso.ds_mul(dso.ds_add(X, dso.ds_from_f64(y)), X)
    check_sum([s.packed[0], s.packed[1]], Z, dso)


# ---- reductions over the trailing dimensions (ds_fused_reduce_rows) ----


def check_rows(hi, lo, Z, dso, init=(0.0, 0.0)):
    """Each row's result against the exact sum of its DS values plus init,
    held as in check_sum (different fold orders: 4x the sequential error or
    the DS bound)."""
    got = host(hi).astype(np.float64) + host(lo).astype(np.float64)
    rows = Z.reshape(got.size, -1, 2)
    for r, g in zip(rows, got.ravel()):
        vals = np.concatenate([r[:, 0].astype(np.float64), r[:, 1].astype(np.float64),
                               np.array(init, np.float64)])
        truth = exact.exact_sum(vals)
        h, l = dso.ds_reduce_ds_seq(r[:, 0], r[:, 1], "add", init)
        ref_err = abs(float(h) + float(l) - truth)
        bound = ds_bound(r[:, 0].astype(np.float64)) if r.shape[0] else 0.0
        assert abs(g - truth) <= max(4 * ref_err, bound), (g, truth, ref_err)


@pytest.mark.parametrize("shape,k", [((37, 3001), 1), ((5, 4096), 1), ((3, 7, 300), 2),
                                     ((1000, 3), 1), ((2, 3, 4), 3), ((513, 64), 1),
                                     ((300, 200), 1), ((7, 1000), 1), ((4099, 9), 1)])
def test_rows_add_mul_sum(fuse, dso, shape, k):
    """sum over the last k dimensions of (a + b) * c: rows folded by a block,
    a warp or smaller lane groups (1 to 16 lanes), several rank-k tails."""
    rng = np.random.default_rng(sum(shape) + k)
    a, b, c = (rng.uniform(-1, 1, shape) for _ in range(3))
    p = fuse.Prepared([(I, 0, 0, 0.0), (I, 1, 0, 0.0), (ADD, 0, 1, 0.0), (I, 2, 0, 0.0),
                       (MUL, 2, 3, 0.0)], ["f64"] * 3, "packed")
    hi, lo = p.reduce_rows([cu(a), cu(b), cu(c)], shape, k)
    assert tuple(hi.shape) == shape[:len(shape) - k]
    Z = dso.ds_mul(dso.ds_add(dso.ds_from_f64(a), dso.ds_from_f64(b)), dso.ds_from_f64(c))
    check_rows(hi, lo, Z, dso)


def test_rows_broadcast_init_and_empty_rows(fuse, dso):
    rng = np.random.default_rng(8)
    x = rng.uniform(-1, 1, (64, 1))
    y = rng.uniform(-1, 1, 2500).astype(np.float32)
    p = fuse.Prepared([(I, 0, 0, 0.0), (I, 1, 0, 0.0), (MUL, 0, 1, 0.0)], ["f64", "f32"],
                      "packed")
    hi, lo = p.reduce_rows([cu(x), cu(y)], (64, 2500), 1, init=(0.5, 2.0 ** -30))
    Z = dso.ds_mul(dso.ds_from_f64(np.broadcast_to(x, (64, 2500))),
                   dso.ds_from_f32(np.broadcast_to(y, (64, 2500))))
    check_rows(hi, lo, Z, dso, init=(0.5, 2.0 ** -30))
    # rows of length 0 hold init, bit for bit
    e = torch.zeros(4, 0, dtype=torch.float64, device="cuda")
    q = fuse.Prepared([(I, 0, 0, 0.0)], ["f64"], "packed")
    h0, l0 = q.reduce_rows([e], (4, 0), 1, init=(1.5, 2.0 ** -30))
    assert np.all(host(h0) == 1.5) and np.all(host(l0) == np.float32(2.0 ** -30))


def test_rows_product_body_and_determinism(fuse, dso):
    rng = np.random.default_rng(9)
    x = 1.0 + 1e-7 * rng.uniform(-1, 1, (16, 5000))
    p = fuse.Prepared([(I, 0, 0, 0.0)], ["f64"], "packed")
    hi, lo = p.reduce_rows([cu(x)], x.shape, 1, "mul", init=(2.0, 0.0))
    first = (host(hi), host(lo))
    hi2, lo2 = p.reduce_rows([cu(x)], x.shape, 1, "mul", init=(2.0, 0.0))
    assert_bits_equal(host(hi2), first[0], "hi")
    assert_bits_equal(host(lo2), first[1], "lo")
    got = first[0].astype(np.float64) + first[1].astype(np.float64)
    for i in range(16):
        h, l = dso.ds_reduce_f64_seq(x[i], body="mul", init=(2.0, 0.0))
        want = float(h) + float(l)
        assert abs(got[i] - want) / abs(want) < 1e-12


def test_dstensor_row_sum_uses_one_kernel(dso):
    from ds_b200 import _lib
    from ds_b200.dstensor import DSTensor
    rng = np.random.default_rng(10)
    x, y = rng.uniform(-1, 1, (40, 3000)), rng.uniform(-1, 1, 3000)
    a = DSTensor.from_f64(cu(x))
    expr = (a + cu(y)) * a
    _lib.profile_reset()
    _lib.profile_enable(True)
    s = expr.sum(dimensions=(-1,))
    torch.cuda.synchronize()
    _lib.profile_enable(False)
    assert _lib.profile_read("fused_reduce")[1] == 1
    assert _lib.profile_read("fused")[1] == 0
    assert s.shape == (40,)
    X = dso.ds_from_f64(x)
    Z = dso.ds_mul(dso.ds_add(X, dso.ds_from_f64(np.broadcast_to(y, x.shape))), X)
    p = s.packed
    check_rows(p[:, 0], p[:, 1], Z, dso)
