"""The DS transform of torch programs on the GPU.

Elementwise results equal, bit for bit, the C oracle composing the same DS
operations (the pass's emitDsAdd / emitDsSub / emitDsMul chain,
DsTransformPass.cpp:282-321, with emitFromFloat at entry and emitToFloat at
the return).  Reductions and products equal the library's own targets
called by hand on the same values (one code path), and their errors
against exact sums stay within the DS bound.
"""
import math

import numpy as np
import pytest
import torch

from conftest import assert_bits_equal
from gpu_util import cu, host
from oracle import exact

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tr():
    from ds_b200 import transform
    return transform


@pytest.fixture(scope="module")
def ops():
    from ds_b200 import ops as _ops
    return _ops


def test_config1_chain_bits(tr, dso):
    """(a + b) * c on 2^20 f64 values (uniform [-1, 1], seed 0) is the
    oracle's ds_fused_add_mul3_to_f64."""
    rng = np.random.default_rng(0)
    a, b, c = (rng.uniform(-1, 1, 1 << 20) for _ in range(3))
    f = tr.ds_transform(lambda a, b, c: (a + b) * c)
    assert f.plan(cu(a), cu(b), cu(c)).launches() == {"fused": 1}
    got = host(f(cu(a), cu(b), cu(c)))
    assert_bits_equal(got, dso.ds_fused_add_mul3_to_f64(a, b, c), "config 1")


def test_mixed_program_bits(tr, dso):
    rng = np.random.default_rng(1)
    x = rng.uniform(-1, 1, (64, 257))
    y = rng.uniform(-1, 1, 257).astype(np.float32)

    @tr.ds_transform
    def f(x, y):
        z = (x + y) * x - 0.1
        return z, -z * 3.0

    z, w = f(cu(x), cu(y))
    X, Y = dso.ds_from_f64(x), dso.ds_from_f32(np.broadcast_to(y, x.shape))
    C = np.broadcast_to(dso.ds_from_f64(np.array(0.1)), x.shape + (2,))
    Z = dso.ds_sub(dso.ds_mul(dso.ds_add(X, Y), X), C)
    W = dso.ds_mul(-Z, np.broadcast_to(dso.ds_from_f64(np.array(3.0)), x.shape + (2,)))
    assert_bits_equal(host(z), dso.ds_to_f64(Z), "z")
    assert_bits_equal(host(w), dso.ds_to_f64(W), "w")


def test_long_chain_bits(tr, dso):
    """600 DS operations, cut into several programs, keep the bits."""
    rng = np.random.default_rng(2)
    x, a = rng.uniform(-1, 1, 4099), rng.uniform(0.999, 1.001, 4099)

    @tr.ds_transform
    def f(x, a):
        for _ in range(300):
            x = x * a + a
        return x

    assert f.plan(cu(x), cu(a)).launches()["fused"] >= 3
    X, A = dso.ds_from_f64(x), dso.ds_from_f64(a)
    for _ in range(300):
        X = dso.ds_add(dso.ds_mul(X, A), A)
    assert_bits_equal(host(f(cu(x), cu(a))), dso.ds_to_f64(X), "chain")


def test_reduce_matches_target(tr, ops, dso):
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, (37, 3001)) * 1e8 + rng.uniform(0, 1, (37, 3001)) * 1e-3

    @tr.ds_transform
    def f(x):
        return (x * x).sum(dim=1), x.sum()

    s1, s = f(cu(x))
    # the row sums run in the product's own kernel (its own tree order):
    # within the DS bound of the exact sums of the DS products, as the
    # packed reduce of the same products is.  Both sum the same DS products
    # in different tree orders, so neither error bounds the other: 4x the
    # unfused error, or the DS bound.  The whole-array sum of the f64
    # argument takes the f64 entry and is held to the sequential DS fold.
    X = dso.ds_from_f64(x)
    Z = dso.ds_mul(X, X)
    truth = np.array([exact.exact_sum(np.concatenate([z[:, 0].astype(np.float64),
                                                      z[:, 1].astype(np.float64)])) for z in Z])
    packed = ops.ds_mul(ops.ds_from_f64(cu(x)), ops.ds_from_f64(cu(x)))
    hi, lo = ops.ds_reduce_packed(packed, dimensions=(1,))
    unfused = host(hi).astype(np.float64) + host(lo).astype(np.float64)
    row_bound = 2.0 ** -46 * np.abs(Z[..., 0]).max(axis=1) * math.log2(3001) * 64
    assert np.all(np.abs(host(s1) - truth) <= np.maximum(4 * np.abs(unfused - truth), row_bound))
    flat = x.ravel()
    truth = exact.exact_sum(flat)
    h, l = dso.ds_reduce_f64_seq(flat)
    ref_err = abs(float(h) + float(l) - truth)
    assert abs(float(host(s)) - truth) <= ref_err


def test_matmul_matches_target(tr, ops):
    rng = np.random.default_rng(4)
    A, B = rng.uniform(-1, 1, (256, 512)), rng.uniform(-1, 1, (512, 384))

    @tr.ds_transform
    def f(a, b):
        return (a @ b) * 2.0, a @ b

    scaled, p = f(cu(A), cu(B))
    want = host(ops.ds_matmul_f64(cu(A), cu(B)))
    assert_bits_equal(host(p), want, "product")
    assert np.max(np.abs(host(p) - A @ B)) < 1e-12
    # the product enters the multiply as its DS split: 2^-48 relative
    assert np.all(np.abs(host(scaled) - 2 * want) <= 2.0 ** -46 * np.abs(want))


def test_batched_and_vector_matmul(tr):
    rng = np.random.default_rng(5)
    f = tr.ds_transform(lambda a, b: a @ b)
    for sa, sb in [((3, 64, 96), (3, 96, 32)), ((2, 64, 96), (96, 32)), ((96,), (96, 32)),
                   ((64, 96), (96,))]:
        a, b = rng.uniform(-1, 1, sa), rng.uniform(-1, 1, sb)
        got = host(f(cu(a), cu(b)))
        assert got.shape == np.matmul(a, b).shape
        assert np.max(np.abs(got - np.matmul(a, b))) < 1e-12, (sa, sb)


def test_layout_and_untouched_ops(tr, dso):
    rng = np.random.default_rng(6)
    a, b = rng.uniform(-1, 1, (48, 80)), rng.uniform(-1, 1, (80, 48))

    @tr.ds_transform
    def f(a, b):
        y = a * b.T
        return y.T + b, torch.exp(y)

    g, e = f(cu(a), cu(b))
    Y = dso.ds_mul(dso.ds_from_f64(a), dso.ds_from_f64(np.ascontiguousarray(b.T)))
    YT = np.ascontiguousarray(Y.transpose(1, 0, 2))
    assert_bits_equal(host(g), dso.ds_to_f64(dso.ds_add(YT, dso.ds_from_f64(b))), "layout")
    assert np.allclose(host(e), np.exp(dso.ds_to_f64(Y)), rtol=1e-15, atol=0)


def test_graph_capture(tr, dso):
    """A transformed function replays inside a CUDA graph."""
    rng = np.random.default_rng(7)
    x, y = cu(rng.uniform(-1, 1, 100_000)), cu(rng.uniform(-1, 1, 100_000))
    f = tr.ds_transform(lambda x, y: ((x + y) * y).sum())
    eager = host(f(x, y))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        f(x, y)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = f(x, y)
    g.replay()
    assert_bits_equal(host(out), eager, "graph")


def test_linear_module(tr, ops, dso):
    """nn.Linear lowers to the DS product then a DS add of the bias: the add
    is the oracle's on the product's values, bit for bit."""
    torch.manual_seed(1)
    lin = torch.nn.Linear(96, 64).double().cuda()
    f = tr.ds_transform(lin)
    x = cu(np.random.default_rng(8).uniform(-1, 1, (128, 96)))
    got = host(f(x))
    with torch.no_grad():
        prod = host(ops.ds_matmul_f64(x, lin.weight.T.contiguous()))
        bias = host(lin.bias)
    want = dso.ds_to_f64(dso.ds_add(dso.ds_from_f64(prod),
                                    dso.ds_from_f64(np.broadcast_to(bias, prod.shape))))
    assert_bits_equal(got, want, "linear")


def test_edge_shapes(tr, dso):
    """0-d and empty tensors, keepdim on a fused full reduction, f32 programs."""
    f = tr.ds_transform(lambda x, y: ((x * y + 1.0).sum(dim=(0, 1), keepdim=True), x * y - y))
    x = np.random.default_rng(9).uniform(-1, 1, (5, 7))
    s, d = f(cu(x), cu(x))
    assert tuple(s.shape) == (1, 1) and tuple(d.shape) == (5, 7)
    X = dso.ds_from_f64(x)
    assert_bits_equal(host(d), dso.ds_to_f64(dso.ds_sub(dso.ds_mul(X, X), X)), "map")
    e, _ = f(torch.zeros(0, 7, dtype=torch.float64, device="cuda"),
             torch.zeros(0, 7, dtype=torch.float64, device="cuda"))
    assert float(host(e).item()) == 0.0
    g = tr.ds_transform(lambda a, b: a * b + 0.5)
    a0 = torch.tensor(3.0, dtype=torch.float64, device="cuda")
    assert float(host(g(a0, a0))) == 9.5
    h = tr.ds_transform(lambda a, b: (a + b) * a)
    u = np.random.default_rng(10).uniform(-1, 1, 1001).astype(np.float32)
    v = np.random.default_rng(11).uniform(-1, 1, 1001).astype(np.float32)
    got = host(h(cu(u), cu(v)))
    U, V = dso.ds_from_f32(u), dso.ds_from_f32(v)
    assert got.dtype == np.float32
    assert_bits_equal(got, dso.ds_to_f32(dso.ds_mul(dso.ds_add(U, V), U)), "f32 program")


def test_graph_mode_replays_with_new_values(tr, dso):
    """graphs=True: the plan is captured once; later calls copy their
    tensors in and replay, with the eager results bit for bit."""
    rng = np.random.default_rng(12)

    def prog(a, b):
        y = (a + b) * b - 0.25
        return y.sum(), y * 2.0

    f = tr.ds_transform(prog, graphs=True)
    eager = tr.ds_transform(prog)
    for i in range(4):
        a, b = cu(rng.uniform(-1, 1, 5000)), cu(rng.uniform(-1, 1, 5000))
        s, y = f(a, b)
        es, ey = eager(a, b)
        assert_bits_equal(host(s), host(es), f"sum {i}")
        assert_bits_equal(host(y), host(ey), f"map {i}")
    assert f.plan(a, b)._graph  # captured
