"""DS reduce on the GPU against exact sums and the reference DS path.

The reference's reduce is XLA's tree over the pass's DS body
(DsTransformPass.cpp:376-448) and no reference test pins its bits, so parity
is measured as error: on f64 input (the config-2 path) the GPU result's error
against math.fsum must be no worse than the reference-order (sequential) DS
fold's error.  Where a case cannot promise that (named in its docstring), it
must stay within a DS-precision bound of the input magnitudes.
"""
import math

import numpy as np
import pytest

from conftest import assert_bits_equal
from gpu_util import cu, host
from oracle import exact

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from ds_b200 import ops as _ops
    return _ops


def config2_inputs(n, seed=1):
    """x_i = s_i*1e8 + u_i*1e-3, s alternating +-1, u ~ U[0,1) (seed 1)."""
    s = np.where(np.arange(n) % 2 == 0, 1.0, -1.0)
    u = np.random.default_rng(seed).uniform(0, 1, n)
    return s * 1e8 + u * 1e-3


def ds_bound(x):
    """Error budget of a DS sum: ~2^-46 of the largest partial magnitude per
    level of a log-depth tree plus the per-thread folds."""
    ax = np.abs(np.asarray(x, np.float64))
    return 2.0 ** -46 * (ax.max() * math.log2(max(ax.size, 2)) * 64 + 1e-300)


@pytest.mark.parametrize("n", [1, 2, 3, 1000, 10_000, 65_537, 1 << 20, (1 << 20) + 37,
                               (1 << 22) + 4095])
def test_config2_sum_error(ops, dso, n):
    """Config 2 (x = +-1e8 alternating + U[0,1) 1e-3): the f64 entry sums each
    thread's values exactly in f64 before its DS tree, so its error is never
    above the sequential DS fold's (which also pays for splitting every x)."""
    x = config2_inputs(n)
    truth = exact.exact_sum(x)
    got = float(host(ops.ds_sum_f64(cu(x))))
    h, l = dso.ds_reduce_f64_seq(x)
    ref = float(h) + float(l)
    f32 = float(np.sum(x.astype(np.float32), dtype=np.float32))
    err, ref_err, f32_err = abs(got - truth), abs(ref - truth), abs(f32 - truth)
    assert err <= ref_err, (err, ref_err)
    if n >= 1000:
        assert err < f32_err / 1000, (err, f32_err)


def test_sum_of_tenths(ops):
    """README.md:199-201: 10,000 x 0.1 (f64 in); the reference DS error is 1.49e-05."""
    x = np.full(10_000, 0.1)
    got = float(host(ops.ds_sum_f64(cu(x))))
    assert abs(got - exact.exact_sum(x)) < 1e-10


def test_triplet_cancellation(ops):
    """handoff.md:191-193: (1e8, 1, -1e8) triplets, n=3333 -> DS error 0."""
    x = np.zeros(3 * 3333)
    x[0::3], x[1::3], x[2::3] = 1e8, 1.0, -1e8
    assert float(host(ops.ds_sum_f64(cu(x)))) == 3333.0


def test_soa_entry_and_f64_entry(ops, dso):
    """ds_reduce on the split inputs (DS values) and the fused f64 entry (which
    sums the f64 inputs exactly per thread) are both within the DS bound, and
    the f64 entry is at least as close to the exact sum of the f64 inputs.
    The SoA entry and the sequential fold add the same DS values, whose
    representation error (the sum of the split errors, common to both)
    dominates; the two folds differ only in order, so neither error bounds the
    other and the SoA entry is held to 4x the sequential error or the DS bound.
    The f64 entry is held to the sequential error itself."""
    x = config2_inputs(100_003, seed=3)
    truth = exact.exact_sum(x)
    sp = dso.ds_from_f64(x)
    hi, lo = ops.ds_reduce(cu(np.ascontiguousarray(sp[:, 0])), cu(np.ascontiguousarray(sp[:, 1])))
    soa = float(np.float64(host(hi))) + float(np.float64(host(lo)))
    f64 = float(host(ops.ds_sum_f64(cu(x))))
    h, l = dso.ds_reduce_f64_seq(x)
    ref_err = abs(float(h) + float(l) - truth)
    assert abs(soa - truth) <= max(4 * ref_err, ds_bound(x))
    assert abs(f64 - truth) <= abs(soa - truth) + ds_bound(x) * 2.0 ** -8
    assert abs(f64 - truth) <= ref_err


@pytest.mark.parametrize("n", [1, 2, 7, 4096, 100_003])
@pytest.mark.parametrize("aligned", [True, False])
def test_packed_entry_matches_soa(ops, dso, n, aligned):
    """ds_reduce_packed on x[..., 2] is the SoA ds_reduce of the same pairs,
    bit for bit (same fold order, vector or scalar loads alike)."""
    from gpu_util import misaligned
    x = config2_inputs(n, seed=n)
    sp = np.ascontiguousarray(dso.ds_from_f64(x))
    put = cu if aligned else misaligned
    hi, lo = ops.ds_reduce(put(np.ascontiguousarray(sp[:, 0])),
                           put(np.ascontiguousarray(sp[:, 1])), init=(0.5, 2.0 ** -30))
    ph, pl = ops.ds_reduce_packed(put(sp), init=(0.5, 2.0 ** -30))
    assert_bits_equal(host(ph), host(hi), "hi")
    assert_bits_equal(host(pl), host(lo), "lo")


def test_packed_entry_segmented(ops, dso):
    x = np.random.default_rng(5).uniform(-1, 1, (37, 300))
    sp = np.ascontiguousarray(dso.ds_from_f64(x.ravel()).reshape(37, 300, 2))
    hi, lo = ops.ds_reduce(cu(np.ascontiguousarray(sp[..., 0])),
                           cu(np.ascontiguousarray(sp[..., 1])), dimensions=(1,))
    ph, pl = ops.ds_reduce_packed(cu(sp), dimensions=(1,))
    assert ph.shape == (37,)
    assert_bits_equal(host(ph), host(hi), "hi")
    assert_bits_equal(host(pl), host(lo), "lo")


def test_packed_entry_rejects_bad_last_dim(ops):
    import torch
    from ds_b200 import _lib
    with pytest.raises(_lib.DsInvalidArgument, match="last dim == 2"):
        ops.ds_reduce_packed(torch.zeros(8, 3, dtype=torch.float32, device="cuda"))


def test_out_argument(ops):
    """Results written into caller-given views equal the allocated results;
    a wrong result shape is rejected before the launch."""
    import torch
    x = cu(config2_inputs(10_000, seed=4))
    hi, lo = ops.ds_reduce_from_f64(x)
    pair = torch.full((2,), 7.0, dtype=torch.float32, device="cuda")
    r = ops.ds_reduce_from_f64(x, out=(pair[0], pair[1]))
    assert r[0].data_ptr() == pair.data_ptr()
    assert_bits_equal(host(pair), np.array([host(hi), host(lo)], np.float32).ravel(), "pair")
    f = torch.empty((), dtype=torch.float64, device="cuda")
    ops.ds_to_f64(pair, out=f)
    assert float(host(f)) == float(np.float64(host(hi))) + float(np.float64(host(lo)))
    with pytest.raises(ValueError, match="shape"):
        ops.ds_reduce_from_f64(x, out=(pair, pair))


def test_deterministic(ops):
    x = cu(config2_inputs(1 << 22, seed=9))
    a = host(ops.ds_sum_f64(x))
    for _ in range(3):
        assert_bits_equal(host(ops.ds_sum_f64(x)), a, "repeat")


def test_empty_returns_init(ops):
    import torch
    x = torch.zeros(0, dtype=torch.float64, device="cuda")
    assert float(host(ops.ds_reduce_f64(x, init=2.5))) == 2.5
    assert float(host(ops.ds_reduce_f64(x, init=-0.0))) == 0.0


def test_init_and_bodies(ops, dso):
    rng = np.random.default_rng(11)
    x = rng.uniform(-1, 1, 50_001)
    got = float(host(ops.ds_reduce_f64(cu(x), init=3.0)))
    assert abs(got - (3.0 + exact.exact_sum(x))) < 1e-11
    got = float(host(ops.ds_reduce_f64(cu(x), init=3.0, body="sub")))
    assert abs(got - (3.0 - exact.exact_sum(x))) < 1e-11
    y = 1.0 + 1e-7 * rng.uniform(-1, 1, 20_000)
    got = float(host(ops.ds_reduce_f64(cu(y), init=1.0, body="mul")))
    h, l = dso.ds_reduce_f64_seq(y, body="mul", init=(1.0, 0.0))
    want = float(h) + float(l)
    assert abs(got - want) / abs(want) < 1e-12


def test_nan_inf_propagate(ops):
    x = np.arange(1000, dtype=np.float64)
    x[17] = np.nan
    assert math.isnan(float(host(ops.ds_sum_f64(cu(x)))))
    x[17] = np.inf
    r = float(host(ops.ds_sum_f64(cu(x))))
    assert math.isinf(r) or math.isnan(r)


@pytest.mark.parametrize("shape,dims", [((37, 1000), (1,)), ((1000, 37), (0,)),
                                        ((6, 50, 7), (1,)), ((4, 3, 500), (1, 2)),
                                        ((300, 2), (0, 1)), ((1 << 18, 8), (0,)),
                                        ((20000, 3, 5), (0,)), ((2, 9000, 4), (1,)),
                                        ((3000, 64), (1,))])
def test_segmented(ops, shape, dims):
    rng = np.random.default_rng(sum(shape))
    x = rng.uniform(-1, 1, shape) * 1e6 + rng.uniform(0, 1, shape) * 1e-6
    got = host(ops.ds_reduce_f64(cu(x), dimensions=dims))
    moved = np.moveaxis(x, dims, list(range(x.ndim - len(dims), x.ndim)))
    flat = moved.reshape(-1, int(np.prod([shape[d] for d in dims])))
    want = np.array([exact.exact_sum(r) for r in flat]).reshape(got.shape)
    # DS recursive-summation bound: a few units of 2^-48 of sum |x| per output
    budget = (2.0 ** -44 * np.abs(flat).sum(axis=1)).reshape(got.shape)
    assert np.all(np.abs(got - want) <= budget)


@pytest.mark.slow
def test_config2_large_property(ops, dso):
    """N = 2^26 (512 MiB): error vs math.fsum no worse than the sequential DS
    fold's."""
    n = 1 << 26
    x = config2_inputs(n)
    got = float(host(ops.ds_sum_f64(cu(x))))
    truth = exact.exact_sum(x)
    h, l = dso.ds_reduce_f64_seq(x)
    ref_err = abs(float(h) + float(l) - truth)
    assert abs(got - truth) <= ref_err


def test_bulk_stream_matches_per_thread_loads_in_accuracy(ops):
    """Long aligned input takes the bulk-copy stream; an unaligned view of
    the same values takes the per-thread-load kernel: both are exact sums
    rounded once here (integers well inside 2^53)."""
    from gpu_util import misaligned
    rng = np.random.default_rng(21)
    x = rng.integers(-2 ** 30, 2 ** 30, (1 << 21) + 3).astype(np.float64)
    want = float(np.sum(x.astype(np.int64)))
    assert float(host(ops.ds_sum_f64(cu(x)))) == want
    assert float(host(ops.ds_sum_f64(misaligned(x)))) == want


def test_bulk_stream_nan_inf(ops):
    x = np.ones((1 << 21) + 9)
    x[(1 << 20) + 3] = np.nan
    assert math.isnan(float(host(ops.ds_sum_f64(cu(x)))))
    x[(1 << 20) + 3] = np.inf
    r = float(host(ops.ds_sum_f64(cu(x))))
    assert math.isinf(r) or math.isnan(r)


def test_variadic_reduce(ops):
    """Several inputs, each with its own body and init, equal the single
    reductions bit for bit (full and segmented)."""
    import torch
    rng = np.random.default_rng(31)
    xs = [cu(rng.uniform(-1, 1, (64, 3001))) for _ in range(3)]
    for dims in (None, (1,)):
        outs = ops.ds_reduce_f64_multi(xs, inits=[0.0, 1.5, 1.0], bodies=["add", "sub", "mul"],
                                       dimensions=dims)
        for x, o, init, body in zip(xs, outs, [0.0, 1.5, 1.0], ["add", "sub", "mul"]):
            want = ops.ds_reduce_f64(x, init=init, dimensions=dims, body=body)
            assert_bits_equal(host(o), host(want), f"{body} {dims}")
    with pytest.raises(Exception):
        ops.ds_reduce_f64_multi([xs[0], torch.zeros(5, dtype=torch.float64, device="cuda")])


SLICED = [((1 << 18, 8), (0,)), ((20000, 3, 5), (0,))]


def _reduce_f64_capi(x, dims, body, workspace_bytes):
    """ds_reduce_f64 through the C ABI with a caller-sized workspace (0: none)."""
    import ctypes
    import torch
    from ds_b200 import _lib as L
    init = torch.zeros((), dtype=torch.float64, device=x.device)
    shape = tuple(s for i, s in enumerate(x.shape) if i not in dims)
    out = torch.empty(shape, dtype=torch.float64, device=x.device)
    ws = torch.empty(max(workspace_bytes, 1), dtype=torch.uint8, device=x.device)
    bx, kx = L.make_buffer(x.data_ptr(), x.shape)
    bi, ki = L.make_buffer(init.data_ptr(), ())
    bo, ko = L.make_buffer(out.data_ptr(), shape)
    cd = (ctypes.c_int64 * len(dims))(*dims)
    st = L.lib().ds_reduce_f64(ctypes.byref(bx), ctypes.byref(bi), cd, len(dims),
                               {"add": L.DS_BODY_ADD, "mul": L.DS_BODY_MUL}[body],
                               ctypes.byref(bo), ctypes.c_void_p(ws.data_ptr()),
                               ctypes.c_size_t(workspace_bytes),
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    L.check(st, "ds_reduce_f64")
    return host(out)


def _columns(x, dims):
    moved = np.moveaxis(x, dims, list(range(x.ndim - len(dims), x.ndim)))
    return moved.reshape(-1, int(np.prod([x.shape[d] for d in dims])))


@pytest.mark.parametrize("shape,dims", SLICED)
def test_sliced_columns_mul_body(ops, dso, shape, dims):
    """The sliced leading-dimension path with the multiply body: slice
    partials start from the identity and init is applied once, at the end.
    Each column's product of up to 2^18 factors 1 + 1e-7 u is checked
    against the exact product (1.5 exp(fsum(log1p(1e-7 u))), good to about
    2^-51), as is the oracle's sequential DS product.  The reference's DS
    multiply (no renormalisation) carries a small systematic error, so 2^18
    factors drift by about 2^-35 in either order (the oracle: 2^-35.2 and
    2^-35.8 on the first two columns): both are held to 2^-32 of the
    product, which a slice's init or identity gone wrong (a factor of 1.5 or
    more) misses by far."""
    rng = np.random.default_rng(41)
    y = 1.0 + 1e-7 * rng.uniform(-1, 1, shape)
    got = host(ops.ds_reduce_f64(cu(y), init=1.5, dimensions=dims, body="mul")).ravel()
    for c, col in enumerate(_columns(y, dims)):
        truth = 1.5 * math.exp(math.fsum(np.log1p(col - 1.0).tolist()))
        h, l = dso.ds_reduce_f64_seq(col, body="mul", init=(1.5, 0.0))
        seq = float(h) + float(l)
        assert abs(seq - truth) <= 2.0 ** -32 * truth, (c, seq, truth)
        assert abs(got[c] - truth) <= 2.0 ** -32 * truth, (c, got[c], truth)


@pytest.mark.parametrize("shape,dims", SLICED)
def test_sliced_columns_packed_and_soa(ops, dso, shape, dims):
    """DS input on the sliced path: the packed and SoA entries give the same
    bits, within the DS bound of the exact column sums of the DS values."""
    rng = np.random.default_rng(43)
    x = rng.uniform(-1, 1, shape) * 1e6 + rng.uniform(0, 1, shape) * 1e-6
    sp = np.ascontiguousarray(dso.ds_from_f64(x.ravel()).reshape(shape + (2,)))
    hi, lo = ops.ds_reduce(cu(np.ascontiguousarray(sp[..., 0])),
                           cu(np.ascontiguousarray(sp[..., 1])), dimensions=dims)
    ph, pl = ops.ds_reduce_packed(cu(sp), dimensions=dims)
    assert_bits_equal(host(ph), host(hi), "hi")
    assert_bits_equal(host(pl), host(lo), "lo")
    got = (host(hi).astype(np.float64) + host(lo).astype(np.float64)).ravel()
    vals = sp[..., 0].astype(np.float64) + sp[..., 1].astype(np.float64)
    cols = _columns(vals, dims)
    want = np.array([exact.exact_sum(c) for c in cols])
    assert np.all(np.abs(got - want) <= 2.0 ** -44 * np.abs(cols).sum(axis=1))


@pytest.mark.parametrize("shape,dims", SLICED)
def test_sliced_columns_with_and_without_workspace(ops, shape, dims):
    """With ds_reduce_workspace_size bytes the reduced dimension is sliced
    across blocks; with none the one-stage kernel runs.  The two fold in
    different orders: integer-valued sums (exact in both) agree bit for bit,
    general inputs agree within the DS bound."""
    from ds_b200 import _lib as L
    import ctypes
    rng = np.random.default_rng(47)
    xi = rng.integers(-2 ** 20, 2 ** 20, shape).astype(np.float64)
    bx, kx = L.make_buffer(0, shape)
    cd = (ctypes.c_int64 * len(dims))(*dims)
    need = int(L.lib().ds_reduce_workspace_size(ctypes.byref(bx), cd, len(dims)))
    assert need > 0  # these shapes are sliced
    d = cu(xi)
    a, b = _reduce_f64_capi(d, dims, "add", need), _reduce_f64_capi(d, dims, "add", 0)
    assert np.array_equal(a.view(np.uint64), b.view(np.uint64))
    assert np.array_equal(a.ravel(), _columns(xi, dims).sum(axis=1))
    xf = rng.uniform(-1, 1, shape) * 1e6 + rng.uniform(0, 1, shape) * 1e-6
    d = cu(xf)
    a, b = _reduce_f64_capi(d, dims, "add", need), _reduce_f64_capi(d, dims, "add", 0)
    cols = _columns(xf, dims)
    want = np.array([exact.exact_sum(c) for c in cols])
    bound = 2.0 ** -44 * np.abs(cols).sum(axis=1)
    assert np.all(np.abs(a.ravel() - want) <= bound) and np.all(np.abs(b.ravel() - want) <= bound)
