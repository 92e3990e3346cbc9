"""Elementwise DS kernels on the GPU, bit-exact against the oracle and the
reference's golden vectors (tests/golden/ds_ref_vectors.npz).

Covers split/recombine, packed add/sub/mul, every fused chain and both
recurrences at empty, odd, tail-heavy and large sizes, unaligned views and
multi-dimensional packed tensors.
"""
import numpy as np
import pytest

from conftest import assert_bits_equal
from gpu_util import cu, host, misaligned

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 2, 3, 5, 4097, 65537, (1 << 20) + 3]


@pytest.fixture(scope="module")
def ops():
    from ds_b200 import ops as _ops
    return _ops


def rand_f64(rng, n, lo=-8, hi=8):
    return rng.uniform(-1, 1, n) * 10.0 ** rng.uniform(lo, hi, n)


# ---- golden vectors (the reference's ds_ref.py) -------------------------------

def test_golden_packed(ops, golden):
    a, b = cu(golden["pk_a"]), cu(golden["pk_b"])
    for name in ("add", "sub", "mul"):
        got = host(getattr(ops, "ds_" + name)(a, b))
        assert_bits_equal(got, golden["pk_" + name], "ds_" + name)


def test_golden_split_recombine(ops, golden):
    with np.errstate(all="ignore"):
        sp = host(ops.ds_from_f64(cu(golden["f64_x"])))
    assert_bits_equal(sp, golden["f64_split"], "ds_from_f64")
    assert_bits_equal(host(ops.ds_to_f64(cu(golden["f64_split"]))), golden["f64_recombine"],
                      "ds_to_f64")


def test_golden_fused(ops, golden):
    x, y, c = cu(golden["fx"]), cu(golden["fy"]), cu(golden["fc"])
    assert_bits_equal(host(ops.ds_fused_add_mul(x, y)), golden["fused_add_mul_packed"], "packed")
    for fn in (ops.ds_fused_add_mul_to_f64, ops.ds_fused_axpy, ops.ds_fused_add_mul_to_f64_cuda):
        assert_bits_equal(host(fn(x, y)), golden["fused_add_mul_to_f64"], fn.__name__)
    assert_bits_equal(host(ops.ds_fused_add_sub_to_f64_cuda(x, y)),
                      golden["fused_add_sub_to_f64"], "add_sub")
    assert_bits_equal(host(ops.ds_fused_add_mul3_to_f64(x, y, c)),
                      golden["fused_add_mul3_to_f64"], "add_mul3")


def test_golden_recurrences(ops, golden):
    x, y = cu(golden["rec_x"]), cu(golden["rec_y"])
    for k in (0, 1, 8):
        assert_bits_equal(host(ops.ds_recurrence_add_mul_to_f64_cuda(x, y, k)),
                          golden[f"rec_add_mul_k{k}"], f"rec k={k}")
    mx, ma, mb = cu(golden["mrec_x"]), cu(golden["mrec_a"]), cu(golden["mrec_b"])
    for k in (1, 4, 16):
        assert_bits_equal(host(ops.ds_recurrence_mul_add_to_f64(mx, ma, mb, k)),
                          golden[f"mrec_k{k}"], f"mul_add k={k}")


# ---- seeded sizes against the oracle --------------------------------------------

@pytest.mark.parametrize("n", SIZES)
def test_split_recombine_vs_oracle(ops, dso, n):
    rng = np.random.default_rng(100 + n)
    x = rand_f64(rng, n, -30, 30)
    assert_bits_equal(host(ops.ds_from_f64(cu(x))), dso.ds_from_f64(x, 8), "from_f64")
    p = dso.ds_from_f64(x, 8)
    assert_bits_equal(host(ops.ds_to_f64(cu(p))), dso.ds_to_f64(p, 8), "to_f64")
    f = rng.standard_normal(n).astype(np.float32)
    assert_bits_equal(host(ops.ds_from_f32(cu(f))), dso.ds_from_f32(f), "from_f32")
    assert_bits_equal(host(ops.ds_to_f32(cu(p))), dso.ds_to_f32(p), "to_f32")


@pytest.mark.parametrize("n", SIZES)
def test_packed_vs_oracle(ops, dso, n):
    rng = np.random.default_rng(200 + n)
    a = dso.ds_from_f64(rand_f64(rng, n, -12, 12), 8)
    b = dso.ds_from_f64(rand_f64(rng, n, -12, 12), 8)
    ta, tb = cu(a), cu(b)
    for name in ("add", "sub", "mul"):
        assert_bits_equal(host(getattr(ops, "ds_" + name)(ta, tb)),
                          getattr(dso, "ds_" + name)(a, b, 8), f"{name} n={n}")


@pytest.mark.parametrize("n", SIZES)
def test_fused_vs_oracle(ops, dso, n):
    rng = np.random.default_rng(300 + n)
    x, y, c = rand_f64(rng, n), rand_f64(rng, n), rand_f64(rng, n)
    tx, ty, tc = cu(x), cu(y), cu(c)
    assert_bits_equal(host(ops.ds_fused_add_mul(tx, ty)), dso.ds_fused_add_mul(x, y, 8), "packed")
    assert_bits_equal(host(ops.ds_fused_add_mul_to_f64(tx, ty)),
                      dso.ds_fused_add_mul_to_f64(x, y, 8), "add_mul")
    assert_bits_equal(host(ops.ds_fused_add_sub_to_f64_cuda(tx, ty)),
                      dso.ds_fused_add_sub_to_f64(x, y, 8), "add_sub")
    assert_bits_equal(host(ops.ds_fused_add_mul3_to_f64(tx, ty, tc)),
                      dso.ds_fused_add_mul3_to_f64(x, y, c, 8), "add_mul3")


@pytest.mark.parametrize("n,k", [(0, 3), (1, 0), (7, 1), (4099, 4), (65537, 16), (1 << 16, 64),
                                 (4097, 1024)])
def test_recurrences_vs_oracle(ops, dso, n, k):
    rng = np.random.default_rng(400 + n + k)
    x = rng.uniform(-1, 1, n)
    a = rng.uniform(0.999, 1.001, n)
    b = rng.uniform(-1e-3, 1e-3, n)
    y = rng.uniform(-1, 1, n)
    assert_bits_equal(host(ops.ds_recurrence_mul_add_to_f64(cu(x), cu(a), cu(b), k)),
                      dso.ds_recurrence_mul_add_to_f64(x, a, b, k, 8), f"mul_add k={k}")
    assert_bits_equal(host(ops.ds_recurrence_add_mul_to_f64_cuda(cu(x), cu(y), k)),
                      dso.ds_recurrence_add_mul_to_f64(x, y, k, 8), f"add_mul k={k}")


def test_recurrences_edge_magnitudes(ops, dso):
    """The recurrences take the product's error term from an FMA only where
    it equals Dekker's; operands and products over the whole f32 range
    (Veltkamp-split overflow near 8.3e34, products near the subnormal range,
    zeros, Inf, NaN) give the oracle's (Dekker's) bits at every k.  The
    edge values sit at the start of the array, so whole warps see them."""
    rng = np.random.default_rng(77)
    n = (1 << 16) + 7
    sign = lambda: np.where(rng.integers(0, 2, n) == 0, 1.0, -1.0)  # noqa: E731
    x = sign() * 2.0 ** rng.uniform(-148, 127, n)
    a = sign() * 2.0 ** rng.uniform(-80, 80, n)
    b = sign() * 2.0 ** rng.uniform(-148, 127, n)
    y = sign() * 2.0 ** rng.uniform(-75, 64, n)
    edges = [0.0, -0.0, np.inf, -np.inf, np.nan, 8.4e34, -8.3e34, 1e-45, 2.0 ** -90,
             2.0 ** 115, 2.0 ** 120, 2.0 ** -126, 2.0 ** -5, 2.0 ** 110]
    for v in (x, a, b, y):
        v[:len(edges)] = edges
        v[len(edges):2 * len(edges)] = edges[::-1]
    # a stretch of ordinary values, where whole warps take the FMA path
    x[4096:8192] = rng.uniform(-1, 1, 4096)
    a[4096:8192] = rng.uniform(0.999, 1.001, 4096)
    y[4096:8192] = rng.uniform(-1, 1, 4096)
    for k in (1, 2, 5, 33):
        assert_bits_equal(host(ops.ds_recurrence_mul_add_to_f64(cu(x), cu(a), cu(b), k)),
                          dso.ds_recurrence_mul_add_to_f64(x, a, b, k, 8), f"mul_add k={k}")
        assert_bits_equal(host(ops.ds_recurrence_add_mul_to_f64_cuda(cu(x), cu(y), k)),
                          dso.ds_recurrence_add_mul_to_f64(x, y, k, 8), f"add_mul k={k}")


def test_unaligned_views(ops, dso):
    """Odd element offsets take the scalar path and give the same bits."""
    rng = np.random.default_rng(5)
    n = 1001
    x, y, c = rand_f64(rng, n), rand_f64(rng, n), rand_f64(rng, n)
    got = host(ops.ds_fused_add_mul3_to_f64(misaligned(x), misaligned(y), misaligned(c)))
    assert_bits_equal(got, dso.ds_fused_add_mul3_to_f64(x, y, c), "unaligned add_mul3")
    a, b = dso.ds_from_f64(x), dso.ds_from_f64(y)
    got = host(ops.ds_mul(misaligned(a), misaligned(b)))
    assert_bits_equal(got, dso.ds_mul(a, b), "unaligned mul")
    assert_bits_equal(host(ops.ds_from_f64(misaligned(x))), dso.ds_from_f64(x), "unaligned split")


def test_multidim_packed(ops, dso):
    rng = np.random.default_rng(6)
    shape = (3, 5, 7)
    a = dso.ds_from_f64(rand_f64(rng, 105).reshape(shape))
    b = dso.ds_from_f64(rand_f64(rng, 105).reshape(shape))
    got = host(ops.ds_add(cu(a), cu(b)))
    assert got.shape == shape + (2,)
    assert_bits_equal(got, dso.ds_add(a, b), "3-d add")


def test_config1_fused_add_mul_vs_numpy(ops, dso):
    """(a + b) * c on 2^20 uniform[-1,1] f64, seed 0: bit-exact vs the oracle and
    close to numpy f64 (DS carries ~48 bits)."""
    rng = np.random.default_rng(0)
    n = 1 << 20
    a, b, c = rng.uniform(-1, 1, n), rng.uniform(-1, 1, n), rng.uniform(-1, 1, n)
    got = host(ops.ds_fused_add_mul3_to_f64(cu(a), cu(b), cu(c)))
    assert_bits_equal(got, dso.ds_fused_add_mul3_to_f64(a, b, c, 8), "config 1")
    ref = (a + b) * c
    rel = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-300)
    assert np.max(np.abs(got - ref)) < 2.0 ** -44 * 4.0


@pytest.mark.slow
def test_large_fused_property(ops, dso):
    """2^26 + 5 elements (above L2): bit-exact against the multi-threaded oracle."""
    rng = np.random.default_rng(7)
    n = (1 << 26) + 5
    a, b, c = rng.uniform(-1, 1, n), rng.uniform(-1, 1, n), rng.uniform(-1, 1, n)
    got = host(ops.ds_fused_add_mul3_to_f64(cu(a), cu(b), cu(c)))
    assert_bits_equal(got, dso.ds_fused_add_mul3_to_f64(a, b, c, 8), "2^26+5")


def test_reference_ffi_smoke_vectors():
    """python/test_ds_add.py and python/test_ds_fused_add_mul_to_f64.py through
    register_ffi_target / ffi_call, as the reference tests call them."""
    import ctypes

    import torch
    from ds_b200 import LIB_PATH, ffi
    lib = ctypes.cdll.LoadLibrary(LIB_PATH)
    ffi.register_ffi_target("ds_from_f64", lib.ds_from_f64, platform="CUDA")
    ffi.register_ffi_target("ds_to_f64", lib.ds_to_f64, platform="CUDA")
    ffi.register_ffi_target("ds_add", lib.ds_add, platform="CUDA")
    f64, f32 = torch.float64, torch.float32

    def ds_from_f64(x):
        return ffi.ffi_call("ds_from_f64", ffi.ShapeDtypeStruct(tuple(x.shape) + (2,), f32),
                            vmap_method="broadcast_all")(x)

    def ds_to_f64(x):
        return ffi.ffi_call("ds_to_f64", ffi.ShapeDtypeStruct(tuple(x.shape[:-1]), f64),
                            vmap_method="broadcast_all")(x)

    def ds_add(a, b):
        return ffi.ffi_call("ds_add", ffi.ShapeDtypeStruct(tuple(a.shape), f32),
                            vmap_method="broadcast_all")(a, b)

    x = torch.tensor([1.0, 2.0, 3.0], dtype=f64, device="cuda")
    y = torch.tensor([4.0, 5.0, 6.0], dtype=f64, device="cuda")
    z = ds_to_f64(ds_add(ds_from_f64(x), ds_from_f64(y)))
    np.testing.assert_allclose(host(z), host(x + y), rtol=1e-6, atol=1e-6)

    ffi.register_ffi_target("ds_fused_add_mul_to_f64", lib.ds_fused_add_mul_to_f64,
                            platform="CUDA")
    x = torch.tensor([1.23456789012345, 2.5, 123456789.12345679], dtype=f64, device="cuda")
    y = torch.tensor([9.87654321098765, 3.0, 1.23456789e-7], dtype=f64, device="cuda")
    out = ffi.ffi_call("ds_fused_add_mul_to_f64", ffi.ShapeDtypeStruct(tuple(x.shape), f64),
                       vmap_method="broadcast_all")(x, y)
    np.testing.assert_allclose(host(out), host((x + y) * y), rtol=1e-5, atol=1e-5)

    # python/test_ds_recurrence_add_mul_to_f64_cuda.py:39-49 (k=8, attribute)
    ffi.register_ffi_target("ds_recurrence_add_mul_to_f64_cuda",
                            lib.ds_recurrence_add_mul_to_f64_cuda, platform="CUDA")
    x = torch.tensor([0.25, 0.5, 0.75], dtype=f64, device="cuda")
    y = torch.tensor([0.2, 0.3, 0.4], dtype=f64, device="cuda")
    out = ffi.ffi_call("ds_recurrence_add_mul_to_f64_cuda",
                       ffi.ShapeDtypeStruct(tuple(x.shape), f64),
                       vmap_method="broadcast_all")(x, y, k=np.int32(8))
    ref = x.clone()
    for _ in range(8):
        ref = (ref + y) * y
    assert np.max(np.abs(host(out) - host(ref))) < 1e-12


def test_invalid_shape_raises_reference_message(ops):
    import torch
    from ds_b200 import DsInvalidArgument, ffi
    a = torch.zeros(4, 3, dtype=torch.float32, device="cuda")
    with pytest.raises(DsInvalidArgument, match="ds.add expects last dim == 2"):
        ffi.ffi_call("ds_add", ffi.ShapeDtypeStruct((4, 3), torch.float32))(a, a)
