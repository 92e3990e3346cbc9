"""Pin the C oracle to the reference's own DS model (tests/ds_ref.py) bit for bit.

The vectors in tests/golden/ds_ref_vectors.npz were produced by importing the
reference's ds_ref.py (see tests/golden/make_golden.py).  Every comparison here
is bit-exact (NaN positions must match).
"""
import numpy as np

from conftest import assert_bits_equal
from oracle import ds_pass_ref


def test_primitives(golden, dso):
    a, b = golden["prim_a"], golden["prim_b"]
    with np.errstate(all="ignore"):
        s, e = dso.two_sum(a, b)
        assert_bits_equal(s, golden["two_sum_s"], "two_sum s")
        assert_bits_equal(e, golden["two_sum_e"], "two_sum e")
        h, l = dso.split(a)
        assert_bits_equal(h, golden["split_hi"], "split hi")
        assert_bits_equal(l, golden["split_lo"], "split lo")
        p, pe = dso.two_prod(a, b)
        assert_bits_equal(p, golden["two_prod_p"], "two_prod p")
        assert_bits_equal(pe, golden["two_prod_e"], "two_prod e")


def test_packed_ops(golden, dso):
    a, b = golden["pk_a"], golden["pk_b"]
    for name in ("add", "sub", "mul"):
        got = getattr(dso, "ds_" + name)(a, b)
        assert_bits_equal(got, golden["pk_" + name], "ds_" + name)
        # the multi-threaded loop gives the same bits
        assert_bits_equal(getattr(dso, "ds_" + name)(a, b, nthreads=4), got, name + " omp")


def test_split_recombine(golden, dso):
    with np.errstate(all="ignore"):
        sp = dso.ds_from_f64(golden["f64_x"])
        assert_bits_equal(sp, golden["f64_split"], "ds_from_f64")
        assert_bits_equal(dso.ds_to_f64(sp), golden["f64_recombine"], "ds_to_f64")


def test_fused_chains(golden, dso):
    x, y, c = golden["fx"], golden["fy"], golden["fc"]
    assert_bits_equal(dso.ds_fused_add_mul(x, y), golden["fused_add_mul_packed"],
                      "fused_add_mul")
    assert_bits_equal(dso.ds_fused_add_mul_to_f64(x, y), golden["fused_add_mul_to_f64"],
                      "fused_add_mul_to_f64")
    assert_bits_equal(dso.ds_fused_add_sub_to_f64(x, y), golden["fused_add_sub_to_f64"],
                      "fused_add_sub_to_f64")
    assert_bits_equal(dso.ds_fused_add_mul3_to_f64(x, y, c),
                      golden["fused_add_mul3_to_f64"], "fused_add_mul3_to_f64")


def test_recurrences(golden, dso):
    for k in (0, 1, 8):
        assert_bits_equal(dso.ds_recurrence_add_mul_to_f64(golden["rec_x"], golden["rec_y"], k),
                          golden[f"rec_add_mul_k{k}"], f"recurrence k={k}")
    for k in (1, 4, 16):
        assert_bits_equal(
            dso.ds_recurrence_mul_add_to_f64(golden["mrec_x"], golden["mrec_a"],
                                             golden["mrec_b"], k),
            golden[f"mrec_k{k}"], f"mul_add recurrence k={k}")


def test_sequential_folds(golden, dso):
    x = golden["sum_x"]
    h, l = dso.ds_reduce_ds_seq(x, np.zeros_like(x))
    assert float(h) + float(l) == float(golden["sum_ref"])
    h, l = dso.ds_dot_f32_seq(golden["dot_a"], golden["dot_b"])
    assert float(h) + float(l) == float(golden["dot_ref"])
    t = golden["trip_x"]
    h, l = dso.ds_dot_f32_seq(t, np.ones_like(t))
    assert float(h) + float(l) == float(golden["trip_dot_ref"]) == 1000.0


def test_pass_restatement_elementwise(golden, dso):
    """The NumPy restatement of the pass's add/sub/mul matches the C oracle bit for bit."""
    a, b = golden["pk_a"], golden["pk_b"]
    with np.errstate(all="ignore"):
        for name in ("add", "sub", "mul"):
            h, l = getattr(ds_pass_ref, "ds_" + name)(a[:, 0], a[:, 1], b[:, 0], b[:, 1])
            assert_bits_equal(np.stack([h, l], -1), golden["pk_" + name], "pass " + name)
        got = ds_pass_ref.fused_add_mul3_f64(golden["fx"], golden["fy"], golden["fc"])
        assert_bits_equal(got, golden["fused_add_mul3_to_f64"], "pass (a+b)*c")


def test_reference_known_answers(dso):
    """Hand-picked vectors of the reference's FFI smoke tests."""
    # python/test_ds_add.py:50-67
    x = np.array([1.0, 2.0, 3.0])
    y = np.array([4.0, 5.0, 6.0])
    z = dso.ds_to_f64(dso.ds_add(dso.ds_from_f64(x), dso.ds_from_f64(y)))
    np.testing.assert_allclose(z, x + y, rtol=1e-6, atol=1e-6)
    # python/test_ds_fused_add_mul_to_f64.py:34-42
    x = np.array([1.23456789012345, 2.5, 123456789.12345679])
    y = np.array([9.87654321098765, 3.0, 1.23456789e-7])
    np.testing.assert_allclose(dso.ds_fused_add_mul_to_f64(x, y), (x + y) * y,
                               rtol=1e-5, atol=1e-5)
    # python/test_pass_correctness.py:57-111 cancellation (x+y)-x against the
    # f64 result of the same expression; improvement > 100x on elements 0 and 1
    # (at x=1e12 the DS precision, ~2^-48 * 1e12, is coarser than y=1e-4).
    x = np.array([1e8, 1e10, 1e12])
    y = np.array([1e-2, 1e-3, 1e-4])
    ref = (x + y) - x
    ds = dso.ds_fused_add_sub_to_f64(x, y)
    x32, y32 = x.astype(np.float32), y.astype(np.float32)
    f32 = ((x32 + y32) - x32).astype(np.float64)
    improvement = np.abs(f32 - ref) / (np.abs(ds - ref) + 1e-30)
    assert improvement[0] > 100 and improvement[1] > 100
    # tests/test_f64_ds.py:88-97 split fidelity
    v = np.array([1.23456789012345e10])
    r = dso.ds_to_f64(dso.ds_from_f64(v))
    assert abs(r[0] - v[0]) / abs(v[0]) < 2.0 ** -46
