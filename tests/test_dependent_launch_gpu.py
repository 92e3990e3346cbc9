"""The library's short kernels are launched as programmatic dependents of
the previous kernel on the stream, and each waits for that kernel before its
first memory access.  These tests rewrite an op's inputs with the kernel
just before it (a torch kernel, or another op of the library) and compare
the result with the same op run again after a device synchronize: the bits
must agree, so no kernel read an input before its producer finished."""
import numpy as np
import pytest

from conftest import assert_bits_equal
from gpu_util import cu, host

pytestmark = pytest.mark.gpu


def quiet(fn):
    """fn's result with the device idle before and after the call."""
    import torch
    torch.cuda.synchronize()
    r = fn()
    torch.cuda.synchronize()
    return host(r)


def test_elementwise_reads_what_the_kernel_before_wrote():
    from ds_b200 import ops
    rng = np.random.default_rng(41)
    x = cu(rng.uniform(-1, 1, (1 << 22) + 3))
    y = cu(rng.uniform(-1, 1, (1 << 22) + 3))
    for k in range(6):
        # a torch kernel rewrites x; the op is launched right behind it
        x.mul_(-1.5 if k % 2 else 0.75)
        got = host(ops.ds_fused_add_mul3_to_f64(x, y, y))
        want = quiet(lambda: ops.ds_fused_add_mul3_to_f64(x, y, y))
        assert_bits_equal(got, want, f"fused add-mul after a torch write, step {k}")


def test_chained_ops_read_the_previous_op_in_full():
    from ds_b200 import ops
    rng = np.random.default_rng(42)
    a = cu(rng.uniform(-1, 1, 3_000_001))
    b = cu(rng.uniform(-1, 1, 3_000_001))
    # each op consumes the previous op's output with no synchronize between
    pa = ops.ds_from_f64(a)
    pb = ops.ds_from_f64(b)
    y = ops.ds_to_f64(ops.ds_mul(ops.ds_add(pa, pb), pb))
    total = ops.ds_sum_f64(y)
    got_y, got_t = host(y), host(total)

    def again():
        return ops.ds_to_f64(ops.ds_mul(ops.ds_add(ops.ds_from_f64(a), ops.ds_from_f64(b)),
                                        ops.ds_from_f64(b)))
    want_y = quiet(again)
    assert_bits_equal(got_y, want_y, "packed chain")
    assert_bits_equal(got_t, quiet(lambda: ops.ds_sum_f64(cu(want_y))), "sum of the chain")


@pytest.mark.parametrize("n", [10_000, 1 << 20, (1 << 24) + 5])
def test_reduce_stages_read_the_kernel_before(n):
    from ds_b200 import ops
    rng = np.random.default_rng(43)
    x = cu(rng.uniform(-1, 1, n))
    for k in range(4):
        x.add_(0.25 * (k + 1))  # a torch kernel right before stage 1
        got = host(ops.ds_sum_f64(x))
        want = quiet(lambda: ops.ds_sum_f64(x))
        assert_bits_equal(got, want, f"sum of {n} after a torch write, step {k}")


def test_sliced_leading_reduce_and_batched_dot_after_a_write():
    from ds_b200 import ops
    rng = np.random.default_rng(44)
    x = cu(rng.uniform(-1, 1, (1 << 18, 8)))
    v = cu(rng.uniform(-1, 1, (64, 1 << 14)))
    w = cu(rng.uniform(-1, 1, (64, 1 << 14)))

    def bdot():
        return ops.ds_dot_general_f64(v, w, lhs_contracting=1, rhs_contracting=1,
                                      lhs_batch=(0,), rhs_batch=(0,))
    for k in range(3):
        x.mul_(-1.0)
        got = host(ops.ds_sum_f64(x, dimensions=(0,)))
        assert_bits_equal(got, quiet(lambda: ops.ds_sum_f64(x, dimensions=(0,))),
                          f"leading-dimension sum, step {k}")
        v.mul_(0.5)
        got = host(bdot())
        assert_bits_equal(got, quiet(bdot), f"batched dot, step {k}")


def test_fused_program_after_a_write_and_in_a_graph():
    import torch
    from ds_b200 import fuse
    rng = np.random.default_rng(45)
    a = cu(rng.uniform(-1, 1, 1 << 20))
    b = cu(rng.uniform(-1, 1, 1 << 20))
    f = fuse.jit(lambda x, y: (x + y) * x - 0.5)
    for k in range(3):
        a.mul_(-1.0)
        got = host(f(f(a, b), b))
        assert_bits_equal(got, quiet(lambda: f(f(a, b), b)), f"fused chain, step {k}")
    # captured: the first program of each replay follows a copy into its input
    src = cu(rng.uniform(-1, 1, 1 << 20))
    f(f(a, b), b)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            a.copy_(src)
            out = f(f(a, b), b)
    torch.cuda.current_stream().wait_stream(s)
    for k in range(3):
        src.mul_(-1.0)
        g.replay()
        got = host(out)
        assert_bits_equal(got, quiet(lambda: f(f(src, b), b)), f"graph replay {k}")
    del g
