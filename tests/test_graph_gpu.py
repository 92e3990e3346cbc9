"""The ops are stream-ordered with no host synchronisation, so a step of
them can be captured once in a CUDA graph and replayed: the graph gives the
same bits as the eager calls (tensor-core product, DS sum, fused program,
elementwise chain)."""
import numpy as np
import pytest

from conftest import assert_bits_equal
from gpu_util import cu, host

pytestmark = pytest.mark.gpu


def test_capture_and_replay():
    import torch
    from ds_b200 import fuse, ops
    rng = np.random.default_rng(12)
    A = cu(rng.uniform(-1, 1, (512, 384)))
    B = cu(rng.uniform(-1, 1, (384, 640)))
    x = cu(rng.uniform(-1, 1, 1 << 21))
    y = cu(rng.uniform(-1, 1, 1 << 21))
    chain = fuse.jit(lambda a, b: (a + b) * a - 0.5)

    def step():
        return (ops.ds_matmul_f64(A, B), ops.ds_sum_f64(x), chain(x, y),
                ops.ds_fused_add_mul_to_f64(x, y))

    eager = [host(t) for t in step()]  # warm-up: one-time setup and compilation
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # second warm-up on the capture stream
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            outs = step()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for got, want, name in zip(outs, eager, ("gemm", "sum", "fused", "chain")):
        assert_bits_equal(host(got), want, name)
    # new inputs copied into the captured buffers flow through the graph
    x.copy_(cu(rng.uniform(-1, 1, 1 << 21)))
    g.replay()
    torch.cuda.synchronize()
    assert_bits_equal(host(outs[1]), host(ops.ds_sum_f64(x)), "sum after update")
    del g
