"""The allocation-free reduce entry point (ds_reduce_f64_noalloc), through the C ABI.

Callers that cannot allocate device memory -- a handler with no scratch
allocator, or code living beside a framework allocator that already holds
most of the GPU -- pass only inputs and outputs to this entry point; its
scratch is a static device array inside the library.  This checks it against
the workspace-taking entry point (ds_reduce_f64) on two calls in a row, the
second of which reuses the array the first one left behind.  Collected last
(file name) so a failing run has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc_sum(L, x, dims):
    init = torch.zeros((), dtype=torch.float64, device=x.device)
    out_shape = tuple(s for i, s in enumerate(x.shape) if i not in dims)
    out = torch.empty(out_shape, dtype=torch.float64, device=x.device)
    bx, kx = L.make_buffer(x.data_ptr(), x.shape)
    bi, ki = L.make_buffer(init.data_ptr(), ())
    bo, ko = L.make_buffer(out.data_ptr(), out_shape)
    cd = (ctypes.c_int64 * max(len(dims), 1))(*dims)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = L.lib().ds_reduce_f64_noalloc(ctypes.byref(bx), ctypes.byref(bi), cd, len(dims),
                                       L.DS_BODY_ADD, ctypes.byref(bo), stream)
    L.check(st, "ds_reduce_f64_noalloc")
    return out


def test_noalloc_matches_workspace_entry():
    from ds_b200 import _lib as L
    from ds_b200 import ops
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(1)
    # Two calls in a row: a multi-block full reduction (block partials in the
    # static array), then a different length over the array's old contents.
    for n in ((1 << 22) + 7, 1_000_003):
        s = np.where(np.arange(n) % 2 == 0, 1.0, -1.0)
        x = torch.from_numpy(s * 1e8 + rng.uniform(0, 1, n) * 1e-3).to(dev)
        got = _noalloc_sum(L, x, (0,))
        want = ops.ds_reduce_f64(x, dimensions=(0,))
        torch.cuda.synchronize()
        assert got.cpu().numpy().tobytes() == want.cpu().numpy().tobytes()
    # A segmented reduction needs no partials and takes the same path.
    y = torch.from_numpy(rng.uniform(-1, 1, (64, 5000))).to(dev)
    got = _noalloc_sum(L, y, (1,))
    want = ops.ds_reduce_f64(y, dimensions=(1,))
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    # Reductions over a leading dimension with few columns slice it across
    # blocks; their slice partials live in the same static array.
    for shape in ((1 << 18, 8), (20000, 3, 5)):
        z = torch.from_numpy(rng.uniform(-1, 1, shape) * 1e6).to(dev)
        got = _noalloc_sum(L, z, (0,))
        want = ops.ds_reduce_f64(z, dimensions=(0,))
        torch.cuda.synchronize()
        assert got.cpu().numpy().tobytes() == want.cpu().numpy().tobytes()
