"""The sharded reduce's exchange kernel on one GPU.

Cross-GPU runs are in test_dist_gpu.py.  Here the other ranks are stand-ins
that cannot wait on this kernel (nothing on the GPU runs them): a world of
one rank exchanging with itself, a world of two whose second rank's record
is already in place before the launch, and a world of two whose second rank
never writes, which must end in the bounded wait's error path -- NaN result,
the error word set, the context still usable.
"""
import ctypes

import numpy as np
import pytest

from conftest import assert_bits_equal
from gpu_util import cu, host

pytestmark = pytest.mark.gpu

RECORD = np.dtype([("hi", "<f4"), ("lo", "<f4"), ("n", "<i8"), ("epoch", "<u8"),
                   ("pad", "<u8")])


@pytest.fixture(scope="module")
def env():
    import torch
    from ds_b200 import _lib, ops
    return torch, _lib, ops


def new_buffer(torch, _lib):
    nbytes = int(_lib.lib().ds_exchange_bytes())
    assert nbytes == 1024
    return torch.zeros(nbytes, dtype=torch.uint8, device="cuda")


def records(buf):
    return host(buf)[:2 * 8 * 32].view(RECORD).reshape(2, 8)


def error_word(buf):
    return int(host(buf)[512:516].view(np.uint32)[0])


def sharded_sum(env, x, init, bufs, rank, epoch, timeout_ms=1000, body=0):
    torch, _lib, ops = env
    L = _lib.lib()
    ib, idims = _lib.make_buffer(x.data_ptr(), tuple(x.shape))
    it = torch.full((), float(init), dtype=torch.float64, device="cuda")
    tb, tdims = _lib.make_buffer(it.data_ptr(), ())
    out = torch.empty((), dtype=torch.float64, device="cuda")
    ob, odims = _lib.make_buffer(out.data_ptr(), ())
    ws_bytes = L.ds_reduce_f64_sharded_workspace_size(ctypes.byref(ib))
    ws = torch.empty(max(int(ws_bytes), 8), dtype=torch.uint8, device="cuda")
    ptrs = (ctypes.c_void_p * len(bufs))(*[b.data_ptr() for b in bufs])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(L.ds_reduce_f64_sharded(ctypes.byref(ib), ctypes.byref(tb), body, ctypes.byref(ob),
                                       ptrs, len(bufs), rank, epoch, timeout_ms,
                                       ctypes.c_void_p(ws.data_ptr()), ws_bytes, stream))
    return out


def inputs(n, seed):
    s = np.where(np.arange(n) % 2 == 0, 1.0, -1.0)
    return s * 1e8 + np.random.default_rng(seed).uniform(0, 1, n) * 1e-3


@pytest.mark.parametrize("n", [100_003, 1 << 22])
def test_world_of_one_matches_local_reduce(env, n):
    """A single rank exchanging with itself folds exactly what the one-GPU
    reduce folds: same partial tree, same init step -> same bits, call after
    call (the parity of the records alternates)."""
    torch, _lib, ops = env
    x = cu(inputs(n, 3))
    want = host(ops.ds_reduce_f64(x, init=0.25))
    buf = new_buffer(torch, _lib)
    for epoch in range(1, 5):
        got = host(sharded_sum(env, x, 0.25, [buf], 0, epoch))
        assert_bits_equal(got, want, f"epoch {epoch}")
    rec = records(buf)
    assert rec[0, 0]["epoch"] == 4 and rec[1, 0]["epoch"] == 3
    assert rec[0, 0]["n"] == n
    assert error_word(buf) == 0


def test_world_of_one_small_and_empty(env):
    torch, _lib, ops = env
    buf = new_buffer(torch, _lib)
    empty = torch.zeros(0, dtype=torch.float64, device="cuda")
    assert float(host(sharded_sum(env, empty, 2.5, [buf], 0, 1))) == 2.5
    x = np.random.default_rng(2).uniform(-1, 1, 5)
    got = float(host(sharded_sum(env, cu(x), 0.0, [buf], 0, 2)))
    assert abs(got - float(np.sum(x))) < 1e-13


def test_two_ranks_with_peer_record_in_place(env, dso):
    """Rank 0 of two: rank 1's total is already in rank 0's buffer, so the
    wait ends at once.  Rank 0 must publish its own total into rank 1's
    buffer and return init + (total_0 + total_1) in DS arithmetic."""
    torch, _lib, ops = env
    own, peer = new_buffer(torch, _lib), new_buffer(torch, _lib)
    epoch = 7
    par = epoch & 1
    p1 = np.zeros(1, RECORD)
    p1["hi"], p1["lo"], p1["n"], p1["epoch"] = np.float32(12345.5), np.float32(1e-4), 10, epoch
    raw = host(own).copy()
    off = (par * 8 + 1) * 32
    raw[off:off + 32] = p1.view(np.uint8)
    own.copy_(torch.from_numpy(raw))
    x = inputs(200_001, 5)
    got = float(host(sharded_sum(env, cu(x), 0.5, [own, peer], 0, epoch)))
    sent = records(peer)[par, 0]
    assert sent["epoch"] == epoch and sent["n"] == x.size
    p0 = np.array([[sent["hi"], sent["lo"]]], np.float32)
    p1v = np.array([[p1["hi"][0], p1["lo"][0]]], np.float32)
    total = dso.ds_add(p0, p1v)
    want = float(dso.ds_to_f64(dso.ds_add(dso.ds_from_f64(np.array([0.5])), total))[0])
    assert got == want
    assert error_word(own) == 0


def test_two_ranks_empty_peer_is_skipped(env):
    torch, _lib, ops = env
    own, peer = new_buffer(torch, _lib), new_buffer(torch, _lib)
    epoch = 2
    raw = host(own).copy()
    rec = np.zeros(1, RECORD)
    rec["hi"], rec["n"], rec["epoch"] = np.float32(99.0), 0, epoch  # n = 0: ignored
    off = ((epoch & 1) * 8 + 1) * 32
    raw[off:off + 32] = rec.view(np.uint8)
    own.copy_(torch.from_numpy(raw))
    x = cu(inputs(100_003, 8))
    want = host(ops.ds_reduce_f64(x, init=0.0))
    got = host(sharded_sum(env, x, 0.0, [own, peer], 0, epoch))
    assert_bits_equal(got, want, "empty peer skipped")


def test_wait_times_out_and_reports(env):
    """The second rank never writes: the bounded wait gives up after
    timeout_ms, the result is NaN, the own error word is 1, and the context
    keeps working."""
    import time
    torch, _lib, ops = env
    own, peer = new_buffer(torch, _lib), new_buffer(torch, _lib)
    x = cu(inputs(10_000, 1))
    t0 = time.perf_counter()
    got = float(host(sharded_sum(env, x, 0.0, [own, peer], 0, 1, timeout_ms=20)))
    elapsed = time.perf_counter() - t0
    assert np.isnan(got)
    assert error_word(own) == 1
    assert elapsed < 5.0
    code = ctypes.c_uint32()
    _lib.check(_lib.lib().ds_exchange_error(ctypes.c_void_p(own.data_ptr()), ctypes.byref(code)))
    assert code.value == 1
    # the context is intact
    assert float(host(ops.ds_sum_f64(cu(np.ones(1000))))) == 1000.0


def test_argument_checks(env):
    torch, _lib, ops = env
    buf = new_buffer(torch, _lib)
    x = cu(np.ones(10))
    with pytest.raises(_lib.DsInvalidArgument, match="epochs start at 1"):
        sharded_sum(env, x, 0.0, [buf], 0, 0)
    with pytest.raises(_lib.DsInvalidArgument, match="rank/world"):
        sharded_sum(env, x, 0.0, [buf], 1, 1)
    with pytest.raises(_lib.DsInvalidArgument, match="timeout"):
        sharded_sum(env, x, 0.0, [buf], 0, 1, timeout_ms=0)
    with pytest.raises(_lib.DsInvalidArgument, match="rank/world"):
        sharded_sum(env, x, 0.0, [buf] * 9, 0, 1)
