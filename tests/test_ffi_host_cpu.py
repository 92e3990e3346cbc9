"""Host logic of the Python mirror of jax.ffi that needs no GPU: the
per-stream workspace cache (how it grows, the size above which nothing is
kept, nothing kept while a CUDA graph is captured) and the dims arrays that
buffers of one shape share.  CPU tensors stand in for device memory."""
import pytest
import torch

MiB = 1 << 20


@pytest.fixture
def ffi(monkeypatch):
    from ds_b200 import ffi as f
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: False)
    monkeypatch.setattr(f, "_workspaces", {})
    return f


def test_workspace_grows_to_powers_of_two_and_is_reused(ffi):
    cpu = torch.device("cpu")
    w1 = ffi._workspace(10, cpu, 7)
    assert w1.numel() == MiB  # the first buffer is 1 MiB
    assert ffi._workspace(MiB, cpu, 7) is w1  # a request that fits reuses it
    w2 = ffi._workspace(MiB + 1, cpu, 7)
    assert w2 is not w1 and w2.numel() == 2 * MiB
    assert ffi._workspace(5 * MiB, cpu, 7).numel() == 8 * MiB
    assert ffi._workspace(100, cpu, 7).numel() == 8 * MiB  # it never shrinks


def test_workspaces_are_per_stream(ffi):
    cpu = torch.device("cpu")
    assert ffi._workspace(100, cpu, 1) is not ffi._workspace(100, cpu, 2)
    assert ffi._workspace(100, cpu, 1) is ffi._workspace(200, cpu, 1)


def test_large_workspaces_are_not_kept(ffi):
    cpu = torch.device("cpu")
    small = ffi._workspace(100, cpu, 3)
    n = ffi._CACHED_WORKSPACE_MAX + 1
    big = ffi._workspace(n, cpu, 3)
    assert big.numel() == n
    assert ffi._workspace(100, cpu, 3) is small  # the large one replaced nothing
    assert ffi._workspace(ffi._CACHED_WORKSPACE_MAX, cpu, 3).numel() == \
        ffi._CACHED_WORKSPACE_MAX  # the limit itself is still cached


def test_nothing_is_kept_while_capturing(ffi, monkeypatch):
    cpu = torch.device("cpu")
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)
    a = ffi._workspace(1000, cpu, 4)
    b = ffi._workspace(1000, cpu, 4)
    assert a is not b and a.numel() == 1000
    assert ffi._workspaces == {}


def test_buffers_of_one_shape_share_their_dims():
    from ds_b200 import _lib
    b1, d1 = _lib.make_buffer(256, (3, 4))
    b2, d2 = _lib.make_buffer(512, [3, 4])
    assert d1 is d2 and list(d1) == [3, 4]
    assert (b1.data, b1.rank, b2.data, b2.rank) == (256, 2, 512, 2)
    _, d3 = _lib.make_buffer(256, (4, 3))
    assert d3 is not d1 and list(d3) == [4, 3]
    _, d0 = _lib.make_buffer(256, ())
    assert len(d0) == 1  # a rank-0 buffer still gets a valid dims pointer
