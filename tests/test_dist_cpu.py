"""Multi-rank host logic with CPU ranks (gloo, world size 2 and 3).

The per-rank GPU reduction and the fold are replaced by the oracle (the
checker), so what runs here is the sharding, the (hi, lo) all-gather and the
fixed-order combine that ds_b200.dist performs on GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_DIR, ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, q):
    import sys
    for p in (ROOT, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        _worker_body(rank, world, n, q)
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, None, repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


def _worker_body(rank, world, n, q):
    if True:
        from ds_b200 import dist as dsd
        from oracle import dso
        rng = np.random.default_rng(1)
        x = np.where(np.arange(n) % 2 == 0, 1e8, -1e8) + rng.uniform(0, 1, n) * 1e-3
        start, stop = dsd.shard_range(n, rank, world)
        local = torch.from_numpy(x[start:stop])

        def local_pair(t):
            # the GPU's f64 entry sums a shard exactly in f64 per thread
            # before its DS tree: stood in for by the exact sum, split
            import math
            s = math.fsum(t.numpy().tolist())
            p = dso.ds_from_f64(np.array([s]))
            return torch.tensor([p[0, 0], p[0, 1]], dtype=torch.float32)

        def combine(pairs, init):
            p = pairs.numpy()
            h, l = dso.ds_reduce_ds_seq(p[:, 0], p[:, 1], init=init)
            return torch.tensor(float(h) + float(l), dtype=torch.float64)

        r = dsd.ds_sum_f64_sharded(local, init=0.5, local_pair=local_pair, combine=combine)
        allr = [torch.zeros((), dtype=torch.float64) for _ in range(world)]
        dist.all_gather(allr, r)
        q.put((rank, float(r), [float(v) for v in allr], (start, stop)))


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_sum_gloo(world):
    n = 100_003
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    errors = [r for r in results if r[1] is None]
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)
    results.sort()
    # every rank holds the same bits
    vals = {v for _, v, _, _ in results}
    assert len(vals) == 1
    for _, v, allv, _ in results:
        assert len(set(allv)) == 1 and allv[0] == v
    # the shards tile [0, n)
    ranges = [rg for *_, rg in results]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    # no farther from the exact sum (+ init) than the reference-order DS
    # fold, whose running sum swings through +-1e8 (DS resolves ~1e8 * 2^-48)
    import math

    from oracle import dso
    rng = np.random.default_rng(1)
    x = np.where(np.arange(n) % 2 == 0, 1e8, -1e8) + rng.uniform(0, 1, n) * 1e-3
    truth = math.fsum(x.tolist()) + 0.5
    h, l = dso.ds_reduce_f64_seq(x, init=(0.5, 0.0))
    seq_err = abs(float(h) + float(l) - truth)
    assert abs(results[0][1] - truth) <= seq_err


def test_shard_range_covers():
    from ds_b200.dist import shard_range
    for n in (0, 1, 7, 4096, 100_003):
        for world in (1, 2, 3, 8):
            parts = [shard_range(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 3, 3)


class _FakeExchangeBackend:
    """Stands in for the CUDA IPC calls: 'addresses' are integers, a handle
    names its owner, and every call is logged.  `fail_open` makes opening
    that rank's handle raise, as a failing cudaIpcOpenMemHandle would."""

    def __init__(self, rank, fail_open=None, error_word=0):
        self.rank, self.fail_open, self.error_word = rank, fail_open, error_word
        self.log = []

    def alloc(self):
        self.log.append(("alloc",))
        return 1000 + self.rank, f"h{self.rank}".encode()

    def open(self, handle):
        owner = int(handle.decode()[1:])
        if owner == self.fail_open:
            raise RuntimeError("open failed")
        self.log.append(("open", owner))
        return 2000 + owner

    def close(self, ptr):
        self.log.append(("close", ptr))

    def free(self, ptr):
        self.log.append(("free", ptr))

    def error(self, ptr):
        return self.error_word


def _exchange_worker(rank, world, port, q):
    import sys
    for p in (ROOT, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from ds_b200 import dist as dsd
        fake = _FakeExchangeBackend(rank)
        ex = dsd.PeerExchange(backend=fake, timeout_ms=250)
        epochs = [ex.next_epoch() for _ in range(3)]
        ptrs = list(ex.ptrs)
        ex.close()
        ex.close()  # idempotent
        try:
            ex.next_epoch()
            after_close = "no error"
        except RuntimeError:
            after_close = "raised"
        # an open that fails frees what was set up and raises
        bad = _FakeExchangeBackend(rank, fail_open=(rank + 1) % world)
        try:
            dsd.PeerExchange(backend=bad)
            failed = "no error"
        except RuntimeError:
            failed = "raised"
        # a timed-out wait recorded in the error word surfaces in check()
        ex2 = dsd.PeerExchange(backend=_FakeExchangeBackend(rank, error_word=1))
        try:
            ex2.check()
            checked = "no error"
        except RuntimeError as e:
            checked = str(e)
        ex2.close()
        q.put((rank, epochs, ptrs, fake.log, after_close, failed, bad.log, checked))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, None, repr(e), None, None, None, None, None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_peer_exchange_host_logic(world):
    """Handles gathered in rank order, the own buffer in its own slot, every
    peer mapped once and unmapped before the free; epochs count 1, 2, 3."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=120) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] is not None for r in results), results
    for rank, epochs, ptrs, log, after_close, failed, bad_log, checked in results:
        assert epochs == [1, 2, 3]
        assert ptrs == [1000 + r if r == rank else 2000 + r for r in range(world)]
        peers = [r for r in range(world) if r != rank]
        assert log == [("alloc",)] + [("open", r) for r in peers] + \
            [("close", 2000 + r) for r in peers] + [("free", 1000 + rank)]
        assert after_close == "raised"
        assert failed == "raised"
        assert bad_log[-1] == ("free", 1000 + rank)  # own buffer released on failure
        assert "timed out" in checked


def _gemm_worker(rank, world, port, q):
    import sys
    for p in (ROOT, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from ds_b200 import dist as dsd
        from oracle import ds_pass_ref
        M, K, N = 101, 64, 48  # 101 rows: the shards differ in length
        rng = np.random.default_rng(8)
        A = rng.integers(-64, 64, (M, K)).astype(np.float64)
        B = torch.from_numpy(rng.integers(-64, 64, (K, N)).astype(np.float64)) if rank == 0 \
            else torch.zeros((K, N), dtype=torch.float64)
        dsd.replicate(B, src=0)
        r0, r1 = dsd.shard_range(M, rank, world)
        # the per-rank product stood in for by the oracle's restatement of the
        # reference pass (exact here: small integers)
        C_local = torch.from_numpy(ds_pass_ref.dot_general_f64(A[r0:r1], B.numpy()))
        C = dsd.gather_rows(C_local)
        q.put((rank, C.numpy(), (r0, r1), B.numpy()))
    except Exception as e:
        q.put((rank, None, repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_row_sharded_gemm_gloo(world):
    """The GEMM's multi-GPU partitioning with CPU ranks: rows of A split by
    shard_range, B replicated from rank 0, every rank's block reassembled by
    gather_rows in rank order, equal on every rank to the single-process
    product."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gemm_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=120) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] is not None for r in results), results
    assert all(p.exitcode == 0 for p in procs)
    from oracle import ds_pass_ref
    rng = np.random.default_rng(8)
    A = rng.integers(-64, 64, (101, 64)).astype(np.float64)
    B = rng.integers(-64, 64, (64, 48)).astype(np.float64)
    want = ds_pass_ref.dot_general_f64(A, B)
    assert np.array_equal(want, A @ B)
    for _, C, _, Bg in results:
        assert np.array_equal(Bg, B)
        assert np.array_equal(C, want)
    spans = [r[2] for r in results]
    assert spans[0][0] == 0 and spans[-1][1] == 101
    assert len({s[1] - s[0] for s in spans}) == 2  # ragged shards exercised
