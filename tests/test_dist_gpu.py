"""Sharded DS ops on 2+ GPUs (one NCCL process per GPU); skipped on one GPU.

- reduce: every rank sums its range, the (hi, lo) partials are all-gathered
  and folded in rank order; all ranks must hold the same bits, close to the
  exact sum of the whole array.  The same through the peer-memory exchange
  (PeerExchange, NVLink P2P stores inside the reduce kernel; NVLS off), call
  after call, with no error word set.
- dot_general: rows of A per rank with B replicated by broadcast; each
  rank's block must equal the single-GPU product of those rows (the
  tensor-core product is exact up to its final rounding, so bit-equal).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG_DIR, ROOT

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    for p in (ROOT, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        from ds_b200 import dist as dsd
        n = 3_000_017
        x = np.where(np.arange(n) % 2 == 0, 1e8, -1e8) + \
            np.random.default_rng(1).uniform(0, 1, n) * 1e-3
        lo, hi = dsd.shard_range(n, rank, world)
        xl = torch.from_numpy(x[lo:hi]).to(dev)
        r = dsd.ds_sum_f64_sharded(xl, init=0.25)
        sums = [torch.zeros((), dtype=torch.float64, device=dev) for _ in range(world)]
        dist.all_gather(sums, r)
        ex = dsd.PeerExchange(timeout_ms=2000)
        peer_vals = [float(dsd.ds_sum_f64_sharded(xl, init=0.25, exchange=ex))
                     for _ in range(5)]
        ex.check()
        ex.close()
        # row-sharded GEMM with B broadcast from rank 0
        rng = np.random.default_rng(2)
        A = rng.uniform(-1, 1, (512, 768))
        B = torch.from_numpy(rng.uniform(-1, 1, (768, 384))).to(dev) if rank == 0 else \
            torch.empty((768, 384), dtype=torch.float64, device=dev)
        dsd.replicate(B, src=0)
        a0, a1 = dsd.shard_range(A.shape[0], rank, world)
        C_local = dsd.ds_matmul_f64_row_sharded(torch.from_numpy(A[a0:a1]).to(dev), B)
        torch.cuda.synchronize()
        q.put((rank, float(r), [float(s) for s in sums], C_local.cpu().numpy(), (a0, a1),
               peer_vals))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, None, repr(e), None, None, None))
        raise
    finally:
        dist.destroy_process_group()


def test_sharded_sum_and_gemm():
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=300) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
    errors = [r for r in results if r[1] is None]
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)
    # identical bits on every rank
    vals = {v for _, v, _, _, _, _ in results}
    assert len(vals) == 1
    for _, v, allv, _, _, _ in results:
        assert set(allv) == {v}
    peer = {pv for *_, pvs in results for pv in pvs}
    assert len(peer) == 1  # every rank, every call
    peer_val = peer.pop()
    import math
    n = 3_000_017
    x = np.where(np.arange(n) % 2 == 0, 1e8, -1e8) + np.random.default_rng(1).uniform(0, 1, n) * 1e-3
    truth = math.fsum(x.tolist()) + 0.25
    from oracle import dso
    h, l = dso.ds_reduce_f64_seq(x, init=(0.25, 0.0))
    seq_err = abs(float(h) + float(l) - truth)
    assert abs(results[0][1] - truth) <= seq_err
    assert abs(peer_val - truth) <= seq_err
    # the row blocks reassemble the single-GPU product
    from ds_b200 import ops
    rng = np.random.default_rng(2)
    A = rng.uniform(-1, 1, (512, 768))
    B = rng.uniform(-1, 1, (768, 384))
    full = ops.ds_matmul_f64(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()).cpu().numpy()
    for _, _, _, C_local, (a0, a1), _ in results:
        assert np.array_equal(C_local, full[a0:a1])
