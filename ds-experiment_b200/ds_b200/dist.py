"""The DS ops sharded over one process per GPU (torch.distributed, NCCL).

The reference has no multi-GPU code; this is the partitioning the ops allow:
- elementwise chains, split/recombine and the recurrences: contiguous ranges
  of the element index per rank, no collective (shard_range / shard);
- reduce: every rank reduces its range to a DS pair on its own GPU and the
  pairs are folded in rank order on every rank, so all ranks hold the same
  bits (a plain sum all-reduce would drop the lo word).  Within one node the
  exchange runs inside the reduce itself (PeerExchange: the final block
  stores its pair into every peer's exchange buffer over NVLink and folds
  what arrives in its own); otherwise the pairs are all-gathered as (hi, lo)
  f32, 8 bytes per rank, and folded by one packed DS reduce launch;
- dot_general: rows of A per rank with B replicated once into every GPU's
  own memory (replicate); no collective inside the product.  Batched dots
  shard the batch dimension.

The local-reduce and combine steps are parameters so that the host logic can
be exercised with CPU ranks (gloo); the defaults are the CUDA ops.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist


def shard_range(n: int, rank: int, world: int) -> Tuple[int, int]:
    """[start, stop) of rank's contiguous share of n items (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("invalid rank/world")
    base, rem = divmod(int(n), int(world))
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def shard(x: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    start, stop = shard_range(x.shape[dim], rank, world)
    return x.narrow(dim, start, stop - start)


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def _split_init(init: float) -> Tuple[float, float]:
    hi = float(np.float32(init))
    lo = float(np.float32(init - hi))
    return hi, lo


def _local_pair_cuda(x_local: torch.Tensor) -> torch.Tensor:
    """This rank's DS partial as f32 [hi, lo], written straight into the
    send buffer of the all-gather."""
    from . import ops
    pair = torch.empty(2, dtype=torch.float32, device=x_local.device)
    ops.ds_reduce_from_f64(x_local, out=(pair[0], pair[1]))
    return pair


def _combine_cuda(pairs: torch.Tensor, init: Tuple[float, float]) -> torch.Tensor:
    """Fold the gathered [world, 2] pairs in rank order (one packed DS
    reduce launch), then recombine to f64."""
    from . import ops
    res = torch.empty(2, dtype=torch.float32, device=pairs.device)
    ops.ds_reduce_packed(pairs, init=init, out=(res[0], res[1]))
    return ops.ds_to_f64(res)


class _CudaExchangeBackend:
    """The exchange-buffer calls of libds_b200 (CUDA IPC)."""

    def __init__(self):
        from . import _lib
        self._lib = _lib
        self.L = _lib.lib()
        self.handle_bytes = int(self.L.ds_exchange_handle_bytes())

    def alloc(self):
        import ctypes
        buf = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(self.handle_bytes)
        self._lib.check(self.L.ds_exchange_alloc(ctypes.byref(buf), handle), "exchange alloc")
        return int(buf.value), handle.raw

    def open(self, handle: bytes) -> int:
        import ctypes
        buf = ctypes.c_void_p()
        self._lib.check(self.L.ds_exchange_open(handle, ctypes.byref(buf)), "exchange open")
        return int(buf.value)

    def close(self, ptr: int) -> None:
        self._lib.check(self.L.ds_exchange_close(ptr), "exchange close")

    def free(self, ptr: int) -> None:
        self._lib.check(self.L.ds_exchange_free(ptr), "exchange free")

    def error(self, ptr: int) -> int:
        import ctypes
        code = ctypes.c_uint32()
        self._lib.check(self.L.ds_exchange_error(ptr, ctypes.byref(code)), "exchange error")
        return int(code.value)


class PeerExchange:
    """Exchange buffers of one node's ranks, each mapped into every rank.

    Construction is collective: every rank allocates its buffer, the CUDA
    IPC handles are all-gathered through the process group, every rank maps
    the others' buffers, and a barrier ends it.  Every use (`next_epoch`)
    must happen on all ranks in the same order, like a collective, and on
    one stream per rank (the calls share a cached workspace).
    `close()` is collective too.  At most 8 ranks.
    """

    MAX_RANKS = 8

    def __init__(self, group=None, timeout_ms: int = 1000, backend=None):
        self.group = group
        self.world, self.rank = _world(group)
        if self.world > self.MAX_RANKS:
            raise ValueError(f"PeerExchange supports at most {self.MAX_RANKS} ranks")
        if timeout_ms <= 0:
            raise ValueError("timeout_ms must be positive")
        self.timeout_ms = int(timeout_ms)
        self.backend = backend or _CudaExchangeBackend()
        self.own, handle = self.backend.alloc()
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs = []
        self._opened = []
        try:
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.ptrs.append(self.own)
                else:
                    p = self.backend.open(h)
                    self._opened.append(p)
                    self.ptrs.append(p)
        except Exception:
            for p in self._opened:
                self.backend.close(p)
            self.backend.free(self.own)
            raise
        self.epoch = 0
        self.closed = False
        self._call_state = None
        dist.barrier(group=group)

    def next_epoch(self) -> int:
        if self.closed:
            raise RuntimeError("PeerExchange is closed")
        self.epoch += 1
        return self.epoch

    def error(self) -> int:
        """The own buffer's sticky error word (waits for the device)."""
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        return self.backend.error(self.own)

    def check(self) -> None:
        code = self.error()
        if code:
            raise RuntimeError(f"PeerExchange rank {self.rank}: a wait for another rank "
                               f"timed out (error word {code}); rebuild the exchange")

    def close(self) -> None:
        """Unmap the peers' buffers and free the own one, after every rank
        has finished using them (two barriers)."""
        if self.closed:
            return
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._opened:
            self.backend.close(p)
        dist.barrier(group=self.group)
        self.backend.free(self.own)
        self.closed = True


def _sum_exchange_cuda(x_local: torch.Tensor, init: float, exchange: PeerExchange,
                       body: int) -> torch.Tensor:
    import ctypes
    from . import _lib, ops
    if x_local.dtype != torch.float64 or not x_local.is_cuda:
        raise ValueError("the peer-exchange sum takes float64 CUDA tensors")
    x = x_local.contiguous()
    L = _lib.lib()
    # per-call host work is kept small: every rank's step waits for the
    # slowest rank, so host time per call adds to the step
    st = exchange._call_state
    if st is None or st["shape"] != tuple(x.shape) or st["device"] != x.device:
        ib, idims = _lib.make_buffer(0, tuple(x.shape))
        ws_bytes = int(L.ds_reduce_f64_sharded_workspace_size(ctypes.byref(ib)))
        st = exchange._call_state = {
            "shape": tuple(x.shape), "device": x.device, "ib": ib, "idims": idims,
            "ws": torch.empty(max(ws_bytes, 8), dtype=torch.uint8, device=x.device),
            "ws_bytes": ws_bytes,
            "ptrs": (ctypes.c_void_p * exchange.world)(*exchange.ptrs),
            "out_dims": (ctypes.c_int64 * 1)(0)}
        st["wsp"] = ctypes.c_void_p(st["ws"].data_ptr())
    ib = st["ib"]
    ib.data = x.data_ptr()
    it = ops._scalar(init, torch.float64, x.device)
    out = torch.empty((), dtype=torch.float64, device=x.device)
    tb = _lib.DsBuffer(it.data_ptr(), st["out_dims"], 0)
    ob = _lib.DsBuffer(out.data_ptr(), st["out_dims"], 0)
    stream = ctypes.c_void_p(_lib.current_stream_ptr(x.device))
    _lib.check(L.ds_reduce_f64_sharded(
        ctypes.byref(ib), ctypes.byref(tb), body, ctypes.byref(ob), st["ptrs"], exchange.world,
        exchange.rank, exchange.next_epoch(), exchange.timeout_ms, st["wsp"], st["ws_bytes"],
        stream), "ds_reduce_f64_sharded")
    return out


def ds_sum_f64_sharded(x_local: torch.Tensor, init: float = 0.0, group=None,
                       local_pair: Optional[Callable] = None,
                       combine: Optional[Callable] = None,
                       exchange: Optional[PeerExchange] = None) -> torch.Tensor:
    """DS sum of the concatenation of every rank's x_local, in rank order.

    Returns the f64 result (0-d) on every rank, bit-identical across ranks.
    With `exchange` (one node): two kernels, the local block partials and
    one block that folds them, trades the totals over peer memory and folds
    those.  Without: the local reduce, one all-gather of 8 bytes per rank,
    one packed reduce of the [world, 2] pairs and one recombine.
    """
    if exchange is not None:
        return _sum_exchange_cuda(x_local, init, exchange, 0)
    world, _ = _world(group)
    local_pair = local_pair or _local_pair_cuda
    combine = combine or _combine_cuda
    pair = local_pair(x_local).to(torch.float32).reshape(2)
    gathered = torch.empty(world * 2, dtype=torch.float32, device=pair.device)
    dist.all_gather_into_tensor(gathered, pair, group=group)
    return combine(gathered.view(world, 2), _split_init(init))


def replicate(t: torch.Tensor, src: int = 0, group=None) -> torch.Tensor:
    """Place src's tensor in every rank's own memory (one broadcast)."""
    dist.broadcast(t, src=src, group=group)
    return t


def ds_matmul_f64_row_sharded(A_local: torch.Tensor, B: torch.Tensor,
                              algorithm: str = "tensor") -> torch.Tensor:
    """This rank's rows of A @ B (B replicated on every rank beforehand)."""
    from . import ops
    return ops.ds_matmul_f64(A_local, B, algorithm=algorithm)


def gather_rows(C_local: torch.Tensor, group=None) -> torch.Tensor:
    """Concatenate every rank's row block, in rank order, on every rank.  The
    blocks may differ in length (shard_range gives the first n mod world
    ranks one row more): each is padded to the longest for one all-gather,
    and the padding is dropped."""
    world, _ = _world(group)
    rows = torch.tensor([C_local.shape[0]], dtype=torch.int64, device=C_local.device)
    counts = torch.empty(world, dtype=torch.int64, device=C_local.device)
    dist.all_gather_into_tensor(counts, rows, group=group)
    counts = [int(c) for c in counts.tolist()]
    most = max(counts)
    tail = tuple(C_local.shape[1:])
    block = C_local.contiguous()
    if C_local.shape[0] < most:
        block = torch.cat([block, torch.zeros((most - C_local.shape[0],) + tail,
                                              dtype=C_local.dtype, device=C_local.device)])
    out = torch.empty((world * most,) + tail, dtype=C_local.dtype, device=C_local.device)
    dist.all_gather_into_tensor(out, block, group=group)
    if all(c == most for c in counts):
        return out
    return torch.cat([out[r * most:r * most + c] for r, c in enumerate(counts)])
