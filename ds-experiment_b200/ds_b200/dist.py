"""The DS ops sharded over one process per GPU (torch.distributed, NCCL).

The reference has no multi-GPU code; this is the partitioning the ops allow:
- elementwise chains, split/recombine and the recurrences: contiguous ranges
  of the element index per rank, no collective (shard_range / shard);
- reduce: every rank reduces its range to a DS pair on its own GPU; the pairs
  are all-gathered as (hi, lo) f32 (8 bytes per rank) and folded in rank
  order on every rank with the DS reduce kernel, so all ranks hold the same
  bits.  A plain sum all-reduce would drop the lo word;
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


def ds_sum_f64_sharded(x_local: torch.Tensor, init: float = 0.0, group=None,
                       local_pair: Optional[Callable] = None,
                       combine: Optional[Callable] = None) -> torch.Tensor:
    """DS sum of the concatenation of every rank's x_local, in rank order.

    Returns the f64 result (0-d) on every rank, bit-identical across ranks.
    Per call: the local reduce, one all-gather of 8 bytes per rank, one
    packed reduce of the [world, 2] pairs and one recombine.
    """
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
    """Concatenate every rank's row block (equal row counts) on every rank."""
    world, _ = _world(group)
    out = torch.empty((world * C_local.shape[0],) + tuple(C_local.shape[1:]),
                      dtype=C_local.dtype, device=C_local.device)
    dist.all_gather_into_tensor(out, C_local.contiguous(), group=group)
    return out
