"""Python functions over the custom-call targets, one per reference op.

They mirror the helper functions of the reference's FFI tests
(python/test_ds_add.py:35-48: ``ds_from_f64(x)``, ``ds_add(a, b)``,
``ds_to_f64(x)``; python/test_ds_recurrence_add_mul_to_f64_cuda.py:24-31),
and add the DS pass's reduce and dot_general (DsTransformPass.cpp:337-448)
as ``ds_reduce*`` and ``ds_dot_general*``.  All take and return torch CUDA
tensors and run on torch's current stream.
"""
from __future__ import annotations

from typing import Iterable, Optional, Sequence

import torch

from . import _lib
from .ffi import ShapeDtypeStruct, ffi_call

F64, F32 = torch.float64, torch.float32

_BODIES = {"add": _lib.DS_BODY_ADD, "sub": _lib.DS_BODY_SUB, "subtract": _lib.DS_BODY_SUB,
           "mul": _lib.DS_BODY_MUL, "multiply": _lib.DS_BODY_MUL}
_ALGOS = {"tensor": _lib.DS_DOT_TENSOR_INT8, "int8": _lib.DS_DOT_TENSOR_INT8,
          "cuda_core": _lib.DS_DOT_CUDA_CORE, "simt": _lib.DS_DOT_CUDA_CORE}


def _sds(shape, dtype):
    return ShapeDtypeStruct(tuple(shape), dtype)


# ---- split / recombine ------------------------------------------------------

def ds_from_f64(x: torch.Tensor) -> torch.Tensor:
    return ffi_call("ds_from_f64", _sds(tuple(x.shape) + (2,), F32))(x)


def ds_to_f64(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    return ffi_call("ds_to_f64", _sds(tuple(x.shape[:-1]), F64))(x, out=out)


def ds_from_f32(x: torch.Tensor) -> torch.Tensor:
    return ffi_call("ds_from_f32", _sds(tuple(x.shape) + (2,), F32))(x)


def ds_to_f32(x: torch.Tensor) -> torch.Tensor:
    return ffi_call("ds_to_f32", _sds(tuple(x.shape[:-1]), F32))(x)


# ---- packed elementwise -------------------------------------------------------

def ds_add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return ffi_call("ds_add", _sds(a.shape, F32))(a, b)


def ds_sub(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return ffi_call("ds_sub", _sds(a.shape, F32))(a, b)


def ds_mul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return ffi_call("ds_mul", _sds(a.shape, F32))(a, b)


# ---- fused f64 chains -----------------------------------------------------------

def ds_fused_add_mul(x, y):
    """(x + y) * y -> packed DS [N, 2]."""
    return ffi_call("ds_fused_add_mul", _sds(tuple(x.shape) + (2,), F32))(x, y)


def ds_fused_add_mul_to_f64(x, y):
    """(x + y) * y -> f64 [N]."""
    return ffi_call("ds_fused_add_mul_to_f64", _sds(x.shape, F64))(x, y)


def ds_fused_axpy(x, y):
    """(x + y) * y -> f64 (the reference op of this name computes this chain)."""
    return ffi_call("ds_fused_axpy", _sds(x.shape, F64))(x, y)


def ds_fused_add_mul_to_f64_cuda(x, y):
    return ffi_call("ds_fused_add_mul_to_f64_cuda", _sds(x.shape, F64))(x, y)


def ds_fused_add_sub_to_f64_cuda(x, y):
    """(x + y) - x -> f64."""
    return ffi_call("ds_fused_add_sub_to_f64_cuda", _sds(x.shape, F64))(x, y)


def ds_recurrence_add_mul_to_f64_cuda(x, y, k: int):
    """z = x; k times z = (z + y) * y."""
    return ffi_call("ds_recurrence_add_mul_to_f64_cuda", _sds(x.shape, F64))(x, y, k=int(k))


def ds_fused_add_mul3_to_f64(a, b, c):
    """(a + b) * c -> f64."""
    return ffi_call("ds_fused_add_mul3_to_f64", _sds(a.shape, F64))(a, b, c)


def ds_recurrence_mul_add_to_f64(x, a, b, k: int):
    """x <- x * a + b, k times."""
    return ffi_call("ds_recurrence_mul_add_to_f64", _sds(x.shape, F64))(x, a, b, k=int(k))


# ---- reduce ---------------------------------------------------------------------

def _reduce_dims(rank: int, dimensions: Optional[Iterable[int]]):
    if dimensions is None:
        return tuple(range(rank))
    dims = sorted(int(d) % rank if rank else int(d) for d in dimensions)
    return tuple(dims)


def _out_shape(shape, dims):
    return tuple(s for i, s in enumerate(shape) if i not in dims)


_SCALARS: dict = {}


def _scalar(value: float, dtype, device) -> torch.Tensor:
    """A 0-d device tensor holding `value`, cached per (device, stream, dtype,
    value) so that repeated calls launch no fill kernel; the cache key holds
    the stream because the fill is ordered only on the stream that made it."""
    if torch.cuda.is_current_stream_capturing():
        # made inside a CUDA graph capture: its fill runs at replay, so it is
        # not kept for eager calls
        return torch.full((), float(value), dtype=dtype, device=device)
    stream = _lib.current_stream_ptr(device)
    key = (device.index, stream, dtype, float(value).hex())  # hex keeps -0.0 apart
    t = _SCALARS.get(key)
    if t is None:
        if len(_SCALARS) > 256:
            _SCALARS.clear()
        t = _SCALARS[key] = torch.full((), float(value), dtype=dtype, device=device)
    return t


def ds_reduce(hi: torch.Tensor, lo: torch.Tensor, init=(0.0, 0.0),
              dimensions: Optional[Sequence[int]] = None, body: str = "add", out=None):
    """DS reduce of SoA (hi, lo) over `dimensions` (default: all) -> (hi, lo)."""
    dims = _reduce_dims(hi.dim(), dimensions)
    ih = _scalar(init[0], F32, hi.device)
    il = _scalar(init[1], F32, hi.device)
    res = _sds(_out_shape(hi.shape, dims), F32)
    return ffi_call("ds_reduce", (res, res))(hi, lo, ih, il, dimensions=dims,
                                             body=_BODIES[body], out=out)


def ds_reduce_packed(x: torch.Tensor, init=(0.0, 0.0),
                     dimensions: Optional[Sequence[int]] = None, body: str = "add", out=None):
    """DS reduce of a packed DS tensor x[..., 2] over `dimensions` of its
    logical shape x.shape[:-1] (default: all) -> (hi, lo)."""
    dims = _reduce_dims(x.dim() - 1, dimensions)
    ih = _scalar(init[0], F32, x.device)
    il = _scalar(init[1], F32, x.device)
    res = _sds(_out_shape(x.shape[:-1], dims), F32)
    return ffi_call("ds_reduce_packed", (res, res))(x, ih, il, dimensions=dims,
                                                    body=_BODIES[body], out=out)


def ds_reduce_f64(x: torch.Tensor, init: float = 0.0,
                  dimensions: Optional[Sequence[int]] = None, body: str = "add", out=None):
    """DS reduce of an f64 tensor -> f64.  The combining step is the DS
    body; with add/sub each thread first accumulates its elements with an
    exact f64 two_sum before the DS tree."""
    dims = _reduce_dims(x.dim(), dimensions)
    it = _scalar(init, F64, x.device)
    return ffi_call("ds_reduce_f64", _sds(_out_shape(x.shape, dims), F64))(
        x, it, dimensions=dims, body=_BODIES[body], out=out)


def ds_reduce_from_f64(x: torch.Tensor, init: float = 0.0,
                       dimensions: Optional[Sequence[int]] = None, body: str = "add", out=None):
    """DS reduce of an f64 tensor with the result kept as a DS pair (hi, lo)."""
    dims = _reduce_dims(x.dim(), dimensions)
    it = _scalar(init, F64, x.device)
    res = _sds(_out_shape(x.shape, dims), F32)
    return ffi_call("ds_reduce_from_f64", (res, res))(x, it, dimensions=dims,
                                                      body=_BODIES[body], out=out)


def ds_reduce_f64_multi(xs, inits=None, dimensions: Optional[Sequence[int]] = None,
                        bodies=None):
    """A variadic reduce: every f64 tensor in `xs` (one shape) reduced over
    `dimensions` with its own body ("add", "sub", "mul") and init -> list."""
    import ctypes
    xs = [x.contiguous() for x in xs]
    n = len(xs)
    inits = [0.0] * n if inits is None else list(inits)
    bodies = ["add"] * n if bodies is None else list(bodies)
    if len(inits) != n or len(bodies) != n:
        raise ValueError("one init and one body per input")
    dims = _reduce_dims(xs[0].dim(), dimensions)
    shape = _out_shape(xs[0].shape, dims)
    dev = xs[0].device
    outs = [torch.empty(shape, dtype=F64, device=dev) for _ in range(n)]
    its = [_scalar(v, F64, dev) for v in inits]
    keep = []

    def bufs(ts):
        arr = (ctypes.POINTER(_lib.DsBuffer) * n)()
        for k, t in enumerate(ts):
            b, d = _lib.make_buffer(t.data_ptr(), tuple(t.shape))
            keep.append((b, d))
            arr[k] = ctypes.pointer(b)
        return arr
    L = _lib.lib()
    cdims = (ctypes.c_int64 * max(len(dims), 1))(*dims)
    ib = bufs(xs)
    ws_bytes = int(L.ds_reduce_workspace_size(ib[0], cdims, len(dims)))
    ws = torch.empty(max(ws_bytes, 8), dtype=torch.uint8, device=dev)
    body_codes = (ctypes.c_int32 * n)(*[_BODIES[b] for b in bodies])
    stream = ctypes.c_void_p(_lib.current_stream_ptr(dev))
    _lib.check(L.ds_reduce_f64_multi(ib, bufs(its), body_codes, n, cdims, len(dims), bufs(outs),
                                     ctypes.c_void_p(ws.data_ptr()), ws_bytes, stream),
               "ds_reduce_f64_multi")
    return outs


def ds_sum_f64(x: torch.Tensor, dimensions=None) -> torch.Tensor:
    return ds_reduce_f64(x, 0.0, dimensions, "add")


# ---- dot_general -------------------------------------------------------------------

def _dims(x, default):
    if x is None:
        return default
    return (int(x),) if isinstance(x, int) else tuple(int(v) for v in x)


def _dot_out_shape(ls, rs, lb, rb, lc, rc):
    """stablehlo.dot_general's result: batch (lhs order), lhs free, rhs free."""
    out = [ls[i] for i in lb]
    out += [d for i, d in enumerate(ls) if i not in lb and i not in lc]
    out += [d for i, d in enumerate(rs) if i not in rb and i not in rc]
    return tuple(out)


def ds_dot_general(lhs_hi, lhs_lo, rhs_hi, rhs_lo, lhs_contracting=None, rhs_contracting=None,
                   lhs_batch=(), rhs_batch=(), algorithm: str = "tensor"):
    """DS dot_general on SoA operands -> (hi, lo), with stablehlo dimension
    numbers: contracting dimensions an int or a sequence (paired in order),
    batching dimensions anywhere.  Defaults: A[..., M, K] @ B[..., K, N]."""
    lb, rb = tuple(lhs_batch), tuple(rhs_batch)
    lc = _dims(lhs_contracting, (lhs_hi.dim() - 1,))
    rc = _dims(rhs_contracting, (len(rb),))
    out = _sds(_dot_out_shape(lhs_hi.shape, rhs_hi.shape, lb, rb, lc, rc), F32)
    return ffi_call("ds_dot_general", (out, out))(
        lhs_hi, lhs_lo, rhs_hi, rhs_lo, lhs_batching_dimensions=lb,
        rhs_batching_dimensions=rb, lhs_contracting_dimensions=lc,
        rhs_contracting_dimensions=rc, algorithm=_ALGOS[algorithm])


def ds_dot_general_f64(lhs, rhs, lhs_contracting=None, rhs_contracting=None, lhs_batch=(),
                       rhs_batch=(), algorithm: str = "tensor"):
    """DS dot_general of f64 operands (split and recombine fused) -> f64,
    with the dimension numbers of ds_dot_general."""
    lb, rb = tuple(lhs_batch), tuple(rhs_batch)
    lc = _dims(lhs_contracting, (lhs.dim() - 1,))
    rc = _dims(rhs_contracting, (len(rb),))
    out = _sds(_dot_out_shape(lhs.shape, rhs.shape, lb, rb, lc, rc), F64)
    return ffi_call("ds_dot_general_f64", out)(
        lhs, rhs, lhs_batching_dimensions=lb,
        rhs_batching_dimensions=rb, lhs_contracting_dimensions=lc,
        rhs_contracting_dimensions=rc, algorithm=_ALGOS[algorithm])


def ds_matmul_f64(A, B, algorithm: str = "tensor"):
    """A[M, K] @ B[K, N] in DS arithmetic, f64 in and out."""
    return ds_dot_general_f64(A, B, algorithm=algorithm)
