"""Fused elementwise DS programs: one kernel per elementwise DAG.

The reference's DS pass turns every f64 add, subtract and multiply of a
function into a chain of f32 StableHLO operations (DsTransformPass.cpp:
282-321), with constants and arguments split by emitFromFloat (:169-187,
:244-257) and broadcast_in_dim applied to hi and lo alike (:259-279); XLA
then fuses what it can, and the reference documents the cliff where it does
not (README.md:53-68).  Here the same lowering is one generated kernel:

    from ds_b200 import fuse

    @fuse.jit
    def f(x, y, z):
        return (x + y) * z - 0.1 * x

    out = f(x, y, z)      # torch CUDA tensors; f64 result computed in DS

`fn` is traced once per argument signature (which arguments are tensors,
their element types and shapes; scalar arguments are baked in as constants)
into a list of operations, which the library turns into CUDA source, compiles
with NVRTC for sm_100a and caches (ds_fused_run in ds_b200.h).  Inputs
broadcast with numpy's rules.  f64 tensors are split on load, f32 tensors
enter as (v, 0), `Packed(t)` marks a packed DS tensor [..., 2].  The result
is f64 if any input is f64, else f32, unless `out_dtype` says otherwise
("f64", "f32" or "packed").
"""
from __future__ import annotations

import ctypes
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch

from . import _lib


class Packed:
    """A packed DS tensor [..., 2] (hi, lo) used as a fused-program input."""

    def __init__(self, t: torch.Tensor):
        if t.dtype != torch.float32 or t.dim() == 0 or t.shape[-1] != 2:
            raise ValueError("Packed expects a float32 tensor with last dim == 2")
        self.t = t


class _Program:
    def __init__(self):
        self.ops: List[Tuple[int, int, int, float]] = []

    def add(self, code, a=0, b=0, value=0.0) -> "Node":
        self.ops.append((code, int(a), int(b), float(value)))
        return Node(self, len(self.ops) - 1)

    def const(self, v: float) -> "Node":
        return self.add(_lib.DS_FUSED_CONST, value=v)


class Node:
    """A traced DS value: arithmetic on Nodes (and Python numbers) records
    operations of the program."""

    def __init__(self, prog: _Program, idx: int):
        self.prog, self.idx = prog, idx

    def _lift(self, other) -> "Node":
        if isinstance(other, Node):
            if other.prog is not self.prog:
                raise ValueError("values of different traces mixed")
            return other
        if isinstance(other, (int, float)):
            return self.prog.const(float(other))
        return NotImplemented

    def _bin(self, code, other, swap=False):
        o = self._lift(other)
        if o is NotImplemented:
            return NotImplemented
        a, b = (o, self) if swap else (self, o)
        return self.prog.add(code, a.idx, b.idx)

    def __add__(self, o):
        return self._bin(_lib.DS_FUSED_ADD, o)

    def __radd__(self, o):
        return self._bin(_lib.DS_FUSED_ADD, o, swap=True)

    def __sub__(self, o):
        return self._bin(_lib.DS_FUSED_SUB, o)

    def __rsub__(self, o):
        return self._bin(_lib.DS_FUSED_SUB, o, swap=True)

    def __mul__(self, o):
        return self._bin(_lib.DS_FUSED_MUL, o)

    def __rmul__(self, o):
        return self._bin(_lib.DS_FUSED_MUL, o, swap=True)

    def __neg__(self):
        return self.prog.add(_lib.DS_FUSED_NEG, self.idx)

    def __pos__(self):
        return self


_TYPES = {torch.float64: _lib.DS_FUSED_F64, torch.float32: _lib.DS_FUSED_F32}
_OUT = {"f64": _lib.DS_FUSED_F64, "f32": _lib.DS_FUSED_F32, "packed": _lib.DS_FUSED_PACKED}


def _broadcast(shapes):
    try:
        return tuple(torch.broadcast_shapes(*shapes))
    except RuntimeError as e:
        raise ValueError(f"fused inputs do not broadcast: {e}") from None


def _kind(a):
    if isinstance(a, Packed):
        return ("packed", tuple(a.t.shape))
    if isinstance(a, torch.Tensor):
        if a.dtype not in _TYPES:
            raise TypeError(f"fused inputs are float64 or float32 tensors, got {a.dtype}")
        return (str(a.dtype), tuple(a.shape))
    if isinstance(a, (int, float)):
        return ("scalar", float(a))
    raise TypeError(f"unsupported fused argument {type(a).__name__}")


class _Compiled:
    def __init__(self, ops, n_inputs):
        self.n_ops = len(ops)
        self.ops = (_lib.DsFusedOp * self.n_ops)(
            *[_lib.DsFusedOp(c, a, b, 0, v) for c, a, b, v in ops])
        self.n_inputs = n_inputs


def trace(fn: Callable, args: Sequence) -> Tuple[list, List[int]]:
    """Record fn's operations for these arguments: (ops, positions of the
    tensor arguments in input order)."""
    prog = _Program()
    traced, tensors = [], []
    for pos, a in enumerate(args):
        if isinstance(a, (int, float)) and not isinstance(a, bool):
            traced.append(float(a))
        else:
            traced.append(prog.add(_lib.DS_FUSED_INPUT, len(tensors)))
            tensors.append(pos)
    result = fn(*traced)
    if not isinstance(result, Node):
        if isinstance(result, (int, float)):
            result = prog.const(float(result))
        else:
            raise TypeError("a fused function must return an expression of its arguments")
    if result.idx != len(prog.ops) - 1:
        # make the result the last operation (a copy: 0 + r would round)
        prog.add(_lib.DS_FUSED_NEG, prog.add(_lib.DS_FUSED_NEG, result.idx).idx)
    return prog.ops, tensors


def _buffers(tensors):
    bufs, keep = [], []
    for t in tensors:
        b, d = _lib.make_buffer(t.data_ptr(), tuple(t.shape))
        bufs.append(b)
        keep.append((b, d))
    return bufs, keep


class jit:
    """Decorator: run `fn` as one fused DS kernel (see the module docstring)."""

    def __init__(self, fn: Callable, out_dtype: Optional[str] = None):
        self.fn = fn
        self.out_dtype = out_dtype
        self._cache: Dict[tuple, Tuple[_Compiled, List[int]]] = {}
        self.__doc__ = fn.__doc__

    def _prepare(self, args):
        key = tuple(_kind(a) for a in args)
        hit = self._cache.get(key)
        if hit is None:
            ops, positions = trace(self.fn, args)
            hit = (_Compiled(ops, len(positions)), positions)
            self._cache[key] = hit
        return hit

    def _io(self, args, positions, out=None):
        tensors, types, logical = [], [], []
        device = None
        for pos in positions:
            a = args[pos]
            if isinstance(a, Packed):
                t, ty, shape = a.t, _lib.DS_FUSED_PACKED, tuple(a.t.shape[:-1])
            else:
                t, ty, shape = a, _TYPES[a.dtype], tuple(a.shape)
            if not t.is_cuda:
                raise ValueError("fused inputs must be CUDA tensors (there is no CPU path)")
            if not t.is_contiguous():
                raise ValueError("fused inputs must be contiguous")
            device = device or t.device
            if t.device != device:
                raise ValueError("fused inputs must be on one device")
            tensors.append(t)
            types.append(ty)
            logical.append(shape)
        if device is None:
            raise ValueError("a fused call needs at least one tensor argument")
        shape = _broadcast(logical)
        out_type = _OUT[self.out_dtype] if self.out_dtype else (
            _lib.DS_FUSED_F64 if _lib.DS_FUSED_F64 in types else _lib.DS_FUSED_F32)
        if out is None:
            if out_type == _lib.DS_FUSED_PACKED:
                out = torch.empty(shape + (2,), dtype=torch.float32, device=device)
            else:
                out = torch.empty(shape, dtype=torch.float64 if out_type == _lib.DS_FUSED_F64
                                  else torch.float32, device=device)
        return tensors, types, out_type, out

    def __call__(self, *args, out: Optional[torch.Tensor] = None):
        comp, positions = self._prepare(args)
        tensors, types, out_type, out = self._io(args, positions, out)
        bufs, keep = _buffers(tensors)
        ob, od = _lib.make_buffer(out.data_ptr(), tuple(out.shape))
        arr = (ctypes.POINTER(_lib.DsBuffer) * max(len(bufs), 1))(
            *[ctypes.pointer(b) for b in bufs])
        ty = (ctypes.c_int32 * max(len(types), 1))(*types)
        dev = out.device
        if dev.index is not None and dev.index != torch.cuda.current_device():
            with torch.cuda.device(dev):
                st = self._run(comp, ty, arr, len(bufs), out_type, ob)
        else:
            st = self._run(comp, ty, arr, len(bufs), out_type, ob)
        _lib.check(st, "ds_fused_run")
        return out

    @staticmethod
    def _run(comp, ty, arr, n, out_type, ob):
        stream = ctypes.c_void_p(_lib.current_stream_ptr())
        return _lib.lib().ds_fused_run(comp.ops, comp.n_ops, ty, arr, n, out_type,
                                       ctypes.byref(ob), stream)

    def source(self, *args) -> str:
        """The CUDA source generated for these arguments (needs no GPU:
        the tensors may live on any device)."""
        comp, positions = self._prepare(args)
        types, bufs, keep = [], [], []
        logical = []
        for pos in positions:
            a = args[pos]
            t = a.t if isinstance(a, Packed) else a
            types.append(_lib.DS_FUSED_PACKED if isinstance(a, Packed) else _TYPES[a.dtype])
            logical.append(tuple(t.shape[:-1]) if isinstance(a, Packed) else tuple(t.shape))
            b, d = _lib.make_buffer(256, tuple(t.shape))  # aligned stand-in pointer
            bufs.append(b)
            keep.append(d)
        shape = _broadcast(logical)
        out_type = _OUT[self.out_dtype] if self.out_dtype else (
            _lib.DS_FUSED_F64 if _lib.DS_FUSED_F64 in types else _lib.DS_FUSED_F32)
        oshape = shape + ((2,) if out_type == _lib.DS_FUSED_PACKED else ())
        ob, od = _lib.make_buffer(256, oshape)
        arr = (ctypes.POINTER(_lib.DsBuffer) * max(len(bufs), 1))(
            *[ctypes.pointer(b) for b in bufs])
        ty = (ctypes.c_int32 * max(len(types), 1))(*types)
        n = ctypes.c_size_t()
        L = _lib.lib()
        _lib.check(L.ds_fused_source(comp.ops, comp.n_ops, ty, arr, len(bufs), out_type,
                                     ctypes.byref(ob), None, 0, ctypes.byref(n)), "source")
        buf = ctypes.create_string_buffer(n.value)
        _lib.check(L.ds_fused_source(comp.ops, comp.n_ops, ty, arr, len(bufs), out_type,
                                     ctypes.byref(ob), buf, n.value, ctypes.byref(n)), "source")
        self._last_check = lambda: _lib.check(L.ds_fused_compile_check(
            comp.ops, comp.n_ops, ty, arr, len(bufs), out_type, ctypes.byref(ob)), "compile")
        return buf.value.decode()

    def compile_check(self, *args) -> None:
        """Generate and compile (NVRTC) for these arguments without running:
        raises on a compilation error.  Needs no GPU."""
        self.source(*args)
        self._last_check()


_KIND = {"f64": _lib.DS_FUSED_F64, "f32": _lib.DS_FUSED_F32, "packed": _lib.DS_FUSED_PACKED}


class Prepared:
    """An operation list with its input kinds and result kind, converted to
    the C structures once and run many times: `prog` holds (code, a, b,
    value) tuples in SSA order (the last is the result), `kinds` the kind of
    each input ("f64", "f32" or "packed"), `out_kind` the result's."""

    def __init__(self, prog, kinds: Sequence[str], out_kind: str):
        if out_kind not in _KIND or any(k not in _KIND for k in kinds):
            raise ValueError("fused kinds are 'f64', 'f32' or 'packed'")
        self.ops = [tuple(o) for o in prog]
        self.kinds = tuple(kinds)
        self.out_kind = out_kind
        self._comp = _Compiled(self.ops, len(self.kinds))
        self._types = (ctypes.c_int32 * max(len(self.kinds), 1))(*[_KIND[k] for k in self.kinds])

    def __call__(self, tensors: Sequence[torch.Tensor], shape) -> torch.Tensor:
        """Run on `tensors` (one per input kind); the result has the logical
        `shape` (the inputs broadcast to it)."""
        if len(tensors) != len(self.kinds) or not tensors:
            raise ValueError(f"the program takes {len(self.kinds)} input tensors")
        tensors = [t.contiguous() for t in tensors]
        device = tensors[0].device
        for t in tensors:
            if not t.is_cuda or t.device != device:
                raise ValueError("fused inputs must be CUDA tensors on one device")
        shape = tuple(shape)
        if self.out_kind == "packed":
            out = torch.empty(shape + (2,), dtype=torch.float32, device=device)
        else:
            out = torch.empty(shape, dtype=torch.float64 if self.out_kind == "f64"
                              else torch.float32, device=device)
        bufs, keep = _buffers(tensors)
        ob, od = _lib.make_buffer(out.data_ptr(), tuple(out.shape))
        arr = (ctypes.POINTER(_lib.DsBuffer) * len(bufs))(*[ctypes.pointer(b) for b in bufs])
        if device.index is not None and device.index != torch.cuda.current_device():
            with torch.cuda.device(device):
                st = jit._run(self._comp, self._types, arr, len(bufs), _KIND[self.out_kind], ob)
        else:
            st = jit._run(self._comp, self._types, arr, len(bufs), _KIND[self.out_kind], ob)
        _lib.check(st, "ds_fused_run")
        return out


    def _reduce_args(self, tensors, shape, body):
        if body not in _BODY:
            raise ValueError("a fused reduction's body is 'add' or 'mul'")
        shape = tuple(int(d) for d in shape)
        dims = (ctypes.c_int64 * max(len(shape), 1))(*shape)
        bufs, keep = _buffers(tensors)
        arr = (ctypes.POINTER(_lib.DsBuffer) * max(len(bufs), 1))(
            *[ctypes.pointer(b) for b in bufs])
        return shape, dims, bufs, keep, arr

    def reduce(self, tensors: Sequence[torch.Tensor], shape, body: str = "add",
               init=(0.0, 0.0)) -> Tuple[torch.Tensor, torch.Tensor]:
        """The program over the logical `shape`, its results combined with
        `body` ("add" or "mul") and the init pair, in one pass over the
        inputs (ds_fused_reduce): (hi, lo) as 0-d f32 tensors."""
        from . import ops  # the init scalars' cache
        if len(tensors) != len(self.kinds) or not tensors:
            raise ValueError(f"the program takes {len(self.kinds)} input tensors")
        tensors = [t.contiguous() for t in tensors]
        device = tensors[0].device
        for t in tensors:
            if not t.is_cuda or t.device != device:
                raise ValueError("fused inputs must be CUDA tensors on one device")
        shape, dims, bufs, keep, arr = self._reduce_args(tensors, shape, body)
        L = _lib.lib()
        with torch.cuda.device(device):
            ws_bytes = int(L.ds_fused_reduce_workspace_size(dims, len(shape)))
            ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=device)
            ih = ops._scalar(init[0], torch.float32, device)
            il = ops._scalar(init[1], torch.float32, device)
            hi = torch.empty((), dtype=torch.float32, device=device)
            lo = torch.empty((), dtype=torch.float32, device=device)
            scal = [_lib.make_buffer(t.data_ptr(), ()) for t in (ih, il, hi, lo)]
            stream = ctypes.c_void_p(_lib.current_stream_ptr())
            st = L.ds_fused_reduce(self._comp.ops, self._comp.n_ops, self._types, arr, len(bufs),
                                   dims, len(shape), _BODY[body],
                                   *[ctypes.byref(b) for b, _ in scal],
                                   ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream)
        _lib.check(st, "ds_fused_reduce")
        return hi, lo

    def reduce_compile_check(self, shapes: Sequence[tuple], shape, body: str = "add") -> None:
        """Generate and compile the reduction kernel for inputs of these
        shapes (no GPU needed; raises on a compilation error)."""
        shape, dims, _, _, _ = self._reduce_args([], shape, body)
        bufs, keep = [], []
        for s in shapes:
            b, d = _lib.make_buffer(256, tuple(s))
            bufs.append(b)
            keep.append(d)
        arr = (ctypes.POINTER(_lib.DsBuffer) * max(len(bufs), 1))(
            *[ctypes.pointer(b) for b in bufs])
        _lib.check(_lib.lib().ds_fused_reduce_compile_check(
            self._comp.ops, self._comp.n_ops, self._types, arr, len(bufs), dims, len(shape),
            _BODY[body]), "compile")


    def reduce_rows(self, tensors: Sequence[torch.Tensor], shape, n_reduced: int,
                    body: str = "add", init=(0.0, 0.0)) -> Tuple[torch.Tensor, torch.Tensor]:
        """The program over the logical `shape`, reduced over its last
        `n_reduced` dimensions in the same kernel (ds_fused_reduce_rows):
        (hi, lo) f32 tensors of shape shape[:-n_reduced]."""
        from . import ops  # the init scalars' cache
        if len(tensors) != len(self.kinds) or not tensors:
            raise ValueError(f"the program takes {len(self.kinds)} input tensors")
        tensors = [t.contiguous() for t in tensors]
        device = tensors[0].device
        for t in tensors:
            if not t.is_cuda or t.device != device:
                raise ValueError("fused inputs must be CUDA tensors on one device")
        shape, dims, bufs, keep, arr = self._reduce_args(tensors, shape, body)
        out_shape = shape[:len(shape) - int(n_reduced)]
        with torch.cuda.device(device):
            ih = ops._scalar(init[0], torch.float32, device)
            il = ops._scalar(init[1], torch.float32, device)
            hi = torch.empty(out_shape, dtype=torch.float32, device=device)
            lo = torch.empty(out_shape, dtype=torch.float32, device=device)
            scal = [_lib.make_buffer(t.data_ptr(), tuple(t.shape)) for t in (ih, il, hi, lo)]
            stream = ctypes.c_void_p(_lib.current_stream_ptr(device))
            st = _lib.lib().ds_fused_reduce_rows(
                self._comp.ops, self._comp.n_ops, self._types, arr, len(bufs), dims, len(shape),
                int(n_reduced), _BODY[body], *[ctypes.byref(b) for b, _ in scal], stream)
        _lib.check(st, "ds_fused_reduce_rows")
        return hi, lo

    def reduce_rows_compile_check(self, shapes: Sequence[tuple], shape, n_reduced: int,
                                  body: str = "add") -> None:
        """Generate and compile the per-row kernel for inputs of these shapes
        (no GPU needed; raises on a compilation error)."""
        shape, dims, _, _, _ = self._reduce_args([], shape, body)
        bufs, keep = [], []
        for s in shapes:
            b, d = _lib.make_buffer(256, tuple(s))
            bufs.append(b)
            keep.append(d)
        arr = (ctypes.POINTER(_lib.DsBuffer) * max(len(bufs), 1))(
            *[ctypes.pointer(b) for b in bufs])
        _lib.check(_lib.lib().ds_fused_reduce_rows_compile_check(
            self._comp.ops, self._comp.n_ops, self._types, arr, len(bufs), dims, len(shape),
            int(n_reduced), _BODY[body]), "compile")


_BODY = {"add": _lib.DS_BODY_ADD, "mul": _lib.DS_BODY_MUL}


def run_program(prog, inputs, out_kind: str, shape) -> torch.Tensor:
    """Run an operation list directly: `prog` holds (code, a, b, value)
    tuples in SSA order, `inputs` (kind, tensor) pairs with kind "f64",
    "f32" or "packed"; the result has the logical `shape` and `out_kind`."""
    return Prepared(prog, [k for k, _ in inputs], out_kind)([t for _, t in inputs], shape)
