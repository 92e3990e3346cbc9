"""Custom-call surface of libds_b200, shaped like the reference's jax.ffi use.

The reference registers its XLA-FFI handlers by target name and calls them
with ``ffi.ffi_call(name, ShapeDtypeStruct(...), vmap_method=...)(*args,
**attrs)`` (python/test_ds_add.py:16-48,
python/test_ds_recurrence_add_mul_to_f64_cuda.py:18-31).  This module keeps
that surface over torch CUDA tensors: ``register_ffi_target(name, lib.<sym>,
platform="CUDA")`` binds a target name to a libds_b200 entry point, and
``ffi_call`` allocates the results, passes torch's current CUDA stream and
raises on a non-OK status.  Every reference target name is registered at
import.  Scratch for ds_reduce / ds_dot_general comes from torch's caching
allocator (the role XLA's scratch allocator plays for an FFI handler); small
scratch is kept per stream and reused, and a reduce's scratch size is asked
once per shape.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, Tuple

import torch

from . import _lib


@dataclass(frozen=True)
class ShapeDtypeStruct:
    shape: Tuple[int, ...]
    dtype: torch.dtype

    def __init__(self, shape, dtype):
        object.__setattr__(self, "shape", tuple(int(d) for d in shape))
        object.__setattr__(self, "dtype", dtype)


F64, F32 = torch.float64, torch.float32


@dataclass(frozen=True)
class _Convention:
    """Operand dtypes, attribute names and result dtypes of one entry point,
    in the order of the reference handler's Bind() (Args, Attrs, Rets)."""
    args: Tuple[torch.dtype, ...]
    attrs: Tuple[str, ...]
    results: Tuple[torch.dtype, ...]
    kind: str = "plain"  # plain | reduce | reduce_f64 | dot | dot_f64


CONVENTIONS: Dict[str, _Convention] = {
    "ds_from_f64": _Convention((F64,), (), (F32,)),
    "ds_to_f64": _Convention((F32,), (), (F64,)),
    "ds_from_f32": _Convention((F32,), (), (F32,)),
    "ds_to_f32": _Convention((F32,), (), (F32,)),
    "ds_add": _Convention((F32, F32), (), (F32,)),
    "ds_sub": _Convention((F32, F32), (), (F32,)),
    "ds_mul": _Convention((F32, F32), (), (F32,)),
    "ds_fused_add_mul": _Convention((F64, F64), (), (F32,)),
    "ds_fused_add_mul_to_f64": _Convention((F64, F64), (), (F64,)),
    "ds_fused_axpy": _Convention((F64, F64), (), (F64,)),
    "ds_fused_add_mul_to_f64_cuda": _Convention((F64, F64), (), (F64,)),
    "ds_fused_add_sub_to_f64_cuda": _Convention((F64, F64), (), (F64,)),
    "ds_recurrence_add_mul_to_f64_cuda": _Convention((F64, F64), ("k",), (F64,)),
    "ds_fused_add_mul3_to_f64": _Convention((F64, F64, F64), (), (F64,)),
    "ds_recurrence_mul_add_to_f64": _Convention((F64, F64, F64), ("k",), (F64,)),
    "ds_reduce": _Convention((F32, F32, F32, F32), ("dimensions", "body"), (F32, F32),
                             "reduce"),
    "ds_reduce_f64": _Convention((F64, F64), ("dimensions", "body"), (F64,), "reduce_f64"),
    "ds_reduce_from_f64": _Convention((F64, F64), ("dimensions", "body"), (F32, F32),
                                      "reduce_from_f64"),
    "ds_reduce_packed": _Convention((F32, F32, F32), ("dimensions", "body"), (F32, F32),
                                    "reduce_packed"),
    "ds_dot_general": _Convention((F32, F32, F32, F32),
                                  ("lhs_batching_dimensions", "rhs_batching_dimensions",
                                   "lhs_contracting_dimensions",
                                   "rhs_contracting_dimensions", "algorithm"),
                                  (F32, F32), "dot"),
    "ds_dot_general_f64": _Convention((F64, F64),
                                      ("lhs_batching_dimensions", "rhs_batching_dimensions",
                                       "lhs_contracting_dimensions",
                                       "rhs_contracting_dimensions", "algorithm"),
                                      (F64,), "dot_f64"),
}

# The reference's target names, each bound to its replacement entry point.
REFERENCE_TARGETS = {
    "ds_from_f64": "ds_from_f64",
    "ds_to_f64": "ds_to_f64",
    "ds_from_f32": "ds_from_f32",
    "ds_to_f32": "ds_to_f32",
    "ds_add": "ds_add",
    "ds_sub": "ds_sub",
    "ds_mul": "ds_mul",
    "ds_fused_add_mul": "ds_fused_add_mul",
    "ds_fused_add_mul_to_f64": "ds_fused_add_mul_to_f64",
    "ds_fused_axpy": "ds_fused_axpy",
    "ds_fused_add_mul_to_f64_cuda": "ds_fused_add_mul_to_f64_cuda",
    "ds_fused_add_sub_to_f64_cuda": "ds_fused_add_sub_to_f64_cuda",
    "ds_recurrence_add_mul_to_f64_cuda": "ds_recurrence_add_mul_to_f64_cuda",
    "ds_fused_add_mul3_to_f64": "ds_fused_add_mul3_to_f64",
    "ds_recurrence_mul_add_to_f64": "ds_recurrence_mul_add_to_f64",
    "ds_reduce": "ds_reduce",
    "ds_reduce_f64": "ds_reduce_f64",
    "ds_reduce_from_f64": "ds_reduce_from_f64",
    "ds_reduce_packed": "ds_reduce_packed",
    "ds_dot_general": "ds_dot_general",
    "ds_dot_general_f64": "ds_dot_general_f64",
}

# target name -> libds_b200 symbol; every reference target is bound at import.
_registry: Dict[str, str] = dict(REFERENCE_TARGETS)


def register_ffi_target(name: str, target, platform: str = "CUDA") -> None:
    """Bind custom-call target `name` to a libds_b200 entry point.

    `target` is a ctypes function of libds_b200 (``lib.ds_add``) or its
    symbol name.  Only platform "CUDA" exists: there is no host fallback.
    """
    if platform.upper() not in ("CUDA", "GPU"):
        raise ValueError(f"platform {platform!r} is not provided; libds_b200 runs on CUDA only")
    sym = target if isinstance(target, str) else getattr(target, "__name__", None)
    if sym not in CONVENTIONS:
        raise ValueError(f"{sym!r} is not a libds_b200 entry point")
    _registry[name] = sym
    _calls.clear()


def registered_targets():
    return sorted(_registry)


def _stream_handle(device=None) -> ctypes.c_void_p:
    return ctypes.c_void_p(_lib.current_stream_ptr(device))


def _check_tensor(t, dtype, what):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{what}: expected a torch.Tensor, got {type(t).__name__}")
    if not t.is_cuda:
        raise ValueError(f"{what}: libds_b200 operates on CUDA tensors only")
    if t.dtype != dtype:
        raise TypeError(f"{what}: expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{what}: tensor must be contiguous (row-major)")


def _buf(t):
    return _lib.make_buffer(t.data_ptr(), t.shape)


# Workspaces up to _CACHED_WORKSPACE_MAX (reduce partials, the residue
# planes of products up to about 1100 x 1100) are kept per (device, stream)
# and reused: calls on one stream run in order, so one buffer serves them
# all, and a call skips an allocation.  The buffer starts at 1 MiB and grows
# to the next power of two a request needs; the one it replaces was
# allocated on the same stream, so torch's allocator hands its memory out
# again only to work ordered after the calls that used it.  Larger ones come
# from torch's allocator each time, so that they are not held.  None is kept
# while a CUDA graph is being captured (its replay may overlap eager calls).
_SMALL_WORKSPACE = 1 << 20
_CACHED_WORKSPACE_MAX = 64 << 20
_workspaces: Dict[tuple, torch.Tensor] = {}


def _workspace(nbytes: int, device, stream: int = 0) -> torch.Tensor:
    nbytes = max(int(nbytes), 1)
    if nbytes > _CACHED_WORKSPACE_MAX or torch.cuda.is_current_stream_capturing():
        return torch.empty(nbytes, dtype=torch.uint8, device=device)
    key = (device.index, stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        if ws is None and len(_workspaces) > 64:
            _workspaces.clear()
        size = max(_SMALL_WORKSPACE, 1 << (nbytes - 1).bit_length())
        ws = _workspaces[key] = torch.empty(size, dtype=torch.uint8, device=device)
    return ws


# ds_reduce_workspace_size by (device, shape, dimensions): a pure function
# of them, asked on every reduce call otherwise.  Likewise the dot_general's
# dimension-number struct and ds_dot_general_workspace_size, by (target,
# device, shapes, algorithm, dimension numbers).
_reduce_ws: Dict[tuple, int] = {}
_dot_setup: Dict[tuple, tuple] = {}
_dims_arrays: Dict[tuple, object] = {}


def _dims_array(dims: tuple):
    arr = _dims_arrays.get(dims)
    if arr is None:
        if len(_dims_arrays) > 256:
            _dims_arrays.clear()
        arr = _dims_arrays[dims] = (ctypes.c_int64 * max(len(dims), 1))(*dims)
    return arr


# (target, result specs) -> the callable ffi_call built for them
_calls: Dict[tuple, object] = {}
_MAX_CALLS = 512


def ffi_call(target_name: str, result_shape_dtypes, vmap_method=None):
    """Return a callable running target `target_name` on torch CUDA tensors.

    result_shape_dtypes: a ShapeDtypeStruct or a sequence of them, one per
    result.  Attributes are keyword arguments, as in jax.ffi.ffi_call.
    vmap_method is accepted for signature compatibility; the entry points
    already take arbitrary leading (batch) dimensions.  Callables are cached
    per target and result specs, so a call site that asks again each time
    pays a dictionary lookup.
    """
    key = (target_name, result_shape_dtypes if isinstance(result_shape_dtypes, ShapeDtypeStruct)
           else tuple(result_shape_dtypes))
    hit = _calls.get(key)
    if hit is not None:
        return hit
    call = _make_call(target_name, result_shape_dtypes)
    if len(_calls) >= _MAX_CALLS:
        _calls.clear()
    _calls[key] = call
    return call


def _make_call(target_name: str, result_shape_dtypes):
    if target_name not in _registry:
        raise KeyError(f"custom-call target {target_name!r} is not registered")
    sym = _registry[target_name]
    conv = CONVENTIONS[sym]
    fn = getattr(_lib.lib(), sym)
    single = isinstance(result_shape_dtypes, ShapeDtypeStruct)
    results_spec = [result_shape_dtypes] if single else list(result_shape_dtypes)
    if len(results_spec) != len(conv.results):
        raise ValueError(f"{target_name}: expected {len(conv.results)} result(s)")
    for spec, dt in zip(results_spec, conv.results):
        if spec.dtype != dt:
            raise TypeError(f"{target_name}: result dtype must be {dt}, got {spec.dtype}")

    def call(*args: torch.Tensor, out=None, **attrs):
        """Run the target.  `out`: optional pre-allocated result tensor(s)
        (contiguous, of the declared shapes and dtypes), as XLA hands a
        handler its result buffers; otherwise results are allocated."""
        if len(args) != len(conv.args):
            raise TypeError(f"{target_name}: expected {len(conv.args)} operand(s), got {len(args)}")
        for i, (t, dt) in enumerate(zip(args, conv.args)):
            _check_tensor(t, dt, f"{target_name} operand {i}")
        unknown = set(attrs) - set(conv.attrs)
        if unknown:
            raise TypeError(f"{target_name}: unknown attribute(s) {sorted(unknown)}")
        device = args[0].device
        if out is not None:
            out = [out] if isinstance(out, torch.Tensor) else list(out)
            if len(out) != len(results_spec):
                raise ValueError(f"{target_name}: expected {len(results_spec)} output tensor(s)")
            for i, (t, s) in enumerate(zip(out, results_spec)):
                _check_tensor(t, s.dtype, f"{target_name} result {i}")
                if tuple(t.shape) != s.shape:
                    raise ValueError(f"{target_name} result {i}: shape {tuple(t.shape)} != {s.shape}")
        if device.index is not None and device.index != torch.cuda.current_device():
            with torch.cuda.device(device):
                return _invoke(args, attrs, device, out)
        return _invoke(args, attrs, device, out)

    def _invoke(args, attrs, device, out):
        outs = out if out is not None else [
            torch.empty(s.shape, dtype=s.dtype, device=device) for s in results_spec]
        keep = []
        bufs = []
        for t in list(args) + outs:
            b, d = _buf(t)
            keep.append(d)
            bufs.append(b)
        refs = [ctypes.byref(b) for b in bufs]
        stream_ptr = _lib.current_stream_ptr(device)
        stream = ctypes.c_void_p(stream_ptr)
        if conv.kind == "plain":
            call_args = refs[:len(args)]
            for name in conv.attrs:
                if name not in attrs:
                    raise TypeError(f"{target_name}: missing attribute {name!r}")
                call_args.append(int(attrs[name]))
            call_args += refs[len(args):]
            status = fn(*call_args, stream)
        elif conv.kind in ("reduce", "reduce_f64", "reduce_from_f64", "reduce_packed"):
            dims = tuple(int(d) for d in attrs.get("dimensions", ()))
            body = int(attrs.get("body", _lib.DS_BODY_ADD))
            cdims = _dims_array(dims)
            shape = tuple(args[0].shape[:-1]) if conv.kind == "reduce_packed" else tuple(args[0].shape)
            wkey = (device.index, shape, dims)
            ws_bytes = _reduce_ws.get(wkey)
            if ws_bytes is None:
                if conv.kind == "reduce_packed":  # sized on the logical shape [..., 2] -> [...]
                    lb, ld = _lib.make_buffer(args[0].data_ptr(), shape)
                    keep.append(ld)
                    ws_bytes = _lib.lib().ds_reduce_workspace_size(ctypes.byref(lb), cdims,
                                                                   len(dims))
                else:
                    ws_bytes = _lib.lib().ds_reduce_workspace_size(refs[0], cdims, len(dims))
                if len(_reduce_ws) > 1024:
                    _reduce_ws.clear()
                _reduce_ws[wkey] = ws_bytes
            ws = _workspace(ws_bytes, device, stream_ptr)
            wsp = ctypes.c_void_p(ws.data_ptr())
            if conv.kind == "reduce":
                status = fn(refs[0], refs[1], refs[2], refs[3], cdims, len(dims), body,
                            refs[4], refs[5], wsp, ws_bytes, stream)
            elif conv.kind == "reduce_f64":
                status = fn(refs[0], refs[1], cdims, len(dims), body, refs[2], wsp,
                            ws_bytes, stream)
            elif conv.kind == "reduce_packed":
                status = fn(refs[0], refs[1], refs[2], cdims, len(dims), body, refs[3], refs[4],
                            wsp, ws_bytes, stream)
            else:
                status = fn(refs[0], refs[1], cdims, len(dims), body, refs[2], refs[3],
                            wsp, ws_bytes, stream)
        else:
            algorithm = int(attrs.get("algorithm", _lib.DS_DOT_TENSOR_INT8))
            rhs = args[2] if conv.kind == "dot" else args[1]
            dkey = (conv.kind, device.index, tuple(args[0].shape), tuple(rhs.shape), algorithm,
                    tuple(attrs.get("lhs_batching_dimensions", ())),
                    tuple(attrs.get("rhs_batching_dimensions", ())),
                    tuple(attrs.get("lhs_contracting_dimensions", ())),
                    tuple(attrs.get("rhs_contracting_dimensions", ())))
            cached = _dot_setup.get(dkey)
            if cached is None:
                dd = _dot_dims(attrs, args[0].dim())
                rhs_ref = refs[2] if conv.kind == "dot" else refs[1]
                ws_bytes = _lib.lib().ds_dot_general_workspace_size(
                    refs[0], rhs_ref, ctypes.byref(dd), algorithm)
                if ws_bytes:  # 0: invalid; the call below reports why
                    if len(_dot_setup) > 1024:
                        _dot_setup.clear()
                    _dot_setup[dkey] = (dd, ws_bytes)
            else:
                dd, ws_bytes = cached
            ws = _workspace(ws_bytes, device, stream_ptr)
            wsp = ctypes.c_void_p(ws.data_ptr())
            if conv.kind == "dot":
                status = fn(refs[0], refs[1], refs[2], refs[3], ctypes.byref(dd), algorithm,
                            refs[4], refs[5], wsp, ws_bytes, stream)
            else:
                status = fn(refs[0], refs[1], ctypes.byref(dd), algorithm, refs[2], wsp,
                            ws_bytes, stream)
        _lib.check(status, target_name)
        return outs[0] if single else tuple(outs)

    return call


def _dot_dims(attrs, lhs_rank) -> _lib.DsDotDims:
    lb = tuple(attrs.get("lhs_batching_dimensions", ()))
    rb = tuple(attrs.get("rhs_batching_dimensions", ()))
    lc = tuple(attrs.get("lhs_contracting_dimensions", (lhs_rank - 1,)))
    rc = tuple(attrs.get("rhs_contracting_dimensions", (len(rb),)))
    return _lib.make_dot_dims(lhs_contracting=lc, rhs_contracting=rc, lhs_batch=lb,
                              rhs_batch=rb)
