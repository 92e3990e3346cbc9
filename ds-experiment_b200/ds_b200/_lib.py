"""ctypes binding of libds_b200.so (the C ABI in include/ds_b200.h).

Loading fails loudly when the library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libds_b200.so")

DS_OK = 0
DS_INVALID_ARGUMENT = 3
DS_INTERNAL = 13

DS_BODY_ADD, DS_BODY_SUB, DS_BODY_MUL = 0, 1, 2
DS_DOT_TENSOR_INT8, DS_DOT_CUDA_CORE = 0, 1


class DsError(RuntimeError):
    """A non-OK ds_status; .code is the xla::ffi::ErrorCode value."""

    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


class DsInvalidArgument(DsError, ValueError):
    pass


class DsInternal(DsError):
    pass


class DsBuffer(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p),
                ("dims", ctypes.POINTER(ctypes.c_int64)),
                ("rank", ctypes.c_int64)]


DS_DOT_MAX_DIMS = 8


class DsDotDims(ctypes.Structure):
    _fields_ = [("n_batch", ctypes.c_int64),
                ("lhs_batch", ctypes.c_int64 * DS_DOT_MAX_DIMS),
                ("rhs_batch", ctypes.c_int64 * DS_DOT_MAX_DIMS),
                ("n_contracting", ctypes.c_int64),
                ("lhs_contracting", ctypes.c_int64 * DS_DOT_MAX_DIMS),
                ("rhs_contracting", ctypes.c_int64 * DS_DOT_MAX_DIMS)]


class DsFusedOp(ctypes.Structure):
    _fields_ = [("code", ctypes.c_int32), ("a", ctypes.c_int32), ("b", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("value", ctypes.c_double)]


DS_FUSED_INPUT, DS_FUSED_CONST, DS_FUSED_ADD, DS_FUSED_SUB, DS_FUSED_MUL, DS_FUSED_NEG = range(6)
DS_FUSED_F64, DS_FUSED_F32, DS_FUSED_PACKED = 0, 1, 2

_BUF = ctypes.POINTER(DsBuffer)
_VP = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_I64P = ctypes.POINTER(ctypes.c_int64)
_DIMS = ctypes.POINTER(DsDotDims)
_OPS = ctypes.POINTER(DsFusedOp)

# name -> (argtypes, restype)
SIGNATURES = {
    "ds_last_error": ([], ctypes.c_char_p),
    "ds_version": ([], ctypes.c_char_p),
    "ds_from_f64": ([_BUF, _BUF, _VP], ctypes.c_int),
    "ds_to_f64": ([_BUF, _BUF, _VP], ctypes.c_int),
    "ds_from_f32": ([_BUF, _BUF, _VP], ctypes.c_int),
    "ds_to_f32": ([_BUF, _BUF, _VP], ctypes.c_int),
    "ds_add": ([_BUF, _BUF, _BUF, _VP], ctypes.c_int),
    "ds_sub": ([_BUF, _BUF, _BUF, _VP], ctypes.c_int),
    "ds_mul": ([_BUF, _BUF, _BUF, _VP], ctypes.c_int),
    "ds_fused_add_mul": ([_BUF, _BUF, _BUF, _VP], ctypes.c_int),
    "ds_fused_add_mul_to_f64": ([_BUF, _BUF, _BUF, _VP], ctypes.c_int),
    "ds_fused_axpy": ([_BUF, _BUF, _BUF, _VP], ctypes.c_int),
    "ds_fused_add_mul_to_f64_cuda": ([_BUF, _BUF, _BUF, _VP], ctypes.c_int),
    "ds_fused_add_sub_to_f64_cuda": ([_BUF, _BUF, _BUF, _VP], ctypes.c_int),
    "ds_recurrence_add_mul_to_f64_cuda": ([_BUF, _BUF, _I32, _BUF, _VP], ctypes.c_int),
    "ds_fused_add_mul3_to_f64": ([_BUF, _BUF, _BUF, _BUF, _VP], ctypes.c_int),
    "ds_recurrence_mul_add_to_f64": ([_BUF, _BUF, _BUF, _I32, _BUF, _VP], ctypes.c_int),
    "ds_reduce_workspace_size": ([_BUF, _I64P, _I64], _SZ),
    "ds_reduce": ([_BUF, _BUF, _BUF, _BUF, _I64P, _I64, _I32, _BUF, _BUF, _VP, _SZ, _VP],
                  ctypes.c_int),
    "ds_reduce_f64": ([_BUF, _BUF, _I64P, _I64, _I32, _BUF, _VP, _SZ, _VP], ctypes.c_int),
    "ds_reduce_from_f64": ([_BUF, _BUF, _I64P, _I64, _I32, _BUF, _BUF, _VP, _SZ, _VP],
                           ctypes.c_int),
    "ds_reduce_f64_noalloc": ([_BUF, _BUF, _I64P, _I64, _I32, _BUF, _VP], ctypes.c_int),
    "ds_reduce_packed": ([_BUF, _BUF, _BUF, _I64P, _I64, _I32, _BUF, _BUF, _VP, _SZ, _VP],
                         ctypes.c_int),
    "ds_reduce_f64_multi": ([ctypes.POINTER(_BUF), ctypes.POINTER(_BUF), ctypes.POINTER(_I32), _I32,
                             _I64P, _I64, ctypes.POINTER(_BUF), _VP, _SZ, _VP], ctypes.c_int),
    "ds_exchange_bytes": ([], _SZ),
    "ds_exchange_handle_bytes": ([], _SZ),
    "ds_exchange_alloc": ([ctypes.POINTER(_VP), _VP], ctypes.c_int),
    "ds_exchange_open": ([_VP, ctypes.POINTER(_VP)], ctypes.c_int),
    "ds_exchange_close": ([_VP], ctypes.c_int),
    "ds_exchange_free": ([_VP], ctypes.c_int),
    "ds_exchange_error": ([_VP, ctypes.POINTER(ctypes.c_uint32)], ctypes.c_int),
    "ds_reduce_f64_sharded_workspace_size": ([_BUF], _SZ),
    "ds_reduce_f64_sharded": ([_BUF, _BUF, _I32, _BUF, ctypes.POINTER(_VP), _I32, _I32,
                               ctypes.c_uint64, _I32, _VP, _SZ, _VP], ctypes.c_int),
    "ds_dot_general_workspace_size": ([_BUF, _BUF, _DIMS, _I32], _SZ),
    "ds_dot_general": ([_BUF, _BUF, _BUF, _BUF, _DIMS, _I32, _BUF, _BUF, _VP, _SZ, _VP],
                       ctypes.c_int),
    "ds_dot_general_f64": ([_BUF, _BUF, _DIMS, _I32, _BUF, _VP, _SZ, _VP], ctypes.c_int),
    "ds_fused_run": ([_OPS, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_BUF), _I32, _I32, _BUF,
                      _VP], ctypes.c_int),
    "ds_fused_source": ([_OPS, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_BUF), _I32, _I32, _BUF,
                         ctypes.c_char_p, _SZ, ctypes.POINTER(_SZ)], ctypes.c_int),
    "ds_fused_compile_check": ([_OPS, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_BUF), _I32, _I32,
                                _BUF], ctypes.c_int),
    "ds_fused_reduce_workspace_size": ([_I64P, _I32], _SZ),
    "ds_fused_reduce": ([_OPS, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_BUF), _I32, _I64P, _I32,
                         _I32, _BUF, _BUF, _BUF, _BUF, _VP, _SZ, _VP], ctypes.c_int),
    "ds_fused_reduce_compile_check": ([_OPS, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_BUF), _I32,
                                       _I64P, _I32, _I32], ctypes.c_int),
    "ds_fused_reduce_rows": ([_OPS, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_BUF), _I32, _I64P,
                              _I32, _I32, _I32, _BUF, _BUF, _BUF, _BUF, _VP], ctypes.c_int),
    "ds_fused_reduce_rows_compile_check": ([_OPS, _I32, ctypes.POINTER(_I32), ctypes.POINTER(_BUF),
                                            _I32, _I64P, _I32, _I32, _I32], ctypes.c_int),
    "ds_dot_tensor_plan": ([_I64, ctypes.POINTER(_I32), ctypes.POINTER(_I32)], ctypes.c_int),
    "ds_dot_tensor_kernel_info": ([ctypes.POINTER(_I32), ctypes.POINTER(_I32)], ctypes.c_int),
    "ds_profile_enable": ([ctypes.c_int], None),
    "ds_profile_select": ([ctypes.c_char_p], None),
    "ds_profile_reset": ([], None),
    "ds_profile_read": ([ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), _I64P], ctypes.c_int),
}


def gemm_info(M: int, N: int, K: int) -> dict:
    """Plan of the tensor-core dot_general for an M x N x K product: int8 GEMMs
    (moduli), bits kept per operand, and the int8 tensor ops it performs
    (2 per MAC, unpadded)."""
    m, b = ctypes.c_int32(), ctypes.c_int32()
    check(lib().ds_dot_tensor_plan(int(K), ctypes.byref(m), ctypes.byref(b)), "plan")
    return {"moduli": m.value, "bits": b.value,
            "tensor_ops_per_launch": float(m.value) * 2.0 * M * N * K}


def gemm_kernel_info() -> dict:
    """Tensor-core GEMM kernel of the current device: CTA pairs of the
    cta_group::2 kernel (0 = the one-CTA kernel) and the occupancy query's
    CUDA error code."""
    p, e = ctypes.c_int32(), ctypes.c_int32()
    check(lib().ds_dot_tensor_kernel_info(ctypes.byref(p), ctypes.byref(e)), "kernel info")
    return {"cta_pairs": p.value, "query_error": e.value,
            "kernel": "cta_pair" if p.value > 0 else "single_cta"}


_raw_stream = getattr(__import__("torch")._C, "_cuda_getCurrentRawStream", None)


def current_stream_ptr(device=None) -> int:
    """The cudaStream_t of torch's current stream on `device` (a
    torch.device, an index, or None for the current device), as an int.
    Uses torch's raw-pointer query when it has one: building a Stream
    object costs several microseconds per call."""
    import torch
    if isinstance(device, torch.device):
        device = device.index
    if device is None:
        device = torch.cuda.current_device()
    if _raw_stream is not None:
        return int(_raw_stream(device))
    return torch.cuda.current_stream(device).cuda_stream


def profile_enable(on: bool = True) -> None:
    lib().ds_profile_enable(1 if on else 0)


def profile_select(names=None) -> None:
    """Record only the kernel families in `names` (an iterable of names);
    None records all."""
    lib().ds_profile_select(",".join(names).encode() if names else None)


def profile_reset() -> None:
    lib().ds_profile_reset()


def profile_read(name: str):
    """(total milliseconds, launch count) of kernel family `name` since the
    last reset; waits for the recorded events."""
    ms = ctypes.c_double()
    n = ctypes.c_int64()
    check(lib().ds_profile_read(name.encode(), ctypes.byref(ms), ctypes.byref(n)), "profile")
    return ms.value, n.value

_lib = None


def lib():
    """Load libds_b200.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python ds-experiment_b200/build.py` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (argtypes, restype) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = L
    return _lib


def last_error() -> str:
    return lib().ds_last_error().decode()


def check(status: int, what: str = "") -> None:
    if status == DS_OK:
        return
    msg = last_error()
    if status == DS_INVALID_ARGUMENT:
        raise DsInvalidArgument(status, msg)
    raise DsInternal(status, f"{what}: {msg}" if what else msg)


_DIMS_TYPES = [ctypes.c_int64 * max(n, 1) for n in range(17)]
# dims arrays by shape: read-only once built, so buffers of one shape share one
_shape_dims: dict = {}


def make_buffer(ptr: int, shape) -> tuple:
    """A DsBuffer for `shape` at device address `ptr`; returns (buffer, dims)
    (keep `dims` alive while the buffer is used)."""
    shape = tuple(shape)
    dims = _shape_dims.get(shape)
    if dims is None:
        n = len(shape)
        dims = (_DIMS_TYPES[n] if n < 17 else ctypes.c_int64 * n)(*shape)
        if len(_shape_dims) > 1024:
            _shape_dims.clear()
        _shape_dims[shape] = dims
    return DsBuffer(ptr, dims, len(shape)), dims


def make_dot_dims(n_batch=0, lhs_contracting=1, rhs_contracting=0, lhs_batch=None,
                  rhs_batch=None) -> DsDotDims:
    """stablehlo dot_general dimension numbers.  Contracting dimensions are an
    int or a sequence (paired in order); batching dimensions default to the
    leading n_batch of each operand."""
    lb = tuple(range(n_batch)) if lhs_batch is None else tuple(lhs_batch)
    rb = tuple(range(n_batch)) if rhs_batch is None else tuple(rhs_batch)
    lc = (lhs_contracting,) if isinstance(lhs_contracting, int) else tuple(lhs_contracting)
    rc = (rhs_contracting,) if isinstance(rhs_contracting, int) else tuple(rhs_contracting)
    if len(lb) != len(rb) or len(lc) != len(rc):
        raise ValueError("dot_general: lhs and rhs dimension lists differ in length")
    if len(lb) > DS_DOT_MAX_DIMS or len(lc) > DS_DOT_MAX_DIMS:
        raise ValueError(f"dot_general: at most {DS_DOT_MAX_DIMS} batching or contracting "
                         "dimensions")
    d = DsDotDims()
    d.n_batch = len(lb)
    for i, (x, y) in enumerate(zip(lb, rb)):
        d.lhs_batch[i] = int(x)
        d.rhs_batch[i] = int(y)
    d.n_contracting = len(lc)
    for i, (x, y) in enumerate(zip(lc, rc)):
        d.lhs_contracting[i] = int(x)
        d.rhs_contracting[i] = int(y)
    return d
