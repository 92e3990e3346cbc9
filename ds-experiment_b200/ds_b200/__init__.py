"""ds_b200: double-single (DS) arithmetic on B200 (sm_100a).

The product is libds_b200.so (C ABI in include/ds_b200.h).  This package is
its Python host side: ``ffi`` mirrors the reference's custom-call surface
(register_ffi_target / ffi_call), ``ops`` has one function per op, and
``dist`` shards the ops over one process per GPU, and ``ds_transform``
rewrites a torch program's f64 / f32 arithmetic to DS the way the
reference's compiler pass does.
"""
from ._lib import (DS_BODY_ADD, DS_BODY_MUL, DS_BODY_SUB, DS_DOT_CUDA_CORE,
                   DS_DOT_TENSOR_INT8, DsError, DsInternal, DsInvalidArgument, LIB_PATH,
                   lib)
from .ffi import ShapeDtypeStruct, ffi_call, register_ffi_target, registered_targets
from .ops import *  # noqa: F401,F403
from .transform import DsFunction, ds_transform

__all__ = [
    "DS_BODY_ADD", "DS_BODY_SUB", "DS_BODY_MUL", "DS_DOT_TENSOR_INT8", "DS_DOT_CUDA_CORE",
    "DsError", "DsInvalidArgument", "DsInternal", "LIB_PATH", "lib", "ShapeDtypeStruct",
    "ffi_call", "register_ffi_target", "registered_targets", "ds_transform", "DsFunction",
]
