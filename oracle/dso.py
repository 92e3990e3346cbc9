"""ctypes wrapper over the C oracle (``libds_oracle.so``).

TEST INFRASTRUCTURE ONLY.  Each function restates a reference CPU handler
(rcast915/ds-experiment ``cpp/``) operation for operation; see ds_oracle.c
for the per-function citations.  Arrays are numpy; packed DS arrays have a
trailing dimension of 2 (hi, lo).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libds_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    src = os.path.join(_HERE, "ds_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
        subprocess.run(["make", "-s", "-C", _HERE, "libds_oracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        for name in ("dso_add", "dso_sub", "dso_mul"):
            getattr(L, name).argtypes = [_f32p, _f32p, _f32p, _i64, ctypes.c_int]
        L.dso_from_f64.argtypes = [_f64p, _f32p, _i64, ctypes.c_int]
        L.dso_to_f64.argtypes = [_f32p, _f64p, _i64, ctypes.c_int]
        L.dso_from_f32.argtypes = [_f32p, _f32p, _i64, ctypes.c_int]
        L.dso_to_f32.argtypes = [_f32p, _f32p, _i64, ctypes.c_int]
        L.dso_fused_add_mul.argtypes = [_f64p, _f64p, _f32p, _i64, ctypes.c_int]
        for name in ("dso_fused_add_mul_to_f64", "dso_fused_add_sub_to_f64"):
            getattr(L, name).argtypes = [_f64p, _f64p, _f64p, _i64, ctypes.c_int]
        L.dso_fused_add_mul3_to_f64.argtypes = [_f64p, _f64p, _f64p, _f64p, _i64,
                                                ctypes.c_int]
        L.dso_recurrence_add_mul_to_f64.argtypes = [_f64p, _f64p, _i32, _f64p, _i64,
                                                    ctypes.c_int]
        L.dso_recurrence_mul_add_to_f64.argtypes = [_f64p, _f64p, _f64p, _i32, _f64p,
                                                    _i64, ctypes.c_int]
        L.dso_reduce_f64_seq.argtypes = [_f64p, _i64, ctypes.c_int, ctypes.c_float,
                                         ctypes.c_float, _f32p, _f32p]
        L.dso_reduce_ds_seq.argtypes = [_f32p, _f32p, _i64, ctypes.c_int,
                                        ctypes.c_float, ctypes.c_float, _f32p, _f32p]
        L.dso_dot_f32_seq.argtypes = [_f32p, _f32p, _i64, _f32p, _f32p]
        for name in ("dso_two_sum", "dso_two_prod"):
            getattr(L, name).argtypes = [_f32p, _f32p, _f32p, _f32p, _i64]
        L.dso_split.argtypes = [_f32p, _f32p, _f32p, _i64]
        L.dso_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p32(a):
    return a.ctypes.data_as(_f32p)


def _p64(a):
    return a.ctypes.data_as(_f64p)


def _c32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _c64(a):
    return np.ascontiguousarray(a, dtype=np.float64)


def max_threads() -> int:
    return int(lib().dso_max_threads())


def _packed_binary(name, a, b, nthreads):
    a, b = _c32(a), _c32(b)
    assert a.shape[-1] == 2 and a.size == b.size
    y = np.empty_like(a)
    getattr(lib(), name)(_p32(a), _p32(b), _p32(y), a.size // 2, nthreads)
    return y


def ds_add(a, b, nthreads=1):
    return _packed_binary("dso_add", a, b, nthreads)


def ds_sub(a, b, nthreads=1):
    return _packed_binary("dso_sub", a, b, nthreads)


def ds_mul(a, b, nthreads=1):
    return _packed_binary("dso_mul", a, b, nthreads)


def ds_from_f64(x, nthreads=1):
    x = _c64(x)
    y = np.empty(x.shape + (2,), np.float32)
    lib().dso_from_f64(_p64(x), _p32(y), x.size, nthreads)
    return y


def ds_to_f64(x, nthreads=1):
    x = _c32(x)
    assert x.shape[-1] == 2
    y = np.empty(x.shape[:-1], np.float64)
    lib().dso_to_f64(_p32(x), _p64(y), x.size // 2, nthreads)
    return y


def ds_from_f32(x, nthreads=1):
    x = _c32(x)
    y = np.empty(x.shape + (2,), np.float32)
    lib().dso_from_f32(_p32(x), _p32(y), x.size, nthreads)
    return y


def ds_to_f32(x, nthreads=1):
    x = _c32(x)
    y = np.empty(x.shape[:-1], np.float32)
    lib().dso_to_f32(_p32(x), _p32(y), x.size // 2, nthreads)
    return y


def ds_fused_add_mul(x, y, nthreads=1):
    x, y = _c64(x), _c64(y)
    out = np.empty(x.shape + (2,), np.float32)
    lib().dso_fused_add_mul(_p64(x), _p64(y), _p32(out), x.size, nthreads)
    return out


def ds_fused_add_mul_to_f64(x, y, nthreads=1):
    x, y = _c64(x), _c64(y)
    out = np.empty_like(x)
    lib().dso_fused_add_mul_to_f64(_p64(x), _p64(y), _p64(out), x.size, nthreads)
    return out


def ds_fused_add_mul3_to_f64(a, b, c, nthreads=1):
    a, b, c = _c64(a), _c64(b), _c64(c)
    out = np.empty_like(a)
    lib().dso_fused_add_mul3_to_f64(_p64(a), _p64(b), _p64(c), _p64(out), a.size,
                                    nthreads)
    return out


def ds_fused_add_sub_to_f64(x, y, nthreads=1):
    x, y = _c64(x), _c64(y)
    out = np.empty_like(x)
    lib().dso_fused_add_sub_to_f64(_p64(x), _p64(y), _p64(out), x.size, nthreads)
    return out


def ds_recurrence_add_mul_to_f64(x, y, k, nthreads=1):
    x, y = _c64(x), _c64(y)
    out = np.empty_like(x)
    lib().dso_recurrence_add_mul_to_f64(_p64(x), _p64(y), int(k), _p64(out), x.size,
                                        nthreads)
    return out


def ds_recurrence_mul_add_to_f64(x, a, b, k, nthreads=1):
    x, a, b = _c64(x), _c64(a), _c64(b)
    out = np.empty_like(x)
    lib().dso_recurrence_mul_add_to_f64(_p64(x), _p64(a), _p64(b), int(k), _p64(out),
                                        x.size, nthreads)
    return out


BODY = {"add": 0, "sub": 1, "mul": 2}


def ds_reduce_f64_seq(x, body="add", init=(0.0, 0.0)):
    """Sequential DS fold of f64 inputs; returns (hi, lo) as np.float32."""
    x = _c64(x).ravel()
    h, l = ctypes.c_float(), ctypes.c_float()
    lib().dso_reduce_f64_seq(_p64(x), x.size, BODY[body], float(init[0]),
                             float(init[1]), ctypes.byref(h), ctypes.byref(l))
    return np.float32(h.value), np.float32(l.value)


def ds_reduce_ds_seq(hi, lo, body="add", init=(0.0, 0.0)):
    hi, lo = _c32(hi).ravel(), _c32(lo).ravel()
    h, l = ctypes.c_float(), ctypes.c_float()
    lib().dso_reduce_ds_seq(_p32(hi), _p32(lo), hi.size, BODY[body], float(init[0]),
                            float(init[1]), ctypes.byref(h), ctypes.byref(l))
    return np.float32(h.value), np.float32(l.value)


def ds_dot_f32_seq(a, b):
    a, b = _c32(a).ravel(), _c32(b).ravel()
    h, l = ctypes.c_float(), ctypes.c_float()
    lib().dso_dot_f32_seq(_p32(a), _p32(b), a.size, ctypes.byref(h), ctypes.byref(l))
    return np.float32(h.value), np.float32(l.value)


def two_sum(a, b):
    a, b = _c32(a).ravel(), _c32(b).ravel()
    s, e = np.empty_like(a), np.empty_like(a)
    lib().dso_two_sum(_p32(a), _p32(b), _p32(s), _p32(e), a.size)
    return s, e


def two_prod(a, b):
    a, b = _c32(a).ravel(), _c32(b).ravel()
    p, e = np.empty_like(a), np.empty_like(a)
    lib().dso_two_prod(_p32(a), _p32(b), _p32(p), _p32(e), a.size)
    return p, e


def split(a):
    a = _c32(a).ravel()
    h, l = np.empty_like(a), np.empty_like(a)
    lib().dso_split(_p32(a), _p32(h), _p32(l), a.size)
    return h, l
