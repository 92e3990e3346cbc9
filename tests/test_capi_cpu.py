"""The C ABI without a GPU: symbols, signatures and the reference's shape errors.

Every shape check runs before any CUDA call, so invalid calls return
DS_INVALID_ARGUMENT with the reference handler's message on a CPU-only host.
"""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "ds_b200.h")


@pytest.fixture(scope="module")
def L():
    import importlib
    build = importlib.import_module("build")  # ds-experiment_b200/build.py
    build.build()
    from ds_b200 import _lib
    return _lib


def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"DS_API\s+[\w\s\*]+?\b(ds_\w+)\s*\(", text)))


def test_header_symbols_exported(L):
    syms = header_symbols()
    assert len(syms) >= 20
    cdll = ctypes.CDLL(L.LIB_PATH)
    for s in syms:
        assert hasattr(cdll, s), f"{s} declared in ds_b200.h but not exported"
    # the Python binding declares a signature for every header entry point
    assert set(syms) == set(L.SIGNATURES), set(syms) ^ set(L.SIGNATURES)


def test_library_loads_and_reports_version(L):
    assert b"sm_100a" in L.lib().ds_version()


def _b(L, shape, ptr=0x1000):
    return L.make_buffer(ptr, shape)


def _call_err(L, name, *args):
    fn = getattr(L.lib(), name)
    st = fn(*args)
    return st, L.last_error()


def test_packed_shape_errors(L):
    a, _ka = _b(L, (4, 2))
    b3, _kb = _b(L, (4, 3))
    y, _ky = _b(L, (4, 2))
    y5, _ky5 = _b(L, (5, 2))
    a3d, _k3 = _b(L, (2, 2, 2))
    r = ctypes.byref
    for name, op in (("ds_add", "ds.add"), ("ds_sub", "ds.sub"), ("ds_mul", "ds.mul")):
        st, msg = _call_err(L, name, r(a), r(b3), r(y), None)
        assert st == L.DS_INVALID_ARGUMENT and msg == f"{op} expects last dim == 2"
        st, msg = _call_err(L, name, r(a), r(a3d), r(y), None)
        assert st == L.DS_INVALID_ARGUMENT and msg == f"{op} input shapes must match"
        st, msg = _call_err(L, name, r(a), r(a), r(y5), None)
        assert st == L.DS_INVALID_ARGUMENT and msg == f"{op} output shape mismatch"


def test_split_recombine_shape_errors(L):
    r = ctypes.byref
    x, _k1 = _b(L, (8,))
    y_bad, _k2 = _b(L, (8, 3))
    y_mis, _k3 = _b(L, (7, 2))
    st, msg = _call_err(L, "ds_from_f64", r(x), r(y_bad), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "ds_from_f64 output last dim must be 2")
    st, msg = _call_err(L, "ds_from_f64", r(x), r(y_mis), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "ds_from_f64 shape mismatch")
    p, _k4 = _b(L, (8, 3))
    st, msg = _call_err(L, "ds_to_f64", r(p), r(x), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "ds_to_f64 input last dim must be 2")
    p2, _k5 = _b(L, (8, 2))
    o7, _k6 = _b(L, (7,))
    st, msg = _call_err(L, "ds_to_f64", r(p2), r(o7), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "ds_to_f64 shape mismatch")
    st, msg = _call_err(L, "ds_from_f32", r(x), r(y_mis), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "ds_from_f32 shape mismatch")
    st, msg = _call_err(L, "ds_to_f32", r(p2), r(o7), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "ds_to_f32 shape mismatch")


def test_fused_shape_errors(L):
    r = ctypes.byref
    x, _1 = _b(L, (8,))
    y7, _2 = _b(L, (7,))
    m, _3 = _b(L, (2, 4))
    o8, _4 = _b(L, (8,))
    o82, _5 = _b(L, (8, 2))
    st, msg = _call_err(L, "ds_fused_add_mul_to_f64_cuda", r(m), r(x), r(o8), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "ds_fused_add_mul_to_f64_cuda expects rank-1 inputs")
    st, msg = _call_err(L, "ds_fused_add_sub_to_f64_cuda", r(x), r(y7), r(o8), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "input lengths must match")
    st, msg = _call_err(L, "ds_fused_add_mul_to_f64", r(x), r(x), r(o82), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "output shape must be [N]")
    st, msg = _call_err(L, "ds_fused_add_mul", r(x), r(x), r(o8), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "output shape must be [N,2]")
    st, msg = _call_err(L, "ds_fused_axpy", r(m), r(x), r(o8), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "ds_fused_axpy expects rank-1 inputs")
    # k < 0 (cpp/ds_recurrence_add_mul_to_f64_cuda.cu:115-117)
    st, msg = _call_err(L, "ds_recurrence_add_mul_to_f64_cuda", r(x), r(x), -1, r(o8), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "k must be nonnegative")
    st, msg = _call_err(L, "ds_recurrence_mul_add_to_f64", r(x), r(x), r(x), -3, r(o8), None)
    assert (st, msg) == (L.DS_INVALID_ARGUMENT, "k must be nonnegative")


def test_null_pointer_rejected(L):
    r = ctypes.byref
    x, _1 = _b(L, (8,), ptr=0)
    y, _2 = _b(L, (8, 2))
    st, msg = _call_err(L, "ds_from_f64", r(x), r(y), None)
    assert st == L.DS_INVALID_ARGUMENT and "null" in msg


def test_reduce_and_dot_shape_errors(L):
    r = ctypes.byref
    x, _1 = _b(L, (4, 5, 6))
    init, _2 = _b(L, ())
    out, _3 = _b(L, (4, 6))
    dims = (ctypes.c_int64 * 2)(0, 2)  # not contiguous
    st, msg = _call_err(L, "ds_reduce_f64", r(x), r(init), dims, 2, 0, r(out), None, 0, None)
    assert st == L.DS_INVALID_ARGUMENT and "contiguous" in msg
    d1 = (ctypes.c_int64 * 1)(1)
    bad, _4 = _b(L, (4, 5))
    st, msg = _call_err(L, "ds_reduce_f64", r(x), r(init), d1, 1, 0, r(bad), None, 0, None)
    assert st == L.DS_INVALID_ARGUMENT and "output shape" in msg
    st, msg = _call_err(L, "ds_reduce_f64", r(x), r(init), d1, 1, 7, r(out), None, 0, None)
    assert st == L.DS_INVALID_ARGUMENT and "body" in msg
    # dot_general: contracting sizes differ
    A, _5 = _b(L, (8, 16))
    B, _6 = _b(L, (15, 4))
    C, _7 = _b(L, (8, 4))
    dd = L.make_dot_dims(0, 1, 0)
    st, msg = _call_err(L, "ds_dot_general_f64", r(A), r(B), r(dd), 0, r(C), None, 0, None)
    assert st == L.DS_INVALID_ARGUMENT and "contracting" in msg
    B2, _8 = _b(L, (16, 4))
    C2, _9 = _b(L, (8, 5))
    st, msg = _call_err(L, "ds_dot_general_f64", r(A), r(B2), r(dd), 0, r(C2), None, 0, None)
    assert st == L.DS_INVALID_ARGUMENT and "output shape" in msg
    st, msg = _call_err(L, "ds_dot_general_f64", r(A), r(B2), r(dd), 9, r(_b(L, (8, 4))[0]),
                        None, 0, None)
    assert st == L.DS_INVALID_ARGUMENT and "algorithm" in msg


def test_ffi_surface_registry():
    from ds_b200 import ffi
    names = ffi.registered_targets()
    for t in ("ds_add", "ds_sub", "ds_mul", "ds_from_f64", "ds_to_f64", "ds_from_f32",
              "ds_to_f32", "ds_fused_add_mul", "ds_fused_add_mul_to_f64", "ds_fused_axpy",
              "ds_fused_add_mul_to_f64_cuda", "ds_fused_add_sub_to_f64_cuda",
              "ds_recurrence_add_mul_to_f64_cuda", "ds_reduce", "ds_dot_general"):
        assert t in names
    with pytest.raises(ValueError):
        ffi.register_ffi_target("ds_add", "ds_add", platform="cpu")


def test_cpu_tensor_rejected():
    import torch
    from ds_b200 import ops
    with pytest.raises(ValueError, match="CUDA"):
        ops.ds_from_f64(torch.zeros(4, dtype=torch.float64))


def test_fused_reduce_argument_errors(L):
    """ds_fused_reduce checks its body, shape, buffers and workspace before
    any launch."""
    r = ctypes.byref
    ops = (L.DsFusedOp * 1)(L.DsFusedOp(L.DS_FUSED_INPUT, 0, 0, 0, 0.0))
    x, _1 = _b(L, (8,))
    arr = (ctypes.POINTER(L.DsBuffer) * 1)(ctypes.pointer(x))
    ty = (ctypes.c_int32 * 1)(L.DS_FUSED_F64)
    dims = (ctypes.c_int64 * 1)(8)
    s, _2 = _b(L, ())
    lib = L.lib()

    def call(body=L.DS_BODY_ADD, rank=1, init=s, ws=None, nbytes=0, d=dims):
        st = lib.ds_fused_reduce(ops, 1, ty, arr, 1, d, rank, body, r(init), r(s), r(s), r(s),
                                 ws, nbytes, None)
        return st, L.last_error()
    st, msg = call(body=L.DS_BODY_SUB)
    assert st == L.DS_INVALID_ARGUMENT and "DS_BODY_ADD or DS_BODY_MUL" in msg
    st, msg = call(rank=9)
    assert st == L.DS_INVALID_ARGUMENT and "8 dimensions" in msg
    null, _3 = _b(L, (), ptr=0)
    st, msg = call(init=null)
    assert st == L.DS_INVALID_ARGUMENT and "null" in msg
    st, msg = call()
    assert st == L.DS_INVALID_ARGUMENT and "workspace" in msg
    need = int(lib.ds_fused_reduce_workspace_size(dims, 1))
    assert need > 0
    # the map's shape does not match the input: rejected by the program checks
    bad = (ctypes.c_int64 * 1)(9)
    st, msg = call(ws=ctypes.c_void_p(0x100000), nbytes=need, d=bad)
    assert st == L.DS_INVALID_ARGUMENT and "broadcast" in msg


def test_fused_reduce_rows_argument_errors(L):
    """ds_fused_reduce_rows checks its body, reduced dimensions, buffers and
    output shape before any launch."""
    r = ctypes.byref
    ops = (L.DsFusedOp * 1)(L.DsFusedOp(L.DS_FUSED_INPUT, 0, 0, 0, 0.0))
    x, _1 = _b(L, (4, 8))
    arr = (ctypes.POINTER(L.DsBuffer) * 1)(ctypes.pointer(x))
    ty = (ctypes.c_int32 * 1)(L.DS_FUSED_F64)
    dims = (ctypes.c_int64 * 2)(4, 8)
    s, _2 = _b(L, ())
    o4, _3 = _b(L, (4,))
    o5, _4 = _b(L, (5,))
    lib = L.lib()

    def call(body=L.DS_BODY_ADD, k=1, out=o4, init=s):
        st = lib.ds_fused_reduce_rows(ops, 1, ty, arr, 1, dims, 2, k, body, r(init), r(s),
                                      r(out), r(out), None)
        return st, L.last_error()
    st, msg = call(body=L.DS_BODY_SUB)
    assert st == L.DS_INVALID_ARGUMENT and "DS_BODY_ADD or DS_BODY_MUL" in msg
    st, msg = call(k=0)
    assert st == L.DS_INVALID_ARGUMENT and "trailing dimensions" in msg
    st, msg = call(k=3)
    assert st == L.DS_INVALID_ARGUMENT and "trailing dimensions" in msg
    st, msg = call(out=o5)
    assert st == L.DS_INVALID_ARGUMENT and "one value per row" in msg
    null, _5 = _b(L, (), ptr=0)
    st, msg = call(init=null)
    assert st == L.DS_INVALID_ARGUMENT and "null" in msg


def test_dot_general_workspace_counts_the_gather_copy(L):
    """An operand whose free dimensions do not nest into one stride ([F1, K,
    F2], contracting over K) is copied to [F1 * F2, K] first: the workspace
    query adds exactly that copy (8 bytes per element, 256-byte aligned) to
    what the nested [54, 64] x [64, 30] product needs; nested layouts, non-
    leading batch dimensions and several contracting dimensions add nothing."""
    import ctypes
    r = ctypes.byref
    A3, _a = _b(L, (6, 64, 9))
    A2, _b2 = _b(L, (54, 64))
    B, _c = _b(L, (64, 30))
    nested = L.lib().ds_dot_general_workspace_size(r(A2), r(B), r(L.make_dot_dims(0, 1, 0)), 0)
    copied = L.lib().ds_dot_general_workspace_size(r(A3), r(B), r(L.make_dot_dims(0, 1, 0)), 0)
    assert nested > 0 and copied == nested + (54 * 64 * 8 + 255) // 256 * 256
    S, _d = _b(L, (40, 3, 64))
    T, _e = _b(L, (64, 3, 36))
    dd = L.make_dot_dims(lhs_contracting=2, rhs_contracting=0, lhs_batch=(1,), rhs_batch=(1,))
    Sb, _f = _b(L, (3, 40, 64))
    Tb, _g = _b(L, (3, 64, 36))
    lead = L.make_dot_dims(1, 2, 1)
    assert L.lib().ds_dot_general_workspace_size(r(S), r(T), r(dd), 0) == \
        L.lib().ds_dot_general_workspace_size(r(Sb), r(Tb), r(lead), 0)
    M3, _h = _b(L, (64, 12, 20))
    N3, _i = _b(L, (12, 20, 48))
    two = L.make_dot_dims(lhs_contracting=(1, 2), rhs_contracting=(0, 1))
    M2, _j = _b(L, (64, 240))
    N2, _k = _b(L, (240, 48))
    flat = L.lib().ds_dot_general_workspace_size(r(M2), r(N2), r(L.make_dot_dims(0, 1, 0)), 0)
    assert L.lib().ds_dot_general_workspace_size(r(M3), r(N3), r(two), 0) == flat
    # contracting pairs listed out of memory order are taken in memory order
    # (the sum does not depend on it): no copy ...
    swapped = L.make_dot_dims(lhs_contracting=(2, 1), rhs_contracting=(1, 0))
    assert L.lib().ds_dot_general_workspace_size(r(M3), r(N3), r(swapped), 0) == flat
    # ... unless no order suits both operands: A[m, a, b] x B[b, a, n] copies one
    # (the smaller, B)
    Bx, _l = _b(L, (20, 12, 48))
    crossed = L.make_dot_dims(lhs_contracting=(2, 1), rhs_contracting=(0, 1))
    assert L.lib().ds_dot_general_workspace_size(r(M3), r(Bx), r(crossed), 0) == \
        flat + (240 * 48 * 8 + 255) // 256 * 256
    # mismatched sizes get no workspace (the call itself reports why)
    bad = L.make_dot_dims(lhs_contracting=(1, 2), rhs_contracting=(1, 0))
    assert L.lib().ds_dot_general_workspace_size(r(M3), r(N3), r(bad), 0) == 0


def test_profile_select_and_read_without_a_gpu(L):
    """The diagnostics bookkeeping needs no device: selecting families,
    enabling, resetting and reading a family that recorded nothing work on
    the host alone."""
    from ds_b200 import _lib
    _lib.profile_select(["ozaki_gemm", "reduce"])
    _lib.profile_enable(True)
    _lib.profile_enable(False)
    _lib.profile_select(None)
    _lib.profile_reset()
    assert _lib.profile_read("ozaki_gemm") == (0.0, 0)
    L.lib().ds_profile_select(b",,reduce,")  # empty names are skipped
    L.lib().ds_profile_select(None)
