"""Fused elementwise programs, host side: tracing, code generation (the
constants' DS split, broadcast index arithmetic), argument checks, and an
NVRTC compilation of the generated source (no GPU needed)."""
import ctypes

import numpy as np
import pytest
import torch

from ds_b200 import _lib, fuse


def f3(x, y, z):
    return (x + y) * z - 0.1 * x


def test_trace_records_ssa_ops():
    t = torch.zeros(2)
    ops, tensors = fuse.trace(f3, [t, t, t])
    # all three arguments are tensors here: three inputs first
    codes = [o[0] for o in ops]
    assert codes[:3] == [_lib.DS_FUSED_INPUT] * 3
    assert codes[3:] == [_lib.DS_FUSED_ADD, _lib.DS_FUSED_MUL, _lib.DS_FUSED_CONST,
                         _lib.DS_FUSED_MUL, _lib.DS_FUSED_SUB]
    assert tensors == [0, 1, 2]


def test_scalar_arguments_become_constants():
    g = fuse.jit(lambda x, c: x * c + 1.0)
    src = g.source(torch.zeros(5, dtype=torch.float64), 0.1)
    hi = np.float32(0.1)
    lo = np.float32(0.1 - float(hi))
    assert f"0x{hi.view(np.uint32):08x}u" in src
    assert f"0x{lo.view(np.uint32):08x}u" in src
    assert "in1" not in src  # one tensor input only


def test_broadcast_index_expressions():
    g = fuse.jit(f3)
    src = g.source(torch.zeros(4, 3, dtype=torch.float64), torch.zeros(3, dtype=torch.float64),
                   torch.zeros(4, 1, dtype=torch.float32))
    assert "from_f64(__ldg(in0 + (i)))" in src          # full
    assert "% 3LL" in src                                # row vector
    assert "__ldg(in2 + ((i / 3LL))), 0.0f" in src       # f32 column vector as (v, 0)
    assert "out[i] = to_f64(" in src


def test_output_types_and_pair_path():
    x32 = torch.zeros(8, dtype=torch.float32)
    src = fuse.jit(lambda a: a * a).source(x32)                          # f32 result
    assert "__fadd_rn(" in src and "reinterpret_cast<const float2*>(in0) + p" in src
    src = fuse.jit(lambda a: a + a, out_dtype="packed").source(torch.zeros(8, dtype=torch.float64))
    assert "make_float4(" in src and "reinterpret_cast<const double2*>(in0) + p" in src
    src = fuse.jit(lambda a: a - 1.0).source(fuse.Packed(torch.zeros(8, 2)))
    assert "ds2{x0.x, x0.y}" in src and "ds2{x0.z, x0.w}" in src
    # a broadcast input takes the one-element loop only
    src = fuse.jit(lambda a, b: a * b).source(torch.zeros(4, 8, dtype=torch.float64),
                                              torch.zeros(8, dtype=torch.float64))
    assert "npairs" not in src and "% 8LL" in src


def test_bad_broadcast_is_rejected():
    g = fuse.jit(lambda a, b: a + b)
    with pytest.raises(ValueError):
        g.source(torch.zeros(4, 3, dtype=torch.float64), torch.zeros(4, dtype=torch.float64))


def test_capi_rejects_bad_programs():
    L = _lib.lib()
    shape = (8,)
    b, d = _lib.make_buffer(1, shape)
    ob, od = _lib.make_buffer(1, shape)
    arr = (ctypes.POINTER(_lib.DsBuffer) * 1)(ctypes.pointer(b))
    ty = (ctypes.c_int32 * 1)(_lib.DS_FUSED_F64)

    def run(ops, n_inputs=1):
        o = (_lib.DsFusedOp * len(ops))(*[_lib.DsFusedOp(*op) for op in ops])
        return L.ds_fused_source(o, len(ops), ty, arr, n_inputs, _lib.DS_FUSED_F64,
                                 ctypes.byref(ob), None, 0, None)

    assert run([(_lib.DS_FUSED_INPUT, 0, 0, 0, 0.0)]) == _lib.DS_OK
    assert run([(_lib.DS_FUSED_INPUT, 1, 0, 0, 0.0)]) == _lib.DS_INVALID_ARGUMENT  # no input 1
    assert run([(_lib.DS_FUSED_ADD, 0, 0, 0, 0.0)]) == _lib.DS_INVALID_ARGUMENT    # forward ref
    assert run([(_lib.DS_FUSED_INPUT, 0, 0, 0, 0.0), (9, 0, 0, 0, 0.0)]) == _lib.DS_INVALID_ARGUMENT
    assert "operands must be earlier" in _lib.last_error() or "unknown" in _lib.last_error()


def test_generated_source_compiles_with_nvrtc():
    g = fuse.jit(f3)
    try:
        g.compile_check(torch.zeros(4, 3, dtype=torch.float64), torch.zeros(3, dtype=torch.float64),
                        torch.zeros(4, 1, dtype=torch.float32))
    except _lib.DsInternal as e:
        if "could not be loaded" in str(e):
            pytest.skip("NVRTC is not available here")
        raise
