"""NumPy restatement of the reference DS compiler pass (stablehlo_pass/DsTransformPass.cpp).

TEST INFRASTRUCTURE ONLY.  The pass rewrites f32/f64 StableHLO into f32 (hi, lo)
pairs held as separate (SoA) tensors; XLA then runs them.  JAX, MLIR and XLA are
not available here, so this module restates the emitted arithmetic on numpy
float32 arrays.  numpy never fuses a multiply into an add, matching the
element-wise StableHLO ops the pass emits.

The reduce and dot_general orders inside XLA are XLA's own (tree reductions,
cuBLAS SGEMM blocking); they are not pinned by any reference test, so the
reduce below folds sequentially (tests/ds_ref.py:89-96) and the GEMM uses
numpy's float32 BLAS matmul.  Parity for those two is judged by error
magnitude, not bits.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def two_sum(a, b):
    """emitTwoSum, DsTransformPass.cpp:76-85."""
    a = np.asarray(a, F32)
    b = np.asarray(b, F32)
    with np.errstate(invalid="ignore", over="ignore"):
        s = a + b
        bb = s - a
        e = (a - (s - bb)) + (b - bb)
    return s, e


def split(a):
    """emitSplit (Veltkamp, 4097), DsTransformPass.cpp:101-108."""
    a = np.asarray(a, F32)
    with np.errstate(invalid="ignore", over="ignore"):
        t = F32(4097.0) * a
        hi = t - (t - a)
        lo = a - hi
    return hi, lo


def two_prod(a, b):
    """emitTwoProd, DsTransformPass.cpp:113-127."""
    a = np.asarray(a, F32)
    b = np.asarray(b, F32)
    with np.errstate(invalid="ignore", over="ignore"):
        p = a * b
        ah, al = split(a)
        bh, bl = split(b)
        e = (((ah * bh - p) + ah * bl) + al * bh) + al * bl
    return p, e


def ds_add(ah, al, bh, bl):
    """emitDsAdd, DsTransformPass.cpp:130-139."""
    with np.errstate(invalid="ignore", over="ignore"):
        s1, e1 = two_sum(ah, bh)
        s2, e2 = two_sum(al, bl)
        t1, t2 = two_sum(s1, s2 + e1)
        return t1, t2 + e2


def ds_sub(ah, al, bh, bl):
    """emitDsSub, DsTransformPass.cpp:143-149 (negate b, then ds_add)."""
    return ds_add(ah, al, -np.asarray(bh, F32), -np.asarray(bl, F32))


def ds_mul(ah, al, bh, bl):
    """emitDsMul, DsTransformPass.cpp:152-164."""
    with np.errstate(invalid="ignore", over="ignore"):
        p1, e1 = two_prod(ah, bh)
        ah = np.asarray(ah, F32)
        al = np.asarray(al, F32)
        bh = np.asarray(bh, F32)
        bl = np.asarray(bl, F32)
        cross = ah * bl + al * bh
        s, e2 = two_sum(p1, cross)
        return s, (e1 + e2) + al * bl


def from_float(v):
    """emitFromFloat, DsTransformPass.cpp:169-187."""
    v = np.asarray(v)
    if v.dtype == np.float32:
        return v, np.zeros_like(v)
    v = v.astype(np.float64)
    hi = v.astype(F32)
    lo = (v - hi.astype(np.float64)).astype(F32)
    return hi, lo


def to_float(hi, lo, dtype=np.float64):
    """emitToFloat, DsTransformPass.cpp:191-196: convert both, then add."""
    return np.asarray(hi).astype(dtype) + np.asarray(lo).astype(dtype)


def dot_general_2d(a_hi, a_lo, b_hi, b_lo):
    """DotGeneralOp handler, DsTransformPass.cpp:337-370, for A[M,K] @ B[K,N].

    Four float32 dots (f32 accumulation, as cuBLAS SGEMM at HIGHEST precision),
    corr = (e1 + e2) + e3, then two_sum(p, corr).
    """
    p = np.matmul(a_hi, b_hi)
    e1 = np.matmul(a_hi, b_lo)
    e2 = np.matmul(a_lo, b_hi)
    e3 = np.matmul(a_lo, b_lo)
    corr = (e1 + e2) + e3
    return two_sum(p, corr)


def dot_general_f64(A, B):
    """f64 in -> split -> DS dot_general -> recombine to f64 (the pass on f64 args)."""
    ah, al = from_float(A)
    bh, bl = from_float(B)
    h, l = dot_general_2d(ah, al, bh, bl)
    return to_float(h, l)


def fused_add_mul3_f64(a, b, c):
    """(a + b) * c through the pass's element-wise rewrites on f64 arguments."""
    ah, al = from_float(a)
    bh, bl = from_float(b)
    ch, cl = from_float(c)
    sh, sl = ds_add(ah, al, bh, bl)
    ph, pl = ds_mul(sh, sl, ch, cl)
    return to_float(ph, pl)
