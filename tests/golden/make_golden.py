"""Generate golden DS vectors from the reference's own Python model.

Run in a container where the reference tree is mounted (read-only):

    python tests/golden/make_golden.py /root/reference

It imports the reference's pure-NumPy DS model ``tests/ds_ref.py`` (two_sum,
Veltkamp split, Dekker two_prod, ds_add/ds_sub/ds_mul, ds_dot, ds_sum) and
evaluates it on seeded inputs, writing ``ds_ref_vectors.npz`` next to this
script.  The f64 split follows ``tests/test_f64_ds.py:_split_f64`` (hi =
float32(x), lo = float32(x - hi)) and the fused chains compose ds_ref's own
primitives in the order of the reference kernels.  The committed .npz is what
the tests read; nothing at test time touches the reference tree.
"""
from __future__ import annotations

import os
import sys

import numpy as np

F32 = np.float32
HERE = os.path.dirname(os.path.abspath(__file__))


def load_ds_ref(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "tests"))
    import ds_ref  # noqa: E402  (reference module, read-only)
    return ds_ref


def split_f64(x):
    """tests/test_f64_ds.py:_split_f64, vectorised."""
    x = np.asarray(x, np.float64)
    hi = x.astype(F32)
    lo = (x - hi.astype(np.float64)).astype(F32)
    return hi, lo


def edge_f32():
    """Edge values the reference suites exercise (NaN, Inf, subnormals, zeros,
    huge magnitudes where the 4097 split overflows, cancellation scales)."""
    v = [0.0, -0.0, 1.0, -1.0, 0.1, 1e8, -1e8, 1e-2, 1.5e-40, -1.5e-40,
         1e-38, 3.4e38, -3.4e38, 1e35, 8.3e34, 8.4e34, np.inf, -np.inf, np.nan,
         1e7, -1e7 + 1, 1e6, 123456789.0, 1.23456789e-7, 2.0 ** -126,
         2.0 ** -149, 2.0 ** 60, 2.0 ** -60, 16777217.0, 0.3333333]
    return np.array(v, F32)


def make(ref_root, out_path):
    ds_ref = load_ds_ref(ref_root)
    rng = np.random.default_rng(20261201)
    out = {}

    # ---- f32 primitives on random + edge operands ------------------------
    n = 1024
    mags = rng.uniform(-45, 38, n)
    a = (rng.uniform(-1, 1, n) * 10.0 ** mags).astype(F32)
    b = (rng.uniform(-1, 1, n) * 10.0 ** rng.uniform(-45, 38, n)).astype(F32)
    e = edge_f32()
    ea, eb = np.meshgrid(e, e, indexing="ij")
    a = np.concatenate([a, ea.ravel()])
    b = np.concatenate([b, eb.ravel()])
    out["prim_a"], out["prim_b"] = a, b
    with np.errstate(all="ignore"):
        s, err = ds_ref.two_sum(a, b)
        out["two_sum_s"], out["two_sum_e"] = np.asarray(s, F32), np.asarray(err, F32)
        h, l = ds_ref.veltkamp_split(a)
        out["split_hi"], out["split_lo"] = np.asarray(h, F32), np.asarray(l, F32)
        p, pe = ds_ref.two_prod(a, b)
        out["two_prod_p"], out["two_prod_e"] = np.asarray(p, F32), np.asarray(pe, F32)

    # ---- packed DS add/sub/mul -------------------------------------------
    m = 2048
    x = rng.uniform(-1, 1, m) * 10.0 ** rng.uniform(-12, 12, m)
    y = rng.uniform(-1, 1, m) * 10.0 ** rng.uniform(-12, 12, m)
    # cancellation-heavy pairs: y close to -x
    x[:256] = rng.uniform(1, 2, 256) * 1e8
    y[:256] = -x[:256] + rng.uniform(-1, 1, 256) * 1e-3
    xh, xl = split_f64(x)
    yh, yl = split_f64(y)
    # append DS pairs built from the edge grid (lo = 0)
    xh = np.concatenate([xh, ea.ravel()])
    xl = np.concatenate([xl, np.zeros(ea.size, F32)])
    yh = np.concatenate([yh, eb.ravel()])
    yl = np.concatenate([yl, np.zeros(eb.size, F32)])
    out["pk_a"] = np.stack([xh, xl], -1)
    out["pk_b"] = np.stack([yh, yl], -1)
    with np.errstate(all="ignore"):
        for name, fn in (("add", ds_ref.ds_add), ("sub", ds_ref.ds_sub),
                         ("mul", ds_ref.ds_mul)):
            rh, rl = fn(xh, xl, yh, yl)
            out["pk_" + name] = np.stack([np.asarray(rh, F32), np.asarray(rl, F32)], -1)

    # ---- f64 split / recombine -------------------------------------------
    z = np.concatenate([
        rng.uniform(-1, 1, 1024) * 10.0 ** rng.uniform(-30, 30, 1024),
        np.array([1.23456789012345e10, 0.1, -0.0, 0.0, 1e300, -1e-300, np.inf,
                  -np.inf, np.nan, 2.0 ** -1074, 3.4028235677973366e38,
                  3.4028236e38, 1.0 + 2.0 ** -40])])
    with np.errstate(all="ignore"):
        zh, zl = split_f64(z)
    out["f64_x"] = z
    out["f64_split"] = np.stack([zh, zl], -1)
    with np.errstate(all="ignore"):
        out["f64_recombine"] = zh.astype(np.float64) + zl.astype(np.float64)

    # ---- fused chains on f64 inputs, composed from ds_ref primitives ----
    k = 4096
    fx = rng.uniform(-1, 1, k) * 10.0 ** rng.uniform(-8, 8, k)
    fy = rng.uniform(-1, 1, k) * 10.0 ** rng.uniform(-8, 8, k)
    fc = rng.uniform(-1, 1, k) * 10.0 ** rng.uniform(-8, 8, k)
    # the reference test vectors (python/test_ds_fused_add_mul_to_f64.py:34-35,
    # python/test_pass_correctness.py cancellation pairs)
    fx = np.concatenate([fx, [1.23456789012345, 2.5, 123456789.12345679, 1e8, 1e10, 1e12]])
    fy = np.concatenate([fy, [9.87654321098765, 3.0, 1.23456789e-7, 1e-2, 1e-3, 1e-4]])
    fc = np.concatenate([fc, [0.5, -2.0, 3.0, 1.0, 1.0, 1.0]])
    out["fx"], out["fy"], out["fc"] = fx, fy, fc
    Xh, Xl = split_f64(fx)
    Yh, Yl = split_f64(fy)
    Ch, Cl = split_f64(fc)
    sh, sl = ds_ref.ds_add(Xh, Xl, Yh, Yl)
    ph, pl = ds_ref.ds_mul(sh, sl, Yh, Yl)
    out["fused_add_mul_packed"] = np.stack([np.asarray(ph, F32), np.asarray(pl, F32)], -1)
    out["fused_add_mul_to_f64"] = np.asarray(ph, F32).astype(np.float64) + np.asarray(pl, F32).astype(np.float64)
    rh, rl = ds_ref.ds_sub(sh, sl, Xh, Xl)
    out["fused_add_sub_to_f64"] = np.asarray(rh, F32).astype(np.float64) + np.asarray(rl, F32).astype(np.float64)
    qh, ql = ds_ref.ds_mul(sh, sl, Ch, Cl)
    out["fused_add_mul3_to_f64"] = np.asarray(qh, F32).astype(np.float64) + np.asarray(ql, F32).astype(np.float64)

    # recurrence (z+y)*y, k=8, on the reference test vectors
    # (python/test_ds_recurrence_add_mul_to_f64_cuda.py:39-41) plus random ones
    rx = np.concatenate([[0.25, 0.5, 0.75], rng.uniform(-1, 1, 509)])
    ry = np.concatenate([[0.2, 0.3, 0.4], rng.uniform(-1, 1, 509)])
    out["rec_x"], out["rec_y"] = rx, ry
    for kk in (0, 1, 8):
        zh, zl = split_f64(rx)
        Yh2, Yl2 = split_f64(ry)
        for _ in range(kk):
            s1h, s1l = ds_ref.ds_add(zh, zl, Yh2, Yl2)
            zh, zl = ds_ref.ds_mul(s1h, s1l, Yh2, Yl2)
        out[f"rec_add_mul_k{kk}"] = np.asarray(zh, F32).astype(np.float64) + np.asarray(zl, F32).astype(np.float64)

    # recurrence x <- x*a + b (seed-3 style distribution), k in {1, 4, 16}
    mx = rng.uniform(-1, 1, 512)
    ma = rng.uniform(0.999, 1.001, 512)
    mb = rng.uniform(-1e-3, 1e-3, 512)
    out["mrec_x"], out["mrec_a"], out["mrec_b"] = mx, ma, mb
    for kk in (1, 4, 16):
        zh, zl = split_f64(mx)
        Ah, Al = split_f64(ma)
        Bh, Bl = split_f64(mb)
        for _ in range(kk):
            th, tl = ds_ref.ds_mul(zh, zl, Ah, Al)
            zh, zl = ds_ref.ds_add(th, tl, Bh, Bl)
        out[f"mrec_k{kk}"] = np.asarray(zh, F32).astype(np.float64) + np.asarray(zl, F32).astype(np.float64)

    # ---- sequential reductions / dots (ds_ref.ds_sum, ds_dot, ds_matmul) ---
    sv = rng.standard_normal(3000).astype(F32)
    out["sum_x"] = sv
    out["sum_ref"] = np.float64(ds_ref.ds_sum(sv))
    da = rng.standard_normal(2000).astype(F32)
    db = rng.standard_normal(2000).astype(F32)
    out["dot_a"], out["dot_b"] = da, db
    out["dot_ref"] = np.float64(ds_ref.ds_dot(da, db))
    # triplet cancellation (tests/test_dot_product.py:76-86), n=1000
    trip = np.zeros(3000, F32)
    trip[0::3], trip[1::3], trip[2::3] = F32(1e8), F32(1.0), F32(-1e8)
    out["trip_x"] = trip
    out["trip_dot_ref"] = np.float64(ds_ref.ds_dot(trip, np.ones(3000, F32)))
    MA = rng.standard_normal((6, 40)).astype(F32)
    MB = rng.standard_normal((40, 5)).astype(F32)
    out["mm_a"], out["mm_b"] = MA, MB
    out["mm_ref"] = ds_ref.ds_matmul(MA, MB)

    np.savez_compressed(out_path, **out)
    return out_path


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <reference tree root>")
    p = make(sys.argv[1], os.path.join(HERE, "ds_ref_vectors.npz"))
    print("wrote", p, os.path.getsize(p), "bytes")
