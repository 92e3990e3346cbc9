"""DS dot_general on the GPU against exact sampled truth and the reference path.

The reference lowers dot_general to four f32 dots with f32 accumulation and a
two_sum (DsTransformPass.cpp:337-370); oracle/ds_pass_ref.py restates it.  No
reference test pins GEMM bits, so parity is error: on every case the GPU
result's error against the exact product (oracle/exact.py) must be no worse
than the reference path's, and within a DS-level bound of sum_k |a_ik b_kj|.
"""
import math

import numpy as np
import pytest

from gpu_util import cu, host
from oracle import ds_pass_ref, exact

pytestmark = pytest.mark.gpu

ALGOS = ["tensor", "cuda_core"]


@pytest.fixture(scope="module")
def ops():
    from ds_b200 import ops as _ops
    return _ops


def ds_of(x):
    """The exact value of the DS split of x (hi + lo)."""
    hi = x.astype(np.float32)
    lo = (x - hi.astype(np.float64)).astype(np.float32)
    return hi.astype(np.float64) + lo.astype(np.float64)


def check_gemm(got, A, B, samples=512, tol_bits=42, ref=None):
    """Sampled-exact error check of C = A @ B (float64 A, B)."""
    M, N = got.shape
    rows, cols = exact.sample_indices(M, N, samples)
    truth = exact.exact_gemm_entries(A, B, rows, cols)
    mag = np.array([np.dot(np.abs(A[r]), np.abs(B[:, c])) for r, c in zip(rows, cols)])
    err = np.abs(got[rows, cols] - truth)
    assert np.all(err <= 2.0 ** -tol_bits * mag + 1e-300), (err / mag).max()
    if ref is not None:
        ref_err = np.abs(ref[rows, cols] - truth)
        assert err.max() <= ref_err.max(), (err.max(), ref_err.max())
    return err.max(), (err / np.maximum(mag, 1e-300)).max()


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("M,N,K", [(1, 7, 5), (5, 1, 9), (33, 17, 65), (128, 256, 128),
                                   (200, 300, 500), (256, 512, 1024),
                                   # rows longer than 4096: A split alone (512 threads a
                                   # row), B's column maxima and split separately
                                   (64, 96, 5000)])
def test_gemm_shapes(ops, algo, M, N, K):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    A = rng.uniform(-1, 1, (M, K))
    B = rng.uniform(-1, 1, (K, N))
    got = host(ops.ds_matmul_f64(cu(A), cu(B), algorithm=algo))
    ref = ds_pass_ref.dot_general_f64(A, B)
    check_gemm(got, A, B, ref=ref)


@pytest.mark.parametrize("algo", ALGOS)
def test_config3_slice(ops, algo):
    """512 x 512 x 4096 slice of the 4096^3 config (A, B ~ U[-1,1], seed 2)."""
    rng = np.random.default_rng(2)
    A = rng.uniform(-1, 1, (512, 4096))
    B = rng.uniform(-1, 1, (4096, 512))
    got = host(ops.ds_matmul_f64(cu(A), cu(B), algorithm=algo))
    ref = ds_pass_ref.dot_general_f64(A, B)
    check_gemm(got, A, B, samples=256, ref=ref)


@pytest.mark.parametrize("algo", ALGOS)
def test_f32_inputs_soa(ops, algo):
    """f32 inputs enter as (v, 0) (emitFromFloat, DsTransformPass.cpp:174-179)."""
    import torch
    rng = np.random.default_rng(3)
    A = rng.standard_normal((96, 160)).astype(np.float32)
    B = rng.standard_normal((160, 80)).astype(np.float32)
    z = lambda a: torch.zeros(a.shape, dtype=torch.float32, device="cuda")
    hi, lo = ops.ds_dot_general(cu(A), z(A), cu(B), z(B), algorithm=algo)
    got = host(hi).astype(np.float64) + host(lo).astype(np.float64)
    A64, B64 = A.astype(np.float64), B.astype(np.float64)
    ref = ds_pass_ref.dot_general_f64(A, B)
    check_gemm(got, A64, B64, samples=300, ref=ref)


@pytest.mark.parametrize("algo", ALGOS)
def test_transposed_and_batched_layouts(ops, algo):
    rng = np.random.default_rng(4)
    At = rng.uniform(-1, 1, (70, 40))   # [K, M]
    Bt = rng.uniform(-1, 1, (50, 70))   # [N, K]
    got = host(ops.ds_dot_general_f64(cu(At), cu(Bt), lhs_contracting=0, rhs_contracting=1,
                                      algorithm=algo))
    check_gemm(got, At.T.copy(), Bt.T.copy(), samples=200)
    Ab = rng.uniform(-1, 1, (3, 20, 30))
    Bb = rng.uniform(-1, 1, (3, 30, 10))
    got = host(ops.ds_dot_general_f64(cu(Ab), cu(Bb), lhs_contracting=2, rhs_contracting=1,
                                      lhs_batch=(0,), rhs_batch=(0,), algorithm=algo))
    for b in range(3):
        check_gemm(got[b], Ab[b], Bb[b], samples=100)


def test_batched_vector_dot(ops):
    """dot_general with batch 0 and contracting 1 on both: config 5's batched dot
    shape (scaled down), entries 1 + 1e-7 u (near-cancellation free sums)."""
    rng = np.random.default_rng(4)
    X = 1.0 + 1e-7 * rng.uniform(-1, 1, (64, 65536))
    Y = 1.0 + 1e-7 * rng.uniform(-1, 1, (64, 65536))
    got = host(ops.ds_dot_general_f64(cu(X), cu(Y), lhs_contracting=1, rhs_contracting=1,
                                      lhs_batch=(0,), rhs_batch=(0,)))
    truth = np.array([exact.exact_dot(X[i], Y[i]) for i in range(64)])
    assert np.max(np.abs(got - truth) / truth) < 2.0 ** -44
    # vector . vector, one long dot product
    v = rng.uniform(-1, 1, 1 << 20)
    w = rng.uniform(-1, 1, 1 << 20)
    d = float(host(ops.ds_dot_general_f64(cu(v), cu(w), lhs_contracting=0, rhs_contracting=0)))
    assert abs(d - exact.exact_dot(v, w)) < 2.0 ** -44 * np.dot(np.abs(v), np.abs(w))


@pytest.mark.parametrize("algo", ALGOS)
def test_reference_edge_cases(ops, algo):
    """tests/test_matmul.py:67-152 and tests/test_dot_product.py:66-176 cases."""
    import torch
    f32 = np.float32

    def mm(A, B):
        A = np.asarray(A, np.float64)
        B = np.asarray(B, np.float64)
        return host(ops.ds_matmul_f64(cu(A), cu(B), algorithm=algo))

    # identity: A @ I == A exactly for DS-representable A
    rng = np.random.default_rng(42)
    A4 = rng.standard_normal((4, 4)).astype(f32).astype(np.float64)
    assert np.array_equal(mm(A4, np.eye(4)), A4)
    # NaN in A row 0 -> that output row has NaN; Inf -> Inf or NaN
    A_nan = np.array([[1.0, np.nan], [3.0, 4.0]])
    r = mm(A_nan, np.ones((2, 2)))
    assert np.all(np.isnan(r[0])) and np.all(np.isfinite(r[1]))
    A_inf = np.array([[1.0, np.inf], [3.0, 4.0]])
    r = mm(A_inf, np.ones((2, 2)))
    assert np.all(np.isinf(r[0]) | np.isnan(r[0])) and np.array_equal(r[1], [7.0, 7.0])
    # subnormal inputs: finite
    r = mm(np.full((3, 4), f32(1.5e-40)), np.ones((4, 3)))
    assert np.all(np.isfinite(r))
    # cancellation rows (test_matmul.py:99-113, :131-148)
    row = np.array([[1e6, -1e6 + 1, 1e6, -1e6 + 1]], f32)
    assert mm(row, np.ones((4, 1)))[0, 0] == 2.0
    trip = np.zeros((1, 99), f32)
    trip[0, 0::3], trip[0, 1::3], trip[0, 2::3] = 1e6, 1.0, -1e6
    assert mm(trip, np.ones((99, 1)))[0, 0] == 33.0
    # zero operand
    assert np.array_equal(mm(np.zeros((5, 6)), rng.random((6, 7))), np.zeros((5, 7)))


def test_precision_highest_256(ops):
    """tests/test_matmul.py:322-341: (A*A) @ B at 256^2 with f32 inputs; DS error
    must not exceed strict-f32 error (the reference's own assertion)."""
    rng = np.random.default_rng(7)
    A = rng.standard_normal((256, 256)).astype(np.float32)
    B = rng.standard_normal((256, 256)).astype(np.float32)
    AA = (A.astype(np.float64) ** 2)
    got = host(ops.ds_matmul_f64(cu(AA), cu(B.astype(np.float64))))
    f64 = AA @ B.astype(np.float64)
    f32 = (A * A) @ B
    assert np.mean(np.abs(got - f64)) <= np.mean(np.abs(f32 - f64))



def test_long_contraction_runs_in_chunks(ops):
    """K above the int32 limit of one u8 residue product (32768) runs as
    chunks on the tensor cores; accuracy stays at the DS level, and an Inf in
    the second chunk reaches the outputs it touches."""
    rng = np.random.default_rng(40)
    M, N, K = 48, 40, 70_001
    A = rng.uniform(-1, 1, (M, K))
    B = rng.uniform(-1, 1, (K, N))
    got = host(ops.ds_matmul_f64(cu(A), cu(B)))
    check_gemm(got, A, B, samples=96, ref=ds_pass_ref.dot_general_f64(A, B))
    A[3, 50_000] = np.inf
    got = host(ops.ds_matmul_f64(cu(A), cu(B)))
    assert np.all(np.isinf(got[3]) | np.isnan(got[3]))
    assert np.all(np.isfinite(np.delete(got, 3, axis=0)))


_ONE_CTA_CHILD = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
from ds_b200 import _lib, ops
assert _lib.gemm_kernel_info()["kernel"] == "single_cta"
rng = np.random.default_rng(31)
A, B = rng.uniform(-1, 1, (512, 1000)), rng.uniform(-1, 1, (1000, 768))
C = ops.ds_matmul_f64(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
sys.stdout.buffer.write(C.cpu().numpy().tobytes())
"""


def test_single_cta_kernel_gives_the_pair_kernels_bits(ops):
    """The one-CTA GEMM (taken when a device cannot co-schedule CTA pairs;
    DS_B200_GEMM_1CTA=1 forces it) computes the same exact residue products,
    so the result equals the pair kernel's bit for bit."""
    import os
    import subprocess
    import sys
    from conftest import PKG_DIR, ROOT
    rng = np.random.default_rng(31)
    A, B = rng.uniform(-1, 1, (512, 1000)), rng.uniform(-1, 1, (1000, 768))
    want = host(ops.ds_matmul_f64(cu(A), cu(B)))
    env = dict(os.environ, DS_B200_GEMM_1CTA="1")
    out = subprocess.run([sys.executable, "-c", _ONE_CTA_CHILD, PKG_DIR, ROOT], env=env,
                         capture_output=True, timeout=600)
    assert out.returncode == 0, out.stderr.decode()[-2000:]
    got = np.frombuffer(out.stdout, dtype=np.float64).reshape(want.shape)
    assert np.array_equal(got.view(np.uint64), want.view(np.uint64))
    check_gemm(got, A, B)


def _wide_cases():
    """Operands whose rows of A or columns of B span many binades, so the
    row (column) maximum that sets the quantisation step does not take part
    in every output.  Seeded; 96 x 640 x 80."""
    M, K, N = 96, 640, 80
    out = {}
    for span in (30, 60):
        rng = np.random.default_rng(100 + span)
        A = rng.uniform(-1, 1, (M, K)) * 2.0 ** -rng.uniform(0, span, (M, K))
        B = rng.uniform(-1, 1, (K, N)) * 2.0 ** -rng.uniform(0, span, (K, N))
        out[f"binades{span}"] = (A, B)
        # a large entry facing a zero: each output is made of the small terms only
        A = rng.uniform(-1, 1, (M, K)) * 2.0 ** -span
        A[:, 0] = 1.0
        B = rng.uniform(-1, 1, (K, N))
        B[0, :] = 0.0
        out[f"large_faces_zero{span}"] = (A, B)
        # the same on the B side, and a large entry facing a small one
        B = rng.uniform(-1, 1, (K, N)) * 2.0 ** -span
        B[3, :] = -4.0
        A = rng.uniform(-1, 1, (M, K))
        A[:, 3] = 2.0 ** -span * rng.uniform(-1, 1, M)
        out[f"large_faces_small{span}"] = (A, B)
    # mixed-sign cancellation inside each row of A
    rng = np.random.default_rng(7)
    A = rng.uniform(-1, 1, (M, K))
    A[:, 1::2] = -A[:, 0::2] * (1 + 2.0 ** -20 * rng.uniform(-1, 1, (M, K // 2)))
    B = 1.0 + 1e-7 * rng.uniform(-1, 1, (K, N))
    out["row_cancellation"] = (A, B)
    # huge entries facing zeros beside ordinary values
    A = rng.uniform(-1, 1, (M, K))
    A[:, 5] = 2.0 ** 40
    B = rng.uniform(-1, 1, (K, N))
    B[5, :] = 0.0
    out["huge_faces_zero"] = (A, B)
    return out


WIDE = _wide_cases()


def assert_no_worse_than_reference(got, A, B, samples=600):
    """Entry by entry: |ours - exact| <= |reference DS path - exact|, or ours
    is within one f64 ulp of the exact value (a correctly rounded f64 cannot
    be beaten, and the reference can land exactly by chance)."""
    M, N = got.shape
    rows, cols = exact.sample_indices(M, N, samples)
    truth = exact.exact_gemm_entries(A, B, rows, cols)
    ref = ds_pass_ref.dot_general_f64(A, B)
    err = np.abs(got[rows, cols] - truth)
    ref_err = np.abs(ref[rows, cols] - truth)
    ulp = np.spacing(np.abs(truth))
    bad = ~((err <= ref_err) | (err <= ulp))
    assert not bad.any(), (int(bad.sum()), err[bad][:4], ref_err[bad][:4], truth[bad][:4])
    return err, ref_err


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("case", sorted(WIDE))
def test_wide_dynamic_range(ops, algo, case):
    """Rows and columns spanning 2^0..2^-30 and 2^0..2^-60, large entries
    facing zeros (outputs made only of small terms), and cancellation inside
    a row: no sampled entry is worse than the reference DS path."""
    A, B = WIDE[case]
    got = host(ops.ds_matmul_f64(cu(A), cu(B), algorithm=algo))
    assert_no_worse_than_reference(got, A, B)


def test_wide_dynamic_range_ds_operands_and_result(ops):
    """The same certificate on SoA DS operands (hi, lo) with a DS result."""
    A, B = WIDE["large_faces_zero60"]
    ah, al = ds_pass_ref.from_float(A)
    bh, bl = ds_pass_ref.from_float(B)
    hi, lo = ops.ds_dot_general(cu(ah), cu(al), cu(bh), cu(bl))
    got = host(hi).astype(np.float64) + host(lo).astype(np.float64)
    A64 = ah.astype(np.float64) + al.astype(np.float64)
    B64 = bh.astype(np.float64) + bl.astype(np.float64)
    # the DS result carries 48 bits: within 2^-46 of the exact value
    rows, cols = exact.sample_indices(*got.shape, 300)
    truth = exact.exact_gemm_entries(A64, B64, rows, cols)
    assert np.all(np.abs(got[rows, cols] - truth) <= 2.0 ** -46 * np.abs(truth))


def test_zero_rows_and_columns_are_exact_zeros(ops):
    """All-zero rows of A and columns of B give +0 outputs without any
    recomputation; the other outputs are unchanged by their presence."""
    rng = np.random.default_rng(11)
    A = rng.uniform(-1, 1, (200, 300))
    B = rng.uniform(-1, 1, (300, 260))
    A[[0, 17, 199]] = 0.0
    B[:, [1, 100]] = 0.0
    got = host(ops.ds_matmul_f64(cu(A), cu(B)))
    assert np.all(got[[0, 17, 199]] == 0.0) and np.all(got[:, [1, 100]] == 0.0)
    assert not np.signbit(got[[0, 17, 199]]).any()
    check_gemm(got, A, B, samples=400, ref=ds_pass_ref.dot_general_f64(A, B))


def test_many_uncertified_outputs_take_the_tiled_recompute(ops):
    """More than 2^20 uncertified outputs (a large entry facing zeros in every
    row): every output is recomputed by the tiled compensated product.  The
    result is no worse than the reference path, and identical across calls."""
    rng = np.random.default_rng(21)
    M, K, N = 1100, 192, 1000
    A = rng.uniform(-1, 1, (M, K)) * 2.0 ** -40
    A[:, 0] = 1.0
    B = rng.uniform(-1, 1, (K, N))
    B[0, :] = 0.0
    dA, dB = cu(A), cu(B)
    got = host(ops.ds_matmul_f64(dA, dB))
    again = host(ops.ds_matmul_f64(dA, dB))
    assert np.array_equal(got.view(np.uint64), again.view(np.uint64))
    assert_no_worse_than_reference(got, A, B, samples=400)


def test_dot_general_dimension_numbers(ops):
    """stablehlo dot_general dimension numbers beyond [batch..., M, K] x
    [batch..., K, N] (the reference's handler clones any of them,
    DsTransformPass.cpp:345-356).  Where the dimensions nest into single
    strides the product reads the operands in place and gives the same bits
    as the 2-D product of the reshaped operands; otherwise one gather copy
    runs first and the result is checked against exact sampled entries."""
    rng = np.random.default_rng(60)
    u = lambda *s: rng.uniform(-1, 1, s)  # noqa: E731
    mm = lambda A, B: host(ops.ds_matmul_f64(cu(A), cu(B)))  # noqa: E731

    def same_bits(got, want):
        assert got.shape == want.shape
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64))

    # [B, S, D] x [D, E], no batch dimensions: [B, S, E]
    A, B = u(3, 70, 96), u(96, 50)
    got = host(ops.ds_dot_general_f64(cu(A), cu(B), lhs_contracting=2, rhs_contracting=0))
    same_bits(got, mm(A.reshape(-1, 96), B).reshape(3, 70, 50))
    # contracting over two dimensions: [M, K1, K2] x [K1, K2, N]
    A, B = u(64, 12, 20), u(12, 20, 48)
    got = host(ops.ds_dot_general_f64(cu(A), cu(B), lhs_contracting=(1, 2),
                                      rhs_contracting=(0, 1)))
    same_bits(got, mm(A.reshape(64, 240), B.reshape(240, 48)))
    # batch dimensions that are not leading: [S, B, K] x [K, B, N] -> [B, S, N]
    A, B = u(40, 3, 64), u(64, 3, 36)
    got = host(ops.ds_dot_general_f64(cu(A), cu(B), lhs_contracting=2, rhs_contracting=0,
                                      lhs_batch=(1,), rhs_batch=(1,)))
    for b in range(3):
        same_bits(got[b], mm(np.ascontiguousarray(A[:, b, :]), np.ascontiguousarray(B[:, b, :])))
    # free dimensions on both sides of a contracting one, and contracting
    # dimensions paired across the operands' orders: these take the gather copy
    A, B = u(6, 64, 9), u(64, 30)            # [F1, K, F2] x [K, N] -> [F1, F2, N]
    got = host(ops.ds_dot_general_f64(cu(A), cu(B), lhs_contracting=1, rhs_contracting=0))
    A2 = A.transpose(0, 2, 1).reshape(54, 64)
    assert got.shape == (6, 9, 30)
    check_gemm(got.reshape(54, 30), A2, B, samples=300, ref=ds_pass_ref.dot_general_f64(A2, B))
    A, B = u(50, 10, 14), u(14, 10, 40)      # A[m, a, b] B[b, a, n], pairs (2, 0), (1, 1)
    got = host(ops.ds_dot_general_f64(cu(A), cu(B), lhs_contracting=(2, 1),
                                      rhs_contracting=(0, 1)))
    A2 = A.transpose(0, 2, 1).reshape(50, 140)
    B2 = B.reshape(140, 40)
    check_gemm(got, A2, B2, samples=300, ref=ds_pass_ref.dot_general_f64(A2, B2))
    # the same through the SoA DS entry
    ah, al = ds_pass_ref.from_float(A)
    bh, bl = ds_pass_ref.from_float(B)
    hi, lo = ops.ds_dot_general(cu(ah), cu(al), cu(bh), cu(bl), lhs_contracting=(2, 1),
                                rhs_contracting=(0, 1))
    got_ds = host(hi).astype(np.float64) + host(lo).astype(np.float64)
    check_gemm(got_ds, ds_of(A2), ds_of(B2), samples=200)
    # no contracting dimension: an outer product [M] x [N] -> [M, N]
    a, b = u(300), u(200)
    got = host(ops.ds_dot_general_f64(cu(a), cu(b), lhs_contracting=(), rhs_contracting=()))
    assert got.shape == (300, 200)
    assert_no_worse_than_reference(got, a[:, None], b[None, :], samples=400)


def test_dot_general_dimension_errors(ops):
    """Mismatched or repeated dimensions are rejected before any launch."""
    import torch
    from ds_b200 import _lib
    A = torch.zeros((4, 5, 6), dtype=torch.float64, device="cuda")
    B = torch.zeros((6, 5, 7), dtype=torch.float64, device="cuda")
    with pytest.raises(_lib.DsInvalidArgument, match="contracting dimensions must match"):
        ops.ds_dot_general_f64(A, B, lhs_contracting=(2, 1), rhs_contracting=(1, 0))
    with pytest.raises(_lib.DsInvalidArgument, match="out of range or repeated"):
        ops.ds_dot_general_f64(A, B, lhs_contracting=(2, 2), rhs_contracting=(0, 0))
    with pytest.raises(_lib.DsInvalidArgument, match="batch dimensions must match"):
        ops.ds_dot_general_f64(A, B, lhs_contracting=2, rhs_contracting=0, lhs_batch=(0,),
                               rhs_batch=(2,))
