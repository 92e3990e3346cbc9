"""Exact ground truth for DS error reports (test infrastructure only).

- sums: math.fsum, correctly rounded sum of the f64 inputs;
- dot products / GEMM entries: every f64 product expanded exactly into two
  f64 terms with Dekker's algorithm (Veltkamp split 2^27+1), then math.fsum.
  A float64 DGEMM is not accurate enough to score a ~48-bit DS result, so
  GEMM errors are measured on a fixed sample of output entries against this.
"""
from __future__ import annotations

import math

import numpy as np

_SPLIT = 134217729.0  # 2**27 + 1


def _split64(a):
    t = _SPLIT * a
    hi = t - (t - a)
    return hi, a - hi


def two_prod64(a, b):
    """Exact a*b = p + e for float64 arrays (no overflow/underflow assumed)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    p = a * b
    ah, al = _split64(a)
    bh, bl = _split64(b)
    e = ((ah * bh - p) + ah * bl + al * bh) + al * bl
    return p, e


def exact_sum(x) -> float:
    return math.fsum(np.asarray(x, np.float64).ravel().tolist())


def exact_dot(a, b) -> float:
    p, e = two_prod64(a, b)
    return math.fsum(np.concatenate([p.ravel(), e.ravel()]).tolist())


def sample_indices(M, N, count, seed=12345):
    rng = np.random.default_rng(seed)
    count = min(count, M * N)
    flat = rng.choice(M * N, size=count, replace=False)
    return flat // N, flat % N


def exact_gemm_entries(A, B, rows, cols):
    """Correctly rounded C[rows[i], cols[i]] of A @ B (A[M,K], B[K,N] float64)."""
    A = np.asarray(A, np.float64)
    B = np.asarray(B, np.float64)
    out = np.empty(len(rows), np.float64)
    for i, (r, c) in enumerate(zip(rows, cols)):
        out[i] = exact_dot(A[r], B[:, c])
    return out
