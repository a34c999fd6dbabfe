"""CPU restatement of the reference's hand-rolled bf16 linear algebra (TEST INFRASTRUCTURE ONLY).

Restates ``ifkfac/bf16_linalg.py`` of the reference (Gsend/ifkfac) in numpy with
explicit bf16 rounding: values are kept in float32 containers and rounded to
the nearest bfloat16 (ties to even) wherever the reference stores a bf16
tensor.  Matrix products accumulate in float32 and round the result to bf16,
which is what torch's bf16 GEMM does on CPU and on tensor cores.  Accumulation
order inside a product can differ from torch's, so agreement with the
reference is to within bf16 rounding, not bitwise (pinned by
``tests/test_oracle_golden.py`` against vectors produced by the reference).

Only tests and the bench's CPU leg may import this module.
"""
from __future__ import annotations

import math

import numpy as np

from .ifk_oracle import bf16_round as _bf


def _norm32(x: np.ndarray) -> np.float32:
    """``_safe_norm`` (``ifkfac/bf16_linalg.py:38-41``): fp32 norm, then bf16."""
    x = x.astype(np.float32)
    return _bf(np.float32(np.sqrt(np.float32(np.dot(x.ravel(), x.ravel()))))).reshape(-1)[0]


def _safe_div(num: np.ndarray, denom, eps: float = 1e-7) -> np.ndarray:
    """``ifkfac/bf16_linalg.py:44-59``: fp32 divide with a magnitude clamp
    |denom| >= eps keeping the sign (sign(0) -> +1), result rounded to bf16."""
    d = np.float32(denom)
    if abs(d) < eps:
        d = np.float32(eps if d >= 0 else -eps)
    return _bf(np.asarray(num, np.float32) / d)


def _mm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """bf16 GEMM: fp32 accumulate, bf16 result."""
    return _bf(a.astype(np.float32) @ b.astype(np.float32))


def block_householder_qr_bf16(A: np.ndarray, block_size: int = 32) -> np.ndarray:
    """Compact-WY blocked Householder QR (``ifkfac/bf16_linalg.py:64-153``).

    Per panel of ``block_size`` columns: unblocked Householder with
    ``alpha = -sign(x0)*||x||`` and unit-norm v (``:105-119``), the T recursion
    ``T[j,:j] = (-2 V[:,:j]^T v_j)^T T[:j,:j]``, ``T[j,j] = 2`` (``:127-137``),
    the in-panel rank-1 update (``:139-143``), then the trailing update
    ``A <- A - V (T (V^T A))`` (``:146-151``).  Returns ``triu(A[:n,:n])``,
    NOT sign-normalised.
    """
    A = _bf(A).copy()
    m, n = A.shape
    assert m >= n
    for i in range(0, n, block_size):
        b = min(block_size, n - i)
        V = np.zeros((m - i, b), np.float32)
        T = np.zeros((b, b), np.float32)
        for j in range(b):
            x = A[i + j:, i + j].copy()
            sgn = np.float32(np.sign(x[0]))
            alpha = _bf(-sgn * _norm32(x)).reshape(-1)[0]
            v = x.copy()
            v[0] = _bf(np.float32(v[0] - alpha)).reshape(-1)[0]
            v_norm = _norm32(v)
            if v_norm == 0.0:
                T[j, j] = 2.0
                continue
            v = _safe_div(v, v_norm)
            V[j:, j] = v
            if j > 0:
                vtv = _mm(V[:, :j].T, V[:, j:j + 1])              # (j, 1)
                T[j, :j] = _mm(_bf(-2.0 * vtv.T), T[:j, :j])[0]
            T[j, j] = 2.0
            panel = A[i + j:, i + j:i + b]
            coeffs = _mm(v[None, :], panel)                        # (1, b-j)
            A[i + j:, i + j:i + b] = _bf(panel - _bf((2.0 * v)[:, None] * coeffs))
        if i + b < n:
            trail = A[i:, i + b:]
            vta = _mm(V.T, trail)
            tvta = _mm(T, vta)
            vtvta = _mm(V, tvta)
            A[i:, i + b:] = _bf(trail - vtvta)
    return np.triu(A[:n, :n])


def solve_triangular_bf16(R: np.ndarray, B: np.ndarray, upper: bool = True) -> np.ndarray:
    """Row-by-row substitution (``ifkfac/bf16_linalg.py:188-242``): each row's
    partial sum is a bf16 GEMM against the solved rows, then a clamped fp32
    divide by the diagonal, stored as bf16."""
    R = _bf(R)
    B = _bf(B)
    n = R.shape[0]
    X = np.zeros_like(B)
    rows = range(n - 1, -1, -1) if upper else range(n)
    for i in rows:
        if upper and i + 1 < n:
            rhs = _bf(B[i:i + 1] - _mm(R[i:i + 1, i + 1:], X[i + 1:]))
        elif (not upper) and i > 0:
            rhs = _bf(B[i:i + 1] - _mm(R[i:i + 1, :i], X[:i]))
        else:
            rhs = B[i:i + 1]
        X[i:i + 1] = _safe_div(rhs, R[i, i])
    return X


def _posdiag(R: np.ndarray) -> np.ndarray:
    s = np.sign(np.diagonal(R)).astype(np.float32)
    s[s == 0] = 1
    return R * s[:, None]


def bf16_factor(X: np.ndarray, damping: float, block_size: int = 32) -> np.ndarray:
    """Damped bf16 factor composed from the reference's bf16 primitives, the
    harness the north star names as the bf16 oracle: blocked QR of the whole
    stack, sign-normalise, scale by 1/sqrt(p), fold [R; sqrt(damping) I] with
    the same QR, sign-normalise (mirrors ``ifkfac/triangular.py:386-421`` and
    ``ifkfac/activation_hooks.py:328-332`` with the bf16 kernels)."""
    p, n = X.shape
    R = _posdiag(block_householder_qr_bf16(_bf(X), block_size))
    R = _bf(R / np.float32(math.sqrt(p)))
    aug = np.concatenate([R, _bf(np.float32(math.sqrt(damping)) * np.eye(n, dtype=np.float32))], 0)
    return _posdiag(block_householder_qr_bf16(aug, block_size))


def bf16_natgrad(grad_W: np.ndarray, R_X: np.ndarray, R_G: np.ndarray) -> np.ndarray:
    """Four bf16 solves in the order of ``apply_vered`` (``ifkfac/triangular.py:630-656``)."""
    g = _bf(grad_W)
    t1 = solve_triangular_bf16(np.ascontiguousarray(R_G.T), g, upper=False)
    t2 = solve_triangular_bf16(R_G, t1, upper=True)
    t3t = solve_triangular_bf16(np.ascontiguousarray(R_X.T), np.ascontiguousarray(t2.T), upper=False)
    t4t = solve_triangular_bf16(R_X, t3t, upper=True)
    return np.ascontiguousarray(t4t.T)
