"""Known-answer tests of the oracles' small linear algebra: the Cholesky and
Cholesky solve of the DiffMPC oracle (torch.linalg.cholesky /
torch.cholesky_solve semantics), the FastMPC build's pivoted 4x4 LU
(backward_pass_kernel.cu:420-496) and PNQP's pivoted solve
(pnqp_kernel.cuh:15-54). The matrices are built from small integers with
power-of-two pivots, so the exact factors are representable in fp32 and the
factorisations must reproduce them exactly. The device kernels are compared
with these oracles in every replay test.
"""

import numpy as np

import oracle as O
from oracle.diffmpc_oracle import _solve4_pivot

F32 = np.float32
L_TRUE = np.array([[2, 0, 0, 0], [1, 1, 0, 0], [3, -1, 2, 0], [1, 2, 1, 4]], F32)
A_SPD = L_TRUE @ L_TRUE.T


def test_cholesky_reproduces_exact_factor():
    L, ok = O.chol4(A_SPD[None].astype(F32))
    assert ok.all()
    assert np.array_equal(L[0], L_TRUE)


def test_cholesky_reads_lower_triangle_and_flags_indefinite():
    A = A_SPD.copy()
    A[0, 3] = 1e6  # upper triangle is never read
    L, ok = O.chol4(A[None])
    assert ok.all() and np.array_equal(L[0], L_TRUE)
    B = A_SPD.copy()
    B[2, 2] = -1.0
    _, ok = O.chol4(B[None])
    assert not ok.any()


def test_cholesky_solve_known_answer():
    x_true = np.array([[1, -2], [3, 0], [-1, 5], [2, 1]], F32)
    R = (A_SPD @ x_true).astype(F32)
    L, _ = O.chol4(A_SPD[None])
    X = O.chol_solve(L, R[None])[0]
    assert np.array_equal(X, x_true)


def test_pivoted_lu_known_answers():
    # needs a row swap at the first step (zero leading pivot)
    P = np.array([[0, 1, 0, 0], [1, 0, 0, 0], [0, 0, 0, 1], [0, 0, 1, 0]], F32)
    A = (P @ A_SPD).astype(F32)
    x_true = np.array([1, -1, 2, -3], F32)
    b = (A @ x_true).astype(F32)
    LU, piv = O.lu_factor4(A[None])
    assert piv[0, 0] != 0
    x = O.lu_solve4(LU, piv, b[None])[0]
    np.testing.assert_allclose(x, x_true, rtol=0, atol=1e-5)
    # a permutation matrix solves exactly
    x = O.lu_solve4(*O.lu_factor4(P[None]), np.array([[4, 3, 2, 1]], F32))[0]
    assert np.array_equal(x, P.T @ np.array([4, 3, 2, 1], F32))


def test_pivoted_lu_tiny_pivot_semantics():
    """A pivot below 1e-10 is replaced by +-1e-10 for the multipliers only; the
    back substitution still divides by the stored (tiny) diagonal, so an
    exactly singular block gives a non-finite solution, as in the reference."""
    A = np.diag(np.array([1.0, 2.0, 0.0, 4.0], F32))[None]
    LU, piv = O.lu_factor4(A)
    with np.errstate(divide="ignore", invalid="ignore"):
        x = O.lu_solve4(LU, piv, np.array([[1, 2, 3, 4]], F32))[0]
    # rows below the zero pivot solve; it and every row above it (0 * inf) do not
    assert x[3] == 1 and not np.isfinite(x[:3]).any()
    # the masked Q_uu of a clamped control: a 1e-11 diagonal and a zero right-hand side give 0
    A = np.diag(np.array([2.0, 1e-11, 4.0, 1.0], F32))[None]
    x = O.lu_solve4(*O.lu_factor4(A), np.array([[2, 0, 8, 1]], F32))[0]
    assert np.array_equal(x, np.array([1, 0, 2, 1], F32))


def test_pnqp_pivoted_solve_known_answer():
    x_true = np.array([2, -1, 0.5, 3], F32)
    x = _solve4_pivot(A_SPD, (A_SPD @ x_true).astype(F32))
    np.testing.assert_allclose(x, x_true, rtol=0, atol=1e-5)
