"""Algorithmic FLOP and byte counts of the fused solve / backward kernels.

FLOPs count what the algorithm has to compute with the model's Jacobian
structure exploited (A = I + dt J_x has 27 off-identity nonzeros, B 15), an
FMA as 2, add/mul/sub/div/sqrt/sin/cos as 1, compares and negations as 0.
Per batch element and time step (see ilqr_device.cuh / ilqr_solve.cu /
ilqr_backward.cu for the expressions counted):

  STEP   87   drone_step: p (6), |w| (6), normalise (3), half-angle (2),
              sin/cos (2), em (3), quat_mult (28), thrust quaternion (4),
              rotation (21), velocity (12)
  CAND  102   candidate control: x - X (10), K dx (4 x 19), a k + a K dx, + U (16)
  COST  435   tau^T C tau over a dense 14x14 block (14 x 27 + 28), c^T tau (27), sums
  QUAD  392   l_tau = C tau + c (14 x 28)
  JAC    57   nonzeros of A, B
  RIC  5290   one Riccati step: B^T V (182), Q_uu (136), q_x (68), q_u (30),
              A^T V (580), Q_xu (300), Q_xx (680), Cholesky (38), 11 solves
              (352), K^T Q_uu (280), v (240), V (2400)
  RICM 5250   masked adjoint step (backward)
  SWEEP 229   dU = K dX + k (80), A dX + B dU (92), Jacobian (57)
  GRADC 784   grad_C block (196 x 4)

  solve(element)    = T (STEP + COST) + I T (RIC + QUAD + JAC)
                      + I T n_alpha (CAND + STEP + COST)
  backward(element) = T (RICM + JAC + SWEEP + GRADC)

with I the iterations the element ran. An accepted candidate becomes the new
nominal trajectory as it was rolled out in the line search
(controller.py:360-415), so acceptance adds no work. These structured counts
are below the dense counts of the same algorithm (a dense Riccati step is
about 9.8 kFLOP); the achieved rates reported against them are conservative.

Compulsory bytes (fp32, read once / written once, zero references and
terminal cost as on the FastMPC surface):
  solve    = 40 (x0) + T (16 U_init + 784 C + 56 c) + 40 (T+1) X + T (16 U + 4 tight)
  backward = 40 (T+1) X + T (16 U + 784 C + 4 tight) + 40 (T+1) dL/dX + 16 T dL/dU
             + 40 grad_x0 + T (784 grad_C + 56 grad_c)
"""

from __future__ import annotations

import numpy as np

STEP, CAND, COST, QUAD, JAC = 87, 102, 435, 392, 57
RIC, RICM, SWEEP, GRADC = 5290, 5250, 229, 784


def solve_flops(T: int, n_alpha: int, iters, accepts=None) -> float:
    """Total solve FLOPs for elements that ran `iters` iterations (an array
    over the batch). `accepts` is accepted for callers that track it; it does
    not change the count."""
    I = np.asarray(iters, dtype=np.float64)
    per = T * (STEP + COST) + I * T * (RIC + QUAD + JAC) + I * T * n_alpha * (CAND + STEP + COST)
    return float(per.sum())


# Dense algorithmic counts of the same algorithm (the reference computes these
# products with dense matmuls): per element, a Riccati step with
# quadraticisation 10.3 kFLOP, a line-search candidate step 0.66 kFLOP, the
# initial rollout and linearisation 1.0 kFLOP per step, the backward
# 10.8 kFLOP per step (masked Riccati, sweep, grad_C).
RIC_DENSE, LS_DENSE, INIT_DENSE, BWD_DENSE = 10300, 660, 1000, 10800


def solve_flops_dense(T: int, n_alpha: int, iters) -> float:
    """F = T [I (10.3k + 0.66k n_alpha) + 1.0k] summed over the batch, I the
    iterations each element ran."""
    I = np.asarray(iters, dtype=np.float64)
    return float((T * (I * (RIC_DENSE + LS_DENSE * n_alpha) + INIT_DENSE)).sum())


def backward_flops_dense(T: int, B: int) -> float:
    return float(B) * T * BWD_DENSE


def backward_flops(T: int, B: int) -> float:
    return float(B) * T * (RICM + JAC + SWEEP + GRADC)


def solve_bytes(T: int, B: int) -> float:
    return float(B) * (40 + T * (16 + 784 + 56) + 40 * (T + 1) + T * (16 + 4))


def backward_bytes(T: int, B: int) -> float:
    return float(B) * (40 * (T + 1) + T * (16 + 784 + 4) + 40 * (T + 1) + 16 * T + 40
                       + T * (784 + 56))


# Dense algorithmic counts for the 13-state rotor model (ilqr_dense.cu), per
# element and time step, an FMA as 2:
#   Riccati step 16.9 kFLOP: l_tau = C tau + c (17 x 17), Jacobian (~100),
#     A^T V and (A^T V) A (2 x 13^3), V B and A^T (V B) (2 x 13^2 x 4),
#     B^T V B (4 x 4 x 13), q_x, q_u, Cholesky and 14 solves (~480),
#     M = Q_uu K + Q_ux (4 x 4 x 13), V and v updates (13 x 13 x 8, 13 x 8)
#   line-search candidate step 0.88 kFLOP: K dx (4 x 13), controls and clamp,
#     1/2 tau^T C tau + c^T tau (17 x 17 + 2 x 17), model step (~80)
#   initial rollout step 0.75 kFLOP (the candidate step without K dx)
#   backward step 18.0 kFLOP: the masked Riccati step without the
#     quadraticisation, the dX/dU sweep (K dX, A dX, B dU) and grad_C (17 x 17 x 4)
R13_RIC_DENSE, R13_LS_DENSE, R13_INIT_DENSE, R13_BWD_DENSE = 16900, 880, 750, 18000


def r13_solve_flops_dense(T: int, n_alpha: int, iters) -> float:
    """F = T [I (16.9k + 0.88k n_alpha) + 0.75k] summed over the batch."""
    I = np.asarray(iters, dtype=np.float64)
    return float((T * (I * (R13_RIC_DENSE + R13_LS_DENSE * n_alpha) + R13_INIT_DENSE)).sum())


def r13_backward_flops_dense(T: int, B: int) -> float:
    return float(B) * T * R13_BWD_DENSE
