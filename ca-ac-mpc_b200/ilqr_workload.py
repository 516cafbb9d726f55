"""Seeded synthetic solve workloads for the batched quadrotor iLQR solver.

The reference publishes no dataset for this path; its policy builds the cost
tensors from a sigmoid MLP (acmpc_public-master/training_modules/
mlp_mpc_policy_diffmpc.py:194-247: diagonal C stored dense, linear term c).
These generators stand in for that with the same shapes and value ranges:

* x0: position (0,0,1) + N(0, 0.1^2), unit quaternion (1,0,0,0),
  velocity N(0, 0.2^2).
* C[b,t]: diagonal, all 14 entries log-uniform in [1e-2, 1e2], drawn
  independently per (b, t), stored dense [B, T, 14, 14] (the operator
  contract is dense).
* c[b,t] = -C[b,t] tau_ref[b] with tau_ref = (r, 1,0,0,0, 0,0,0, m g, 0,0,0)
  and r uniform in a 10 m cube (or on a sphere of given radius: the
  long-horizon stress case uses 15 m so that the control box binds).
* U_init = hover (fc = 0.752 * 9.8066, zero body rates).
* Control box [0, -10, -10, -4] .. [34, 10, 10, 4] (mlp_mpc_policy_diffmpc.py:132-134).
* Backward seeds dL/dX, dL/dU ~ N(0, 1).

Elements are drawn in blocks of 1024 from generators keyed by (seed, block),
so the first n elements of a batch are identical whatever the batch size:
tests can take a prefix of a large workload.
"""

from __future__ import annotations

import numpy as np

NX, NU, N = 10, 4, 14
MASS = 0.752
G = 9.8066
HOVER_THRUST = MASS * G
U_MIN = np.array([0.0, -10.0, -10.0, -4.0], dtype=np.float32)
U_MAX = np.array([34.0, 10.0, 10.0, 4.0], dtype=np.float32)
BLOCK = 1024

# The five workloads the reference's benchmark plan names (batch, horizon,
# iterations, step sizes, target radius or cube half-width, backward?).
CONFIGS = {
    "latency_b16_t5": dict(B=16, T=5, max_iter=10, alphas=(1.0, 0.8, 0.5, 0.2, 0.1),
                           target="cube", r=5.0, backward=True),
    "b1024_t10": dict(B=1024, T=10, max_iter=10, alphas=(1.0, 0.8, 0.5, 0.2, 0.1),
                      target="cube", r=5.0, backward=True),
    "rollout_b16384_t20": dict(B=16384, T=20, max_iter=5, alphas=(1.0, 0.8, 0.5, 0.2, 0.1),
                               target="cube", r=5.0, backward=True),
    "inference_b262144_t10": dict(B=262144, T=10, max_iter=10, alphas=(1.0, 0.8, 0.5, 0.2, 0.1),
                                  target="cube", r=5.0, backward=False),
    "stress_b65536_t50": dict(B=65536, T=50, max_iter=8, alphas=(1.0, 0.5, 0.25, 0.125),
                              target="sphere", r=15.0, backward=True),
}
DT = 0.05
REG_EPS = 1e-6
CONVERGE_TOL = 1e-6


def _block_inputs(seed: int, block: int, T: int, target: str, r: float):
    rng = np.random.default_rng([seed, block])
    x0 = np.zeros((BLOCK, NX))
    x0[:, 0:3] = np.array([0.0, 0.0, 1.0]) + rng.normal(0.0, 0.1, (BLOCK, 3))
    x0[:, 3] = 1.0
    x0[:, 7:10] = rng.normal(0.0, 0.2, (BLOCK, 3))
    diag = np.exp(rng.uniform(np.log(1e-2), np.log(1e2), (BLOCK, T, N)))
    if target == "cube":
        ref = rng.uniform(-r, r, (BLOCK, 3))
    else:
        d = rng.normal(size=(BLOCK, 3))
        ref = r * d / np.linalg.norm(d, axis=1, keepdims=True)
    return x0, diag, ref


def make_inputs(B: int, T: int, seed: int = 0, target: str = "cube", r: float = 5.0,
                offset: int = 0):
    """Solve inputs for a batch of B elements and horizon T (float32 numpy).

    `offset` (a multiple of 1024) selects elements [offset, offset + B) of the
    seeded stream. Returns dict(x0 [B,10], C [B,T,14,14], c [B,T,14], U_init [B,T,4]).
    """
    assert offset % BLOCK == 0
    b_off = offset // BLOCK
    x0 = np.empty((B, NX), dtype=np.float32)
    C = np.zeros((B, T, N, N), dtype=np.float32)
    c = np.empty((B, T, N), dtype=np.float32)
    idx = np.arange(N)
    for blk in range((B + BLOCK - 1) // BLOCK):
        lo, hi = blk * BLOCK, min(B, (blk + 1) * BLOCK)
        n = hi - lo
        bx0, bdiag, bref = _block_inputs(seed, blk + b_off, T, target, r)
        x0[lo:hi] = bx0[:n]
        d32 = bdiag[:n].astype(np.float32)
        C[lo:hi, :, idx, idx] = d32
        tau = np.zeros((n, N), dtype=np.float32)
        tau[:, 0:3] = bref[:n]
        tau[:, 3] = 1.0
        tau[:, 10] = np.float32(HOVER_THRUST)
        # c = -C tau_ref; C is diagonal so the product is exact per entry.
        c[lo:hi] = -(d32 * tau[:, None, :])
    U_init = np.zeros((B, T, NU), dtype=np.float32)
    U_init[:, :, 0] = np.float32(HOVER_THRUST)
    return dict(x0=x0, C=C, c=c, U_init=U_init)


def make_backward_seeds(B: int, T: int, seed: int = 1, offset: int = 0, nx: int = NX):
    """Upstream gradients dL/dX [B,T+1,nx], dL/dU [B,T,4] ~ N(0,1)."""
    assert offset % BLOCK == 0
    gX = np.empty((B, T + 1, nx), dtype=np.float32)
    gU = np.empty((B, T, NU), dtype=np.float32)
    for blk in range((B + BLOCK - 1) // BLOCK):
        lo, hi = blk * BLOCK, min(B, (blk + 1) * BLOCK)
        rng = np.random.default_rng([seed, blk + offset // BLOCK])
        gX[lo:hi] = rng.normal(size=(BLOCK, T + 1, nx))[: hi - lo]
        gU[lo:hi] = rng.normal(size=(BLOCK, T, NU))[: hi - lo]
    return gX, gU


def make_dense_costs(B: int, T: int, seed: int = 7, asymmetric: bool = False):
    """General (non-diagonal) cost tensors for testing the dense-C path:
    C = G G^T / 14 + diag(log-uniform) (SPD), optionally plus a skew part;
    c ~ N(0, 5^2); terminal C_f SPD, c_f, references x_ref/u_ref ~ N(0, 0.1)."""
    rng = np.random.default_rng(seed)
    Gm = rng.normal(size=(B, T, N, N)) * 0.3
    C = Gm @ np.swapaxes(Gm, -1, -2) / N
    C += np.eye(N) * np.exp(rng.uniform(np.log(1e-1), np.log(1e1), (B, T, N)))[..., None]
    if asymmetric:
        S = rng.normal(size=(B, T, N, N)) * 0.05
        C = C + (S - np.swapaxes(S, -1, -2))
    c = rng.normal(0.0, 5.0, size=(B, T, N))
    Gf = rng.normal(size=(B, N, N)) * 0.3
    C_f = Gf @ np.swapaxes(Gf, -1, -2) / N
    c_f = rng.normal(0.0, 1.0, size=(B, N))
    x_ref = rng.normal(0.0, 0.1, size=(B, T + 1, NX))
    u_ref = rng.normal(0.0, 0.1, size=(B, T, NU))
    f = lambda a: a.astype(np.float32)
    return dict(C=f(C), c=f(c), C_final=f(C_f), c_final=f(c_f), x_ref=f(x_ref), u_ref=f(u_ref))


def config_inputs(name: str, B: int | None = None, seed: int = 0):
    """Inputs for one of CONFIGS (optionally only its first B elements)."""
    cfg = CONFIGS[name]
    nb = cfg["B"] if B is None else B
    inp = make_inputs(nb, cfg["T"], seed=seed, target=cfg["target"], r=cfg["r"])
    return cfg, inp


# --------------------------------------------------------------------------
# 13-state rotor-thrust quadrotor (rotor13): state p, q, v, w; four rotor
# thrusts as fractions of 8.5 N in the box [0, 1]; mass 0.75 kg.
# --------------------------------------------------------------------------

NX13 = 13
N13 = NX13 + NU
MASS13 = 0.75
F_MAX13 = 8.5
HOVER_U13 = MASS13 * G / (4.0 * F_MAX13)
U_MIN13 = np.zeros(NU, dtype=np.float32)
U_MAX13 = np.ones(NU, dtype=np.float32)


def make_rotor13_inputs(B: int, T: int, seed: int = 0, target: str = "cube", r: float = 5.0,
                        offset: int = 0):
    """Rotor13 solve inputs with the same draws as make_inputs:
    x0 = hover at (0,0,1) + N(0, 0.1^2) position and N(0, 0.2^2) velocity
    noise, identity attitude, zero body rates; C[b,t] diagonal, all 17
    entries log-uniform in [1e-2, 1e2]; c[b,t] = -C[b,t] tau_ref[b] with
    tau_ref = (r, 1,0,0,0, 0,0,0, 0,0,0, hover x4) and r in a 10 m cube (or
    on a sphere); U_init = hover thrust on every rotor.
    Returns dict(x0 [B,13], C [B,T,17,17], c [B,T,17], U_init [B,T,4])."""
    assert offset % BLOCK == 0
    b_off = offset // BLOCK
    x0 = np.zeros((B, NX13), dtype=np.float32)
    C = np.zeros((B, T, N13, N13), dtype=np.float32)
    c = np.empty((B, T, N13), dtype=np.float32)
    idx = np.arange(N13)
    for blk in range((B + BLOCK - 1) // BLOCK):
        lo, hi = blk * BLOCK, min(B, (blk + 1) * BLOCK)
        n = hi - lo
        rng = np.random.default_rng([seed, 13, blk + b_off])
        p0 = np.array([0.0, 0.0, 1.0]) + rng.normal(0.0, 0.1, (BLOCK, 3))
        v0 = rng.normal(0.0, 0.2, (BLOCK, 3))
        diag = np.exp(rng.uniform(np.log(1e-2), np.log(1e2), (BLOCK, T, N13)))
        if target == "cube":
            ref = rng.uniform(-r, r, (BLOCK, 3))
        else:
            d = rng.normal(size=(BLOCK, 3))
            ref = r * d / np.linalg.norm(d, axis=1, keepdims=True)
        x0[lo:hi, 0:3] = p0[:n]
        x0[lo:hi, 3] = 1.0
        x0[lo:hi, 7:10] = v0[:n]
        d32 = diag[:n].astype(np.float32)
        C[lo:hi, :, idx, idx] = d32
        tau = np.zeros((n, N13), dtype=np.float32)
        tau[:, 0:3] = ref[:n]
        tau[:, 3] = 1.0
        tau[:, NX13:] = np.float32(HOVER_U13)
        c[lo:hi] = -(d32 * tau[:, None, :])
    U_init = np.full((B, T, NU), np.float32(HOVER_U13), dtype=np.float32)
    return dict(x0=x0, C=C, c=c, U_init=U_init)


def rotor13_config_inputs(name: str, B: int | None = None, seed: int = 0):
    """Rotor13 inputs for one of CONFIGS (optionally its first B elements)."""
    cfg = CONFIGS[name]
    nb = cfg["B"] if B is None else B
    return cfg, make_rotor13_inputs(nb, cfg["T"], seed=seed, target=cfg["target"], r=cfg["r"])
