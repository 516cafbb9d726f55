"""mpc.pytorch-style MPC operator backed by the B200 iLQR solver.

Drop-in for the reference's differentialMPCPerformance/mpc_compat.py: same
names (QuadCost, GradMethods, FastMPC, MPC, DroneMPCFunction), same call
`MPC(n_state, n_ctrl, T, ...)(x_init, QuadCost(C, c), dx)` returning
(x [T+1,B,nx], u [T,B,nu], objs [T,B]), same layout normalisation and
defaults (mpc_compat.py:80-125, 453-616). Differentiable w.r.t. x_init, C and
c (and C_final, c_final, x_ref, u_ref through DroneMPCFunction) iff
torch.is_grad_enabled() and backprop; otherwise runs under inference_mode.

Behind it: one fused CUDA kernel for the whole forward solve and one for the
implicit-differentiation backward (ilqr_native.solve / .backward), with the
reference DiffMPC's numerics (DifferentialMPC/controller.py): step-size grid
(1, .8, .5, .2, .1) unless overridden (alphas= or ACMPC_DIFFMPC_ALPHAS),
regularisation added twice in the gain solve, strict-improvement acceptance,
isclose tight mask, masked adjoint Riccati with unmasked value update.
n_state=10 is the reference's CTBR quadrotor; n_state=13 selects the 13-state
rotor-thrust rigid body (ilqr_native.rotor13_solve / .rotor13_backward), the
same solver on a model DiffMPC would linearise with GradMethod.AUTO_DIFF.

numerics="fastmpc" (or ACMPC_FASTMPC_NUMERICS=fastmpc) selects instead the
numerics of the reference FastMPC extension's CUDA build
(differentialMPCPerformance/cpp): PNQP-aware Riccati pass, step sizes
(1, .5, .25, .1) with u = U + alpha k + K dx, the quaternion renormalising
step, batch-wide convergence checked every fourth iteration, and its masked
adjoint backward (ilqr_native.fastmpc_solve / .fastmpc_backward).
"""

from __future__ import annotations

import os
from enum import Enum
from typing import NamedTuple, Optional, Union

import torch
from torch import Tensor, nn

try:
    from . import ilqr_native as _nat
    from .drone_ilqr import load_drone_ilqr_ext
except ImportError:
    import ilqr_native as _nat
    from drone_ilqr import load_drone_ilqr_ext

HOVER_THRUST = 0.752 * 9.8066  # mpc_compat.py:117


class QuadCost(NamedTuple):
    """Quadratic cost: 0.5 * z^T C z + c^T z where z = [x; u]"""
    C: Tensor  # [T, B, n, n] or [T, n, n] or [n, n]
    c: Optional[Tensor] = None  # [T, B, n] or [T, n] or [n]


class GradMethods(Enum):
    AUTO_DIFF = 1
    FINITE_DIFF = 2
    ANALYTIC = 3
    ANALYTIC_CHECK = 4


def _outer(x: Tensor, y: Tensor) -> Tensor:
    """Batched outer product: x[..., i] * y[..., j] -> [..., i, j]."""
    return x.unsqueeze(-1) * y.unsqueeze(-2)


# Cached zero tensors keyed by (device, dtype, shape); never written into, and
# never returned as an output (mpc_compat.py:66-77).
_ZERO_CACHE: dict = {}


def _zeros(shape, device, dtype) -> Tensor:
    key = (device, dtype, tuple(shape))
    t = _ZERO_CACHE.get(key)
    if t is None:
        t = torch.zeros(shape, device=device, dtype=dtype)
        _ZERO_CACHE[key] = t
    return t


def _normalize_cost(C: Tensor, c: Optional[Tensor], B: int, T: int, n: int,
                    device, dtype) -> tuple:
    """Bring (C, c) to [B, T, n, n] / [B, T, n] float32 contiguous (mpc_compat.py:80-96)."""
    if C.ndim == 2:
        C = C.unsqueeze(0).unsqueeze(0).expand(T, B, n, n)
    elif C.ndim == 3:
        C = C.unsqueeze(1).expand(T, B, n, n)
    if c is None:
        c = _zeros((T, B, n), device, dtype)
    elif c.ndim == 1:
        c = c.unsqueeze(0).unsqueeze(0).expand(T, B, n)
    elif c.ndim == 2:
        c = c.unsqueeze(1).expand(T, B, n)
    return C.permute(1, 0, 2, 3).contiguous().float(), c.permute(1, 0, 2).contiguous().float()


def _normalize_cost_tm(C: Tensor, c: Optional[Tensor], B: int, T: int, n: int, device, dtype) -> tuple:
    """(C, c) as time-major [T, B, n, n] / [T, B, n] float32 contiguous: the
    QuadCost layout itself, passed to the kernels without the reference's
    transpose to batch-major (a contiguous float32 [T, B, n, n] C is used as
    is, and its gradient comes back in the same layout)."""
    if C.ndim == 2:
        C = C.unsqueeze(0).unsqueeze(0).expand(T, B, n, n)
    elif C.ndim == 3:
        C = C.unsqueeze(1).expand(T, B, n, n)
    if c is None:
        c = _zeros((T, B, n), device, dtype)
    elif c.ndim == 1:
        c = c.unsqueeze(0).unsqueeze(0).expand(T, B, n)
    elif c.ndim == 2:
        c = c.unsqueeze(1).expand(T, B, n)
    return C.contiguous().float(), c.contiguous().float()


def _normalize_bounds(u_lower, u_upper, nu, device, dtype):
    """Flatten box bounds to [nu] float32 (mpc_compat.py:99-110); (None, None)
    when either is missing."""
    if u_lower is None or u_upper is None:
        return None, None

    def _flatten(b: Tensor) -> Tensor:
        if b.ndim == 3:
            return b[0, 0, :].contiguous()
        if b.ndim == 1:
            return b.contiguous()
        return b.flatten()[:nu].contiguous()
    return (_flatten(u_lower).to(device=device, dtype=torch.float32).contiguous(),
            _flatten(u_upper).to(device=device, dtype=torch.float32).contiguous())


def _normalize_init(u_init, B, T, nu, device, dtype, nx: int = 10) -> Tensor:
    """U_init as [B, T, nu] float32; hover thrust when absent (mpc_compat.py:113-125;
    for the 13-state rotor model, the hover fraction on every rotor)."""
    if u_init is None:
        out = torch.zeros(B, T, nu, device=device, dtype=torch.float32)
        if nx == _nat.NX13:
            out[:] = _nat.HOVER_U13
        else:
            out[:, :, 0] = HOVER_THRUST
        return out
    if u_init.ndim == 3:
        out = u_init.permute(1, 0, 2)
    elif u_init.shape == (nu, B):
        out = u_init.t().unsqueeze(1).expand(B, T, nu)
    else:
        out = u_init.unsqueeze(0).expand(B, T, nu)
    return out.to(device=device).contiguous().float()


def _f32(t):
    return None if t is None else t.to(torch.float32).contiguous()


class DroneMPCFunction(torch.autograd.Function):
    """Differentiable batched iLQR solve.

    forward(x0 [B,10], C [B,T,n,n], c [B,T,n], C_final [B,n,n] or None,
    c_final [B,n] or None, x_ref [B,T+1,nx] or None, u_ref [B,T,nu] or None,
    solver_cfg) -> (X [B,T+1,nx], U [B,T,nu]) (C, c time-major [T,B,...] when
    solver_cfg["time_major"]), as the reference's
    DroneMPCFunction (mpc_compat.py:128-185). backward runs the fused
    implicit-diff kernel (ILQRSolve.backward semantics, controller.py:68-133):
    gradients w.r.t. x0, C, c, C_final, c_final, x_ref, u_ref.
    solver_cfg["nx"] == 13 selects the 13-state rotor-thrust model.
    """

    @staticmethod
    def forward(ctx, x0, C_bt, c_bt, C_final, c_final, x_ref, u_ref, solver_cfg):
        r13 = solver_cfg.get("nx", _nat.NX) == _nat.NX13
        ctx.r13 = r13
        ctx.time_major = bool(solver_cfg.get("time_major", False))
        out = (_nat.rotor13_solve if r13 else _nat.solve)(
            _f32(x0), _f32(solver_cfg["U_init"]), _f32(C_bt), _f32(c_bt), _f32(C_final),
            _f32(c_final), _f32(x_ref), _f32(u_ref), solver_cfg.get("u_min"), solver_cfg.get("u_max"),
            dt=solver_cfg["dt"], max_iter=solver_cfg["lqr_iter"], reg_eps=solver_cfg["eps"],
            converge_tol=solver_cfg.get("converge_tol", 1e-6),
            alphas=solver_cfg.get("alphas", _nat.DEFAULT_ALPHAS), time_major=ctx.time_major)
        X, U = out["X"], out["U"]
        ctx.save_for_backward(X, U, _f32(C_bt), _f32(C_final) if C_final is not None else None,
                              _f32(x_ref) if x_ref is not None else None, out["tight"])
        ctx.dt = float(solver_cfg["dt"])
        ctx.reg_eps = float(solver_cfg.get("reg_eps", solver_cfg["eps"]))
        return X, U

    @staticmethod
    def backward(ctx, grad_X, grad_U):
        X, U, C_bt, C_final, x_ref, tight = ctx.saved_tensors
        need = ctx.needs_input_grad
        names = ("x0", "C", "c", "C_final", "c_final", "x_ref", "u_ref")
        want = tuple(nm for nm, nd in zip(names, need[:7]) if nd)
        if not want:
            return (None,) * 8
        gX = torch.zeros_like(X) if grad_X is None else grad_X.to(torch.float32).contiguous()
        gU = torch.zeros_like(U) if grad_U is None else grad_U.to(torch.float32).contiguous()
        bwd = _nat.rotor13_backward if ctx.r13 else _nat.backward
        g = bwd(X, U, C_bt, gX, gU, C_final=C_final, x_ref=x_ref, tight=tight,
                dt=ctx.dt, reg_eps=ctx.reg_eps, need=want, time_major=ctx.time_major)
        return tuple(g.get(nm) for nm in names) + (None,)


class SigmoidQuadCost(NamedTuple):
    """Diagonal quadratic costs given as the policy's sigmoid output
    [B, 28 T] instead of dense C, c. The policy builds C, c from this tensor
    in a Python loop over t (_build_cost_tensors,
    training_modules/mlp_mpc_policy_diffmpc.py:194-247); passing it here
    builds them inside the kernels, and autograd returns the gradient of
    sigmoid_cost. Results equal a QuadCost of the C, c the policy would build.
    range_pt defaults to range_q * mass * 9.806, as in the policy."""
    sigmoid_cost: Tensor
    eps: float = 0.1
    range_q: float = 100000.0
    range_p: float = 100000.0
    mass: float = 0.752
    range_pt: Optional[float] = None

    def spec(self):
        return _nat.SigmoidCostSpec(self.eps, self.range_q, self.range_p, self.mass, self.range_pt)


def _sigmoid_index(T: int, device) -> Tensor:
    """[T, 14] positions in x_q / x_p of each tau entry: _build_cost_tensors
    (training_modules/mlp_mpc_policy_diffmpc.py:204-243) slices the sigmoid
    output into blocks of T steps, p (3), q (4), v (3), w (3), thrust (1), and
    lists them in tau order p, q, v, thrust, w."""
    t = torch.arange(T, device=device)
    cols = [3 * t + i for i in range(3)] + [3 * T + 4 * t + i for i in range(4)]
    cols += [7 * T + 3 * t + i for i in range(3)] + [13 * T + t] + [10 * T + 3 * t + i for i in range(3)]
    return torch.stack(cols, dim=1)


def _sigmoid_to_dense_tm(sc: Tensor, T: int, spec) -> tuple:
    """Dense time-major C [T,B,14,14] (diagonal) and c [T,B,14] from the
    policy's sigmoid output [B, 28 T], differentiable, with
    _build_cost_tensors' operations (mlp_mpc_policy_diffmpc.py:194-247):
    x_q = s * range_q + eps on the diagonal, c = (x_p - 0.5) * range_p, and
    for the thrust entry c = -(x_p * range_pt + eps). For the FastMPC numerics
    mode, whose kernels read dense costs."""
    idx = _sigmoid_index(T, sc.device)
    x_q = sc[:, :14 * T] * spec.range_q + spec.eps
    x_p = sc[:, 14 * T:]
    xp = x_p[:, idx]
    c = (xp - 0.5) * spec.range_p
    c_thrust = -(xp[..., 10] * spec.range_pt + spec.eps)
    c = torch.cat([c[..., :10], c_thrust.unsqueeze(-1), c[..., 11:]], dim=-1)
    C = torch.diag_embed(x_q[:, idx])
    return C.transpose(0, 1).contiguous(), c.transpose(0, 1).contiguous()


class SigmoidMPCFunction(torch.autograd.Function):
    """DroneMPCFunction for SigmoidQuadCost: forward(x0 [B,10],
    sigmoid_cost [B,28T], solver_cfg) -> (X, U); backward returns the
    gradients of x0 and sigmoid_cost."""

    @staticmethod
    def forward(ctx, x0, sigmoid_cost, solver_cfg):
        spec = solver_cfg["sigmoid_spec"]
        sc = _f32(sigmoid_cost)
        out = _nat.solve_sigmoid(
            _f32(x0), _f32(solver_cfg["U_init"]), sc, spec, solver_cfg.get("u_min"), solver_cfg.get("u_max"),
            dt=solver_cfg["dt"], max_iter=solver_cfg["lqr_iter"], reg_eps=solver_cfg["eps"],
            converge_tol=solver_cfg.get("converge_tol", 1e-6),
            alphas=solver_cfg.get("alphas", _nat.DEFAULT_ALPHAS))
        X, U = out["X"], out["U"]
        ctx.save_for_backward(X, U, sc, out["tight"])
        ctx.spec = spec
        ctx.dt = float(solver_cfg["dt"])
        ctx.reg_eps = float(solver_cfg.get("reg_eps", solver_cfg["eps"]))
        return X, U

    @staticmethod
    def backward(ctx, grad_X, grad_U):
        X, U, sc, tight = ctx.saved_tensors
        need = ctx.needs_input_grad
        want = tuple(nm for nm, nd in zip(("x0", "sigmoid_cost"), need[:2]) if nd)
        if not want:
            return None, None, None
        gX = torch.zeros_like(X) if grad_X is None else grad_X.to(torch.float32).contiguous()
        gU = torch.zeros_like(U) if grad_U is None else grad_U.to(torch.float32).contiguous()
        g = _nat.backward_sigmoid(X, U, sc, gX, gU, ctx.spec, tight=tight, dt=ctx.dt,
                                  reg_eps=ctx.reg_eps, need=want)
        return g.get("x0"), g.get("sigmoid_cost"), None


class FastMPCNumericsFunction(torch.autograd.Function):
    """The reference FastMPC operator's autograd function with its own
    numerics (differentialMPCPerformance/mpc_compat.py:128-450 on the CUDA
    build): forward(x0 [B,10], C [T,B,14,14], c [T,B,14], solver_cfg) ->
    (X [B,T+1,10], U [B,T,4]); backward returns the gradients of x0, C, c."""

    @staticmethod
    def forward(ctx, x0, C_tb, c_tb, solver_cfg):
        C32 = _f32(C_tb)
        out = _nat.fastmpc_solve(
            _f32(x0), _f32(solver_cfg["U_init"]), C32, _f32(c_tb), None, None, None, None,
            solver_cfg.get("u_min"), solver_cfg.get("u_max"), dt=solver_cfg["dt"], max_iter=solver_cfg["lqr_iter"],
            reg_eps=solver_cfg["eps"], converge_tol=solver_cfg.get("converge_tol", 1e-6),
            alphas=solver_cfg.get("alphas", _nat.FASTMPC_ALPHAS), time_major=True)
        X, U = out["X"], out["U"]
        bounded = solver_cfg.get("u_min") is not None
        ctx.save_for_backward(X, U, out["X_lin"], out["U_lin"], C32, out["tight"] if bounded else None)
        ctx.dt = float(solver_cfg["dt"])
        ctx.reg_eps = float(solver_cfg.get("reg_eps", solver_cfg["eps"]))
        return X, U

    @staticmethod
    def backward(ctx, grad_X, grad_U):
        X, U, X_lin, U_lin, C32, tight = ctx.saved_tensors
        want = tuple(nm for nm, nd in zip(("x0", "C", "c"), ctx.needs_input_grad[:3]) if nd)
        if not want:
            return None, None, None, None
        gX = torch.zeros_like(X) if grad_X is None else grad_X.to(torch.float32).contiguous()
        gU = torch.zeros_like(U) if grad_U is None else grad_U.to(torch.float32).contiguous()
        g = _nat.fastmpc_backward(X, U, X_lin, U_lin, C32, gX, gU, tight=tight, dt=ctx.dt, reg_eps=ctx.reg_eps,
                                  need=want, time_major=True)
        return g.get("x0"), g.get("C"), g.get("c"), None


class FastMPC(nn.Module):
    """Drop-in replacement for mpc.pytorch's MPC class (mpc_compat.py:453-612).

    Only u_lower/u_upper/u_init/lqr_iter/eps/backprop influence the solve, as
    in the reference; the extra keyword `alphas` selects the line-search step
    sizes (default DiffMPC's (1, .8, .5, .2, .1), or ACMPC_DIFFMPC_ALPHAS).
    n_state selects the model: 10 is the reference's CTBR quadrotor, 13 the
    rotor-thrust rigid body (four rotor thrusts in [0, 1]; dense QuadCost only).
    numerics: "diffmpc" (default) or "fastmpc" (the reference FastMPC build's
    own numerics; 10-state model; a SigmoidQuadCost is turned into the dense
    costs the policy would build; ACMPC_FASTMPC_NUMERICS sets the default).
    """

    def __init__(self, n_state: int, n_ctrl: int, T: int, u_lower: Optional[Tensor] = None,
                 u_upper: Optional[Tensor] = None, u_init: Optional[Tensor] = None,
                 lqr_iter: int = 20, verbose: int = -1, exit_unconverged: bool = False,
                 detach_unconverged: bool = True, linesearch_decay: float = 0.2,
                 max_linesearch_iter: int = 10, grad_method: GradMethods = GradMethods.ANALYTIC,
                 eps: float = 1e-6, n_batch: Optional[int] = None, backprop: bool = True,
                 slew_rate_penalty: Optional[float] = None, prev_ctrl: Optional[Tensor] = None,
                 alphas=None, numerics: Optional[str] = None, **kwargs):
        super().__init__()
        numerics = (numerics or os.environ.get("ACMPC_FASTMPC_NUMERICS", "diffmpc")).strip().lower()
        if numerics not in ("diffmpc", "fastmpc"):
            raise ValueError(f"numerics must be 'diffmpc' or 'fastmpc', not {numerics!r}")
        if numerics == "fastmpc" and n_state != _nat.NX:
            raise ValueError("the FastMPC numerics mode runs the 10-state model")
        self.numerics = numerics
        if n_state not in (_nat.NX, _nat.NX13) or n_ctrl != _nat.NU:
            raise ValueError(f"the solver's models have n_state {_nat.NX} or {_nat.NX13} and n_ctrl={_nat.NU}")
        self.n_state = n_state
        self.n_ctrl = n_ctrl
        self.T = T
        self.u_lower = u_lower
        self.u_upper = u_upper
        self.u_init = u_init
        self.lqr_iter = lqr_iter
        self.verbose = verbose
        self.eps = eps
        self.n_batch = n_batch
        self.backprop = backprop
        self.alphas = tuple(alphas) if alphas is not None else None
        self._ext = None
        self._dt = 0.02
        self._bounds_key = None
        self._bounds = (None, None)

    def _get_ext(self):
        if self._ext is None:
            self._ext = load_drone_ilqr_ext()
        return self._ext

    def _alphas(self):
        if self.alphas is not None:
            return self.alphas
        if self.numerics == "fastmpc":
            return _nat.FASTMPC_ALPHAS
        env = os.environ.get("ACMPC_DIFFMPC_ALPHAS")
        if env:
            return tuple(float(x.strip()) for x in env.split(",") if x.strip())
        return _nat.DEFAULT_ALPHAS

    def _get_bounds(self, device, dtype):
        lo, hi = self.u_lower, self.u_upper
        key = (id(lo), getattr(lo, "_version", None), id(hi), getattr(hi, "_version", None), device)
        if key != self._bounds_key:
            self._bounds = _normalize_bounds(lo, hi, self.n_ctrl, device, dtype)
            self._bounds_key = key
        return self._bounds

    def forward(self, x_init: Tensor, cost: Union[QuadCost, SigmoidQuadCost, nn.Module], dx: nn.Module):
        assert isinstance(cost, (QuadCost, SigmoidQuadCost)), "Only QuadCost (or SigmoidQuadCost) supported"
        B = x_init.size(0)
        T = self.T
        nx, nu = self.n_state, self.n_ctrl
        n = nx + nu
        device = x_init.device
        dtype = x_init.dtype
        dt = getattr(dx, "dt", 0.02)
        self._get_ext()
        sigm = isinstance(cost, SigmoidQuadCost)
        r13 = nx == _nat.NX13
        if sigm and r13:
            raise ValueError("SigmoidQuadCost builds the 10-state policy's costs; use QuadCost with n_state=13")
        if sigm and self.numerics == "fastmpc":
            # the FastMPC kernels read dense costs: build the policy's C, c on
            # the device (autograd carries the gradient back to the sigmoid output)
            C_tb, c_tb = _sigmoid_to_dense_tm(cost.sigmoid_cost.to(torch.float32), T, cost.spec())
            sigm = False
        elif not sigm:
            C_tb, c_tb = _normalize_cost_tm(cost.C, cost.c, B, T, n, device, dtype)
        u_min, u_max = self._get_bounds(device, dtype)
        U_init = _normalize_init(self.u_init, B, T, nu, device, dtype, nx)
        x0 = x_init.float().contiguous()
        cfg = {"U_init": U_init, "u_min": u_min, "u_max": u_max, "dt": float(dt),
               "lqr_iter": self.lqr_iter, "eps": self.eps, "converge_tol": 1e-6,
               "reg_eps": self.eps, "nx": nx, "nu": nu, "alphas": self._alphas(), "time_major": True}
        if sigm:
            cfg["sigmoid_spec"] = cost.spec()
            if torch.is_grad_enabled() and self.backprop:
                X, U = SigmoidMPCFunction.apply(x0, cost.sigmoid_cost, cfg)
            else:
                with torch.inference_mode():
                    out = _nat.solve_sigmoid(x0, U_init, _f32(cost.sigmoid_cost), cfg["sigmoid_spec"], u_min,
                                             u_max, dt=float(dt), max_iter=self.lqr_iter, reg_eps=self.eps,
                                             converge_tol=1e-6, alphas=self._alphas())
                X, U = out["X"], out["U"]
        elif self.numerics == "fastmpc":
            if torch.is_grad_enabled() and self.backprop:
                X, U = FastMPCNumericsFunction.apply(x0, C_tb, c_tb, cfg)
            else:
                with torch.inference_mode():
                    out = _nat.fastmpc_solve(x0, U_init, C_tb, c_tb, None, None, None, None, u_min, u_max,
                                             dt=float(dt), max_iter=self.lqr_iter, reg_eps=self.eps,
                                             converge_tol=1e-6, alphas=self._alphas(), time_major=True)
                X, U = out["X"], out["U"]
        elif torch.is_grad_enabled() and self.backprop:
            X, U = DroneMPCFunction.apply(x0, C_tb, c_tb, None, None, None, None, cfg)
        else:
            with torch.inference_mode():
                out = (_nat.rotor13_solve if r13 else _nat.solve)(
                    x0, U_init, C_tb, c_tb, None, None, None, None, u_min, u_max,
                    dt=float(dt), max_iter=self.lqr_iter, reg_eps=self.eps,
                    converge_tol=1e-6, alphas=self._alphas(), time_major=True)
            X, U = out["X"], out["U"]
        x_out = X.permute(1, 0, 2).contiguous()
        u_out = U.permute(1, 0, 2).contiguous()
        if dtype != torch.float32:
            x_out = x_out.to(dtype)
            u_out = u_out.to(dtype)
        objs = torch.zeros(T, B, device=device, dtype=dtype)
        return x_out, u_out, objs


# Alias for drop-in replacement
MPC = FastMPC
