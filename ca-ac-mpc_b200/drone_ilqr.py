"""Loader for the B200 iLQR solver, mirroring the reference's drone_ilqr.py.

`load_drone_ilqr_ext()` (differentialMPCPerformance/drone_ilqr.py:69-180)
returns an object with the reference extension's entry points and return
tuples (cpp/drone_ilqr_ext.cpp:1321-1386). Instead of JIT-compiling a torch
extension it loads the prebuilt C-ABI library libilqr_b200.so from this
directory (built in-tree by csrc/build.py). The numerics are the reference's
DiffMPC ones (DifferentialMPC/controller.py) by default; numerics="fastmpc"
(or ACMPC_FASTMPC_NUMERICS=fastmpc) gives the reference extension's own: its
solve, its masked adjoint Riccati and its assembly (cpp/drone_ilqr_ext.cpp).

There is no CPU path: the entry points require CUDA float32 tensors and the
loader raises if the library is missing.
"""

from __future__ import annotations

import os
from pathlib import Path
from typing import Optional

import torch

try:
    from . import ilqr_native as _nat
except ImportError:
    import ilqr_native as _nat

_EXT = {}
_CUDA_KERNELS = None
NX, NU, N = _nat.NX, _nat.NU, _nat.N


def _alphas_from_env():
    """Step-size grid: DiffMPC's default (controller.py:211), or the policy's
    ACMPC_DIFFMPC_ALPHAS override (mlp_mpc_policy_diffmpc.py:142-144)."""
    env = os.environ.get("ACMPC_DIFFMPC_ALPHAS")
    if env:
        return tuple(float(x.strip()) for x in env.split(",") if x.strip())
    return _nat.DEFAULT_ALPHAS


def _expand_batch(t: torch.Tensor, B: int, full_dim: int) -> torch.Tensor:
    if t.dim() == full_dim - 1:
        t = t.unsqueeze(0)
    if t.shape[0] == 1 and B > 1:
        t = t.expand(B, *t.shape[1:])
    return t


class DroneIlqrExt:
    """Object returned by load_drone_ilqr_ext(); `numerics` is "diffmpc" or
    "fastmpc"."""

    CUDA_GRAPHS_ENABLED = True

    def __init__(self, numerics: str = "diffmpc"):
        if numerics not in ("diffmpc", "fastmpc"):
            raise ValueError(f"numerics must be 'diffmpc' or 'fastmpc', not {numerics!r}")
        self.numerics = numerics
        _nat.lib()
        self._graphs_enabled = False
        self._graph_debug = False
        self._graph_status = (False, 0, 0)

    # ---- drone_ilqr_solve (cpp/drone_ilqr_ext.cpp:664-1064) -----------------
    def drone_ilqr_solve(self, x0, U_init, C, c, C_final, c_final, x_ref, u_ref, u_min, u_max,
                         dt, max_iter, reg_eps, converge_tol):
        """Returns (X, U, l_xx, l_uu, l_xu, l_xxN, A_lin, B_lin, tight_mask, converged)."""
        B = x0.shape[0]
        T = U_init.shape[1]
        dev = x0.device
        f = lambda t: t.to(device=dev, dtype=torch.float32).contiguous()
        C_b = f(_expand_batch(C, B, 4))
        c_b = f(_expand_batch(c, B, 3))
        C_f = f(_expand_batch(C_final, B, 3))
        c_f = f(_expand_batch(c_final, B, 2))
        xr = _expand_batch(x_ref, B, 3)
        if xr.shape[1] == 1:
            xr = xr.expand(B, T + 1, NX)
        ur = _expand_batch(u_ref, B, 3)
        if ur.shape[1] == 1:
            ur = ur.expand(B, T, NU)
        xr, ur = f(xr), f(ur)
        has_bounds = u_min.numel() > 0 and u_max.numel() > 0
        lo = f(u_min.reshape(-1)[:NU]) if has_bounds else None
        hi = f(u_max.reshape(-1)[:NU]) if has_bounds else None
        l_xx = C_b[..., :NX, :NX].contiguous()
        l_uu = C_b[..., NX:, NX:].contiguous()
        l_xu = C_b[..., :NX, NX:].contiguous()
        l_xxN = C_f[..., :NX, :NX].contiguous()
        if self.numerics == "fastmpc":
            # the extension's own loop; A_lin, B_lin where its last Riccati
            # pass linearised (drone_ilqr_ext.cpp:771-795, 1063)
            out = _nat.fastmpc_solve(f(x0), f(U_init), C_b, c_b, C_f, c_f, xr, ur, lo, hi, dt=float(dt),
                                     max_iter=int(max_iter), reg_eps=float(reg_eps),
                                     converge_tol=float(converge_tol))
            A_lin, B_lin = _nat.fastmpc_linearize(out["X_lin"], out["U_lin"], float(dt))
            converged = bool(int(out["batch_info"][0]))
            return (out["X"], out["U"], l_xx, l_uu, l_xu, l_xxN, A_lin, B_lin, out["tight"].bool(), converged)
        out = _nat.solve(f(x0), f(U_init), C_b, c_b, C_f, c_f, xr, ur, lo, hi, dt=float(dt),
                         max_iter=int(max_iter), reg_eps=float(reg_eps),
                         converge_tol=float(converge_tol), alphas=_alphas_from_env(),
                         want_stats=True)
        X, U = out["X"], out["U"]
        A_lin, B_lin = _nat.linearize(X, U, float(dt))
        converged = _nat.converged_flag(out["stall_iter"], out["stall_gap"], out["status"],
                                        int(max_iter), float(converge_tol))
        return (X, U, l_xx, l_uu, l_xu, l_xxN, A_lin, B_lin, out["tight"].bool(), converged)

    # ---- drone_backward_pass_batched (cpp/drone_ilqr_ext.cpp:1066-1177) ------
    def drone_backward_pass_batched(self, A_lin, Bm_lin, l_xx, l_uu, l_xu, l_x, l_u, l_xxN, l_xN,
                                    tight_mask, reg_eps):
        """Masked adjoint Riccati (DiffMPC semantics, or the extension's own
        with numerics="fastmpc"); returns (K, k, v0)."""
        f = lambda t: t.to(torch.float32).contiguous()
        tm = None
        if isinstance(tight_mask, torch.Tensor) and tight_mask.numel() > 0:
            tm = tight_mask.to(torch.uint8).contiguous()
        if self.numerics == "fastmpc":
            return _nat.fastmpc_adjoint_lqr(f(A_lin), f(Bm_lin), f(l_xx), f(l_uu), f(l_xu), f(l_x), f(l_u),
                                            f(l_xxN), f(l_xN), tm, float(reg_eps))
        return _nat.adjoint_lqr(f(A_lin), f(Bm_lin), f(l_xx), f(l_uu), f(l_xu), f(l_x), f(l_u),
                                f(l_xxN), f(l_xN), tm, float(reg_eps))

    # ---- drone_implicit_diff_assembly (cpp/drone_ilqr_ext.cpp:1221-1278) -----
    def drone_implicit_diff_assembly(self, K_seq, k_seq, v0, A_lin, Bm_lin, X, U, x_ref, u_ref,
                                     compute_xref=False, compute_uref=False,
                                     compute_C_final=False, compute_c_final=False):
        """Returns (grad_C, grad_c, grad_x0, grad_xref, grad_uref, grad_C_final,
        grad_c_final); skipped outputs are None."""
        f = lambda t: None if t is None else t.to(torch.float32).contiguous()
        if self.numerics == "fastmpc":
            return _nat.fastmpc_assembly(f(K_seq), f(k_seq), f(v0), f(A_lin), f(Bm_lin), f(X), f(U), f(x_ref),
                                         f(u_ref), bool(compute_xref), bool(compute_uref), bool(compute_C_final),
                                         bool(compute_c_final))
        return _nat.implicit_diff_assembly(f(K_seq), f(k_seq), f(v0), f(A_lin), f(Bm_lin), f(X),
                                           f(U), f(x_ref), f(u_ref), bool(compute_xref),
                                           bool(compute_uref), bool(compute_C_final),
                                           bool(compute_c_final))

    # ---- drone_pnqp4_batch (cpp/drone_ilqr_ext.cpp:1285-1316) ----------------
    def drone_pnqp4_batch(self, H, q, lower, upper, x_init=None):
        """n independent 4-d box QPs: returns (x* [n,4], free_mask [n,4]).
        An empty or absent x_init starts from the unconstrained solution."""
        f = lambda t: t.to(torch.float32).contiguous()
        xi = None if x_init is None or x_init.numel() == 0 else f(x_init)
        return _nat.pnqp4_batch(f(H), f(q), f(lower), f(upper), xi)

    # ---- CUDA-graph helpers (cpp/drone_ilqr_ext.cpp:1181-1212) ---------------
    def clear_cuda_graph_cache(self):
        self._graph_status = (False, 0, 0)

    def get_cuda_graph_status(self):
        return self._graph_status

    def set_cuda_graph_debug(self, enable: bool):
        self._graph_debug = bool(enable)

    def enable_cuda_graphs(self, enable: bool):
        self._graphs_enabled = bool(enable)
        if not enable:
            self.clear_cuda_graph_cache()

    # Direct access to the fused kernels (used by mpc_compat).
    solve = staticmethod(_nat.solve)
    backward = staticmethod(_nat.backward)
    dynamics = staticmethod(_nat.dynamics)
    linearize = staticmethod(_nat.linearize)


def load_drone_ilqr_ext(*, build_directory: Optional[Path] = None, verbose: bool = False,
                        force_rebuild: bool = False, with_fused_kernels: bool = True,
                        numerics: Optional[str] = None):
    """Return the solver extension object (one per numerics, loaded once). The
    keyword arguments of the reference loader are accepted; the library is
    prebuilt in-tree. numerics: "diffmpc" (default) or "fastmpc", the default
    taken from ACMPC_FASTMPC_NUMERICS."""
    numerics = (numerics or os.environ.get("ACMPC_FASTMPC_NUMERICS", "diffmpc")).strip().lower()
    if numerics in _EXT and not force_rebuild:
        return _EXT[numerics]
    if force_rebuild:
        import importlib.util
        spec = importlib.util.spec_from_file_location(
            "ilqr_build", os.path.join(os.path.dirname(os.path.abspath(__file__)), "csrc", "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build(verbose=verbose)
    _EXT[numerics] = DroneIlqrExt(numerics)
    return _EXT[numerics]


def load_drone_cuda_kernels(*, build_directory: Optional[Path] = None, verbose: bool = False,
                            force_rebuild: bool = False):
    """Mirror of the reference's kernel loader (drone_ilqr.py:14-66): returns
    the native module exposing the model step and Jacobian kernels."""
    global _CUDA_KERNELS
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA not available, cannot load CUDA kernels")
    if _CUDA_KERNELS is None or force_rebuild:
        _nat.lib()
        _CUDA_KERNELS = _nat
    return _CUDA_KERNELS
