"""TEST AND BASELINE INFRASTRUCTURE ONLY -- the reference FastMPC extension's CUDA build,
re-executed on the GPU: its own kernels (oracle/_ref/libfastmpc_ref.so, built
from the reference's sources with its own flags by
oracle/build_fastmpc_ref.py) driven by a torch restatement of the host code
around them:

- solve: drone_ilqr_solve's CUDA branch (differentialMPCPerformance/cpp/
  drone_ilqr_ext.cpp:664-1064): clamp and rollout, compute_cost (:620-663),
  then per iteration the Jacobian kernel, the quadraticisation in ATen ops
  (:797-823), the PNQP-aware Riccati kernel (:826-870), the fused forward
  kernel (:952-980), the candidate costs in ATen ops (:984-1001), min / where
  updates (:1003-1027) and the periodic convergence read (:1029-1049);
- backward: the operator's CUDA path (differentialMPCPerformance/
  mpc_compat.py:217-258): drone_backward_pass_batched (drone_ilqr_ext.cpp:
  1066-1123) and drone_implicit_diff_assembly (:1221-1278).

A recorded decision trace can be replayed, as for the oracles. Only the GPU
parity tests, the fixture generator tests/golden/make_fastmpc_golden.py and
the benchmark's reference-baseline leg (which times the existing FastMPC
CUDA build beside the product) import this module.
"""

from __future__ import annotations

import ctypes
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "oracle", "_ref", "libfastmpc_ref.so")
NX, NU, N = 10, 4, 14
ALPHAS = (1.0, 0.5, 0.25, 0.1)  # drone_ilqr_ext.cpp:736
CHECK_PERIOD = 4                # drone_ilqr_ext.cpp:763

_lib = None


def available() -> bool:
    return os.path.exists(LIB)


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(LIB)
        P, F, I = ctypes.c_void_p, ctypes.c_float, ctypes.c_int
        sig = {
            "fmref_step_jacobian": [P, P, P, P, P, F, I, P],
            "fmref_rollout": [P, P, P, F, I, I, P],
            "fmref_forward": [P, P, P, P, P, P, F, I, I, I, I, P, P, P, P, P],
            "fmref_riccati": [P] * 10 + [F, I, I, P, P, P, P],
            "fmref_riccati_pnqp": [P] * 12 + [F, I, I, P, P, P, P, P],
            "fmref_assembly": [P] * 16 + [I, I, P],
            "fmref_pnqp4": [P] * 7 + [I, P],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _chk(st, what):
    if st != 0:
        raise RuntimeError(f"{what}: CUDA error {st}")


def _f32(t):
    return t.to(torch.float32).contiguous()


def compute_cost(X, U, x_ref, u_ref, C, c, C_f, c_f):
    """drone_ilqr_ext.cpp:620-663."""
    T = U.shape[1]
    z = torch.cat([X[:, :T].reshape(-1, NX) - x_ref[:, :T].reshape(-1, NX),
                   U.reshape(-1, NU) - u_ref[:, :T].reshape(-1, NU)], -1).unsqueeze(-1)
    zt = z.transpose(-1, -2)
    quad = 0.5 * torch.matmul(zt, torch.matmul(C.reshape(-1, N, N), z)).squeeze(-1).squeeze(-1)
    lin = torch.matmul(zt, c.reshape(-1, N).unsqueeze(-1)).squeeze(-1).squeeze(-1)
    cost_run = (quad + lin).view(-1, T).sum(1)
    zN = torch.cat([X[:, T] - x_ref[:, T], torch.zeros_like(U[:, 0])], -1).unsqueeze(-1)
    zNt = zN.transpose(-1, -2)
    quadN = 0.5 * torch.matmul(zNt, torch.matmul(C_f, zN)).squeeze(-1).squeeze(-1)
    linN = torch.matmul(zNt, c_f.unsqueeze(-1)).squeeze(-1).squeeze(-1)
    return cost_run + quadN + linN


def solve(x0, U_init, C, c, u_min=None, u_max=None, dt=0.05, max_iter=5, reg=1e-6, tol=1e-6, forced=None,
          forced_stop=0):
    """drone_ilqr_solve on the reference's kernels, with the FastMPC operator's
    zero terminal cost and references. forced [B, max_iter] (int, the trace
    convention of the oracles) and forced_stop replay decisions. Returns
    dict(X, U, tight, A_lin, B_lin, l_xx, l_uu, l_xu, converged, iters, trace,
    costs [B, max_iter, 4] and best_before [B, max_iter] of each iteration)."""
    L = lib()
    dev = x0.device
    x0, U_init, C, c = _f32(x0), _f32(U_init), _f32(C), _f32(c)
    B, T = U_init.shape[:2]
    zeros = lambda *s: torch.zeros(*s, device=dev)
    C_f, c_f, x_ref, u_ref = zeros(B, N, N), zeros(B, N), zeros(B, T + 1, NX), zeros(B, T, NU)
    bounded = u_min is not None
    U = torch.clamp(U_init, _f32(u_min), _f32(u_max)) if bounded else U_init.clone()
    X = torch.empty(B, T + 1, NX, device=dev)
    _chk(L.fmref_rollout(_p(x0), _p(U), _p(X), dt, B, T, _s()), "rollout")
    best = compute_cost(X, U, x_ref, u_ref, C, c, C_f, c_f)
    alphas = torch.tensor(ALPHAS, device=dev)
    nA = len(ALPHAS)
    free = torch.empty(B, T, NU, device=dev)
    lo, hi = (_f32(u_min), _f32(u_max)) if bounded else (None, None)
    converged, iters = False, 0
    A_lin = B_lin = l_xx = l_uu = l_xu = None
    trace = torch.full((B, max_iter), -128, dtype=torch.long, device=dev)
    cand_costs = torch.full((B, max_iter, nA), float("nan"), device=dev)
    best_before = torch.full((B, max_iter), float("nan"), device=dev)
    for it in range(max_iter):
        iters = it + 1
        xf = X[:, :T].reshape(-1, NX).contiguous()
        uf = U.reshape(-1, NU).contiguous()
        A = torch.empty(B * T, NX, NX, device=dev)
        Bm = torch.empty(B * T, NX, NU, device=dev)
        xn = torch.empty(B * T, NX, device=dev)
        _chk(L.fmref_step_jacobian(_p(xf), _p(uf), _p(xn), _p(A), _p(Bm), dt, B * T, _s()), "jacobian")
        A_lin, B_lin = A.view(B, T, NX, NX), Bm.view(B, T, NX, NU)
        Cfl = C.reshape(-1, N, N)
        cfl = c.reshape(-1, N)
        lxx, luu, lxu = Cfl[:, :NX, :NX], Cfl[:, NX:, NX:], Cfl[:, :NX, NX:]
        ex = (X[:, :T] - x_ref[:, :T]).reshape(-1, NX).unsqueeze(-1)
        eu = (U - u_ref).reshape(-1, NU).unsqueeze(-1)
        lx = torch.matmul(lxx, ex).squeeze(-1) + torch.matmul(lxu, eu).squeeze(-1) + cfl[:, :NX]
        lu = torch.matmul(lxu.transpose(-1, -2), ex).squeeze(-1) + torch.matmul(luu, eu).squeeze(-1) + cfl[:, NX:]
        l_xx = lxx.contiguous().view(B, T, NX, NX)
        l_uu = luu.contiguous().view(B, T, NU, NU)
        l_xu = lxu.contiguous().view(B, T, NX, NU)
        l_x = lx.contiguous().view(B, T, NX)
        l_u = lu.contiguous().view(B, T, NU)
        # l_xxN goes to the kernel as the data pointer of the view
        # C_f[:, :nx, :nx] (drone_ilqr_ext.cpp:822, 841), which the kernel
        # indexes as a contiguous [B, 10, 10] block; C_f is zero here.
        l_xxN_ptr = C_f
        l_xN = torch.matmul(C_f[:, :NX, :NX], (X[:, T] - x_ref[:, T]).unsqueeze(-1)).squeeze(-1) + c_f[:, :NX]
        l_xN = l_xN.contiguous()
        K = torch.empty(B, T, NU, NX, device=dev)
        k = torch.empty(B, T, NU, device=dev)
        if bounded:
            _chk(L.fmref_riccati_pnqp(_p(A), _p(Bm), _p(l_xx), _p(l_uu), _p(l_xu), _p(l_x), _p(l_u),
                                      _p(l_xxN_ptr), _p(l_xN), _p(U), _p(lo), _p(hi), reg, B, T, _p(K), _p(k),
                                      None, _p(free), _s()), "riccati_pnqp")
        else:
            _chk(L.fmref_riccati(_p(A), _p(Bm), _p(l_xx), _p(l_uu), _p(l_xu), _p(l_x), _p(l_u), _p(l_xxN_ptr),
                                 _p(l_xN), None, reg, B, T, _p(K), _p(k), None, _s()), "riccati")
        Xc = torch.empty(B * nA, T + 1, NX, device=dev)
        Uc = torch.empty(B * nA, T, NU, device=dev)
        _chk(L.fmref_forward(_p(x0), _p(X), _p(U), _p(K), _p(k), _p(alphas), dt, B, nA, T, int(bounded), _p(lo),
                             _p(hi), _p(Xc), _p(Uc), _s()), "forward")
        Xv, Uv = Xc.view(B, nA, T + 1, NX), Uc.view(B, nA, T, NU)
        z_run = torch.cat([Xv[:, :, :T] - x_ref[:, :T].unsqueeze(1), Uv - u_ref.unsqueeze(1)], -1)
        Cz = torch.matmul(C.unsqueeze(1), z_run.unsqueeze(-1)).squeeze(-1)
        cost_run = ((0.5 * (z_run * Cz)).sum(-1) + (z_run * c.unsqueeze(1)).sum(-1)).sum(-1)
        z_N = torch.cat([Xv[:, :, T] - x_ref[:, T].unsqueeze(1), torch.zeros(B, nA, NU, device=dev)], -1)
        CfzN = torch.matmul(C_f.unsqueeze(1), z_N.unsqueeze(-1)).squeeze(-1)
        costs = cost_run + ((0.5 * (z_N * CfzN)).sum(-1) + (z_N * c_f.unsqueeze(1)).sum(-1))
        new, idx = costs.min(1)
        improved = new < best
        cand_costs[:, it] = costs
        best_before[:, it] = best
        if forced is not None:
            f = forced[:, it].to(dev).long()
            improved = f >= 0
            idx = torch.where(improved, f, -f - 1).clamp(0, nA - 1)
            new = costs.gather(1, idx.view(B, 1)).squeeze(1)
        trace[:, it] = torch.where(improved, idx, -idx - 1)
        Xb = Xv.gather(1, idx.view(B, 1, 1, 1).expand(B, 1, T + 1, NX)).squeeze(1)
        Ub = Uv.gather(1, idx.view(B, 1, 1, 1).expand(B, 1, T, NU)).squeeze(1)
        X = torch.where(improved.view(B, 1, 1), Xb, X)
        U = torch.where(improved.view(B, 1, 1), Ub, U)
        nb = torch.where(improved, new, best)
        improvement = (best - nb).abs().max()
        best = nb
        if it % CHECK_PERIOD == CHECK_PERIOD - 1 or it == max_iter - 1:
            stop = improvement.item() < tol
            if forced is not None and forced_stop and it + 1 < max_iter:
                stop = it + 1 == forced_stop
            if stop:
                converged = True
                break
    tight = (free < 0.5) if bounded else torch.zeros(B, T, NU, dtype=torch.bool, device=dev)
    return dict(X=X, U=U, tight=tight, A_lin=A_lin, B_lin=B_lin, l_xx=l_xx, l_uu=l_uu, l_xu=l_xu,
                converged=converged, iters=iters, trace=trace, costs=cand_costs, best_before=best_before)


def backward(res, grad_X, grad_U, reg=1e-6):
    """The operator's backward on the CUDA path with the FastMPC operator's zero
    terminal cost and references. Returns dict(x0, C, c)."""
    L = lib()
    X, U = res["X"].contiguous(), res["U"].contiguous()
    B, T = U.shape[:2]
    dev = X.device
    gX, gU = _f32(grad_X), _f32(grad_U)
    l_x = (-gX[:, :T]).contiguous()
    l_u = (-gU).contiguous()
    l_xN = (-gX[:, -1]).contiguous()
    l_xxN = torch.zeros(B, NX, NX, device=dev)
    K = torch.zeros(B, T, NU, NX, device=dev)
    k = torch.zeros(B, T, NU, device=dev)
    v0 = torch.zeros(B, NX, device=dev)
    tight = res["tight"].to(torch.uint8).contiguous()
    _chk(L.fmref_riccati(_p(res["A_lin"]), _p(res["B_lin"]), _p(res["l_xx"]), _p(res["l_uu"]), _p(res["l_xu"]),
                         _p(l_x), _p(l_u), _p(l_xxN), _p(l_xN), _p(tight), reg, B, T, _p(K), _p(k), _p(v0), _s()),
         "adjoint riccati")
    zeros = lambda *s: torch.zeros(*s, device=dev)
    x_ref, u_ref = zeros(B, T + 1, NX), zeros(B, T, NU)
    gC, gc, gx0 = zeros(B, T, N, N), zeros(B, T, N), zeros(B, NX)
    _chk(L.fmref_assembly(_p(K), _p(k), _p(v0), _p(res["A_lin"]), _p(res["B_lin"]), _p(X), _p(U), _p(x_ref),
                          _p(u_ref), _p(gC), _p(gc), _p(gx0), None, None, None, None, B, T, _s()), "assembly")
    return dict(x0=gx0, C=gC, c=gc)


def pnqp4_batch(H, q, lower, upper, x_init=None):
    """The reference's batched PNQP-4 kernel (pnqp_kernel.cu:43,
    ext.drone_pnqp4_batch): (x* [n,4], free mask [n,4])."""
    L = lib()
    H, q, lower, upper = _f32(H), _f32(q), _f32(lower), _f32(upper)
    n = H.shape[0]
    x = torch.empty(n, 4, device=H.device)
    fm = torch.empty(n, 4, device=H.device)
    _chk(L.fmref_pnqp4(_p(H), _p(q), _p(lower), _p(upper), _p(None if x_init is None else _f32(x_init)), _p(x),
                       _p(fm), n, _s()), "pnqp4")
    return x, fm

