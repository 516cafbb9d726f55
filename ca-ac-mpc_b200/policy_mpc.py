"""The MPC part of the policy's actor as one batched call.

CustomNetworkDiffMPC.forward_actor (acmpc_public-master/training_modules/
mlp_mpc_policy_diffmpc.py:300-434) splits the batch into chunks of
ACMPC_MPC_CHUNK (1024) elements; for each chunk it builds dense C, c with a
Python loop over t, solves, copies X, U into the nominal buffers and reads a
NaN/inf flag back to the host (`.cpu().item()`, one sync per chunk). It then
keeps U[:, 0] as the next warm start and normalises the first action.

PolicyMPC.actor does the same with one solve over the whole batch: the costs
are built inside the kernels from the sigmoid output (SigmoidQuadCost), the
warm start stays on the device, and the per-chunk NaN/inf count is formed on
the device; nothing reads back to the host. Per-element results do not depend
on the chunking (elements are independent), so the actions equal the
reference loop's on the same solver.
"""

from __future__ import annotations

import os
from typing import Optional

import torch
from torch import Tensor

import ilqr_native as _nat
import mpc_compat

GZ = 9.8066  # drone.py:187, and the hover thrust of _hover_u_init (:249-252)


class PolicyMPC:
    """Solver state of the actor: the warm start u_prev [B, 4] (kept on the
    device between calls made without gradients, as the reference does) and
    the last predictions [B, T, 14].

    Constants follow DroneDx (drone.py:166-203): mass, thrust_max per rotor,
    omega_max; the control box is [4 thrust_min, -omega_max] ..
    [4 thrust_max, omega_max] (mlp_mpc_policy_diffmpc.py:166-177). numerics:
    as FastMPC's ("diffmpc" by default, or "fastmpc")."""

    def __init__(self, T: int, dt: float, lqr_iter: Optional[int] = None, eps: float = 0.1,
                 alphas=None, mass: float = 0.752, thrust_min: float = 0.0, thrust_max: float = 8.5,
                 omega_max=(10.0, 10.0, 4.0), grad_mode: str = "diff", chunk: Optional[int] = None,
                 device=None, numerics: Optional[str] = None):
        self.T = int(T)
        self.dt = float(dt)
        self.lqr_iter = int(os.environ.get("ACMPC_MPC_MAX_ITER", "1")) if lqr_iter is None else int(lqr_iter)
        self.eps = float(eps)
        self.mass = float(mass)
        self.thrust_max = float(thrust_max)
        self.device = torch.device("cuda") if device is None else torch.device(device)
        self.omega_max = torch.tensor(omega_max, dtype=torch.float32, device=self.device)
        self.grad_mode = grad_mode
        # chunk length of the reference's NaN/inf metric (ACMPC_MPC_CHUNK)
        self.chunk = int(os.environ.get("ACMPC_MPC_CHUNK", "1024")) if chunk is None else int(chunk)
        lo = torch.tensor([4.0 * thrust_min, -omega_max[0], -omega_max[1], -omega_max[2]], device=self.device)
        hi = torch.tensor([4.0 * thrust_max, omega_max[0], omega_max[1], omega_max[2]], device=self.device)
        self.solver = mpc_compat.FastMPC(10, 4, self.T, u_lower=lo.view(1, 1, 4).expand(self.T, 1, 4),
                                         u_upper=hi.view(1, 1, 4).expand(self.T, 1, 4),
                                         lqr_iter=self.lqr_iter, eps=self.eps, alphas=alphas, numerics=numerics)
        self._dx = type("Dx", (), {"dt": self.dt})()
        self.u_prev: Optional[Tensor] = None
        self.predictions: Optional[Tensor] = None
        self.naninf_chunks: Optional[Tensor] = None  # device scalar; read it when needed

    def actor(self, sigmoid_cost: Tensor, states: Tensor) -> Tensor:
        """Normalised first actions [B, 4] (thrust, body rates) for states
        [B, >= 10] and the policy network's sigmoid output [B, 28 T]."""
        states = states.float()
        if states.ndimension() == 1:
            states = states.unsqueeze(0)
        x0 = states[:, 0:10].to(self.device)
        B = x0.shape[0]
        warm = not torch.is_grad_enabled()
        if warm and (self.u_prev is None or self.u_prev.shape[0] != B):
            self.u_prev = torch.zeros(B, 4, device=self.device)
            self.u_prev[:, 0] = self.mass * GZ
        if warm:
            u_init = self.u_prev.unsqueeze(1).expand(-1, self.T, -1)
        else:
            u_init = torch.zeros(B, self.T, 4, device=self.device)
            u_init[:, :, 0] = self.mass * GZ
        self.solver.u_init = u_init.permute(1, 0, 2).contiguous()
        self.solver.backprop = self.grad_mode == "diff"
        cost = mpc_compat.SigmoidQuadCost(sigmoid_cost.to(self.device), mass=self.mass)
        if self.grad_mode == "stop" and torch.is_grad_enabled():
            with torch.no_grad():
                X_tbn, U_tbn, _ = self.solver(x0, cost, self._dx)
        else:
            X_tbn, U_tbn, _ = self.solver(x0, cost, self._dx)
        X = X_tbn.permute(1, 0, 2)
        U = U_tbn.permute(1, 0, 2)
        nom_x, nom_u = X[:, :self.T, :], U
        if warm:
            self.u_prev = nom_u[:, 0, :].detach().clone()
        self.predictions = torch.cat((nom_x, nom_u), dim=2).detach()
        bad = (~torch.isfinite(U.detach())).flatten(1).any(dim=1)
        self.naninf_chunks = torch.stack([c.any() for c in torch.split(bad, self.chunk)]).sum()
        thrust = nom_u[:, 0, 0] / self.mass
        omegas = nom_u[:, 0, 1:4]
        max_acc = (self.thrust_max * 4) / self.mass
        force_std = max(1e-6, max_acc - GZ)
        thrust_normalized = (thrust - GZ) / force_std
        omegas_normalized = omegas / self.omega_max
        return torch.cat((thrust_normalized.unsqueeze(1), omegas_normalized), dim=1)


__all__ = ["PolicyMPC"]
