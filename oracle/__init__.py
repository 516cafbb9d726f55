"""TEST INFRASTRUCTURE ONLY -- the CPU oracle for the batched iLQR solver.

This package is a numpy restatement of the reference's DiffMPC algorithm
(DifferentialMPC/controller.py, DifferentialMPC/cost.py) and of its quadrotor
model (acmpc_public-master/diff_mpc_drones/drone.py). It exists to check the
CUDA solver: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg may import it. The product path (the C-ABI library and the Python surface
in ca-ac-mpc_b200/) never imports, links or executes anything here.

fastmpc_oracle.py restates the reference FastMPC extension's CUDA build (its
own numerics mode of the same solver).

Pinning: the oracle is checked against golden vectors produced by running the
reference DiffMPC itself (tests/golden/make_golden.py, which imports the
reference from its source tree in the build container); see
tests/test_oracle_golden.py.
"""

from .diffmpc_oracle import *  # noqa: F401,F403
from .rotor13_model import *  # noqa: F401,F403
from .fastmpc_oracle import *  # noqa: F401,F403
