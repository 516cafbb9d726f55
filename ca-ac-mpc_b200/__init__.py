"""B200 batched differentiable iLQR solver for the quadrotor MPC of
prisma-lab/CA-AC-MPC (drop-in for its differentialMPCPerformance/ backend).

Put this directory on sys.path and import as the reference's callers do:

    from mpc_compat import FastMPC, QuadCost   # or MPC
    from drone_ilqr import load_drone_ilqr_ext

Contents: mpc_compat.py / drone_ilqr.py (the reference-facing surface),
ilqr_native.py (ctypes binding of libilqr_b200.so, the C ABI declared in
include/ilqr_b200.h), csrc/ (CUDA sources and build script),
ilqr_workload.py (seeded synthetic workloads), ilqr_costmodel.py
(algorithmic FLOP / byte counts for the roofline).
"""
