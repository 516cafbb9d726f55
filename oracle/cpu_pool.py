"""TEST AND BASELINE INFRASTRUCTURE ONLY -- runs the reference's CPU algorithm
over a process pool, for the benchmark's CPU-baseline leg and its reference
arm: either the reference DiffMPC solver itself (impl "reference": the
sources oracle/stage_diffmpc_ref.py staged, one torch thread per worker,
oracle/diffmpc_ref.py) or the numpy restatement of it (impl "port":
oracle/diffmpc_oracle.py). The pool uses the spawn start method. Each worker
generates its own chunk of the workload and times only the solve (and
backward)."""

from __future__ import annotations

import multiprocessing as mp
import os
import time

os.environ.setdefault("OMP_NUM_THREADS", "1")
os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
os.environ.setdefault("MKL_NUM_THREADS", "1")


def _solve_chunk(args):
    """fwd(+bwd) of the first n elements of the 1024-element block at `lo` of
    a workload; returns (n, seconds)."""
    import sys
    root, pkg, name, lo, n, seed, impl = args
    for p in (root, pkg):
        if p not in sys.path:
            sys.path.insert(0, p)
    import ilqr_workload as wl
    cfg = wl.CONFIGS[name]
    T = cfg["T"]
    inp = wl.make_inputs(max(n, 1024), T, seed=seed, target=cfg["target"], r=cfg["r"], offset=lo)
    gX, gU = wl.make_backward_seeds(max(n, 1024), T, offset=lo)
    inp = {k: v[:n] for k, v in inp.items()}
    gX, gU = gX[:n], gU[:n]
    if impl == "reference":
        import warnings

        import torch
        from oracle import diffmpc_ref as R
        warnings.filterwarnings("ignore")
        torch.set_num_threads(1)
        t0 = time.perf_counter()
        R.solve_fwd_bwd(inp, T, cfg["max_iter"], cfg["alphas"], wl.DT, wl.U_MIN, wl.U_MAX, gX, gU)
        return n, time.perf_counter() - t0
    from oracle import diffmpc_oracle as O
    t0 = time.perf_counter()
    r = O.solve(inp["x0"], inp["U_init"], inp["C"], inp["c"], u_min=wl.U_MIN, u_max=wl.U_MAX,
                dt=wl.DT, max_iter=cfg["max_iter"], alphas=cfg["alphas"])
    if cfg["backward"]:
        O.backward(r["X"], r["U"], inp["C"], None, None, None, r["tight"], gX, gU, wl.DT, wl.REG_EPS)
    return n, time.perf_counter() - t0


class OraclePool:
    """Spawned worker pool; `run(name, chunks, chunk)` solves `chunks` chunks of
    `chunk` elements (one per worker) and returns (elements, seconds), the
    seconds being the slowest worker's compute time. `impl` is "reference"
    (DiffMPC itself) or "port" (the numpy restatement)."""

    def __init__(self, workers: int, root: str, pkg: str, impl: str = "port"):
        assert impl in ("reference", "port")
        self.workers, self.impl = workers, impl
        self.root, self.pkg = root, pkg
        self.pool = mp.get_context("spawn").Pool(workers)
        self.pool.map(_solve_chunk, [(root, pkg, "latency_b16_t5", 0, 1, 0, impl)] * workers)

    def run(self, name: str, chunks: int, chunk: int, seed: int = 0):
        assert chunk <= 1024 or chunk % 1024 == 0
        step = max(chunk, 1024)
        tasks = [(self.root, self.pkg, name, i * step, chunk, seed, self.impl) for i in range(chunks)]
        res = self.pool.map(_solve_chunk, tasks, chunksize=1)
        return sum(n for n, _ in res), max(t for _, t in res)

    def close(self):
        self.pool.close()
        self.pool.join()
