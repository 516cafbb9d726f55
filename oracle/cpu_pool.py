"""TEST INFRASTRUCTURE ONLY -- runs the oracle over a process pool, for the
benchmark's CPU-baseline leg (the reference's CPU algorithm timed on host
cores). Workers import numpy and the oracle only; the pool uses the spawn
start method. Each worker generates its own chunk of the workload and times
only the solve (and backward)."""

from __future__ import annotations

import multiprocessing as mp
import os
import time

os.environ.setdefault("OMP_NUM_THREADS", "1")
os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
os.environ.setdefault("MKL_NUM_THREADS", "1")


def _solve_chunk(args):
    """fwd(+bwd) of elements [lo, lo + n) of a workload; returns (n, seconds)."""
    import sys
    root, pkg, name, lo, n, seed = args
    for p in (root, pkg):
        if p not in sys.path:
            sys.path.insert(0, p)
    import ilqr_workload as wl
    from oracle import diffmpc_oracle as O
    cfg = wl.CONFIGS[name]
    T = cfg["T"]
    inp = wl.make_inputs(n, T, seed=seed, target=cfg["target"], r=cfg["r"], offset=lo)
    gX, gU = wl.make_backward_seeds(n, T, offset=lo)
    t0 = time.perf_counter()
    r = O.solve(inp["x0"], inp["U_init"], inp["C"], inp["c"], u_min=wl.U_MIN, u_max=wl.U_MAX,
                dt=wl.DT, max_iter=cfg["max_iter"], alphas=cfg["alphas"])
    if cfg["backward"]:
        O.backward(r["X"], r["U"], inp["C"], None, None, None, r["tight"], gX, gU, wl.DT, wl.REG_EPS)
    return n, time.perf_counter() - t0


class OraclePool:
    """Spawned worker pool; `run(name, chunks, chunk)` solves `chunks` chunks of
    `chunk` elements (one per worker) and returns (elements, seconds), the
    seconds being the slowest worker's compute time."""

    def __init__(self, workers: int, root: str, pkg: str):
        self.workers = workers
        self.root, self.pkg = root, pkg
        self.pool = mp.get_context("spawn").Pool(workers)
        self.pool.map(_solve_chunk, [(root, pkg, "latency_b16_t5", 0, 1, 0)] * workers)

    def run(self, name: str, chunks: int, chunk: int, seed: int = 0):
        assert chunk % 1024 == 0
        tasks = [(self.root, self.pkg, name, i * chunk, chunk, seed) for i in range(chunks)]
        res = self.pool.map(_solve_chunk, tasks, chunksize=1)
        return sum(n for n, _ in res), max(t for _, t in res)

    def close(self):
        self.pool.close()
        self.pool.join()
