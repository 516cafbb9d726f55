"""The no-allocation solve entry point (ilqr_b200_solve_f32_noalloc).

It serves hosts that cannot allocate device memory while running (for
example a control loop whose GPU memory is fixed at start-up, or a plugin
whose host owns the allocator): the caller passes inputs and outputs, and the
solver's scratch comes from a fixed array inside the library. These tests call
it through the C ABI and compare it with the workspace-taking entry point.
The file sorts last so that a run stopping at its first failure has already
run every other test; it also passes on its own in a fresh process."""

import ctypes

import numpy as np
import pytest
import torch

import ilqr_native as nat
import ilqr_workload as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SCRATCH_BYTES = 16 << 20
STATUS_NOALLOC_LIMIT = 6


def _fn():
    L = nat.lib()
    f = L.ilqr_b200_solve_f32_noalloc
    P, I64, I32, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float
    f.argtypes = [P] * 10 + [I64, I32, F, I32, F, F, P, I32, P] + [P] * 9 + [P]
    f.restype = I32
    return f


def _inputs(name, B):
    cfg, inp = wl.config_inputs(name, B=B)
    t = {k: torch.from_numpy(v).to(DEV) for k, v in inp.items()}
    return cfg, t


def _outputs(B, T, max_iter):
    return dict(X=torch.empty(B, T + 1, 10, device=DEV), U=torch.empty(B, T, 4, device=DEV),
                tight=torch.empty(B, T, 4, device=DEV, dtype=torch.uint8),
                trace=torch.empty(B, max_iter, device=DEV, dtype=torch.int8),
                iters=torch.empty(B, device=DEV, dtype=torch.int32),
                status=torch.empty(B, device=DEV, dtype=torch.int32),
                best=torch.empty(B, device=DEV))


def _call_noalloc(f, cfg, t, lo, hi, out):
    p = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    al = (ctypes.c_float * len(cfg["alphas"]))(*cfg["alphas"])
    B, T = t["U_init"].shape[:2]
    return f(p(t["x0"]), p(t["U_init"]), p(t["C"]), p(t["c"]), None, None, None, None, p(lo), p(hi),
             B, T, wl.DT, cfg["max_iter"], wl.REG_EPS, wl.CONVERGE_TOL,
             ctypes.cast(al, ctypes.c_void_p), len(cfg["alphas"]), None, p(out["X"]), p(out["U"]),
             p(out["tight"]), p(out["trace"]), p(out["iters"]), p(out["status"]), p(out["best"]), None, None,
             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    f = _fn()
    lo, hi = torch.from_numpy(wl.U_MIN).to(DEV), torch.from_numpy(wl.U_MAX).to(DEV)
    cases = [("rollout_b16384_t20", 1024), ("latency_b16_t5", 16)]
    results = []
    for name, B in cases:  # two calls in a row, different sizes; the scratch is reused
        cfg, t = _inputs(name, B)
        out = _outputs(B, cfg["T"], cfg["max_iter"])
        assert _call_noalloc(f, cfg, t, lo, hi, out) == 0
        results.append((cfg, t, out))
    torch.cuda.synchronize()
    for cfg, t, out in results:
        ref = nat.solve(t["x0"], t["U_init"], t["C"], t["c"], None, None, None, None, lo, hi,
                        dt=wl.DT, max_iter=cfg["max_iter"], reg_eps=wl.REG_EPS,
                        alphas=cfg["alphas"], want_trace=True, want_stats=True)
        torch.cuda.synchronize()
        # Same kernel, same inputs, scratch written before it is read: the
        # results are the same bits, on the second call as on the first.
        for k in ("X", "U", "tight", "trace"):
            assert torch.equal(out[k], ref[k]), k
        assert torch.equal(out["iters"], ref["iters"])
        assert torch.equal(out["status"], ref["status"].to(torch.int32))
        assert torch.equal(out["best"], ref["best_cost"])


def test_noalloc_rejects_problems_beyond_the_fixed_scratch():
    f = _fn()
    need = ctypes.c_size_t()
    nat.lib().ilqr_b200_solve_workspace_size(1184, 20, ctypes.byref(need))
    assert need.value <= SCRATCH_BYTES
    nat.lib().ilqr_b200_solve_workspace_size(1185, 20, ctypes.byref(need))
    assert need.value > SCRATCH_BYTES
    cfg, t = _inputs("rollout_b16384_t20", 1)
    fake = ctypes.c_void_p(t["C"].data_ptr())
    al = (ctypes.c_float * 5)(*cfg["alphas"])
    st = f(*([fake] * 4 + [None] * 6), 1185, 20, wl.DT, 5, wl.REG_EPS, wl.CONVERGE_TOL,
           ctypes.cast(al, ctypes.c_void_p), 5, None, fake, fake, None, None, None, None, None, None,
           None, None)
    assert st == STATUS_NOALLOC_LIMIT
    assert b"no-allocation" in nat.lib().ilqr_b200_status_string(st)
