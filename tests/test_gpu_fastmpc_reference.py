"""The FastMPC numerics mode against the reference's own CUDA kernels.

tests/fastmpc_ref.py re-executes the reference FastMPC extension's CUDA build
on the GPU: its kernels, compiled from the reference sources with its own
flags (--use_fast_math) into oracle/_ref/, driven by a torch restatement of
its host loop. The B200 solve records its line-search decisions and batch
stop; the re-executed reference replays them, and X, U must agree to 1e-4
(relative to the element's largest magnitude), the tight masks on 99 % of
entries, and the gradients of x0, C, c to 1e-3. The cases use the FastMPC
operator's zero terminal cost and references, as the operator does.
"""

import numpy as np
import pytest
import torch

import fastmpc_ref as ref
import ilqr_native as nat
import ilqr_workload as wl

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref.available(),
                                 reason="oracle/_ref/libfastmpc_ref.so not built (needs the reference sources)")]
DEV = "cuda"
LO = np.array([0.0, -10.0, -10.0, -4.0], np.float32)
HI = np.array([34.0, 10.0, 10.0, 4.0], np.float32)


def _t(a):
    return None if a is None else torch.as_tensor(np.ascontiguousarray(a)).to(DEV, torch.float32)


def _rel(a, b):
    a = a.double().cpu().numpy()
    b = b.double().cpu().numpy()
    ax = tuple(range(1, a.ndim))
    scale = np.maximum(np.abs(b).max(axis=ax, keepdims=True), 1.0)
    return (np.abs(a - b) / scale).max(axis=ax)


def _case(name):
    if name == "cfg1_b16_t5":
        return wl.make_inputs(16, 5, seed=0), True, 10
    if name == "cfg2_b64_t10":
        return wl.make_inputs(64, 10, seed=1), True, 10
    if name == "cfg3_b48_t20":
        return wl.make_inputs(48, 20, seed=2), True, 5
    if name == "dense_b8_t6":
        d = wl.make_inputs(8, 6, seed=3)
        extra = wl.make_dense_costs(8, 6, seed=4)
        return dict(d, C=extra["C"], c=extra["c"]), True, 6
    if name == "nobox_b8_t5":
        return wl.make_inputs(8, 5, seed=5), False, 5
    if name == "ragged_b13_t7":
        return wl.make_inputs(13, 7, seed=6, r=15.0), True, 9
    raise KeyError(name)


CASES = ["cfg1_b16_t5", "cfg2_b64_t10", "cfg3_b48_t20", "dense_b8_t6", "nobox_b8_t5", "ragged_b13_t7"]


@pytest.mark.parametrize("name", CASES)
def test_fastmpc_matches_reference_kernels(name):
    d, boxed, iters = _case(name)
    lo, hi = (_t(LO), _t(HI)) if boxed else (None, None)
    ours = nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=lo, u_max=hi, dt=0.05,
                             max_iter=iters, want_trace=True)
    run = int(ours["batch_info"][1])
    r = ref.solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), lo, hi, dt=0.05, max_iter=iters,
                  forced=ours["trace"].long(), forced_stop=run)
    assert r["iters"] == run
    for k in ("X", "U"):
        err = _rel(ours[k], r[k])
        assert err.max() <= 1e-4, (k, float(err.max()), int(err.argmax()))
    agree = (ours["tight"].bool() == r["tight"]).float().mean().item()
    assert agree >= 0.99, agree
    # the backward at each side's own solution
    B, T = d["U_init"].shape[:2]
    gX, gU = (_t(a) for a in wl.make_backward_seeds(B, T))
    g = nat.fastmpc_backward(ours["X"], ours["U"], ours["X_lin"], ours["U_lin"], _t(d["C"]), gX, gU,
                             tight=ours["tight"] if boxed else None, dt=0.05)
    rg = ref.backward(r, gX, gU)
    for k in ("x0", "C", "c"):
        err = _rel(g[k], rg[k])
        assert err.max() <= 1e-3, (k, float(err.max()), int(err.argmax()))


@pytest.mark.parametrize("name", ["cfg1_b16_t5", "cfg2_b64_t10", "cfg3_b48_t20"])
def test_free_run_parts_from_reference_only_at_ties(name):
    """Without replay each side decides for itself. An element whose decisions
    match the reference's ends within 1e-4 of it; where they part, the first
    differing decision is a near-tie in the reference's own costs: two step
    sizes within 1e-5 of each other (relative), or an accept/reject call on an
    improvement below 1e-5 of the cost."""
    d, boxed, iters = _case(name)
    ours = nat.fastmpc_solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), u_min=_t(LO), u_max=_t(HI),
                             dt=0.05, max_iter=iters, want_trace=True)
    r = ref.solve(_t(d["x0"]), _t(d["U_init"]), _t(d["C"]), _t(d["c"]), _t(LO), _t(HI), dt=0.05, max_iter=iters)
    n = min(int(ours["batch_info"][1]), r["iters"])
    to = ours["trace"][:, :n].long().cpu().numpy()
    tr = r["trace"][:, :n].cpu().numpy()
    costs = r["costs"][:, :n].double().cpu().numpy()
    best = r["best_before"][:, :n].double().cpu().numpy()
    err = _rel(ours["U"], r["U"])
    parted = 0
    for b in range(to.shape[0]):
        diff = np.nonzero(to[b] != tr[b])[0]
        if diff.size == 0:
            if int(ours["batch_info"][1]) == r["iters"]:
                assert err[b] <= 1e-4, (b, err[b])
            continue
        parted += 1
        i = diff[0]
        c = costs[b, i]
        scale = max(np.abs(c).max(), abs(best[b, i]), 1e-30)
        jo, jr = to[b, i], tr[b, i]
        if jo >= 0 and jr >= 0:
            gap = abs(c[jo] - c[jr])
        else:
            j = jo if jo >= 0 else jr
            gap = abs(c[j] - best[b, i]) if j >= 0 else abs(c[-jo - 1] - c[-jr - 1])
        assert gap <= 1e-5 * scale, (b, i, jo, jr, gap / scale)
    assert parted < to.shape[0]


def test_pnqp4_batch_matches_reference_kernel():
    """drone_pnqp4_batch against the reference's own PNQP-4 kernel on the
    golden problems (mpc.pytorch pnqp's set) and on the box QPs of a solve:
    the same optimum to 1e-4 and the same free mask, cold and warm started."""
    import os
    from parity import GOLDEN_DIR
    d = np.load(os.path.join(GOLDEN_DIR, "pnqp4_n256.npz"))
    H, q, lo, hi = (_t(d[k]) for k in ("H", "q", "lower", "upper"))
    for x_init in (None, _t(d["opt_x"].astype(np.float32))):
        x, fm = nat.pnqp4_batch(H, q, lo, hi, x_init)
        rx, rfm = ref.pnqp4_batch(H, q, lo, hi, x_init)
        scale = torch.clamp(rx.abs().amax(1, keepdim=True), min=1.0)
        close = ((x - rx).abs() / scale).amax(1) <= 1e-4
        assert close.float().mean().item() >= 0.98, close.float().mean().item()
        assert torch.equal(fm[close], rfm[close])

