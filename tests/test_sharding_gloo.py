"""Multi-rank batch sharding on CPU (gloo, world size 2): each rank solves its
contiguous shard with the oracle and runs the backward, the first actions
and the gradients (dL/dx0, dL/dc) are all-gathered with the same helpers the
GPU benchmark uses, and the gathered results equal the single-process solve
and backward bit for bit (batch elements are independent)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import ilqr_shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, B, T, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ca-ac-mpc_b200")]
    import torch.distributed as dist
    import ilqr_shard as sh
    import ilqr_workload as wl
    import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        inp = wl.make_inputs(B, T, seed=0)
        lo, hi = sh.shard_bounds(B, rank, world)
        r = O.solve(inp["x0"][lo:hi], inp["U_init"][lo:hi], inp["C"][lo:hi], inp["c"][lo:hi],
                    u_min=wl.U_MIN, u_max=wl.U_MAX, dt=wl.DT, max_iter=3)
        acts = sh.gather_first_actions(torch.from_numpy(r["U"]), B)
        gX, gU = wl.make_backward_seeds(B, T)
        gr = O.backward(r["X"], r["U"], inp["C"][lo:hi], None, None, None, r["tight"], gX[lo:hi], gU[lo:hi],
                        wl.DT, wl.REG_EPS)
        gl = {"x0": torch.from_numpy(gr["grad_x0"]), "c": torch.from_numpy(gr["grad_c"])}
        gg = sh.gather_gradients(gl, B, keys=("x0", "c"))
        acts2, gg2 = sh.gather_actions_and_gradients(torch.from_numpy(r["U"]), gl, B, keys=("x0", "c"))
        assert torch.equal(acts2, acts) and torch.equal(gg2["x0"], gg["x0"]) and torch.equal(gg2["c"], gg["c"])
        if rank == 0:
            q.put((acts.numpy(), gg["x0"].numpy(), gg["c"].numpy()))
    finally:
        dist.destroy_process_group()


def test_shard_bounds_cover_batch():
    for B in (0, 1, 7, 64, 1001):
        for W in (1, 2, 3, 8):
            spans = [ilqr_shard.shard_bounds(B, r, W) for r in range(W)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


@pytest.mark.parametrize("B", [64, 37])
def test_gloo_two_ranks_match_single_process(B):
    import ilqr_workload as wl
    import oracle as O
    T = 5
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, B, T, q)) for r in range(2)]
    for p in procs:
        p.start()
    got, gx0, gc = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    inp = wl.make_inputs(B, T, seed=0)
    ref = O.solve(inp["x0"], inp["U_init"], inp["C"], inp["c"], u_min=wl.U_MIN, u_max=wl.U_MAX,
                  dt=wl.DT, max_iter=3)
    assert np.array_equal(got, ref["U"][:, 0, :])
    gX, gU = wl.make_backward_seeds(B, T)
    gr = O.backward(ref["X"], ref["U"], inp["C"], None, None, None, ref["tight"], gX, gU, wl.DT, wl.REG_EPS)
    assert gx0.shape == (B, 10) and gc.shape == (B, T, 14)
    assert np.array_equal(gx0, gr["grad_x0"])
    assert np.array_equal(gc, gr["grad_c"])
