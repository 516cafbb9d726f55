"""CPU tests: the C-ABI library loads and exports what include/ilqr_b200.h
declares, argument validation (no GPU needed), host-side surface logic, the
synthetic workload generator, and the global converged-flag reconstruction."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

import ilqr_native as nat
import ilqr_workload as wl
import mpc_compat
import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    src = open(os.path.join(ROOT, "include", "ilqr_b200.h")).read()
    return sorted(set(re.findall(r"\b(ilqr_b200_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = nat.lib()
    declared = _header_functions()
    assert declared, "no declarations parsed"
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing
    assert sorted(nat.EXPORTED_SYMBOLS) == declared
    assert L.ilqr_b200_abi_version() == 1


def test_status_strings():
    L = nat.lib()
    for code in range(6):
        assert L.ilqr_b200_status_string(code)
    assert b"unknown" in L.ilqr_b200_status_string(99)


def test_workspace_sizes():
    L = nat.lib()
    n = ctypes.c_size_t()
    assert L.ilqr_b200_solve_workspace_size(16384, 20, ctypes.byref(n)) == 0
    assert n.value == (6 * 21 * 16 + 20 * (40 + 4 + 32)) * 16384 * 4
    assert L.ilqr_b200_backward_workspace_size(33, 5, ctypes.byref(n)) == 0
    assert n.value == 5 * 44 * 64 * 4
    assert L.ilqr_b200_solve_workspace_size(-1, 20, ctypes.byref(n)) == 1
    assert L.ilqr_b200_solve_workspace_size(4, 0, ctypes.byref(n)) == 1


def test_size_limits_reject_before_the_byte_count_can_wrap():
    """B beyond ILQR_MAX_BATCH or T beyond ILQR_MAX_HORIZON is rejected by
    every workspace query (B = 2^61 at T = 20 would wrap the byte count to
    0), and so by every entry point that sizes its workspace with them."""
    L = nat.lib()
    n = ctypes.c_size_t(12345)
    big_b, big_t = (1 << 61), 65537
    assert L.ilqr_b200_solve_workspace_size(2**31 - 1, 20, ctypes.byref(n)) == 0
    assert n.value > 0
    for q in (L.ilqr_b200_solve_workspace_size, L.ilqr_b200_backward_workspace_size,
              L.ilqr_b200_rotor13_backward_workspace_size, L.ilqr_b200_fastmpc_backward_workspace_size):
        assert q(big_b, 20, ctypes.byref(n)) == 1
        assert q(2**31, 20, ctypes.byref(n)) == 1
        assert q(16, big_t, ctypes.byref(n)) == 1
    for q in (L.ilqr_b200_rotor13_solve_workspace_size, L.ilqr_b200_fastmpc_solve_workspace_size):
        assert q(big_b, 20, 5, ctypes.byref(n)) == 1
        assert q(16, big_t, 5, ctypes.byref(n)) == 1
    # the entry points return that status instead of passing a wrapped size
    assert L.ilqr_b200_solve_f32(*_solve_args(B=big_b)) == 1
    f = L.ilqr_b200_solve_f32_noalloc
    P, I64, I32, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float
    f.argtypes = [P] * 10 + [I64, I32, F, I32, F, F, P, I32, P] + [P] * 9 + [P]
    f.restype = I32
    assert f(*(_solve_args(B=big_b)[:-3] + [None])) == 1


def test_rotor13_workspace_sizes():
    """Rotor13 solve: (n_alpha + 1) slots of (T + 1) records of 20 floats plus
    K_t columns and k_t ([T][14] float4) per element; backward: the gains."""
    L = nat.lib()
    n = ctypes.c_size_t()
    assert L.ilqr_b200_rotor13_solve_workspace_size(16384, 20, 5, ctypes.byref(n)) == 0
    assert n.value == (6 * 21 * 20 + 20 * 14 * 4) * 16384 * 4
    assert L.ilqr_b200_rotor13_solve_workspace_size(3, 4, 8, ctypes.byref(n)) == 0
    assert n.value == (9 * 5 * 20 + 4 * 56) * 3 * 4
    assert L.ilqr_b200_rotor13_backward_workspace_size(33, 5, ctypes.byref(n)) == 0
    assert n.value == 5 * 56 * 33 * 4
    assert L.ilqr_b200_rotor13_solve_workspace_size(4, 5, 9, ctypes.byref(n)) == 1
    assert L.ilqr_b200_rotor13_solve_workspace_size(4, 0, 5, ctypes.byref(n)) == 1


def test_rotor13_argument_validation_without_gpu():
    L = nat.lib()
    f = L.ilqr_b200_rotor13_solve_f32
    assert f(*_solve_args(n_alpha=0)) == 1
    assert f(*_solve_args(n_alpha=9)) == 1
    assert f(*_solve_args(x0=None)) == 1
    assert f(*_solve_args(u_min=ctypes.c_void_p(0x10000))) == 1
    assert f(*_solve_args(ws_bytes=16)) == 3
    assert f(*_solve_args(ws=ctypes.c_void_p(0x10004))) == 2      # workspace misaligned
    assert f(*_solve_args(B=0)) == 0
    fake = ctypes.c_void_p(0x10000)
    args = [fake, fake, fake, None, None, None, None, fake, fake, 4, 5, 0.05, 1e-6,
            fake, fake, fake, None, None, None, None, fake, 1 << 30, None]
    g = L.ilqr_b200_rotor13_backward_f32
    bad = list(args); bad[0] = None
    assert g(*bad) == 1
    bad = list(args); bad[-2] = 0
    assert g(*bad) == 3


def test_rotor13_surface_without_gpu():
    """FastMPC(13, 4, T) selects the rotor model, defaults U_init to the
    hover fraction, refuses SigmoidQuadCost and CPU tensors."""
    B, T = 2, 3
    m = mpc_compat.FastMPC(13, 4, T, lqr_iter=2)
    init = mpc_compat._normalize_init(None, B, T, 4, torch.device("cpu"), torch.float32, 13)
    assert torch.allclose(init, torch.full((B, T, 4), nat.HOVER_U13))
    x = torch.zeros(B, 13)
    x[:, 3] = 1
    with pytest.raises(ValueError):
        m(x, mpc_compat.SigmoidQuadCost(torch.zeros(B, 28 * T)), type("Dx", (), {"dt": 0.05})())
    C = torch.eye(17).expand(T, B, 17, 17)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(x, mpc_compat.QuadCost(C, None), type("Dx", (), {"dt": 0.05})())
    with pytest.raises(ValueError):
        mpc_compat.FastMPC(12, 4, T)


def test_fastmpc_numerics_surface_without_gpu(monkeypatch):
    """numerics="fastmpc" (or ACMPC_FASTMPC_NUMERICS) selects the reference
    FastMPC build's numerics: its step sizes by default, the 10-state model
    only, and no CPU path; SigmoidQuadCost is turned into the policy's dense
    costs (bit for bit the policy's construction)."""
    B, T = 2, 3
    m = mpc_compat.FastMPC(10, 4, T, lqr_iter=2, numerics="fastmpc")
    assert m.numerics == "fastmpc" and m._alphas() == nat.FASTMPC_ALPHAS == (1.0, 0.5, 0.25, 0.1)
    assert mpc_compat.FastMPC(10, 4, T).numerics == "diffmpc"
    monkeypatch.setenv("ACMPC_FASTMPC_NUMERICS", "fastmpc")
    assert mpc_compat.FastMPC(10, 4, T).numerics == "fastmpc"
    with pytest.raises(ValueError):
        mpc_compat.FastMPC(13, 4, T, numerics="fastmpc")
    with pytest.raises(ValueError):
        mpc_compat.FastMPC(10, 4, T, numerics="mpc.pytorch")
    x = torch.zeros(B, 10)
    x[:, 3] = 1
    C = torch.eye(14).expand(T, B, 14, 14)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(x, mpc_compat.QuadCost(C, None), type("Dx", (), {"dt": 0.05})())
    rng = np.random.default_rng(0)
    sc = rng.uniform(size=(B, 28 * T)).astype(np.float32)
    Ct, ct = mpc_compat._sigmoid_to_dense_tm(torch.from_numpy(sc), T, nat.SigmoidCostSpec())
    Cr, cr = O.sigmoid_costs(sc, T)
    assert np.array_equal(Ct.transpose(0, 1).numpy(), Cr) and np.array_equal(ct.transpose(0, 1).numpy(), cr)


def test_extension_numerics_option(monkeypatch):
    """load_drone_ilqr_ext keeps one extension object per numerics; the
    default follows ACMPC_FASTMPC_NUMERICS; unknown numerics are refused; the
    FastMPC compat entry points reject bad sizes before touching the GPU."""
    import drone_ilqr
    a = drone_ilqr.load_drone_ilqr_ext(numerics="fastmpc")
    b = drone_ilqr.load_drone_ilqr_ext(numerics="diffmpc")
    assert a.numerics == "fastmpc" and b.numerics == "diffmpc" and a is not b
    assert drone_ilqr.load_drone_ilqr_ext(numerics="fastmpc") is a
    monkeypatch.setenv("ACMPC_FASTMPC_NUMERICS", "fastmpc")
    assert drone_ilqr.load_drone_ilqr_ext() is a
    with pytest.raises(ValueError):
        drone_ilqr.DroneIlqrExt("mpc.pytorch")
    L = nat.lib()
    fake = ctypes.c_void_p(0x10000)
    assert L.ilqr_b200_fastmpc_linearize_f32(fake, fake, 4, 0, 0.05, fake, fake, None) == 1
    assert L.ilqr_b200_fastmpc_linearize_f32(None, fake, 4, 5, 0.05, fake, fake, None) == 1
    assert L.ilqr_b200_fastmpc_adjoint_lqr_f32(*([fake] * 9), None, 4, 5, 1e-6, None, fake, fake, None) == 1
    assert L.ilqr_b200_fastmpc_assembly_f32(*([fake] * 7), None, None, 4, 5, fake, None, fake, *([None] * 4),
                                            None) == 1
    assert L.ilqr_b200_fastmpc_assembly_f32(*([fake] * 7), None, None, 0, 5, *([None] * 7), None) == 0


def test_fastmpc_workspace_sizes_and_argument_validation():
    L = nat.lib()
    n = ctypes.c_size_t(0)
    assert L.ilqr_b200_fastmpc_solve_workspace_size(16384, 20, 4, ctypes.byref(n)) == 0
    assert n.value == 256 + 16384 * (5 * 21 * 16 + 20 * 44 + 20 * 4 + 5) * 4
    assert L.ilqr_b200_fastmpc_backward_workspace_size(16384, 20, ctypes.byref(n)) == 0
    assert n.value == 256 + 16384 * 20 * 44 * 4
    assert L.ilqr_b200_fastmpc_solve_workspace_size(4, 5, 9, ctypes.byref(n)) != 0
    fake = ctypes.c_void_p(0x10000)
    al = ctypes.cast((ctypes.c_float * 4)(1, .5, .25, .1), ctypes.c_void_p)

    def solve(**over):
        a = dict(x0=fake, U_init=fake, C=fake, c=fake, C_final=None, c_final=None, x_ref=None, u_ref=None,
                 u_min=None, u_max=None, B=4, T=5, dt=0.05, max_iter=3, reg=1e-6, tol=1e-6, alphas=al, n_alpha=4,
                 layout=0, forced=None, forced_stop=0, X=fake, U=fake, tight=None, X_lin=None, U_lin=None,
                 trace=None, best=None, info=None, ws=None, ws_bytes=0, stream=None)
        a.update(over)
        return L.ilqr_b200_fastmpc_solve_f32(*a.values())

    # each rejected before anything touches the device
    assert solve(layout=2) == 1
    assert solve(u_min=fake) == 1
    assert solve(forced_stop=2) == 1
    assert solve(n_alpha=0) == 1
    assert solve() == 3  # no workspace
    assert solve(B=0) == 0


def _solve_args(**over):
    fake = ctypes.c_void_p(0x10000)
    a = dict(x0=fake, U_init=fake, C=fake, c=fake, C_final=None, c_final=None, x_ref=None,
             u_ref=None, u_min=None, u_max=None, B=4, T=5, dt=0.05, max_iter=3, reg=1e-6, tol=1e-6,
             alphas=ctypes.cast((ctypes.c_float * 5)(1, .8, .5, .2, .1), ctypes.c_void_p), n_alpha=5,
             forced=None, X=fake, U=fake, tight=None, trace=None, iters=None, status=None, best=None,
             s_it=None, s_gap=None, ws=fake, ws_bytes=1 << 30, stream=None)
    a.update(over)
    return list(a.values())


def test_solve_argument_validation_without_gpu():
    """Invalid calls are rejected on the host before any CUDA call."""
    L = nat.lib()
    f = L.ilqr_b200_solve_f32
    assert f(*_solve_args(n_alpha=0)) == 1
    assert f(*_solve_args(n_alpha=9)) == 1
    assert f(*_solve_args(T=0)) == 1
    assert f(*_solve_args(x0=None)) == 1
    assert f(*_solve_args(u_min=ctypes.c_void_p(0x10000))) == 1  # u_max missing
    assert f(*_solve_args(C=ctypes.c_void_p(0x10004))) == 2      # misaligned
    assert f(*_solve_args(ws_bytes=16)) == 3                     # workspace too small
    assert f(*_solve_args(ws=None)) == 3
    assert f(*_solve_args(B=0)) == 0                             # empty batch: no-op


def test_backward_argument_validation_without_gpu():
    L = nat.lib()
    fake = ctypes.c_void_p(0x10000)
    args = [fake, fake, fake, None, None, None, None, fake, fake, 4, 5, 0.05, 1e-6,
            fake, fake, fake, None, None, None, None, fake, 1 << 30, None]
    f = L.ilqr_b200_backward_f32
    bad = list(args); bad[13 + 1] = ctypes.c_void_p(0x10008)  # grad_C misaligned
    assert f(*bad) == 2
    bad = list(args); bad[0] = None
    assert f(*bad) == 1
    bad = list(args); bad[-2] = 0
    assert f(*bad) == 3


def test_no_cpu_fallback():
    """The product path refuses CPU tensors instead of computing on the CPU."""
    B, T = 2, 3
    m = mpc_compat.FastMPC(10, 4, T, lqr_iter=2)
    x = torch.zeros(B, 10)
    x[:, 3] = 1
    C = torch.eye(14).expand(T, B, 14, 14)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(x, mpc_compat.QuadCost(C, None), type("Dx", (), {"dt": 0.05})())


def test_normalize_cost_layouts():
    B, T, n = 3, 4, 14
    C2 = torch.randn(n, n)
    Cb, cb = mpc_compat._normalize_cost(C2, None, B, T, n, torch.device("cpu"), torch.float32)
    assert Cb.shape == (B, T, n, n) and cb.shape == (B, T, n)
    assert torch.equal(Cb[2, 3], C2) and torch.count_nonzero(cb) == 0
    C4 = torch.randn(T, B, n, n)
    c3 = torch.randn(T, B, n)
    Cb, cb = mpc_compat._normalize_cost(C4, c3, B, T, n, torch.device("cpu"), torch.float32)
    assert torch.equal(Cb[1, 2], C4[2, 1]) and torch.equal(cb[1, 2], c3[2, 1])
    c1 = torch.randn(n)
    _, cb = mpc_compat._normalize_cost(C4, c1, B, T, n, torch.device("cpu"), torch.float32)
    assert torch.equal(cb[2, 3], c1)
    # The time-major form the operator hands to the kernels is the same data
    # without the transpose, for every accepted shape of C and c.
    cpu = torch.device("cpu")
    for C, c in ((C2, None), (C4, c3), (C4, c1), (torch.randn(T, n, n), torch.randn(T, n))):
        Cb, cb = mpc_compat._normalize_cost(C, c, B, T, n, cpu, torch.float32)
        Ct, ct = mpc_compat._normalize_cost_tm(C, c, B, T, n, cpu, torch.float32)
        assert Ct.is_contiguous() and ct.is_contiguous()
        assert torch.equal(Ct, Cb.transpose(0, 1)) and torch.equal(ct, cb.transpose(0, 1))


def test_normalize_bounds_and_init():
    lo = torch.zeros(5, 1, 4)
    lo[..., 1:] = -3
    hi = torch.ones(5, 1, 4) * 3
    a, b = mpc_compat._normalize_bounds(lo, hi, 4, torch.device("cpu"), torch.float32)
    assert a.tolist() == [0, -3, -3, -3] and b.tolist() == [3, 3, 3, 3]
    assert mpc_compat._normalize_bounds(None, hi, 4, "cpu", torch.float32) == (None, None)
    U = mpc_compat._normalize_init(None, 2, 3, 4, torch.device("cpu"), torch.float32)
    assert U.shape == (2, 3, 4) and torch.allclose(U[..., 0], torch.tensor(0.752 * 9.8066))
    ui = torch.randn(3, 2, 4)
    assert torch.equal(mpc_compat._normalize_init(ui, 2, 3, 4, torch.device("cpu"), torch.float32),
                       ui.permute(1, 0, 2))
    ub = torch.randn(4, 2)
    out = mpc_compat._normalize_init(ub, 2, 3, 4, torch.device("cpu"), torch.float32)
    assert torch.equal(out[1, 2], ub[:, 1])


def test_workload_prefix_and_structure():
    a = wl.make_inputs(40, 6, seed=0)
    b = wl.make_inputs(1030, 6, seed=0)
    for k in a:
        assert np.array_equal(a[k], b[k][:40]), k
    C = b["C"]
    off = C.copy()
    idx = np.arange(14)
    off[:, :, idx, idx] = 0
    assert not off.any()
    d = C[:, :, idx, idx]
    assert d.min() >= 1e-2 * (1 - 1e-6) and d.max() <= 1e2 * (1 + 1e-6)
    tau = -b["c"] / d
    assert np.allclose(tau[..., 3], 1.0) and np.allclose(tau[..., 10], 0.752 * 9.8066, rtol=1e-6)
    gX, gU = wl.make_backward_seeds(40, 6)
    gX2, gU2 = wl.make_backward_seeds(2000, 6)
    assert np.array_equal(gX, gX2[:40]) and np.array_equal(gU, gU2[:40])


@pytest.mark.parametrize("stall,gap,iters,expect", [
    ([1, 2, 3], [0.0, 0.0, 0.0], 10, True),      # all stall with zero gap
    ([1, 9, 3], [1.0, 1.0, 1.0], 10, False),     # last stall at 9, gap large, no 3 strikes
    ([1, 7, 3], [1.0, 1.0, 1.0], 10, True),      # third strike at 9 < 10
    ([10, 10], [0.0, 0.0], 10, False),           # never stalled; finiteness decides
])
def test_converged_flag_matches_oracle(stall, gap, iters, expect):
    s = np.array(stall)
    g = np.array(gap)
    ref = O.global_converged_flag(s, g, iters, 1e-6, all_finite=False)
    got = nat.converged_flag(torch.tensor(s), torch.tensor(g), torch.tensor([2, 0]), iters, 1e-6)
    assert ref == got == expect
