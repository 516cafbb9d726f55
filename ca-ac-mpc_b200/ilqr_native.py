"""ctypes binding of libilqr_b200.so (the C ABI in include/ilqr_b200.h).

Tensor-level wrappers: they check device/dtype/shape/contiguity, allocate the
outputs and the scratch workspace through torch's caching allocator, enqueue
the CUDA work on torch's current stream and map a non-zero status to a
RuntimeError, as the reference extension's TORCH_CHECKs do
(differentialMPCPerformance/cpp/drone_ilqr_ext.cpp:1080-1088). There is no CPU
fallback: loading fails loudly if the library is missing, and every entry
point requires CUDA tensors.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional, Sequence

import torch

NX, NU, N = 10, 4, 14
NOT_RUN = -128
DEFAULT_ALPHAS = (1.0, 0.8, 0.5, 0.2, 0.1)  # DifferentialMPC/controller.py:211
HOVER_THRUST = 0.752 * 9.8066  # hover U_init (mlp_mpc_policy_diffmpc.py:249-252)
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libilqr_b200.so")

_lib = None
_lib_lock = threading.Lock()

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F = ctypes.c_float


def lib():
    """Load the solver library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python ca-ac-mpc_b200/csrc/build.py` "
                "(or __graft_entry__.build()); there is no CPU fallback")
        L = ctypes.CDLL(LIB_PATH)
        sig = {
            "ilqr_b200_abi_version": ([], _I32),
            "ilqr_b200_status_string": ([_I32], ctypes.c_char_p),
            "ilqr_b200_check_device": ([_I32], _I32),
            "ilqr_b200_solve_workspace_size": ([_I64, _I32, ctypes.POINTER(ctypes.c_size_t)], _I32),
            "ilqr_b200_backward_workspace_size": ([_I64, _I32, ctypes.POINTER(ctypes.c_size_t)], _I32),
            "ilqr_b200_solve_f32": ([_P] * 10 + [_I64, _I32, _F, _I32, _F, _F, _P, _I32, _P]
                                    + [_P] * 9 + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_backward_f32": ([_P] * 9 + [_I64, _I32, _F, _F] + [_P] * 7
                                       + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_solve_sigmoid_f32": ([_P] * 3 + [_F] * 4 + [_P] * 2 + [_I64, _I32, _F, _I32, _F, _F, _P, _I32, _P]
                                            + [_P] * 9 + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_backward_sigmoid_f32": ([_P] * 3 + [_F] * 4 + [_P] * 3 + [_I64, _I32, _F, _F] + [_P] * 2
                                               + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_dynamics_f32": ([_P, _P, _I64, _F, _P, _P], _I32),
            "ilqr_b200_pnqp4_batch_f32": ([_P] * 5 + [_I64, _P, _P, _P], _I32),
            "ilqr_b200_linearize_f32": ([_P, _P, _I64, _I32, _F, _P, _P, _P], _I32),
            "ilqr_b200_adjoint_lqr_f32": ([_P] * 10 + [_I64, _I32, _F, _P, _P, _P, _P], _I32),
            "ilqr_b200_implicit_diff_assembly_f32": ([_P] * 9 + [_I64, _I32] + [_P] * 7 + [_P], _I32),
            "ilqr_b200_rotor13_solve_workspace_size": ([_I64, _I32, _I32, ctypes.POINTER(ctypes.c_size_t)], _I32),
            "ilqr_b200_rotor13_backward_workspace_size": ([_I64, _I32, ctypes.POINTER(ctypes.c_size_t)], _I32),
            "ilqr_b200_rotor13_solve_f32": ([_P] * 10 + [_I64, _I32, _F, _I32, _F, _F, _P, _I32, _P]
                                            + [_P] * 9 + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_rotor13_backward_f32": ([_P] * 9 + [_I64, _I32, _F, _F] + [_P] * 7
                                               + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_rotor13_dynamics_f32": ([_P, _P, _I64, _F, _P, _P], _I32),
            "ilqr_b200_solve_tm_f32": ([_P] * 10 + [_I64, _I32, _F, _I32, _F, _F, _P, _I32, _P]
                                       + [_P] * 9 + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_backward_tm_f32": ([_P] * 9 + [_I64, _I32, _F, _F] + [_P] * 7
                                          + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_rotor13_solve_tm_f32": ([_P] * 10 + [_I64, _I32, _F, _I32, _F, _F, _P, _I32, _P]
                                               + [_P] * 9 + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_rotor13_backward_tm_f32": ([_P] * 9 + [_I64, _I32, _F, _F] + [_P] * 7
                                                  + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_rotor13_linearize_f32": ([_P, _P, _I64, _I32, _F, _P, _P, _P], _I32),
            "ilqr_b200_fastmpc_solve_workspace_size": ([_I64, _I32, _I32, ctypes.POINTER(ctypes.c_size_t)], _I32),
            "ilqr_b200_fastmpc_backward_workspace_size": ([_I64, _I32, ctypes.POINTER(ctypes.c_size_t)], _I32),
            "ilqr_b200_fastmpc_solve_f32": ([_P] * 10 + [_I64, _I32, _F, _I32, _F, _F, _P, _I32, _I32, _P, _I32]
                                            + [_P] * 8 + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_fastmpc_backward_f32": ([_P] * 11 + [_I64, _I32, _F, _F, _I32] + [_P] * 7
                                               + [_P, ctypes.c_size_t, _P], _I32),
            "ilqr_b200_fastmpc_linearize_f32": ([_P, _P, _I64, _I32, _F, _P, _P, _P], _I32),
            "ilqr_b200_fastmpc_adjoint_lqr_f32": ([_P] * 10 + [_I64, _I32, _F, _P, _P, _P, _P], _I32),
            "ilqr_b200_fastmpc_assembly_f32": ([_P] * 9 + [_I64, _I32] + [_P] * 7 + [_P], _I32),
        }
        for name, (argt, rest) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = argt
            fn.restype = rest
        if L.ilqr_b200_abi_version() != 1:
            raise RuntimeError("libilqr_b200.so ABI version mismatch")
        _lib = L
    return _lib


EXPORTED_SYMBOLS = (
    "ilqr_b200_abi_version", "ilqr_b200_status_string", "ilqr_b200_check_device",
    "ilqr_b200_solve_workspace_size", "ilqr_b200_backward_workspace_size",
    "ilqr_b200_solve_f32", "ilqr_b200_backward_f32", "ilqr_b200_dynamics_f32",
    "ilqr_b200_linearize_f32", "ilqr_b200_adjoint_lqr_f32",
    "ilqr_b200_implicit_diff_assembly_f32", "ilqr_b200_solve_f32_noalloc",
    "ilqr_b200_solve_sigmoid_f32", "ilqr_b200_backward_sigmoid_f32", "ilqr_b200_pnqp4_batch_f32",
    "ilqr_b200_rotor13_solve_workspace_size", "ilqr_b200_rotor13_backward_workspace_size",
    "ilqr_b200_rotor13_solve_f32", "ilqr_b200_rotor13_backward_f32", "ilqr_b200_rotor13_dynamics_f32",
    "ilqr_b200_rotor13_linearize_f32", "ilqr_b200_solve_tm_f32", "ilqr_b200_backward_tm_f32",
    "ilqr_b200_rotor13_solve_tm_f32", "ilqr_b200_rotor13_backward_tm_f32",
    "ilqr_b200_fastmpc_solve_workspace_size", "ilqr_b200_fastmpc_backward_workspace_size",
    "ilqr_b200_fastmpc_solve_f32", "ilqr_b200_fastmpc_backward_f32", "ilqr_b200_fastmpc_linearize_f32",
    "ilqr_b200_fastmpc_adjoint_lqr_f32", "ilqr_b200_fastmpc_assembly_f32",
)


def _check(status: int, what: str):
    if status != 0:
        msg = lib().ilqr_b200_status_string(status).decode()
        raise RuntimeError(f"{what} failed: {msg} (status {status})")


def _ptr(t: Optional[torch.Tensor]):
    # a plain int: the declared c_void_p argtypes convert it (cheaper than a
    # c_void_p object per argument on the latency path)
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device):
    """torch's current stream on `device` as a cudaStream_t (the raw handle
    getter when this torch has it: a per-call saving on the latency path)."""
    if _raw_stream is not None:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


def _req(t: torch.Tensor, name: str, shape, device, dtype=torch.float32):
    # the common case in one test; the checks below name what is wrong
    if (isinstance(t, torch.Tensor) and t.dtype is dtype and t.shape == tuple(shape) and t.device == device
            and t.is_contiguous()):
        return t
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (no CPU path)")
    if t.device != device:
        raise RuntimeError(f"{name} is on {t.device}, expected {device}")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")
    if tuple(t.shape) != tuple(shape):
        raise RuntimeError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    return t


def _opt(t, name, shape, device, dtype=torch.float32):
    return None if t is None else _req(t, name, shape, device, dtype)


_checked_devices = set()


def _cuda_device(t, name):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor: the solver has no CPU path")
    return t.device


def _device_ok(device: torch.device):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _checked_devices:
        _check(lib().ilqr_b200_check_device(idx), "device check")
        _checked_devices.add(idx)


_ws_sizes = {}
_alpha_arrays = {}


def _alpha_array(al):
    """The step sizes as a C float array, one per distinct tuple (kept alive
    here, so the pointer passed to the library stays valid)."""
    key = tuple(al)
    arr = _alpha_arrays.get(key)
    if arr is None:
        arr = _alpha_arrays[key] = (ctypes.c_float * len(key))(*key)
    return arr


def workspace_bytes(kind: str, B: int, T: int) -> int:
    key = (kind, B, T)
    n_cached = _ws_sizes.get(key)
    if n_cached is not None:
        return n_cached
    n = ctypes.c_size_t(0)
    fn = lib().ilqr_b200_solve_workspace_size if kind == "solve" else lib().ilqr_b200_backward_workspace_size
    _check(fn(B, T, ctypes.byref(n)), "workspace query")
    _ws_sizes[key] = int(n.value)
    return _ws_sizes[key]


def solve(x0, U_init, C, c, C_final=None, c_final=None, x_ref=None, u_ref=None,
          u_min=None, u_max=None, dt=0.05, max_iter=10, reg_eps=1e-6, converge_tol=1e-6,
          alphas: Sequence[float] = DEFAULT_ALPHAS, forced_trace=None, want_trace=False,
          want_stats=False, time_major=False):
    """Batched iLQR solve (DifferentiableMPCController.solve_step semantics).

    Returns dict(X [B,T+1,10], U [B,T,4], tight [B,T,4] uint8) plus, when
    requested, trace [B,max_iter] int8 and per-element iters / status /
    best_cost / stall_iter / stall_gap. time_major: C [T,B,14,14] and
    c [T,B,14] (mpc.pytorch's layout) instead of [B,T,...].
    """
    L = lib()
    dev = _cuda_device(x0, "x0")
    _device_ok(dev)
    B = x0.shape[0]
    T = U_init.shape[1]
    _req(x0, "x0", (B, NX), dev)
    _req(U_init, "U_init", (B, T, NU), dev)
    bt = (T, B) if time_major else (B, T)
    _req(C, "C", (*bt, N, N), dev)
    _req(c, "c", (*bt, N), dev)
    _opt(C_final, "C_final", (B, N, N), dev)
    _opt(c_final, "c_final", (B, N), dev)
    _opt(x_ref, "x_ref", (B, T + 1, NX), dev)
    _opt(u_ref, "u_ref", (B, T, NU), dev)
    if (u_min is None) != (u_max is None):
        raise RuntimeError("u_min and u_max must both be given or both be None")
    _opt(u_min, "u_min", (NU,), dev)
    _opt(u_max, "u_max", (NU,), dev)
    _opt(forced_trace, "forced_trace", (B, max_iter), dev, torch.int8)
    al = [float(a) for a in alphas]
    if not 1 <= len(al) <= 8:
        raise RuntimeError("between 1 and 8 line-search step sizes are supported")
    if C_final is None and c_final is not None:
        C_final = torch.zeros(B, N, N, device=dev)
    X = torch.empty(B, T + 1, NX, device=dev)
    U = torch.empty(B, T, NU, device=dev)
    tight = torch.empty(B, T, NU, device=dev, dtype=torch.uint8)
    out = dict(X=X, U=U, tight=tight)
    trace = iters = status = best = s_it = s_gap = None
    if want_trace:
        trace = out["trace"] = torch.empty(B, max_iter, device=dev, dtype=torch.int8)
    if want_stats:
        iters = out["iters"] = torch.empty(B, device=dev, dtype=torch.int32)
        status = out["status"] = torch.empty(B, device=dev, dtype=torch.int32)
        best = out["best_cost"] = torch.empty(B, device=dev)
        s_it = out["stall_iter"] = torch.empty(B, device=dev, dtype=torch.int32)
        s_gap = out["stall_gap"] = torch.empty(B, device=dev)
    nbytes = workspace_bytes("solve", B, T)
    ws = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
    a_arr = _alpha_array(al)
    fn = L.ilqr_b200_solve_tm_f32 if time_major else L.ilqr_b200_solve_f32
    st = fn(
        _ptr(x0), _ptr(U_init), _ptr(C), _ptr(c), _ptr(C_final), _ptr(c_final), _ptr(x_ref),
        _ptr(u_ref), _ptr(u_min), _ptr(u_max), B, T, float(dt), int(max_iter), float(reg_eps),
        float(converge_tol), ctypes.cast(a_arr, ctypes.c_void_p), len(al), _ptr(forced_trace), _ptr(X), _ptr(U), _ptr(tight),
        _ptr(trace), _ptr(iters), _ptr(status), _ptr(best), _ptr(s_it), _ptr(s_gap),
        _ptr(ws), nbytes, _stream(dev))
    _check(st, "ilqr_b200_solve_f32")
    return out


def backward(X, U, C, grad_X, grad_U, C_final=None, x_ref=None, u_ref=None, tight=None,
             dt=0.05, reg_eps=1e-6, need=("x0", "C", "c"), time_major=False):
    """Fused implicit-diff backward at a solved (X, U) (ILQRSolve.backward
    semantics). `need` selects outputs among x0, C, c, C_final, c_final,
    x_ref, u_ref; returns a dict with those keys. time_major: C and the
    gradients of C, c are [T,B,...]."""
    L = lib()
    dev = _cuda_device(X, "X")
    _device_ok(dev)
    B, T1, _ = X.shape
    T = T1 - 1
    _req(X, "X", (B, T + 1, NX), dev)
    _req(U, "U", (B, T, NU), dev)
    bt = (T, B) if time_major else (B, T)
    _req(C, "C", (*bt, N, N), dev)
    _req(grad_X, "grad_X", (B, T + 1, NX), dev)
    _req(grad_U, "grad_U", (B, T, NU), dev)
    _opt(C_final, "C_final", (B, N, N), dev)
    _opt(x_ref, "x_ref", (B, T + 1, NX), dev)
    _opt(u_ref, "u_ref", (B, T, NU), dev)
    _opt(tight, "tight_mask", (B, T, NU), dev, torch.uint8)
    shapes = dict(x0=(B, NX), C=(*bt, N, N), c=(*bt, N), C_final=(B, N, N), c_final=(B, N),
                  x_ref=(B, T + 1, NX), u_ref=(B, T, NU))
    out = {k: torch.empty(shapes[k], device=dev) for k in need}
    nbytes = workspace_bytes("backward", B, T)
    ws = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
    g = lambda k: _ptr(out.get(k))
    fn = L.ilqr_b200_backward_tm_f32 if time_major else L.ilqr_b200_backward_f32
    st = fn(
        _ptr(X), _ptr(U), _ptr(C), _ptr(C_final), _ptr(x_ref), _ptr(u_ref), _ptr(tight),
        _ptr(grad_X), _ptr(grad_U), B, T, float(dt), float(reg_eps),
        g("x0"), g("C"), g("c"), g("C_final"), g("c_final"), g("x_ref"), g("u_ref"),
        _ptr(ws), nbytes, _stream(dev))
    _check(st, "ilqr_b200_backward_f32")
    return out


class SigmoidCostSpec:
    """Constants of the policy's cost construction from its sigmoid output
    (_build_cost_tensors, training_modules/mlp_mpc_policy_diffmpc.py:194-247):
    x_q = s * range_q + eps, c = (x_p - 0.5) * range_p, thrust c =
    -(x_p * range_pt + eps) with range_pt = range_q * mass * 9.806."""

    def __init__(self, eps: float = 0.1, range_q: float = 100000.0, range_p: float = 100000.0,
                 mass: float = 0.752, range_pt: Optional[float] = None):
        self.eps = float(eps)
        self.range_q = float(range_q)
        self.range_p = float(range_p)
        self.range_pt = float(range_q * mass * 9.806 if range_pt is None else range_pt)

    def args(self):
        return (self.eps, self.range_q, self.range_p, self.range_pt)


def solve_sigmoid(x0, U_init, sigmoid_cost, spec: Optional[SigmoidCostSpec] = None, u_min=None, u_max=None,
                  dt=0.05, max_iter=10, reg_eps=1e-6, converge_tol=1e-6,
                  alphas: Sequence[float] = DEFAULT_ALPHAS, forced_trace=None, want_trace=False,
                  want_stats=False):
    """solve() with the costs built in the kernel from the policy's sigmoid
    output [B, 28 T] (zero terminal cost and references, as in the policy).
    Returns the same dict as solve()."""
    L = lib()
    spec = spec or SigmoidCostSpec()
    dev = _cuda_device(x0, "x0")
    _device_ok(dev)
    B = x0.shape[0]
    T = U_init.shape[1]
    _req(x0, "x0", (B, NX), dev)
    _req(U_init, "U_init", (B, T, NU), dev)
    _req(sigmoid_cost, "sigmoid_cost", (B, 2 * N * T), dev)
    if (u_min is None) != (u_max is None):
        raise RuntimeError("u_min and u_max must both be given or both be None")
    _opt(u_min, "u_min", (NU,), dev)
    _opt(u_max, "u_max", (NU,), dev)
    _opt(forced_trace, "forced_trace", (B, max_iter), dev, torch.int8)
    al = [float(a) for a in alphas]
    if not 1 <= len(al) <= 8:
        raise RuntimeError("between 1 and 8 line-search step sizes are supported")
    out = dict(X=torch.empty(B, T + 1, NX, device=dev), U=torch.empty(B, T, NU, device=dev),
               tight=torch.empty(B, T, NU, device=dev, dtype=torch.uint8))
    trace = iters = status = best = s_it = s_gap = None
    if want_trace:
        trace = out["trace"] = torch.empty(B, max_iter, device=dev, dtype=torch.int8)
    if want_stats:
        iters = out["iters"] = torch.empty(B, device=dev, dtype=torch.int32)
        status = out["status"] = torch.empty(B, device=dev, dtype=torch.int32)
        best = out["best_cost"] = torch.empty(B, device=dev)
        s_it = out["stall_iter"] = torch.empty(B, device=dev, dtype=torch.int32)
        s_gap = out["stall_gap"] = torch.empty(B, device=dev)
    nbytes = workspace_bytes("solve", B, T)
    ws = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
    a_arr = _alpha_array(al)
    st = L.ilqr_b200_solve_sigmoid_f32(
        _ptr(x0), _ptr(U_init), _ptr(sigmoid_cost), *spec.args(), _ptr(u_min), _ptr(u_max),
        B, T, float(dt), int(max_iter), float(reg_eps), float(converge_tol),
        ctypes.cast(a_arr, ctypes.c_void_p), len(al), _ptr(forced_trace), _ptr(out["X"]), _ptr(out["U"]),
        _ptr(out["tight"]), _ptr(trace), _ptr(iters), _ptr(status), _ptr(best), _ptr(s_it), _ptr(s_gap),
        _ptr(ws), nbytes, _stream(dev))
    _check(st, "ilqr_b200_solve_sigmoid_f32")
    return out


def backward_sigmoid(X, U, sigmoid_cost, grad_X, grad_U, spec: Optional[SigmoidCostSpec] = None,
                     tight=None, dt=0.05, reg_eps=1e-6, need=("x0", "sigmoid_cost")):
    """backward() for solve_sigmoid(): returns a dict with the gradients of
    x0 [B, 10] and of the sigmoid cost row [B, 28 T] (as selected by need)."""
    L = lib()
    spec = spec or SigmoidCostSpec()
    dev = _cuda_device(X, "X")
    _device_ok(dev)
    B, T1, _ = X.shape
    T = T1 - 1
    _req(X, "X", (B, T + 1, NX), dev)
    _req(U, "U", (B, T, NU), dev)
    _req(sigmoid_cost, "sigmoid_cost", (B, 2 * N * T), dev)
    _req(grad_X, "grad_X", (B, T + 1, NX), dev)
    _req(grad_U, "grad_U", (B, T, NU), dev)
    _opt(tight, "tight_mask", (B, T, NU), dev, torch.uint8)
    shapes = dict(x0=(B, NX), sigmoid_cost=(B, 2 * N * T))
    out = {k: torch.empty(shapes[k], device=dev) for k in need}
    nbytes = workspace_bytes("backward", B, T)
    ws = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
    st = L.ilqr_b200_backward_sigmoid_f32(
        _ptr(X), _ptr(U), _ptr(sigmoid_cost), *spec.args(), _ptr(tight), _ptr(grad_X), _ptr(grad_U),
        B, T, float(dt), float(reg_eps), _ptr(out.get("x0")), _ptr(out.get("sigmoid_cost")),
        _ptr(ws), nbytes, _stream(dev))
    _check(st, "ilqr_b200_backward_sigmoid_f32")
    return out


class CapturedSolve:
    """A fixed-shape solve (and optionally its backward) captured once into a
    CUDA graph and replayed: the launch sequence a control loop repeats every
    tick (solve, then backward) costs one graph launch instead of the host work
    of two entry-point calls. Inputs are copied into static device buffers on
    the current stream; the returned tensors are static buffers that the next
    call overwrites. Dense costs (C, c) by default, or the policy's sigmoid
    output when spec is a SigmoidCostSpec."""

    def __init__(self, B: int, T: int, device=None, u_min=None, u_max=None, dt=0.05, max_iter=10,
                 reg_eps=1e-6, alphas: Sequence[float] = DEFAULT_ALPHAS, with_backward: bool = True,
                 need=("x0", "C", "c"), spec: Optional[SigmoidCostSpec] = None):
        dev = torch.device("cuda") if device is None else torch.device(device)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        _device_ok(dev)
        self.B, self.T, self.spec = B, T, spec
        z = lambda *sh: torch.zeros(*sh, device=dev)
        self.x0, self.U_init = z(B, NX), z(B, T, NU)
        self.U_init[:, :, 0] = HOVER_THRUST
        if spec is None:
            self.C, self.c = z(B, T, N, N), z(B, T, N)
            eye = torch.eye(N, device=dev)
            self.C.copy_(eye.expand(B, T, N, N))
        else:
            self.sc = torch.full((B, 2 * N * T), 0.5, device=dev)
        self.gX, self.gU = z(B, T + 1, NX), z(B, T, NU)
        self.lo = None if u_min is None else u_min.to(dev, torch.float32).contiguous()
        self.hi = None if u_max is None else u_max.to(dev, torch.float32).contiguous()
        kw = dict(dt=dt, max_iter=max_iter, reg_eps=reg_eps, alphas=alphas)
        bwd = dict(dt=dt, reg_eps=reg_eps)

        def run():
            if spec is None:
                out = solve(self.x0, self.U_init, self.C, self.c, None, None, None, None, self.lo, self.hi, **kw)
                g = backward(out["X"], out["U"], self.C, self.gX, self.gU, tight=out["tight"], need=need,
                             **bwd) if with_backward else {}
            else:
                out = solve_sigmoid(self.x0, self.U_init, self.sc, spec, self.lo, self.hi, **kw)
                g = backward_sigmoid(out["X"], out["U"], self.sc, self.gX, self.gU, spec, tight=out["tight"],
                                     **bwd) if with_backward else {}
            return out, g

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            run()  # warm-up outside the capture (library load, first-call work)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out, self.grads = run()

    def __call__(self, x0, U_init=None, C=None, c=None, grad_X=None, grad_U=None, sigmoid_cost=None):
        self.x0.copy_(x0)
        if U_init is not None:
            self.U_init.copy_(U_init)
        if self.spec is None:
            self.C.copy_(C)
            self.c.copy_(c)
        else:
            self.sc.copy_(sigmoid_cost)
        if grad_X is not None:
            self.gX.copy_(grad_X)
        if grad_U is not None:
            self.gU.copy_(grad_U)
        self.graph.replay()
        return self.out, self.grads


class BoundSolve:
    """A fixed-shape solve (and optionally its backward) with everything but
    the inputs prepared once: outputs and workspaces allocated, arguments
    validated and packed for the C ABI. A call checks that the inputs have the
    bound shapes, device and dtype, swaps their pointers into the packed
    arguments and makes one C call per kernel on the current stream; no
    copies and no allocation. The returned tensors are the bound outputs,
    overwritten by the next call. For latency-bound control loops that call
    the solver with the same shapes every tick."""

    def __init__(self, B: int, T: int, device=None, u_min=None, u_max=None, dt=0.05, max_iter=10,
                 reg_eps=1e-6, alphas: Sequence[float] = DEFAULT_ALPHAS, with_backward: bool = True,
                 need=("x0", "C", "c")):
        L = lib()
        dev = torch.device("cuda") if device is None else torch.device(device)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        _device_ok(dev)
        self.dev, self.B, self.T = dev, B, T
        self.lo = None if u_min is None else u_min.to(dev, torch.float32).contiguous()
        self.hi = None if u_max is None else u_max.to(dev, torch.float32).contiguous()
        if (self.lo is None) != (self.hi is None):
            raise RuntimeError("u_min and u_max must both be given or both be None")
        al = [float(a) for a in alphas]
        if not 1 <= len(al) <= 8:
            raise RuntimeError("between 1 and 8 line-search step sizes are supported")
        self._al = (ctypes.c_float * len(al))(*al)
        self.out = dict(X=torch.empty(B, T + 1, NX, device=dev), U=torch.empty(B, T, NU, device=dev),
                        tight=torch.empty(B, T, NU, device=dev, dtype=torch.uint8))
        nb = workspace_bytes("solve", B, T)
        self._ws = torch.empty(max(nb, 1), device=dev, dtype=torch.uint8)
        o = self.out
        # argument list of ilqr_b200_solve_f32; inputs at 0..3 are set per call
        self._sargs = [None, None, None, None, None, None, None, None, _ptr(self.lo), _ptr(self.hi), B, T,
                       float(dt), int(max_iter), float(reg_eps), 1e-6, ctypes.cast(self._al, ctypes.c_void_p),
                       len(al), None, _ptr(o["X"]), _ptr(o["U"]), _ptr(o["tight"]), None, None, None, None,
                       None, None, _ptr(self._ws), nb, None]
        self.grads = {}
        self._bargs = None
        if with_backward:
            shapes = dict(x0=(B, NX), C=(B, T, N, N), c=(B, T, N), C_final=(B, N, N), c_final=(B, N),
                          x_ref=(B, T + 1, NX), u_ref=(B, T, NU))
            self.grads = {k: torch.empty(shapes[k], device=dev) for k in need}
            nbb = workspace_bytes("backward", B, T)
            self._wsb = torch.empty(max(nbb, 1), device=dev, dtype=torch.uint8)
            gp = lambda k: _ptr(self.grads.get(k))
            # argument list of ilqr_b200_backward_f32; C, grad_X, grad_U set per call
            self._bargs = [_ptr(o["X"]), _ptr(o["U"]), None, None, None, None, _ptr(o["tight"]), None, None, B, T,
                           float(dt), float(reg_eps), gp("x0"), gp("C"), gp("c"), gp("C_final"), gp("c_final"),
                           gp("x_ref"), gp("u_ref"), _ptr(self._wsb), nbb, None]
        self._solve = L.ilqr_b200_solve_f32
        self._backward = L.ilqr_b200_backward_f32

    def _check(self, t, name, shape):
        if t.device != self.dev or t.dtype != torch.float32 or tuple(t.shape) != shape or not t.is_contiguous():
            raise RuntimeError(f"{name} must be a contiguous float32 {shape} tensor on {self.dev}")
        return t.data_ptr()

    def __call__(self, x0, U_init, C, c, grad_X=None, grad_U=None):
        B, T = self.B, self.T
        a = self._sargs
        a[0] = self._check(x0, "x0", (B, NX))
        a[1] = self._check(U_init, "U_init", (B, T, NU))
        a[2] = cp = self._check(C, "C", (B, T, N, N))
        a[3] = self._check(c, "c", (B, T, N))
        stream = _stream(self.dev)
        a[-1] = stream
        _check(self._solve(*a), "ilqr_b200_solve_f32")
        if self._bargs is not None and grad_X is not None:
            b = self._bargs
            b[2] = cp
            b[7] = self._check(grad_X, "grad_X", (B, T + 1, NX))
            b[8] = self._check(grad_U, "grad_U", (B, T, NU))
            b[-1] = stream
            _check(self._backward(*b), "ilqr_b200_backward_f32")
        return self.out, self.grads


def pnqp4_batch(H, q, lower, upper, x_init=None):
    """n independent 4-d box QPs by projected Newton (drone_pnqp4_batch):
    returns (x* [n,4], free_mask [n,4])."""
    dev = _cuda_device(H, "H")
    _device_ok(dev)
    n = H.shape[0]
    _req(H, "H", (n, 4, 4), dev)
    for t, nm in ((q, "q"), (lower, "lower"), (upper, "upper")):
        _req(t, nm, (n, 4), dev)
    if x_init is not None and x_init.numel() == 0:
        x_init = None
    _opt(x_init, "x_init", (n, 4), dev)
    x = torch.empty(n, 4, device=dev)
    fm = torch.empty(n, 4, device=dev)
    _check(lib().ilqr_b200_pnqp4_batch_f32(_ptr(H), _ptr(q), _ptr(lower), _ptr(upper), _ptr(x_init), n,
                                           _ptr(x), _ptr(fm), _stream(dev)), "ilqr_b200_pnqp4_batch_f32")
    return x, fm


def dynamics(x, u, dt):
    dev = _cuda_device(x, "x")
    _device_ok(dev)
    n = x.shape[0]
    _req(x, "x", (n, NX), dev)
    _req(u, "u", (n, NU), dev)
    xn = torch.empty_like(x)
    _check(lib().ilqr_b200_dynamics_f32(_ptr(x), _ptr(u), n, float(dt), _ptr(xn), _stream(dev)),
           "ilqr_b200_dynamics_f32")
    return xn


def linearize(X, U, dt):
    dev = _cuda_device(X, "X")
    _device_ok(dev)
    B, T = U.shape[:2]
    _req(X, "X", (B, T + 1, NX), dev)
    _req(U, "U", (B, T, NU), dev)
    A = torch.empty(B, T, NX, NX, device=dev)
    Bm = torch.empty(B, T, NX, NU, device=dev)
    _check(lib().ilqr_b200_linearize_f32(_ptr(X), _ptr(U), B, T, float(dt), _ptr(A), _ptr(Bm),
                                         _stream(dev)), "ilqr_b200_linearize_f32")
    return A, Bm


def adjoint_lqr(A, Bm, l_xx, l_uu, l_xu, l_x, l_u, l_xxN, l_xN, tight, reg_eps):
    dev = _cuda_device(A, "A_lin")
    _device_ok(dev)
    B, T = A.shape[:2]
    for t, nm, sh in ((A, "A_lin", (B, T, NX, NX)), (Bm, "Bm_lin", (B, T, NX, NU)),
                      (l_xx, "l_xx", (B, T, NX, NX)), (l_uu, "l_uu", (B, T, NU, NU)),
                      (l_xu, "l_xu", (B, T, NX, NU)), (l_x, "l_x", (B, T, NX)), (l_u, "l_u", (B, T, NU)),
                      (l_xxN, "l_xxN", (B, NX, NX)), (l_xN, "l_xN", (B, NX))):
        _req(t, nm, sh, dev)
    _opt(tight, "tight_mask", (B, T, NU), dev, torch.uint8)
    K = torch.empty(B, T, NU, NX, device=dev)
    k = torch.empty(B, T, NU, device=dev)
    v0 = torch.empty(B, NX, device=dev)
    _check(lib().ilqr_b200_adjoint_lqr_f32(
        _ptr(A), _ptr(Bm), _ptr(l_xx), _ptr(l_uu), _ptr(l_xu), _ptr(l_x), _ptr(l_u), _ptr(l_xxN),
        _ptr(l_xN), _ptr(tight), B, T, float(reg_eps), _ptr(K), _ptr(k), _ptr(v0), _stream(dev)),
        "ilqr_b200_adjoint_lqr_f32")
    return K, k, v0


def implicit_diff_assembly(K, k, v0, A, Bm, X, U, x_ref=None, u_ref=None, need_xref=False,
                           need_uref=False, need_C_final=False, need_c_final=False):
    dev = _cuda_device(K, "K")
    _device_ok(dev)
    B, T = K.shape[:2]
    for t, nm, sh in ((K, "K", (B, T, NU, NX)), (k, "k", (B, T, NU)), (v0, "v0", (B, NX)),
                      (A, "A_lin", (B, T, NX, NX)), (Bm, "Bm_lin", (B, T, NX, NU)),
                      (X, "X", (B, T + 1, NX)), (U, "U", (B, T, NU))):
        _req(t, nm, sh, dev)
    _opt(x_ref, "x_ref", (B, T + 1, NX), dev)
    _opt(u_ref, "u_ref", (B, T, NU), dev)
    gC = torch.empty(B, T, N, N, device=dev)
    gc = torch.empty(B, T, N, device=dev)
    gx0 = torch.empty(B, NX, device=dev)
    gxr = torch.empty(B, T + 1, NX, device=dev) if need_xref else None
    gur = torch.empty(B, T, NU, device=dev) if need_uref else None
    gCf = torch.empty(B, N, N, device=dev) if need_C_final else None
    gcf = torch.empty(B, N, device=dev) if need_c_final else None
    _check(lib().ilqr_b200_implicit_diff_assembly_f32(
        _ptr(K), _ptr(k), _ptr(v0), _ptr(A), _ptr(Bm), _ptr(X), _ptr(U), _ptr(x_ref), _ptr(u_ref),
        B, T, _ptr(gC), _ptr(gc), _ptr(gx0), _ptr(gxr), _ptr(gur), _ptr(gCf), _ptr(gcf),
        _stream(dev)), "ilqr_b200_implicit_diff_assembly_f32")
    return gC, gc, gx0, gxr, gur, gCf, gcf


def converged_flag(stall_iter, stall_gap, status, max_iter, converge_tol):
    """The reference's global `converged` (controller.py:396-423) from the
    per-element stall iteration and gap: the loop breaks at s = max(stall_iter)
    if the largest gap is below converge_tol, else at s + 2 if that is still
    inside max_iter; a loop that runs out reports convergence iff X, U are
    finite. One device reduction and one host read."""
    if stall_iter.numel() == 0:
        return True
    s = int(stall_iter.max().item())
    if s < max_iter:
        gap = float(stall_gap.max().item())
        if (gap == gap and gap < converge_tol) or s + 2 <= max_iter - 1:
            return True
    return not bool(((status & 2) != 0).any().item())


# ---------------------------------------------------------------------------
# 13-state rotor-thrust quadrotor (state p, q, v, w; four rotor thrusts as
# fractions of F_MAX13 in [0, 1]): the same solver on DiffMPC's model-generic
# path (DifferentialMPC/controller.py:147-160, 607-615).
# ---------------------------------------------------------------------------

NX13 = 13
N13 = NX13 + NU
MASS13 = 0.75
F_MAX13 = 8.5
HOVER_U13 = MASS13 * 9.8066 / (4.0 * F_MAX13)  # per-rotor hover thrust fraction


def rotor13_solve(x0, U_init, C, c, C_final=None, c_final=None, x_ref=None, u_ref=None,
                  u_min=None, u_max=None, dt=0.05, max_iter=10, reg_eps=1e-6, converge_tol=1e-6,
                  alphas: Sequence[float] = DEFAULT_ALPHAS, forced_trace=None, want_trace=False,
                  want_stats=False, time_major=False):
    """solve() for the rotor model: X [B,T+1,13], U [B,T,4], C [B,T,17,17]
    ([T,B,17,17] and c [T,B,17] when time_major)."""
    L = lib()
    dev = _cuda_device(x0, "x0")
    _device_ok(dev)
    B = x0.shape[0]
    T = U_init.shape[1]
    _req(x0, "x0", (B, NX13), dev)
    _req(U_init, "U_init", (B, T, NU), dev)
    bt = (T, B) if time_major else (B, T)
    _req(C, "C", (*bt, N13, N13), dev)
    _req(c, "c", (*bt, N13), dev)
    _opt(C_final, "C_final", (B, N13, N13), dev)
    _opt(c_final, "c_final", (B, N13), dev)
    _opt(x_ref, "x_ref", (B, T + 1, NX13), dev)
    _opt(u_ref, "u_ref", (B, T, NU), dev)
    if (u_min is None) != (u_max is None):
        raise RuntimeError("u_min and u_max must both be given or both be None")
    _opt(u_min, "u_min", (NU,), dev)
    _opt(u_max, "u_max", (NU,), dev)
    _opt(forced_trace, "forced_trace", (B, max_iter), dev, torch.int8)
    al = [float(a) for a in alphas]
    if not 1 <= len(al) <= 8:
        raise RuntimeError("between 1 and 8 line-search step sizes are supported")
    if C_final is None and c_final is not None:
        C_final = torch.zeros(B, N13, N13, device=dev)
    X = torch.empty(B, T + 1, NX13, device=dev)
    U = torch.empty(B, T, NU, device=dev)
    tight = torch.empty(B, T, NU, device=dev, dtype=torch.uint8)
    out = dict(X=X, U=U, tight=tight)
    trace = iters = status = best = s_it = s_gap = None
    if want_trace:
        trace = out["trace"] = torch.empty(B, max_iter, device=dev, dtype=torch.int8)
    if want_stats:
        iters = out["iters"] = torch.empty(B, device=dev, dtype=torch.int32)
        status = out["status"] = torch.empty(B, device=dev, dtype=torch.int32)
        best = out["best_cost"] = torch.empty(B, device=dev)
        s_it = out["stall_iter"] = torch.empty(B, device=dev, dtype=torch.int32)
        s_gap = out["stall_gap"] = torch.empty(B, device=dev)
    n = ctypes.c_size_t(0)
    _check(L.ilqr_b200_rotor13_solve_workspace_size(B, T, len(al), ctypes.byref(n)), "workspace query")
    nbytes = int(n.value)
    ws = torch.empty(max(nbytes, 16), device=dev, dtype=torch.uint8)
    a_arr = _alpha_array(al)
    fn = L.ilqr_b200_rotor13_solve_tm_f32 if time_major else L.ilqr_b200_rotor13_solve_f32
    st = fn(
        _ptr(x0), _ptr(U_init), _ptr(C), _ptr(c), _ptr(C_final), _ptr(c_final), _ptr(x_ref),
        _ptr(u_ref), _ptr(u_min), _ptr(u_max), B, T, float(dt), int(max_iter), float(reg_eps),
        float(converge_tol), ctypes.cast(a_arr, ctypes.c_void_p), len(al), _ptr(forced_trace), _ptr(X), _ptr(U),
        _ptr(tight), _ptr(trace), _ptr(iters), _ptr(status), _ptr(best), _ptr(s_it), _ptr(s_gap),
        _ptr(ws), nbytes, _stream(dev))
    _check(st, "ilqr_b200_rotor13_solve_f32")
    return out


def rotor13_backward(X, U, C, grad_X, grad_U, C_final=None, x_ref=None, u_ref=None, tight=None,
                     dt=0.05, reg_eps=1e-6, need=("x0", "C", "c"), time_major=False):
    """backward() for the rotor model; `need` and `time_major` as there."""
    L = lib()
    dev = _cuda_device(X, "X")
    _device_ok(dev)
    B, T1, _ = X.shape
    T = T1 - 1
    _req(X, "X", (B, T + 1, NX13), dev)
    _req(U, "U", (B, T, NU), dev)
    bt = (T, B) if time_major else (B, T)
    _req(C, "C", (*bt, N13, N13), dev)
    _req(grad_X, "grad_X", (B, T + 1, NX13), dev)
    _req(grad_U, "grad_U", (B, T, NU), dev)
    _opt(C_final, "C_final", (B, N13, N13), dev)
    _opt(x_ref, "x_ref", (B, T + 1, NX13), dev)
    _opt(u_ref, "u_ref", (B, T, NU), dev)
    _opt(tight, "tight_mask", (B, T, NU), dev, torch.uint8)
    shapes = dict(x0=(B, NX13), C=(*bt, N13, N13), c=(*bt, N13), C_final=(B, N13, N13),
                  c_final=(B, N13), x_ref=(B, T + 1, NX13), u_ref=(B, T, NU))
    out = {k: torch.empty(shapes[k], device=dev) for k in need}
    n = ctypes.c_size_t(0)
    _check(L.ilqr_b200_rotor13_backward_workspace_size(B, T, ctypes.byref(n)), "workspace query")
    nbytes = int(n.value)
    ws = torch.empty(max(nbytes, 16), device=dev, dtype=torch.uint8)
    g = lambda k: _ptr(out.get(k))
    fn = L.ilqr_b200_rotor13_backward_tm_f32 if time_major else L.ilqr_b200_rotor13_backward_f32
    st = fn(
        _ptr(X), _ptr(U), _ptr(C), _ptr(C_final), _ptr(x_ref), _ptr(u_ref), _ptr(tight),
        _ptr(grad_X), _ptr(grad_U), B, T, float(dt), float(reg_eps),
        g("x0"), g("C"), g("c"), g("C_final"), g("c_final"), g("x_ref"), g("u_ref"),
        _ptr(ws), nbytes, _stream(dev))
    _check(st, "ilqr_b200_rotor13_backward_f32")
    return out


def rotor13_dynamics(x, u, dt):
    """One rotor-model step for x [n,13], u [n,4]."""
    dev = _cuda_device(x, "x")
    n = x.shape[0]
    _req(x, "x", (n, NX13), dev)
    _req(u, "u", (n, NU), dev)
    xn = torch.empty(n, NX13, device=dev)
    _check(lib().ilqr_b200_rotor13_dynamics_f32(_ptr(x), _ptr(u), n, float(dt), _ptr(xn), _stream(dev)),
           "ilqr_b200_rotor13_dynamics_f32")
    return xn


def rotor13_linearize(X, U, dt):
    """Rotor-model Jacobians A [B,T,13,13], B [B,T,13,4] at (X_t, U_t)."""
    dev = _cuda_device(X, "X")
    B, T1, _ = X.shape
    T = T1 - 1
    _req(X, "X", (B, T + 1, NX13), dev)
    _req(U, "U", (B, T, NU), dev)
    A = torch.empty(B, T, NX13, NX13, device=dev)
    Bm = torch.empty(B, T, NX13, NU, device=dev)
    _check(lib().ilqr_b200_rotor13_linearize_f32(_ptr(X), _ptr(U), B, T, float(dt), _ptr(A), _ptr(Bm),
                                                _stream(dev)), "ilqr_b200_rotor13_linearize_f32")
    return A, Bm


# --------------------------------------------------------------------------
# FastMPC numerics mode (the reference FastMPC extension's CUDA build)
# --------------------------------------------------------------------------

FASTMPC_ALPHAS = (1.0, 0.5, 0.25, 0.1)  # drone_ilqr_ext.cpp:736


def fastmpc_solve(x0, U_init, C, c, C_final=None, c_final=None, x_ref=None, u_ref=None, u_min=None, u_max=None,
                  dt=0.05, max_iter=10, reg_eps=1e-6, converge_tol=1e-6,
                  alphas: Sequence[float] = FASTMPC_ALPHAS, forced_trace=None, forced_stop=0, want_trace=False,
                  time_major=False):
    """Batched solve with the reference FastMPC build's numerics
    (ext.drone_ilqr_solve, drone_ilqr_ext.cpp:664-1064).

    Returns dict(X [B,T+1,10], U [B,T,4], tight [B,T,4] uint8, X_lin, U_lin
    (where the last Riccati pass linearised; the backward's A, B),
    best_cost [B], batch_info [2] int32 (converged, iterations run)) plus
    trace [B,max_iter] int8 when requested. time_major: C [T,B,14,14] and
    c [T,B,14]."""
    L = lib()
    dev = _cuda_device(x0, "x0")
    _device_ok(dev)
    B = x0.shape[0]
    T = U_init.shape[1]
    _req(x0, "x0", (B, NX), dev)
    _req(U_init, "U_init", (B, T, NU), dev)
    bt = (T, B) if time_major else (B, T)
    _req(C, "C", (*bt, N, N), dev)
    _req(c, "c", (*bt, N), dev)
    _opt(C_final, "C_final", (B, N, N), dev)
    _opt(c_final, "c_final", (B, N), dev)
    _opt(x_ref, "x_ref", (B, T + 1, NX), dev)
    _opt(u_ref, "u_ref", (B, T, NU), dev)
    if (u_min is None) != (u_max is None):
        raise RuntimeError("u_min and u_max must both be given or both be None")
    _opt(u_min, "u_min", (NU,), dev)
    _opt(u_max, "u_max", (NU,), dev)
    _opt(forced_trace, "forced_trace", (B, max_iter), dev, torch.int8)
    al = [float(a) for a in alphas]
    if not 1 <= len(al) <= 8:
        raise RuntimeError("between 1 and 8 line-search step sizes are supported")
    X = torch.empty(B, T + 1, NX, device=dev)
    U = torch.empty(B, T, NU, device=dev)
    out = dict(X=X, U=U, tight=torch.empty(B, T, NU, device=dev, dtype=torch.uint8),
               X_lin=torch.empty(B, T + 1, NX, device=dev), U_lin=torch.empty(B, T, NU, device=dev),
               best_cost=torch.empty(B, device=dev), batch_info=torch.zeros(2, device=dev, dtype=torch.int32))
    if want_trace:
        out["trace"] = torch.empty(B, max_iter, device=dev, dtype=torch.int8)
    n = ctypes.c_size_t(0)
    _check(L.ilqr_b200_fastmpc_solve_workspace_size(B, T, len(al), ctypes.byref(n)), "workspace query")
    nbytes = int(n.value)
    ws = torch.empty(max(nbytes, 16), device=dev, dtype=torch.uint8)
    a_arr = _alpha_array(al)
    st = L.ilqr_b200_fastmpc_solve_f32(
        _ptr(x0), _ptr(U_init), _ptr(C), _ptr(c), _ptr(C_final), _ptr(c_final), _ptr(x_ref), _ptr(u_ref),
        _ptr(u_min), _ptr(u_max), B, T, float(dt), int(max_iter), float(reg_eps), float(converge_tol),
        ctypes.cast(a_arr, ctypes.c_void_p), len(al), 1 if time_major else 0, _ptr(forced_trace), int(forced_stop),
        _ptr(X), _ptr(U), _ptr(out["tight"]), _ptr(out["X_lin"]), _ptr(out["U_lin"]), _ptr(out.get("trace")),
        _ptr(out["best_cost"]), _ptr(out["batch_info"]), _ptr(ws), nbytes, _stream(dev))
    _check(st, "ilqr_b200_fastmpc_solve_f32")
    return out


def fastmpc_backward(X, U, X_lin, U_lin, C, grad_X, grad_U, tight=None, C_final=None, x_ref=None, u_ref=None,
                     dt=0.05, reg_eps=1e-6, need=("x0", "C", "c"), time_major=False):
    """The reference FastMPC operator's backward on its CUDA path
    (mpc_compat.py:188-258: drone_backward_pass_batched then
    drone_implicit_diff_assembly). `need` selects outputs among x0, C, c,
    C_final, c_final, x_ref, u_ref."""
    L = lib()
    dev = _cuda_device(X, "X")
    _device_ok(dev)
    B, T1, _ = X.shape
    T = T1 - 1
    _req(X, "X", (B, T + 1, NX), dev)
    _req(U, "U", (B, T, NU), dev)
    _req(X_lin, "X_lin", (B, T + 1, NX), dev)
    _req(U_lin, "U_lin", (B, T, NU), dev)
    bt = (T, B) if time_major else (B, T)
    _req(C, "C", (*bt, N, N), dev)
    _req(grad_X, "grad_X", (B, T + 1, NX), dev)
    _req(grad_U, "grad_U", (B, T, NU), dev)
    _opt(C_final, "C_final", (B, N, N), dev)
    _opt(x_ref, "x_ref", (B, T + 1, NX), dev)
    _opt(u_ref, "u_ref", (B, T, NU), dev)
    _opt(tight, "tight_mask", (B, T, NU), dev, torch.uint8)
    shapes = dict(x0=(B, NX), C=(*bt, N, N), c=(*bt, N), C_final=(B, N, N), c_final=(B, N),
                  x_ref=(B, T + 1, NX), u_ref=(B, T, NU))
    out = {k: torch.empty(shapes[k], device=dev) for k in need}
    n = ctypes.c_size_t(0)
    _check(L.ilqr_b200_fastmpc_backward_workspace_size(B, T, ctypes.byref(n)), "workspace query")
    nbytes = int(n.value)
    ws = torch.empty(max(nbytes, 16), device=dev, dtype=torch.uint8)
    g = lambda k: _ptr(out.get(k))
    st = L.ilqr_b200_fastmpc_backward_f32(
        _ptr(X), _ptr(U), _ptr(X_lin), _ptr(U_lin), _ptr(C), _ptr(C_final), _ptr(x_ref), _ptr(u_ref), _ptr(tight),
        _ptr(grad_X), _ptr(grad_U), B, T, float(dt), float(reg_eps), 1 if time_major else 0,
        g("x0"), g("C"), g("c"), g("C_final"), g("c_final"), g("x_ref"), g("u_ref"), _ptr(ws), nbytes,
        _stream(dev))
    _check(st, "ilqr_b200_fastmpc_backward_f32")
    return out


def fastmpc_linearize(X, U, dt):
    """A [B,T,10,10], B [B,T,10,4] of the FastMPC build's Jacobian at (X_t, U_t)."""
    dev = _cuda_device(X, "X")
    _device_ok(dev)
    B, T1, _ = X.shape
    T = T1 - 1
    _req(X, "X", (B, T + 1, NX), dev)
    _req(U, "U", (B, T, NU), dev)
    A = torch.empty(B, T, NX, NX, device=dev)
    Bm = torch.empty(B, T, NX, NU, device=dev)
    _check(lib().ilqr_b200_fastmpc_linearize_f32(_ptr(X), _ptr(U), B, T, float(dt), _ptr(A), _ptr(Bm), _stream(dev)),
           "ilqr_b200_fastmpc_linearize_f32")
    return A, Bm


def fastmpc_adjoint_lqr(A, Bm, l_xx, l_uu, l_xu, l_x, l_u, l_xxN, l_xN, tight=None, reg_eps=1e-6):
    """ext.drone_backward_pass_batched of the FastMPC build: (K, k, v0)."""
    dev = _cuda_device(A, "A")
    _device_ok(dev)
    B, T = A.shape[:2]
    for t_, nm, sh in ((A, "A", (B, T, NX, NX)), (Bm, "B", (B, T, NX, NU)), (l_xx, "l_xx", (B, T, NX, NX)),
                       (l_uu, "l_uu", (B, T, NU, NU)), (l_xu, "l_xu", (B, T, NX, NU)), (l_x, "l_x", (B, T, NX)),
                       (l_u, "l_u", (B, T, NU)), (l_xxN, "l_xxN", (B, NX, NX)), (l_xN, "l_xN", (B, NX))):
        _req(t_, nm, sh, dev)
    _opt(tight, "tight_mask", (B, T, NU), dev, torch.uint8)
    K = torch.empty(B, T, NU, NX, device=dev)
    k = torch.empty(B, T, NU, device=dev)
    v0 = torch.empty(B, NX, device=dev)
    _check(lib().ilqr_b200_fastmpc_adjoint_lqr_f32(
        _ptr(A), _ptr(Bm), _ptr(l_xx), _ptr(l_uu), _ptr(l_xu), _ptr(l_x), _ptr(l_u), _ptr(l_xxN), _ptr(l_xN),
        _ptr(tight), B, T, float(reg_eps), _ptr(K), _ptr(k), _ptr(v0), _stream(dev)),
        "ilqr_b200_fastmpc_adjoint_lqr_f32")
    return K, k, v0


def fastmpc_assembly(K, k, v0, A, Bm, X, U, x_ref=None, u_ref=None, compute_xref=False, compute_uref=False,
                     compute_C_final=False, compute_c_final=False):
    """ext.drone_implicit_diff_assembly of the FastMPC build: (grad_C, grad_c,
    grad_x0, grad_xref, grad_uref, grad_C_final, grad_c_final), None where
    not requested."""
    dev = _cuda_device(X, "X")
    _device_ok(dev)
    B, T1, _ = X.shape
    T = T1 - 1
    for t_, nm, sh in ((K, "K", (B, T, NU, NX)), (k, "k", (B, T, NU)), (v0, "v0", (B, NX)),
                       (A, "A", (B, T, NX, NX)), (Bm, "B", (B, T, NX, NU)), (X, "X", (B, T + 1, NX)),
                       (U, "U", (B, T, NU))):
        _req(t_, nm, sh, dev)
    _opt(x_ref, "x_ref", (B, T + 1, NX), dev)
    _opt(u_ref, "u_ref", (B, T, NU), dev)
    e = lambda *sh: torch.empty(*sh, device=dev)
    gC, gc, gx0 = e(B, T, N, N), e(B, T, N), e(B, NX)
    gxr = e(B, T + 1, NX) if compute_xref else None
    gur = e(B, T, NU) if compute_uref else None
    gCf = e(B, N, N) if compute_C_final else None
    gcf = e(B, N) if compute_c_final else None
    _check(lib().ilqr_b200_fastmpc_assembly_f32(
        _ptr(K), _ptr(k), _ptr(v0), _ptr(A), _ptr(Bm), _ptr(X), _ptr(U), _ptr(x_ref), _ptr(u_ref), B, T, _ptr(gC),
        _ptr(gc), _ptr(gx0), _ptr(gxr), _ptr(gur), _ptr(gCf), _ptr(gcf), _stream(dev)),
        "ilqr_b200_fastmpc_assembly_f32")
    return gC, gc, gx0, gxr, gur, gCf, gcf

