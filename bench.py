#!/usr/bin/env python
"""Benchmark: batched differentiable iLQR, fwd+bwd solves/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one forward solve (all iLQR iterations) plus the implicit-diff
backward of a global batch of 16384 quadrotor MPC problems with horizon 20
and 5 iterations (the training-scale rollout workload). With N ranks the
batch is sharded by rank (rank r solves the contiguous slice
shard_bounds(16384, r, N)) and the first actions and dL/dx0 are all-gathered
over NCCL inside the step (strong scaling). Rank 0 prints one JSON line; the
larger sections (rotor13 model, FastMPC numerics, sigmoid costs, policy
actor step) go to earlier lines that start with "#section".

  value  global-batch solves/s with inputs resident in HBM (device time, max
         over ranks); the cost blocks (257 MB) exceed the 126 MB L2.
  e2e    the same through the reference-facing operator
         (mpc_compat.MPC(...)(x_init, QuadCost(C, c), dx) + autograd backward)
         with host buffers: every step copies its inputs from pinned host
         memory and reads the actions and dL/dx0 back.
  cpu_baseline  the reference DiffMPC solver itself (staged from the
         reference's sources into oracle/_ref/diffmpc) on the host cores,
         one process per core, over a bounded sample; the numpy port of it
         beside it.
  fastmpc_ref_cuda  the reference FastMPC extension's own CUDA kernels
         (oracle/_ref/libfastmpc_ref.so) through a torch restatement of its
         host loop, on the same inputs and GPU.
  --impl reference: the reference's CPU solver on all host cores (DiffMPC
         itself when staged, else the numpy port), over a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "ca-ac-mpc_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "iLQR fwd+bwd solves/s @B=16384,T=20 at 1/2/4/8 B200; p50 latency @B=16,T=5"
WORKLOAD = "rollout_b16384_t20"


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sigmoid", action="store_true",
                    help="skip the section for costs given as the policy's sigmoid output")
    ap.add_argument("--no-fastmpc", action="store_true",
                    help="skip the FastMPC-numerics section")
    ap.add_argument("--no-rotor13", action="store_true",
                    help="skip the section for the 13-state rotor-thrust model")
    ap.add_argument("--all-configs", action="store_true",
                    help="instead of the benchmark line: one JSON line per workload configuration "
                         "(both models, 1 GPU, device-resident)")
    ap.add_argument("--latency-reps", type=int, default=200)
    ap.add_argument("--batch", type=int, default=None,
                    help="global batch (default: the workload's 16384); for profiling runs")
    ap.add_argument("--no-ref-baselines", action="store_true",
                    help="skip the reference FastMPC CUDA build and the DiffMPC CPU baseline")
    ap.add_argument("--no-weak", action="store_true",
                    help="skip the weak-scaling figure (16384 elements per rank) of runs with N > 1")
    ap.add_argument("--no-inference", action="store_true",
                    help="skip the sharded inference configuration (B=262144, T=10) of runs with N > 1")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    # NVML clocks-event reason bits: sw_power_cap, hw_slowdown,
    # sw_thermal_slowdown, hw_thermal_slowdown (nvml.h)
    NVML_BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                 ("sw_power_cap", 0x4))

    def __init__(self, index: int, pci=None):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._first = threading.Event()
        self._t = None
        self._nvml = None
        if pci is not None:
            try:  # read-only NVML queries, every 2 ms: several samples even in a short timed region
                import pynvml
                pynvml.nvmlInit()
                self._nvml = (pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(pci))
            except Exception:
                self._nvml = None

    def _sample_nvml(self):
        nv, h = self._nvml
        try:
            reasons_fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
            r = reasons_fn(h)
            self.samples.append([str(self.index), str(sm), str(mx), "", ""]
                                + ["Active" if r & bit else "Not Active" for _, bit in self.NVML_BITS])
        except Exception:
            pass

    def _run_nvml(self):
        while not self._stop.is_set():
            self._sample_nvml()
            self._first.set()
            self._stop.wait(0.002)

    def _run(self):
        if self._nvml is not None:
            return self._run_nvml()
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._first.set()
            self._stop.wait(0.2)

    def __enter__(self):
        # the first sample is taken before the timed region opens and a last
        # one when it closes, so even a region of a few milliseconds has two
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        self._first.wait(6.0)
        return self

    def __exit__(self, *a):
        if self._nvml is not None:
            self._sample_nvml()
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples), "source": "nvml" if self._nvml is not None else "nvidia-smi"}


# ---------------------------------------------------------------------------
# Shared config and the reference's CPU solver (baseline leg, reference arm)
# ---------------------------------------------------------------------------
def headline_config(world: int):
    """The config object of the benchmark line, shared by both arms."""
    import ilqr_workload as wl
    cfg = wl.CONFIGS[WORKLOAD]
    return {"workload": WORKLOAD, "B": cfg["B"], "T": cfg["T"], "iters": cfg["max_iter"],
            "alphas": list(cfg["alphas"]), "dt": wl.DT, "control_box": True,
            "parallelism": f"batch sharded by rank over {world}",
            "l2": "inputs > L2 (C 257 MB), no flush"}


def cpu_rate(impl: str, workers: int, chunk: int, reps: int = 1):
    """Element solves/s of the reference's CPU solver ("reference": DiffMPC
    itself, "port": its numpy restatement) over `workers` spawned processes
    of `chunk` elements each (best of `reps`)."""
    from oracle.cpu_pool import OraclePool
    pool = OraclePool(workers, ROOT, PKG, impl)
    try:
        best = None
        for _ in range(reps):
            n, t = pool.run(WORKLOAD, workers, chunk)
            best = t if best is None else min(best, t)
        return n / best, n, best
    finally:
        pool.close()


def diffmpc_staged() -> bool:
    from oracle import diffmpc_ref
    return diffmpc_ref.available()


def run_reference(args):
    """The reference's own CPU implementation of the path on the host cores:
    DiffMPC itself (one single-threaded process per core, 256-element chunks)
    when its sources are staged in oracle/_ref/diffmpc, else the numpy port.
    Only rank 0 works; the other ranks exit."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    import ilqr_workload as wl
    cores = len(os.sched_getaffinity(0))
    from oracle.cpu_pool import OraclePool
    impl = "reference" if diffmpc_staged() else "port"
    chunk = 256 if impl == "reference" else 1024
    pool = OraclePool(cores, ROOT, PKG, impl)
    try:
        for _ in range(args.warmup):
            pool.run(WORKLOAD, cores, chunk)
        times = []
        n = 0
        for _ in range(args.steps):
            n, t = pool.run(WORKLOAD, cores, chunk)
            times.append(t)
    finally:
        pool.close()
    cfg = wl.CONFIGS[WORKLOAD]
    step = statistics.mean(times)
    value = n / step
    what = "DiffMPC itself" if impl == "reference" else "numpy port of DiffMPC"
    sample = f"{n} of {cfg['B']} elements/step, {cores} procs x {chunk}, {what}"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "solves/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": headline_config(world),
        "cpu_baseline": {"value": value, "unit": "solves/s", "cores": cores,
                         "kind": "reference" if impl == "reference" else "port", "sample": sample},
        "e2e": {"value": value, "unit": "solves/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def fp32_peak_tflops(torch, device):
    """Measured FP32 FMA throughput of this GPU (8 independent FMA chains per
    thread, 8 CTAs x 256 threads per SM), best of 5 launches."""
    import ctypes
    L = ctypes.CDLL(os.path.join(PKG, "libilqr_probe.so"))
    L.ilqr_probe_fma.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    L.ilqr_probe_fma_flops.restype = ctypes.c_double
    L.ilqr_probe_fma_flops.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    blocks, threads, iters = sms * 8, 256, 4096
    out = torch.empty(blocks * threads, device=device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    best = 0.0
    for _ in range(6):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        L.ilqr_probe_fma(ctypes.c_void_p(out.data_ptr()), blocks, threads, iters, stream)
        e1.record()
        torch.cuda.synchronize()
        best = max(best, L.ilqr_probe_fma_flops(blocks, threads, iters) / (e0.elapsed_time(e1) * 1e-3) / 1e12)
    return best


def time_streaming(torch, dev, stream, host, compute, warm, steps, barrier):
    """Seconds for `steps` calls of compute(device_buffers) with host inputs
    streamed: the host tensors of call k + 1 are copied into the other half of
    a device double buffer on a second stream while call k computes, as a
    data loader prefetches the next batch. compute enqueues one call's work
    and its result read-back on `stream`; every call's copies and read-back
    are inside the timed region."""
    cstream = torch.cuda.Stream(dev)
    bufs = [[torch.empty_like(h, device=dev) for h in host] for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    for f_ in free:
        f_.record(stream)

    def prefetch(k):
        i = k % 2
        with torch.cuda.stream(cstream):
            cstream.wait_event(free[i])
            for dst, src in zip(bufs[i], host):
                dst.copy_(src, non_blocking=True)
            ready[i].record(cstream)

    def run(n):
        prefetch(0)
        if n > 1:
            prefetch(1)
        for k in range(n):
            i = k % 2
            stream.wait_event(ready[i])
            compute(bufs[i])
            free[i].record(stream)
            if k + 2 < n:
                prefetch(k + 2)

    run(warm)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    cstream.wait_event(e0)
    run(steps)
    e1.record(stream)
    barrier()
    return e0.elapsed_time(e1) * 1e-3


def gpu_pci_bus_id(torch, dev_index):
    """NVML PCI bus id of a CUDA device (None if torch does not report it)."""
    try:
        pr = torch.cuda.get_device_properties(dev_index)
        return f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
    except Exception:
        return None


def bind_to_gpu_numa_node(torch, dev_index):
    """Pin this process to the host CPUs NVML reports as local to its GPU, so
    the pinned host buffers of the end-to-end measurement are allocated and
    read on the GPU's own socket. Process-local; returns the CPUs chosen (None
    if NVML or the PCI address is not available)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(dev_index)
        bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = ((os.cpu_count() or 64) + 63) // 64
        masks = pynvml.nvmlDeviceGetCpuAffinity(h, words)
        cpus = {w * 64 + bit for w, m in enumerate(masks) for bit in range(64) if (m >> bit) & 1}
        cpus &= set(os.sched_getaffinity(0))
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return sorted(cpus)
    except Exception:
        return None


def shard_inputs(wl, B_glob, T, lo, hi, cfg, seed=0):
    """Inputs of elements [lo, hi) of the seeded global batch (the block
    generators make any 1024-aligned slice directly; other slices are cut
    from the generated prefix)."""
    if lo % wl.BLOCK == 0:
        return wl.make_inputs(hi - lo, T, seed=seed, target=cfg["target"], r=cfg["r"], offset=lo)
    full = wl.make_inputs(hi, T, seed=seed, target=cfg["target"], r=cfg["r"])
    return {k: v[lo:hi] for k, v in full.items()}


def kernel_source_sha(names):
    """Short hash of the kernel sources a committed profile describes."""
    import hashlib
    h = hashlib.sha256()
    for n in names:
        with open(os.path.join(PKG, "csrc", n), "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


def solve_variant(B: int) -> str:
    """The solve kernel a batch of B elements launches (the library's own
    choice, PAIR_MAX_B and pick_solve_tier in csrc/): the pair layout up to 4096
    elements, else the team layout at 8 CTAs per SM while the grid fits one
    such wave, at 12 up to one such wave, at 19 up to 1.5 waves of 12, and at
    12 beyond."""
    if B <= 4096:
        return "pair"
    grid = (B + 5) // 6
    if grid <= 148 * 8:
        tier = 8
    elif grid <= 148 * 12 or 2 * grid > 3 * 148 * 12:
        tier = 12
    else:
        tier = 19
    return f"team_tier{tier}" + ("_seg" if solve_segmented(B, 5) else "")


def solve_segmented(B: int, max_iter: int) -> bool:
    """Whether the library runs this solve as a chain of launches (launch_solve
    in csrc/ilqr_solve.cu: team layout beyond one 8-CTA wave, max_iter >= 4, no
    forced trace, ILQR_B200_SEGMENT not 0), each later launch on the elements
    still improving, compacted."""
    if os.environ.get("ILQR_B200_SEGMENT", "1").startswith("0"):
        return False
    return B > 4096 and (B + 5) // 6 > 148 * 8 and max_iter >= 4


def solve_launches(B: int, max_iter: int) -> int:
    """Kernel launches of one solve: two (a split after max_iter - 2) up to
    5 iterations, else one per iteration."""
    if not solve_segmented(B, max_iter):
        return 1
    return 2 if max_iter <= 5 else max_iter


SOLVE_SOURCES = ("ilqr_solve.cu", "ilqr_team.cuh", "ilqr_pair.cuh", "ilqr_device.cuh")


def committed_traffic(variant: str, B: int, T: int):
    """DRAM bytes per launch of this solve variant from the committed ncu
    summary (profiles/solve_kernel_traffic.json), scaled to B elements. Only
    returned while the kernel sources still hash to the captured ones; else
    (None, why)."""
    try:
        prof = json.load(open(os.path.join(ROOT, "profiles", "solve_kernel_traffic.json")))
    except Exception:
        return None, "no committed capture"
    e = prof.get(f"{variant}_t{T}")
    if e is None:
        return None, f"no capture of {variant} at T={T}"
    if e.get("source_sha") != kernel_source_sha(SOLVE_SOURCES):
        return None, f"capture of {variant} is stale (kernel sources changed)"
    return e["dram_bytes_per_launch"] * B / e["B"], f"{e['summary']} (B={e['B']}, scaled per element)"


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    import ilqr_costmodel as cm
    import ilqr_native as nat
    import ilqr_shard
    import ilqr_workload as wl
    import mpc_compat

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    all_cpus = os.sched_getaffinity(0)
    numa_cpus = bind_to_gpu_numa_node(torch, local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    cfg = wl.CONFIGS[WORKLOAD]
    B_glob, T, iters, alphas = cfg["B"], cfg["T"], cfg["max_iter"], cfg["alphas"]
    if args.batch is not None:
        B_glob = args.batch
    # The global batch is one seeded set of problems; rank r solves the
    # contiguous slice shard_bounds(B_glob, r, world) of it.
    s_lo, s_hi = ilqr_shard.shard_bounds(B_glob, rank, world)
    B = s_hi - s_lo
    inp = shard_inputs(wl, B_glob, T, s_lo, s_hi, cfg)
    gXn, gUn = (a[s_lo:s_hi] for a in wl.make_backward_seeds(B_glob, T, seed=1))
    d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in inp.items()}
    gX, gU = torch.from_numpy(np.ascontiguousarray(gXn)).to(dev), torch.from_numpy(np.ascontiguousarray(gUn)).to(dev)
    lo, hi = torch.from_numpy(wl.U_MIN).to(dev), torch.from_numpy(wl.U_MAX).to(dev)

    stream = torch.cuda.current_stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def step(timing=None):
        if timing is not None:
            timing[0].record(stream)
        out = nat.solve(d["x0"], d["U_init"], d["C"], d["c"], None, None, None, None, lo, hi,
                        dt=wl.DT, max_iter=iters, reg_eps=wl.REG_EPS, alphas=alphas)
        if timing is not None:
            timing[1].record(stream)
        g = nat.backward(out["X"], out["U"], d["C"], gX, gU, tight=out["tight"], dt=wl.DT,
                         reg_eps=wl.REG_EPS, need=("x0", "C", "c"))
        if timing is not None:
            timing[2].record(stream)
        if world > 1:
            # actions and dL/dx0 of every shard to rank 0 (one all-gather over NCCL)
            ilqr_shard.gather_actions_and_gradients(out["U"], g, B_glob, keys=("x0",))
        if timing is not None:
            timing[3].record(stream)
        return out, g

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world > 1:
            t = torch.tensor([x], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
        return x

    # ---- device-resident throughput ---------------------------------------
    # The step (solve, backward and, for N > 1, the NCCL gather) is captured
    # once in a CUDA graph and the timed region replays it K times, so that
    # the time is the GPU's and not the host's enqueueing of about twenty
    # small launches (at 2048 elements per GPU the two are comparable). An
    # eager loop with events between the kernels gives the per-kernel times.
    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    timings = [(ev(), ev(), ev(), ev()) for _ in range(args.steps)]
    e_start, e_end = ev(), ev()
    e_start.record(stream)
    for i in range(args.steps):
        step(timings[i])
    e_end.record(stream)
    barrier()
    eager_per_step = max_over_ranks(e_start.elapsed_time(e_end) * 1e-3) / args.steps
    solve_ms = [a.elapsed_time(b) for a, b, _, _ in timings]
    bwd_ms = [b.elapsed_time(c) for _, b, c, _ in timings]
    gather_ms = max_over_ranks(statistics.mean(c.elapsed_time(e) for _, _, c, e in timings))
    graph = None
    try:
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                step()
        stream.wait_stream(side)
        for _ in range(max(3, args.warmup)):
            graph.replay()
        barrier()
    except Exception as exc:  # capture not possible here: time the eager loop
        graph = None
        print(f"#note step graph capture failed ({type(exc).__name__}: {exc}); eager timing", flush=True)
        barrier()
    t_start, t_end = ev(), ev()
    with Clocks(local, gpu_pci_bus_id(torch, dev.index)) as clk:
        barrier()
        t_start.record(stream)
        for i in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                step()
        t_end.record(stream)
        barrier()
    elapsed = max_over_ranks(t_start.elapsed_time(t_end) * 1e-3)
    per_step = elapsed / args.steps
    value = B_glob / per_step

    # ---- algorithmic counts for the roofline (same inputs -> same iterations)
    st = nat.solve(d["x0"], d["U_init"], d["C"], d["c"], None, None, None, None, lo, hi, dt=wl.DT,
                   max_iter=iters, reg_eps=wl.REG_EPS, alphas=alphas, want_stats=True)
    it_n = st["iters"].cpu().numpy()
    acc_n = np.minimum(it_n, st["stall_iter"].cpu().numpy())
    # algorithmic = the dense per-unit counts of the algorithm (ilqr_costmodel:
    # RIC_DENSE ...); the structured counts (Jacobian sparsity exploited) are
    # reported beside them
    f_solve = cm.solve_flops_dense(T, len(alphas), it_n)
    f_bwd = cm.backward_flops_dense(T, B)
    f_solve_s = cm.solve_flops(T, len(alphas), it_n, acc_n)
    f_bwd_s = cm.backward_flops(T, B)
    peak_fp32 = fp32_peak_tflops(torch, dev)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    t_solve = statistics.mean(solve_ms) * 1e-3
    t_bwd = statistics.mean(bwd_ms) * 1e-3
    variant = solve_variant(B)
    traffic, traffic_note = committed_traffic(variant, B, T)
    roofline = {
        "bound": "fp32", "kernel": f"solve ({variant})",
        "achieved": f_solve / t_solve / 1e12, "peak": peak_fp32, "unit": "TFLOP/s",
        "frac": f_solve / t_solve / 1e12 / peak_fp32, "traffic": traffic, "traffic_source": traffic_note,
        "peak_source": "measured FMA probe on this GPU (no FP32 figure in MEASURED_PEAKS.json)",
        "algorithmic_flops_per_launch": f_solve, "mean_launch_ms": t_solve * 1e3,
        "flop_count": "dense per-unit counts: T [I (10.3k + 0.66k n_alpha) + 1.0k] per element (ilqr_costmodel)",
        "structured": {"flops_per_launch": f_solve_s, "achieved": f_solve_s / t_solve / 1e12,
                       "frac": f_solve_s / t_solve / 1e12 / peak_fp32,
                       "note": "counts with the Jacobian sparsity exploited (ilqr_costmodel.solve_flops)"},
        "hbm": {"algorithmic_bytes_per_launch": cm.solve_bytes(T, B),
                "achieved_gbs": cm.solve_bytes(T, B) / t_solve / 1e9, "peak_gbs": hbm_peak,
                "frac": cm.solve_bytes(T, B) / t_solve / 1e9 / hbm_peak,
                "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
        "backward_kernel": {"mean_launch_ms": t_bwd * 1e3, "tflops": f_bwd / t_bwd / 1e12,
                            "fp32_frac": f_bwd / t_bwd / 1e12 / peak_fp32,
                            "structured_fp32_frac": f_bwd_s / t_bwd / 1e12 / peak_fp32,
                            "gbs": cm.backward_bytes(T, B) / t_bwd / 1e9,
                            "hbm_frac": cm.backward_bytes(T, B) / t_bwd / 1e9 / hbm_peak},
    }

    # ---- end to end through the reference-facing operator, host buffers -----
    e2e = None
    if not args.no_e2e:
        pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
        h_x0 = pin(inp["x0"])
        h_C = pin(np.transpose(inp["C"], (1, 0, 2, 3)))   # mpc.pytorch layout [T, B, n, n]
        h_c = pin(np.transpose(inp["c"], (1, 0, 2)))
        h_gX = pin(np.transpose(gXn, (1, 0, 2)))
        h_gU = pin(np.transpose(gUn, (1, 0, 2)))
        h_act = torch.empty(B_glob, 4).pin_memory()
        h_gx0 = torch.empty(B_glob, 10).pin_memory()
        mpc = mpc_compat.MPC(10, 4, T, u_lower=lo.view(1, 1, 4).expand(T, 1, 4),
                             u_upper=hi.view(1, 1, 4).expand(T, 1, 4), lqr_iter=iters,
                             eps=wl.REG_EPS, alphas=alphas)
        dyn = type("Dyn", (), {"dt": wl.DT})()

        def e2e_step():
            x0 = h_x0.to(dev, non_blocking=True).requires_grad_(True)
            C = h_C.to(dev, non_blocking=True).requires_grad_(True)
            c = h_c.to(dev, non_blocking=True).requires_grad_(True)
            gx = h_gX.to(dev, non_blocking=True)
            gu = h_gU.to(dev, non_blocking=True)
            x, u, _ = mpc(x0, mpc_compat.QuadCost(C, c), dyn)
            ((x * gx).sum() + (u * gu).sum()).backward()
            act = u[0].detach()
            gx0 = x0.grad
            if world > 1:
                act, gg = ilqr_shard.gather_actions_and_gradients(u.detach().permute(1, 0, 2), {"x0": gx0}, B_glob)
                gx0 = gg["x0"]
            h_act.copy_(act, non_blocking=True)
            h_gx0.copy_(gx0, non_blocking=True)

        for _ in range(max(3, args.warmup)):
            e2e_step()
        barrier()
        e0, e1 = ev(), ev()
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        barrier()
        el_seq = e0.elapsed_time(e1) * 1e-3
        if world > 1:
            t = torch.tensor([el_seq], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            el_seq = float(t.item())

        host = (h_x0, h_C, h_c, h_gX, h_gU)

        def e2e_compute(bufs):
            bx0, bC, bc, bgx, bgu = bufs
            x0 = bx0.detach().requires_grad_(True)
            C = bC.detach().requires_grad_(True)
            c = bc.detach().requires_grad_(True)
            x, u, _ = mpc(x0, mpc_compat.QuadCost(C, c), dyn)
            ((x * bgx).sum() + (u * bgu).sum()).backward()
            act = u[0].detach()
            gx0 = x0.grad
            if world > 1:
                act, gg = ilqr_shard.gather_actions_and_gradients(u.detach().permute(1, 0, 2), {"x0": gx0}, B_glob)
                gx0 = gg["x0"]
            h_act.copy_(act, non_blocking=True)
            h_gx0.copy_(gx0, non_blocking=True)

        el = time_streaming(torch, dev, stream, host, e2e_compute, max(3, args.warmup), args.steps, barrier)

        # The same operator call with its inputs already on the device: the
        # operator's own cost (layout normalisation, autograd) over the kernels.
        dev_in = [h.to(dev) for h in host]
        for _ in range(max(3, args.warmup)):
            e2e_compute(dev_in)
        barrier()
        e0, e1 = ev(), ev()
        e0.record(stream)
        for _ in range(args.steps):
            e2e_compute(dev_in)
        e1.record(stream)
        barrier()
        el_dev = e0.elapsed_time(e1) * 1e-3
        if world > 1:
            t = torch.tensor([el_dev], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            el_dev = float(t.item())
        del dev_in
        if world > 1:
            t = torch.tensor([el], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            el = float(t.item())
        h2d = sum(t.numel() * 4 for t in host)
        e2e = {"value": B_glob / (el / args.steps), "unit": "solves/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": (h_act.numel() + h_gx0.numel()) * 4,
               "ms_per_step": el / args.steps * 1e3,
               "path": "mpc_compat.MPC(...)(x_init, QuadCost(C, c), dx) + autograd backward",
               "streaming": "inputs of step k+1 copied on a second stream while step k computes (double buffer)",
               "sequential": {"value": B_glob / (el_seq / args.steps), "ms_per_step": el_seq / args.steps * 1e3,
                              "note": "copies and compute of each step back to back on one stream"},
               "operator_device_resident": {"value": B_glob / (el_dev / args.steps),
                                            "ms_per_step": el_dev / args.steps * 1e3,
                                            "note": "the same operator call and backward on device tensors"}}

    # ---- p50 latency, B=16 T=5, 10 iterations, fwd+bwd ----------------------
    lat = None
    if rank == 0 and args.latency_reps > 0:
        lc, li = wl.config_inputs("latency_b16_t5")
        ld = {k: torch.from_numpy(v).to(dev) for k, v in li.items()}
        lgx, lgu = (torch.from_numpy(a).to(dev) for a in wl.make_backward_seeds(16, lc["T"]))
        samples = []
        for r in range(args.latency_reps + 10):
            a, b = ev(), ev()
            a.record(stream)
            o = nat.solve(ld["x0"], ld["U_init"], ld["C"], ld["c"], None, None, None, None, lo, hi,
                          dt=wl.DT, max_iter=lc["max_iter"], alphas=lc["alphas"])
            nat.backward(o["X"], o["U"], ld["C"], lgx, lgu, tight=o["tight"], dt=wl.DT,
                         need=("x0", "C", "c"))
            b.record(stream)
            b.synchronize()
            if r >= 10:
                samples.append(a.elapsed_time(b) * 1e3)
        # the same step replayed from a CUDA graph (ilqr_native.CapturedSolve):
        # inputs copied into its static buffers, then one graph launch
        cap = nat.CapturedSolve(16, lc["T"], dev, lo, hi, dt=wl.DT, max_iter=lc["max_iter"],
                                alphas=lc["alphas"])
        gsamples = []
        for r in range(args.latency_reps + 10):
            a, b = ev(), ev()
            a.record(stream)
            cap(ld["x0"], ld["U_init"], ld["C"], ld["c"], lgx, lgu)
            b.record(stream)
            b.synchronize()
            if r >= 10:
                gsamples.append(a.elapsed_time(b) * 1e3)
        # the same step through ilqr_native.BoundSolve (arguments prepared once)
        bound = nat.BoundSolve(16, lc["T"], dev, lo, hi, dt=wl.DT, max_iter=lc["max_iter"], alphas=lc["alphas"])
        bsamples = []
        for r in range(args.latency_reps + 10):
            a, b = ev(), ev()
            a.record(stream)
            bound(ld["x0"], ld["U_init"], ld["C"], ld["c"], lgx, lgu)
            b.record(stream)
            b.synchronize()
            if r >= 10:
                bsamples.append(a.elapsed_time(b) * 1e3)
        lat = {"p50_us": statistics.median(samples), "p90_us": sorted(samples)[int(0.9 * len(samples))],
               "p50_bound_us": statistics.median(bsamples),
               "p90_bound_us": sorted(bsamples)[int(0.9 * len(bsamples))],
               "bound": "ilqr_native.BoundSolve: solve + backward entry points with arguments prepared once",
               "reps": len(samples), "config": "B=16, T=5, 10 iterations, fwd+bwd, device-resident",
               "p50_graph_us": statistics.median(gsamples),
               "p90_graph_us": sorted(gsamples)[int(0.9 * len(gsamples))],
               "graph": "ilqr_native.CapturedSolve: input copies + one CUDA graph replay of solve + backward"}

    # ---- costs from the policy's sigmoid output [B, 28 T] (SigmoidQuadCost) ----
    # Same batch, horizon, iterations and model; the costs are the diagonal
    # ones the policy builds from its sigmoid output, built inside the kernels.
    sig = None
    if not args.no_sigmoid and world == 1:
        rng = np.random.default_rng(100 + rank)
        scn = (1.0 / (1.0 + np.exp(-rng.normal(0.0, 1.5, (B, 28 * T))))).astype(np.float32)
        sc = torch.from_numpy(scn).to(dev)
        spec = nat.SigmoidCostSpec()

        def sig_step(timing=None):
            if timing is not None:
                timing[0].record(stream)
            o = nat.solve_sigmoid(d["x0"], d["U_init"], sc, spec, lo, hi, dt=wl.DT, max_iter=iters,
                                  reg_eps=wl.REG_EPS, alphas=alphas)
            if timing is not None:
                timing[1].record(stream)
            nat.backward_sigmoid(o["X"], o["U"], sc, gX, gU, spec, tight=o["tight"], dt=wl.DT,
                                 reg_eps=wl.REG_EPS)
            if timing is not None:
                timing[2].record(stream)

        for _ in range(max(3, args.warmup)):
            sig_step()
        barrier()
        stim = [(ev(), ev(), ev()) for _ in range(args.steps)]
        s0, s1 = ev(), ev()
        s0.record(stream)
        for i in range(args.steps):
            sig_step(stim[i])
        s1.record(stream)
        barrier()
        sel = s0.elapsed_time(s1) * 1e-3
        if world > 1:
            t = torch.tensor([sel], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sel = float(t.item())
        # end to end through FastMPC / SigmoidQuadCost with host buffers
        pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
        h_x0, h_sc = pin(inp["x0"]), pin(scn)
        h_gX, h_gU = pin(np.transpose(gXn, (1, 0, 2))), pin(np.transpose(gUn, (1, 0, 2)))
        h_act, h_gx0 = torch.empty(B, 4).pin_memory(), torch.empty(B, 10).pin_memory()
        smpc = mpc_compat.MPC(10, 4, T, u_lower=lo.view(1, 1, 4).expand(T, 1, 4),
                              u_upper=hi.view(1, 1, 4).expand(T, 1, 4), lqr_iter=iters,
                              eps=wl.REG_EPS, alphas=alphas)
        sdyn = type("Dyn", (), {"dt": wl.DT})()

        def sig_e2e():
            x0 = h_x0.to(dev, non_blocking=True).requires_grad_(True)
            scd = h_sc.to(dev, non_blocking=True).requires_grad_(True)
            gx = h_gX.to(dev, non_blocking=True)
            gu = h_gU.to(dev, non_blocking=True)
            x, u, _ = smpc(x0, mpc_compat.SigmoidQuadCost(scd), sdyn)
            ((x * gx).sum() + (u * gu).sum()).backward()
            h_act.copy_(u[0].detach(), non_blocking=True)
            h_gx0.copy_(x0.grad, non_blocking=True)

        for _ in range(max(3, args.warmup)):
            sig_e2e()
        barrier()
        e0, e1 = ev(), ev()
        e0.record(stream)
        for _ in range(args.steps):
            sig_e2e()
        e1.record(stream)
        barrier()
        sel_e2e = e0.elapsed_time(e1) * 1e-3
        if world > 1:
            t = torch.tensor([sel_e2e], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sel_e2e = float(t.item())
        def sig_compute(bufs):
            bx0, bsc, bgx, bgu = bufs
            x0 = bx0.detach().requires_grad_(True)
            scd = bsc.detach().requires_grad_(True)
            x, u, _ = smpc(x0, mpc_compat.SigmoidQuadCost(scd), sdyn)
            ((x * bgx).sum() + (u * bgu).sum()).backward()
            h_act.copy_(u[0].detach(), non_blocking=True)
            h_gx0.copy_(x0.grad, non_blocking=True)

        sel_str = time_streaming(torch, dev, stream, (h_x0, h_sc, h_gX, h_gU), sig_compute, max(3, args.warmup),
                                 args.steps, barrier)
        if world > 1:
            t = torch.tensor([sel_str], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sel_str = float(t.item())
        h2d = sum(t.numel() * 4 for t in (h_x0, h_sc, h_gX, h_gU))
        sig = {"workload": f"policy_sigmoid_b{B}_t{T}", "value": world * B / (sel / args.steps),
               "unit": "solves/s", "ms_per_step": sel / args.steps * 1e3,
               "kernel_ms": {"solve_mean": statistics.mean(a.elapsed_time(b) for a, b, _ in stim),
                             "backward_mean": statistics.mean(b.elapsed_time(c) for _, b, c in stim)},
               "input": "sigmoid output [B, 28 T] (28 floats per element and step instead of 210)",
               "e2e": {"value": world * B / (sel_str / args.steps), "unit": "solves/s",
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": (h_act.numel() + h_gx0.numel()) * 4,
                       "ms_per_step": sel_str / args.steps * 1e3,
                       "path": "mpc_compat.MPC(...)(x_init, SigmoidQuadCost(s), dx) + autograd backward",
                       "streaming": "inputs of step k+1 copied on a second stream while step k computes (double buffer)",
                       "sequential": {"value": world * B / (sel_e2e / args.steps),
                                      "ms_per_step": sel_e2e / args.steps * 1e3}}}

    # ---- the policy actor's MPC step: one call vs the reference's chunk loop ---
    # PolicyMPC.actor against a restatement of forward_actor's loop
    # (mlp_mpc_policy_diffmpc.py:326-402): 1024-element chunks, dense costs
    # built with a Python loop over t, one host read per chunk. Both run on
    # this solver, without gradients (evaluation), rank 0 only.
    actor = None
    if rank == 0 and not args.no_sigmoid and world == 1:
        import policy_mpc
        pm = policy_mpc.PolicyMPC(T, wl.DT, lqr_iter=iters, eps=wl.REG_EPS, alphas=alphas, device=dev)
        sc_all = sc
        st_all = d["x0"]

        def build_dense(s_chunk):
            n_c = s_chunk.shape[0]
            x_q = s_chunk[:, :14 * T] * 100000.0 + 0.1
            x_p = s_chunk[:, 14 * T:]
            Cc = torch.zeros(n_c, T, 14, 14, device=dev)
            cc = torch.zeros(n_c, T, 14, device=dev)
            for t_ in range(T):
                dv = torch.cat([x_q[:, 3 * t_:3 * t_ + 3], x_q[:, 3 * T + 4 * t_:3 * T + 4 * t_ + 4],
                                x_q[:, 7 * T + 3 * t_:7 * T + 3 * t_ + 3], x_q[:, 13 * T + t_:13 * T + t_ + 1],
                                x_q[:, 10 * T + 3 * t_:10 * T + 3 * t_ + 3]], dim=1)
                Cc[:, t_] = torch.diag_embed(dv)
                cc[:, t_] = torch.cat([(x_p[:, 3 * t_:3 * t_ + 3] - 0.5) * 1e5,
                                       (x_p[:, 3 * T + 4 * t_:3 * T + 4 * t_ + 4] - 0.5) * 1e5,
                                       (x_p[:, 7 * T + 3 * t_:7 * T + 3 * t_ + 3] - 0.5) * 1e5,
                                       -(x_p[:, 13 * T + t_:13 * T + t_ + 1] * (1e5 * 0.752 * 9.806) + 0.1),
                                       (x_p[:, 10 * T + 3 * t_:10 * T + 3 * t_ + 3] - 0.5) * 1e5], dim=1)
            return Cc, cc

        loop_mpc = mpc_compat.MPC(10, 4, T, u_lower=lo.view(1, 1, 4).expand(T, 1, 4),
                                  u_upper=hi.view(1, 1, 4).expand(T, 1, 4), lqr_iter=iters,
                                  eps=wl.REG_EPS, alphas=alphas)
        ldyn = type("Dyn", (), {"dt": wl.DT})()
        u_prev = torch.zeros(B, 4, device=dev)
        u_prev[:, 0] = 0.752 * 9.8066

        def chunk_loop():
            nom_u = torch.zeros(B, T, 4, device=dev)
            bad = 0
            for s0_ in range(0, B, 1024):
                e_ = min(B, s0_ + 1024)
                Cc, cc = build_dense(sc_all[s0_:e_])
                loop_mpc.u_init = u_prev[s0_:e_].unsqueeze(1).expand(-1, T, -1).permute(1, 0, 2).contiguous()
                _, U_tbn, _ = loop_mpc(st_all[s0_:e_], mpc_compat.QuadCost(Cc.permute(1, 0, 2, 3).contiguous(),
                                                                           cc.permute(1, 0, 2).contiguous()), ldyn)
                nom_u[s0_:e_] = U_tbn.permute(1, 0, 2)
                bad += int((~torch.isfinite(U_tbn)).any().cpu().item())
            return nom_u

        def timed(fn, reps):
            out = []
            for _ in range(reps + 2):
                a, b_ = ev(), ev()
                a.record(stream)
                with torch.no_grad():
                    fn()
                b_.record(stream)
                b_.synchronize()
                out.append(a.elapsed_time(b_))
            return statistics.median(out[2:])

        one = timed(lambda: pm.actor(sc_all, st_all), max(3, args.steps // 2))
        loop = timed(chunk_loop, max(3, args.steps // 2))
        actor = {"B": B, "T": T, "iters": iters, "one_call_ms": one, "reference_chunk_loop_ms": loop,
                 "note": "no gradients; the chunk loop is the reference's forward_actor loop on this solver"}

    # ---- 13-state rotor-thrust model (ilqr_dense.cu) ---------------------------
    # The benchmark configurations' rigid body (four rotor thrusts in [0, 1]),
    # same batch, horizon, iterations and step sizes, dense C [B,T,17,17].
    r13 = None
    if not args.no_rotor13 and world == 1:
        ri = wl.make_rotor13_inputs(B, T, seed=rank, target=cfg["target"], r=cfg["r"])
        rd = {k: torch.from_numpy(v).to(dev) for k, v in ri.items()}
        rgXn, rgUn = wl.make_backward_seeds(B, T, seed=1 + rank, nx=wl.NX13)
        rgX, rgU = torch.from_numpy(rgXn).to(dev), torch.from_numpy(rgUn).to(dev)
        rlo, rhi = torch.from_numpy(wl.U_MIN13).to(dev), torch.from_numpy(wl.U_MAX13).to(dev)
        r_iters = []

        def r13_step(timing=None):
            if timing is not None:
                timing[0].record(stream)
            o = nat.rotor13_solve(rd["x0"], rd["U_init"], rd["C"], rd["c"], u_min=rlo, u_max=rhi, dt=wl.DT,
                                  max_iter=iters, reg_eps=wl.REG_EPS, alphas=alphas, want_stats=timing is not None)
            if timing is not None:
                timing[1].record(stream)
                r_iters.append(o["iters"])
            nat.rotor13_backward(o["X"], o["U"], rd["C"], rgX, rgU, tight=o["tight"], dt=wl.DT,
                                 reg_eps=wl.REG_EPS)
            if timing is not None:
                timing[2].record(stream)

        for _ in range(max(3, args.warmup)):
            r13_step()
        barrier()
        rtim = [(ev(), ev(), ev()) for _ in range(args.steps)]
        r0, r1 = ev(), ev()
        r0.record(stream)
        for i in range(args.steps):
            r13_step(rtim[i])
        r1.record(stream)
        barrier()
        rel_s = r0.elapsed_time(r1) * 1e-3
        if world > 1:
            t = torch.tensor([rel_s], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            rel_s = float(t.item())
        r_solve = statistics.mean(a.elapsed_time(b_) for a, b_, _ in rtim)
        r_bwd = statistics.mean(b_.elapsed_time(c_) for _, b_, c_ in rtim)
        it_np = torch.stack(r_iters).float().mean(0).cpu().numpy()
        fl_s = cm.r13_solve_flops_dense(T, len(alphas), it_np)
        fl_b = cm.r13_backward_flops_dense(T, B)
        # end to end through FastMPC(13, 4, T) with host buffers
        r13_e2e_res = None
        pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
        h_x0 = pin(ri["x0"])
        h_C = pin(np.transpose(ri["C"], (1, 0, 2, 3)))
        h_c = pin(np.transpose(ri["c"], (1, 0, 2)))
        h_gX, h_gU = pin(np.transpose(rgXn, (1, 0, 2))), pin(np.transpose(rgUn, (1, 0, 2)))
        h_act, h_gx0 = torch.empty(B, 4).pin_memory(), torch.empty(B, wl.NX13).pin_memory()
        rmpc = mpc_compat.MPC(wl.NX13, 4, T, u_lower=rlo.view(1, 1, 4).expand(T, 1, 4),
                              u_upper=rhi.view(1, 1, 4).expand(T, 1, 4), lqr_iter=iters,
                              eps=wl.REG_EPS, alphas=alphas)
        rdyn = type("Dyn", (), {"dt": wl.DT})()

        def r13_e2e():
            x0 = h_x0.to(dev, non_blocking=True).requires_grad_(True)
            Cd = h_C.to(dev, non_blocking=True).requires_grad_(True)
            cd = h_c.to(dev, non_blocking=True).requires_grad_(True)
            gx = h_gX.to(dev, non_blocking=True)
            gu = h_gU.to(dev, non_blocking=True)
            x, u, _ = rmpc(x0, mpc_compat.QuadCost(Cd, cd), rdyn)
            ((x * gx).sum() + (u * gu).sum()).backward()
            h_act.copy_(u[0].detach(), non_blocking=True)
            h_gx0.copy_(x0.grad, non_blocking=True)

        if not args.no_e2e:
            for _ in range(max(3, args.warmup)):
                r13_e2e()
            barrier()
            e0, e1 = ev(), ev()
            e0.record(stream)
            for _ in range(args.steps):
                r13_e2e()
            e1.record(stream)
            barrier()
            rel_e2e = e0.elapsed_time(e1) * 1e-3
            if world > 1:
                t = torch.tensor([rel_e2e], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                rel_e2e = float(t.item())
            def r13_compute(bufs):
                bx0, bC, bc, bgx, bgu = bufs
                x0 = bx0.detach().requires_grad_(True)
                Cd = bC.detach().requires_grad_(True)
                cd = bc.detach().requires_grad_(True)
                x, u, _ = rmpc(x0, mpc_compat.QuadCost(Cd, cd), rdyn)
                ((x * bgx).sum() + (u * bgu).sum()).backward()
                h_act.copy_(u[0].detach(), non_blocking=True)
                h_gx0.copy_(x0.grad, non_blocking=True)

            rel_str = time_streaming(torch, dev, stream, (h_x0, h_C, h_c, h_gX, h_gU), r13_compute,
                                     max(3, args.warmup), args.steps, barrier)
            if world > 1:
                t = torch.tensor([rel_str], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                rel_str = float(t.item())
            h2d = sum(t.numel() * 4 for t in (h_x0, h_C, h_c, h_gX, h_gU))
            r13_e2e_res = {"value": world * B / (rel_str / args.steps), "unit": "solves/s",
                           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": (h_act.numel() + h_gx0.numel()) * 4,
                           "ms_per_step": rel_str / args.steps * 1e3,
                           "path": "mpc_compat.MPC(13, 4, T)(x_init, QuadCost(C, c), dx) + autograd backward",
                           "streaming": "inputs of step k+1 copied on a second stream while step k computes",
                           "sequential": {"value": world * B / (rel_e2e / args.steps),
                                          "ms_per_step": rel_e2e / args.steps * 1e3}}
        # latency: B = 16, T = 5, 10 iterations, solve + backward, device-resident
        lc13 = wl.CONFIGS["latency_b16_t5"]
        li = wl.make_rotor13_inputs(16, lc13["T"], seed=rank, target=lc13["target"], r=lc13["r"])
        ld13 = {k: torch.from_numpy(v).to(dev) for k, v in li.items()}
        lgx13, lgu13 = [torch.from_numpy(a).to(dev) for a in wl.make_backward_seeds(16, lc13["T"], nx=wl.NX13)]
        lsamp = []
        for rep in range(args.latency_reps + 10):
            a, b_ = ev(), ev()
            a.record(stream)
            o = nat.rotor13_solve(ld13["x0"], ld13["U_init"], ld13["C"], ld13["c"], u_min=rlo, u_max=rhi,
                                  dt=wl.DT, max_iter=lc13["max_iter"], reg_eps=wl.REG_EPS, alphas=lc13["alphas"])
            nat.rotor13_backward(o["X"], o["U"], ld13["C"], lgx13, lgu13, tight=o["tight"], dt=wl.DT,
                                 reg_eps=wl.REG_EPS)
            b_.record(stream)
            b_.synchronize()
            if rep >= 10:
                lsamp.append(a.elapsed_time(b_) * 1e3)
        r13 = {"workload": f"rotor13_b{B}_t{T}", "value": world * B / (rel_s / args.steps), "unit": "solves/s",
               "ms_per_step": rel_s / args.steps * 1e3,
               "model": "13-state rotor-thrust rigid body (p, q, v, w; 4 rotor thrusts in [0,1] x 8.5 N), "
                        "dense C [B,T,17,17]",
               "kernel_ms": {"solve_mean": r_solve, "backward_mean": r_bwd},
               "mean_iters": float(it_np.mean()),
               "roofline": {"bound": "fp32", "unit": "TFLOP/s", "peak": peak_fp32,
                            "solve_achieved": fl_s / (r_solve * 1e-3) / 1e12,
                            "backward_achieved": fl_b / (r_bwd * 1e-3) / 1e12,
                            "solve_frac": fl_s / (r_solve * 1e-3) / 1e12 / peak_fp32,
                            "backward_frac": fl_b / (r_bwd * 1e-3) / 1e12 / peak_fp32,
                            "count": "dense per-unit counts (ilqr_costmodel: Riccati 16.9k, candidate 0.88k, "
                                     "initial 0.75k, backward 18.0k FLOP per element and step)"},
               "e2e": r13_e2e_res,
               "latency_b16_t5": ({"p50_us": statistics.median(lsamp),
                                   "p90_us": sorted(lsamp)[int(0.9 * len(lsamp))], "reps": len(lsamp),
                                   "config": "B=16, T=5, 10 iterations, fwd+bwd, device-resident, eager"}
                                  if lsamp else None)}

    # ---- FastMPC numerics mode (ilqr_fastmpc.cu) --------------------------------
    # The reference FastMPC extension's own numerics on the same inputs: PNQP
    # box QP in every Riccati step, step sizes (1, .5, .25, .1), batch-wide
    # convergence. Device-resident solve + backward, then the operator call
    # MPC(..., numerics="fastmpc") with autograd on the same device tensors.
    fmr = None
    if not args.no_fastmpc and world == 1:
        fm_alphas = nat.FASTMPC_ALPHAS
        fm_tim = [(ev(), ev(), ev()) for _ in range(args.steps)]
        fm_info = []

        def fm_step(timing=None):
            if timing is not None:
                timing[0].record(stream)
            o = nat.fastmpc_solve(d["x0"], d["U_init"], d["C"], d["c"], u_min=lo, u_max=hi, dt=wl.DT,
                                  max_iter=iters, reg_eps=wl.REG_EPS, alphas=fm_alphas)
            if timing is not None:
                timing[1].record(stream)
                fm_info.append(o["batch_info"])
            nat.fastmpc_backward(o["X"], o["U"], o["X_lin"], o["U_lin"], d["C"], gX, gU, tight=o["tight"], dt=wl.DT,
                                 reg_eps=wl.REG_EPS)
            if timing is not None:
                timing[2].record(stream)
            return o

        for _ in range(max(3, args.warmup)):
            fm_last = fm_step()
        barrier()
        f0, f1 = ev(), ev()
        f0.record(stream)
        for i in range(args.steps):
            fm_step(fm_tim[i])
        f1.record(stream)
        barrier()
        fel = f0.elapsed_time(f1) * 1e-3
        if world > 1:
            t = torch.tensor([fel], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            fel = float(t.item())
        fmpc = mpc_compat.MPC(10, 4, T, u_lower=lo.view(1, 1, 4).expand(T, 1, 4),
                              u_upper=hi.view(1, 1, 4).expand(T, 1, 4), lqr_iter=iters, eps=wl.REG_EPS,
                              numerics="fastmpc")
        fdyn = type("Dyn", (), {"dt": wl.DT})()
        fC = d["C"].transpose(0, 1).contiguous()
        fc_ = d["c"].transpose(0, 1).contiguous()
        fgX, fgU = gX.transpose(0, 1).contiguous(), gU.transpose(0, 1).contiguous()

        def fm_op():
            x0 = d["x0"].detach().requires_grad_(True)
            Cd = fC.detach().requires_grad_(True)
            cd = fc_.detach().requires_grad_(True)
            x, u, _ = fmpc(x0, mpc_compat.QuadCost(Cd, cd), fdyn)
            ((x * fgX).sum() + (u * fgU).sum()).backward()

        for _ in range(max(3, args.warmup)):
            fm_op()
        barrier()
        f0.record(stream)
        for _ in range(args.steps):
            fm_op()
        f1.record(stream)
        barrier()
        fop = f0.elapsed_time(f1) * 1e-3
        del fC, fc_, fgX, fgU
        info = torch.stack(fm_info).float().mean(0).cpu().numpy()
        fmr = {"workload": WORKLOAD, "value": world * B / (fel / args.steps), "unit": "solves/s",
               "ms_per_step": fel / args.steps * 1e3,
               "numerics": "reference FastMPC CUDA build: PNQP-aware Riccati, alphas (1, .5, .25, .1), "
                           "batch convergence every 4 iterations",
               "kernel_ms": {"solve_mean": statistics.mean(a.elapsed_time(b_) for a, b_, _ in fm_tim),
                             "backward_mean": statistics.mean(b_.elapsed_time(c_) for _, b_, c_ in fm_tim)},
               "iterations_run": float(info[1]), "tight_fraction": float(fm_last["tight"].float().mean()),
               "operator_device_resident": {"value": world * B / (fop / args.steps),
                                            "ms_per_step": fop / args.steps * 1e3,
                                            "path": "mpc_compat.MPC(..., numerics='fastmpc') + autograd"}}

    # ---- weak scaling: every rank its own 16384 elements (N > 1) ----------------
    weak = None
    if world > 1 and not args.no_weak:
        Bw = cfg["B"]
        wi = wl.make_inputs(Bw, T, seed=100 + rank, target=cfg["target"], r=cfg["r"])
        wd = {k: torch.from_numpy(v).to(dev) for k, v in wi.items()}
        wgX, wgU = (torch.from_numpy(a).to(dev) for a in wl.make_backward_seeds(Bw, T, seed=200 + rank))

        def wstep():
            o = nat.solve(wd["x0"], wd["U_init"], wd["C"], wd["c"], None, None, None, None, lo, hi,
                          dt=wl.DT, max_iter=iters, reg_eps=wl.REG_EPS, alphas=alphas)
            gw = nat.backward(o["X"], o["U"], wd["C"], wgX, wgU, tight=o["tight"], dt=wl.DT,
                              reg_eps=wl.REG_EPS, need=("x0", "C", "c"))
            ilqr_shard.gather_actions_and_gradients(o["U"], gw, Bw * world, keys=("x0",))

        for _ in range(max(3, args.warmup)):
            wstep()
        barrier()
        e0, e1 = ev(), ev()
        e0.record(stream)
        for _ in range(args.steps):
            wstep()
        e1.record(stream)
        barrier()
        wel = max_over_ranks(e0.elapsed_time(e1) * 1e-3) / args.steps
        weak = {"value": float(f"{world * Bw / wel:.5g}"), "ms": float(f"{wel * 1e3:.4g}"), "B_per_gpu": Bw}
        del wd, wgX, wgU
        torch.cuda.empty_cache()

    # ---- the inference configuration sharded over the ranks (N > 1) -------------
    infer = None
    if world > 1 and not args.no_inference:
        c4 = wl.CONFIGS["inference_b262144_t10"]
        B4, T4 = c4["B"], c4["T"]
        i_lo, i_hi = ilqr_shard.shard_bounds(B4, rank, world)
        ii = shard_inputs(wl, B4, T4, i_lo, i_hi, c4)
        idv = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in ii.items()}

        def icall():
            o = nat.solve(idv["x0"], idv["U_init"], idv["C"], idv["c"], None, None, None, None, lo, hi,
                          dt=wl.DT, max_iter=c4["max_iter"], reg_eps=wl.REG_EPS, alphas=c4["alphas"])
            return ilqr_shard.gather_first_actions(o["U"], B4)

        for _ in range(3):
            icall()
        barrier()
        reps = 5
        e0, e1 = ev(), ev()
        e0.record(stream)
        for _ in range(reps):
            icall()
        e1.record(stream)
        barrier()
        iel = max_over_ranks(e0.elapsed_time(e1) * 1e-3) / reps
        infer = {"value": float(f"{B4 / iel:.5g}"), "ms": float(f"{iel * 1e3:.4g}"), "B": B4, "T": T4,
                 "iters": c4["max_iter"]}
        del idv
        torch.cuda.empty_cache()

    # ---- the reference FastMPC extension's CUDA kernels (rank 0, N=1) ------------
    fm_ref = None
    if rank == 0 and world == 1 and not args.no_ref_baselines:
        from oracle import fastmpc_ref_cuda as fref
        if fref.available():
            def fref_step():
                r_ = fref.solve(d["x0"], d["U_init"], d["C"], d["c"], lo, hi, dt=wl.DT, max_iter=iters,
                                reg=wl.REG_EPS)
                fref.backward(r_, gX, gU, reg=wl.REG_EPS)

            for _ in range(2):
                fref_step()
            torch.cuda.synchronize()
            reps = 5
            e0, e1 = ev(), ev()
            e0.record(stream)
            for _ in range(reps):
                fref_step()
            e1.record(stream)
            torch.cuda.synchronize()
            fms = e0.elapsed_time(e1) / reps
            fm_ref = {"value": B / (fms * 1e-3), "ms": fms,
                      "what": "reference FastMPC CUDA kernels (oracle/_ref) via its restated host loop, "
                              "same inputs, fwd+bwd"}

    # ---- CPU baselines (rank 0, N=1): DiffMPC itself and the numpy port ----------
    cpu = port = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        os.sched_setaffinity(0, all_cpus)  # the CPU baseline uses every host core
        cores = len(os.sched_getaffinity(0))
        rate_p, n_p, _ = cpu_rate("port", cores, 1024)
        port = {"value": rate_p, "cores": cores, "sample": f"{n_p} elements, {cores} procs x 1024"}
        if not args.no_ref_baselines and diffmpc_staged():
            rate, n, _ = cpu_rate("reference", cores, 256)
            cpu = {"value": rate, "unit": "solves/s", "cores": cores, "kind": "reference",
                   "sample": f"DiffMPC itself, fwd+bwd, {n} of {B} elements, {cores} procs x 256"}
        else:
            cpu = {"value": rate_p, "unit": "solves/s", "cores": cores, "kind": "port",
                   "sample": f"numpy port, fwd+bwd, {n_p} of {B} elements, {cores} procs x 1024"}

    graph_used = graph is not None
    del graph  # (a graph holding NCCL work must go before the process group)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    # the bulky sections, each on a line of its own before the benchmark line
    for name, sec in (("roofline", roofline), ("e2e", e2e), ("latency_b16_t5", lat),
                      ("policy_sigmoid_cost", sig), ("policy_actor_step", actor), ("rotor13", r13),
                      ("fastmpc_numerics", fmr)):
        if sec is not None:
            print(f"#section {name} " + json.dumps(sec), flush=True)
    rnd = lambda x, k=4: None if x is None else float(f"{x:.{k}g}")
    line = {
        "metric": METRIC, "value": value, "unit": "solves/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": per_step * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": headline_config(world),
        "roofline": {"bound": "fp32", "achieved": rnd(roofline["achieved"]), "peak": rnd(roofline["peak"]),
                     "unit": "TFLOP/s", "frac": rnd(roofline["frac"]), "traffic": traffic,
                     "kernel": roofline["kernel"], "B": B},
        "cpu_baseline": cpu,
        "e2e": None if e2e is None else {k: e2e[k] for k in ("value", "unit", "h2d_bytes_per_step",
                                                             "d2h_bytes_per_step")},
        "gpu_launches": (solve_launches(B, iters) + 1) * args.steps, "clocks": clk.summary(),
        "latency_b16_t5_p50_us": None if lat is None else rnd(lat["p50_us"]),
        "kernel_ms": {"solve": rnd(statistics.mean(solve_ms)), "bwd": rnd(statistics.mean(bwd_ms)),
                      "gather": rnd(gather_ms) if world > 1 else None, "eager_step": rnd(eager_per_step * 1e3),
                      "graph": graph_used},
        "weak_b16384_per_gpu": weak,
        "inference_b262144_t10": infer,
        "fastmpc_ref_cuda": None if fm_ref is None else {"value": rnd(fm_ref["value"]), "ms": rnd(fm_ref["ms"])},
        "cpu_port": None if port is None else {"value": rnd(port["value"]), "cores": port["cores"]},
    }
    print(json.dumps(line), flush=True)


def run_sharded_inference(args):
    """The inference configuration as specified (B=262144, T=10, 10
    iterations, forward only) sharded over the ranks of torch.distributed.run:
    each rank solves its B / world elements, then the first actions of all
    ranks are all-gathered (NCCL) into every rank's [B, 4] tensor. Time per
    call is the max over ranks; rank 0 prints one JSON line per model."""
    import datetime

    import torch
    import torch.distributed as dist

    import ilqr_native as nat
    import ilqr_shard
    import ilqr_workload as wl
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    stream = torch.cuda.current_stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)
    cfg = wl.CONFIGS["inference_b262144_t10"]
    B, T = cfg["B"], cfg["T"]
    lo_, hi_ = ilqr_shard.shard_bounds(B, rank, world)
    nb = hi_ - lo_
    for model in ("drone10", "rotor13"):
        r13 = model == "rotor13"
        mk = wl.make_rotor13_inputs if r13 else wl.make_inputs
        inp = mk(nb, T, seed=rank, target=cfg["target"], r=cfg["r"])
        d = {k: torch.from_numpy(v).to(dev) for k, v in inp.items()}
        tl = torch.from_numpy(wl.U_MIN13 if r13 else wl.U_MIN).to(dev)
        th = torch.from_numpy(wl.U_MAX13 if r13 else wl.U_MAX).to(dev)
        solve = nat.rotor13_solve if r13 else nat.solve

        def call():
            o = solve(d["x0"], d["U_init"], d["C"], d["c"], u_min=tl, u_max=th, dt=wl.DT,
                      max_iter=cfg["max_iter"], reg_eps=wl.REG_EPS, alphas=cfg["alphas"])
            return ilqr_shard.gather_first_actions(o["U"], B)

        for _ in range(max(3, args.warmup)):
            call()
        dist.barrier()
        torch.cuda.synchronize()
        reps = max(3, min(args.steps, 10))
        e0, e1 = ev(), ev()
        e0.record(stream)
        for _ in range(reps):
            acts = call()
        e1.record(stream)
        dist.barrier()
        torch.cuda.synchronize()
        el = torch.tensor([e0.elapsed_time(e1) / reps], device=dev)
        dist.all_reduce(el, op=dist.ReduceOp.MAX)
        ms = float(el.item())
        if rank == 0:
            print(json.dumps({"model": model, "workload": "inference_b262144_t10", "B": B, "T": T,
                              "iters": cfg["max_iter"], "n_gpus": world, "elements_per_gpu": nb,
                              "ms_per_call_max_over_ranks": ms, "solves_per_s": B / (ms * 1e-3),
                              "actions_gathered": list(acts.shape), "reps": reps,
                              "per_call": "forward solve of the rank's shard + NCCL all-gather of the first actions",
                              "data": "synthetic (seeded)", "device_resident": True}), flush=True)
        del d
        torch.cuda.empty_cache()
    dist.barrier()
    dist.destroy_process_group()


def run_all_configs(args):
    """Every workload configuration on one GPU, for both models: fwd (+bwd
    where the configuration has it) solves/s with device-resident inputs,
    the mean iterations the elements ran, and the solve / backward kernel
    times. Batch sizes above 65536 run as consecutive 65536-element slices
    (the solve is per element; the slices reuse one workspace size). Under
    torch.distributed.run (WORLD_SIZE > 1) only the sharded inference
    configuration runs (run_sharded_inference)."""
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_sharded_inference(args)
        return
    import numpy as np
    import torch

    import ilqr_native as nat
    import ilqr_workload as wl
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)
    for model in ("drone10", "rotor13"):
        r13 = model == "rotor13"
        for name, cfg in wl.CONFIGS.items():
            if r13 and name == "stress_b65536_t50":
                continue  # the reference's own fp32 solve fails there on this model
            B, T, iters, alphas = cfg["B"], cfg["T"], cfg["max_iter"], cfg["alphas"]
            sl = min(B, 65536)
            if r13:
                inp = wl.make_rotor13_inputs(sl, T, seed=0, target=cfg["target"], r=cfg["r"])
                lo, hi = wl.U_MIN13, wl.U_MAX13
                gXn, gUn = wl.make_backward_seeds(sl, T, nx=wl.NX13)
            else:
                inp = wl.make_inputs(sl, T, seed=0, target=cfg["target"], r=cfg["r"])
                lo, hi = wl.U_MIN, wl.U_MAX
                gXn, gUn = wl.make_backward_seeds(sl, T)
            d = {k: torch.from_numpy(v).to(dev) for k, v in inp.items()}
            gX, gU = torch.from_numpy(gXn).to(dev), torch.from_numpy(gUn).to(dev)
            tl, th = torch.from_numpy(lo).to(dev), torch.from_numpy(hi).to(dev)
            solve = nat.rotor13_solve if r13 else nat.solve
            bwd = nat.rotor13_backward if r13 else nat.backward
            its = []

            def one(timing):
                timing[0].record(stream)
                o = solve(d["x0"], d["U_init"], d["C"], d["c"], u_min=tl, u_max=th, dt=wl.DT, max_iter=iters,
                          reg_eps=wl.REG_EPS, alphas=alphas, want_stats=True)
                timing[1].record(stream)
                its.append(o["iters"])
                if cfg["backward"]:
                    bwd(o["X"], o["U"], d["C"], gX, gU, tight=o["tight"], dt=wl.DT, reg_eps=wl.REG_EPS)
                timing[2].record(stream)

            n_sl = B // sl
            for _ in range(max(3, args.warmup)):
                one((ev(), ev(), ev()))
            torch.cuda.synchronize()
            reps = max(3, args.steps // 2) if B <= 1024 else max(3, min(args.steps, 10))
            tims = [[(ev(), ev(), ev()) for _ in range(n_sl)] for _ in range(reps)]
            for r in range(reps):
                for k in range(n_sl):
                    one(tims[r][k])
            torch.cuda.synchronize()
            step_ms = [sum(a.elapsed_time(c) for a, _, c in tims[r]) for r in range(reps)]
            solve_ms = statistics.mean(sum(a.elapsed_time(b_) for a, b_, _ in tims[r]) for r in range(reps))
            bwd_ms = statistics.mean(sum(b_.elapsed_time(c) for _, b_, c in tims[r]) for r in range(reps))
            med = statistics.median(step_ms)
            line = {"model": model, "workload": name, "B": B, "T": T, "iters": iters, "alphas": list(alphas),
                    "backward": cfg["backward"], "slices": n_sl,
                    "ms_per_call_p50": med, "solves_per_s": B / (med * 1e-3),
                    "solve_ms": solve_ms, "backward_ms": bwd_ms,
                    "mean_iters_run": float(torch.stack(its[-n_sl:]).float().mean().item()),
                    "reps": reps, "data": "synthetic (seeded)", "device_resident": True}
            print(json.dumps(line), flush=True)
            del d, gX, gU
            torch.cuda.empty_cache()


def main():
    args = _args()
    if args.impl == "reference":
        run_reference(args)
    elif args.all_configs:
        run_all_configs(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
