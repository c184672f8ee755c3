"""Benchmark: wide-MLP data-parallel training through MiniTensor's API on B200.

Workload (the multi-GPU configuration of the benchmark set): MLP
1024 -> 8192 -> 8192 -> 8192 -> 1000 with ReLU and softmax cross entropy,
Adam(lr=1e-3), Float32, global batch 65536 split evenly over the ranks,
gradients all-reduced with NCCL.  Inputs are seeded synthetic N(0,1) rows with
Int64 labels uniform in [0, 1000) (no dataset is involved).  A step is one full
training iteration (forward, backward, all-reduce, Adam update, leafify) of the
unchanged MiniTensor front-end running on the CUDA backend.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --case gemm|chain|reduce|log_softmax|gather|scatter_add|concat|uniform|normal|adamw|spiral ...

`value` times K steps on device-resident inputs (CUDA events on the backend's
stream, barrier + synchronize on both sides, max over ranks).  `e2e` times steps
through the public workload API from pinned host buffers: every step copies its
inputs host -> device and reads the loss back.  `--impl reference` runs the
reference CPU backend (oracle/_ref, built from the unmodified sources) on the
host cores.  One JSON line is printed by rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "wide_mlp_train_samples_per_s"
WIDTHS = (1024, 8192, 8192, 8192, 1000)
GLOBAL_BATCH = 65536
LR = 1e-3
SEED = 2026


def flops_per_sample(widths=WIDTHS) -> float:
    macs = sum(a * b for a, b in zip(widths[:-1], widths[1:]))
    # forward 2*MACs, backward 4*MACs except no input gradient for the first layer
    return 6.0 * macs - 2.0 * widths[0] * widths[1]


def config(n_gpus: int) -> dict:
    return {
        "workload": "wide MLP 1024-8192-8192-8192-1000 ReLU + softmax CE, Adam lr=1e-3, global batch 65536 "
                    "split over ranks, NCCL gradient all-reduce",
        "global_batch": GLOBAL_BATCH,
        "per_rank_batch": GLOBAL_BATCH // n_gpus,
        "parameters": sum(a * b + b for a, b in zip(WIDTHS[:-1], WIDTHS[1:])),
        "flop_per_step": flops_per_sample() * GLOBAL_BATCH,
        "parallelism": f"dp{n_gpus}",
        "l2": "inputs and weights larger than the 126 MB L2 (no flush needed)",
        "batches": f"{BATCHES} distinct seeded batches per rank, resident; step s uses batch s mod {BATCHES}",
    }


# ---------------------------------------------------------------- helpers --

BATCHES = 4  # distinct seeded batches per rank, cycled step by step


def make_batch(rank: int, batch: int, index: int = 0):
    import numpy as np
    import torch

    rng = np.random.default_rng([SEED, rank, index])
    x = torch.empty((batch, WIDTHS[0]), dtype=torch.float32, pin_memory=True)
    y = torch.empty((batch,), dtype=torch.int64, pin_memory=True)
    x.numpy()[:] = rng.standard_normal((batch, WIDTHS[0]), dtype=np.float32)
    y.numpy()[:] = rng.integers(0, WIDTHS[-1], batch)
    return x, y


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.out = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        if not self.out:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def measure_tf32_peak() -> float:
    """Dense TF32 tensor throughput of cuBLAS (torch.matmul, 8192^3, best of 10): the
    3xTF32 roofline is a third of it.  TF32 is not in the driver's peak file."""
    import torch

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    n = 8192
    a = torch.randn(n, n, device="cuda")
    b = torch.randn(n, n, device="cuda")
    for _ in range(3):
        torch.matmul(a, b)
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch.matmul(a, b)
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b
    return 2 * n ** 3 / (best * 1e-3) / 1e12


def read_traffic(name: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    path = ROOT / "profiles" / "traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith(name + " "):
            try:
                return float(line.split()[1])
            except (IndexError, ValueError):
                return None
    return None


def cpu_reference_sample(batch: int, steps: int, warm: int = 0) -> dict:
    """The reference CPU backend (oracle/_ref) training the same model on one core:
    `warm` untimed steps, then `steps` timed ones."""
    import numpy as np

    from minitensor_cpp_b200.frontend import Frontend, MlpTrainer
    from oracle import refkernels

    fe = Frontend(refkernels.LIB_PATH)
    tr = MlpTrainer(fe, -1, WIDTHS[0], WIDTHS[1], len(WIDTHS) - 2, WIDTHS[-1], seed=SEED, lr=LR)
    tr.materialize()
    rng = np.random.default_rng([SEED, 99])
    x = rng.standard_normal((batch, WIDTHS[0]), dtype=np.float32)
    y = rng.integers(0, WIDTHS[-1], batch).astype(np.int64)
    tr.load_batch(x.ctypes.data, y.ctypes.data, batch)
    for _ in range(warm):
        tr.step_resident(read_loss=True)
    t0 = time.perf_counter()
    for _ in range(steps):
        tr.step_resident(read_loss=True)
    dt = time.perf_counter() - t0
    tr.close()
    return {"samples": batch * steps, "seconds": dt}


def _worker(args):
    batch, steps, warm = args
    return cpu_reference_sample(batch, steps, warm)


# ------------------------------------------------------- single-kernel cases --
# `python bench.py --case NAME [options]` runs one kernel of the backend alone
# on cuda:0 (operands made with torch, device memory only), for ncu captures
# and for timing one kernel: the set-up call, --warm-s seconds of untimed calls,
# then --reps calls back to back (prepared ABI calls) between two CUDA events on
# the current stream.  It prints one JSON line with the mean time per call.
# Under a profiler pass --warm-s 0 --reps 1: the launches are then the set-up
# call and one timed call.

def _case_ms(fn, reps: int, warm_s: float) -> float:
    import torch

    fn()  # set-up call: NVRTC / tensor-map preparation, not timed
    torch.cuda.synchronize()
    t0 = time.perf_counter()  # untimed calls so the SM clock has left idle
    while time.perf_counter() - t0 < warm_s:
        fn()
        torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        fn()
    stop.record()
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / reps


def adamw_program(lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, c1=0.1, c2=0.001):
    """AdamW's per-parameter update as one fused program: registers 0..3 are
    p, g, m, v; outputs p', m', v' (the evaluator builds the same cluster for
    AdamW::update_parameter, src/nn/optimizers/adamw.cpp:67-97)."""
    from minitensor_cpp_b200 import abi

    C, M, A, D, S = abi.CONST, abi.MULTIPLY, abi.ADD, abi.DIVIDE, abi.SUBTRACT
    prog = [(C, 4, 0, 0, b1), (M, 5, 4, 2, 0.0), (C, 6, 0, 0, 1 - b1), (M, 7, 6, 1, 0.0), (A, 8, 5, 7, 0.0),
            (C, 9, 0, 0, b2), (M, 10, 9, 3, 0.0), (C, 11, 0, 0, 1 - b2), (M, 12, 11, 1, 0.0), (M, 13, 12, 1, 0.0),
            (A, 14, 10, 13, 0.0), (C, 15, 0, 0, c1), (D, 16, 8, 15, 0.0), (C, 17, 0, 0, c2), (D, 18, 14, 17, 0.0),
            (C, 21, 0, 0, lr), (M, 22, 21, 16, 0.0), (abi.SQRT, 23, 18, 0, 0.0), (C, 24, 0, 0, eps),
            (A, 25, 23, 24, 0.0), (D, 26, 22, 25, 0.0), (S, 27, 0, 26, 0.0)]
    return prog, [27, 8, 14]


def _case(a) -> dict:
    """One kernel case; returns its figures (ms per call and the rate)."""
    import torch

    from minitensor_cpp_b200 import abi

    V = abi.View.of
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    run = lambda call: _case_ms(call, a.reps, a.warm_s)
    if a.case == "gemm":
        algo = {"auto": abi.GEMM_AUTO, "simt": abi.GEMM_SIMT, "3xtf32": abi.GEMM_3XTF32,
                "simt_ffma": abi.GEMM_SIMT_FFMA}[a.algo]
        m = a.m or a.n
        lead = (a.batch,) if a.batch > 1 else ()
        A = torch.randn(*lead, a.k, m, device="cuda", generator=g).transpose(-1, -2) if a.at else \
            torch.randn(*lead, m, a.k, device="cuda", generator=g)
        B = torch.randn(*lead, a.n, a.k, device="cuda", generator=g).transpose(-1, -2) if a.bt else \
            torch.randn(*lead, a.k, a.n, device="cuda", generator=g)
        C = torch.empty(*lead, m, a.n, device="cuda")
        ms = run(abi.matmul(V(A), V(B), V(C), algo, prepare=True))
        return {"ms": ms, "tflops": 2.0 * a.batch * m * a.n * a.k / ms / 1e9}
    if a.case == "chain":
        n = a.n
        u = lambda *s: torch.rand(*s, device="cuda", generator=g) * 2 - 1
        A, Bs, row, col = u(n, n), u(n, n), u(1, n), u(n, 1)
        E, Y = torch.empty(n, 1, device="cuda"), torch.empty(n, n, device="cuda")
        abi.fused([(abi.NEGATE, 1, 0, 0, 0.0), (abi.EXP, 2, 1, 0, 0.0)], [V(col)], [2], [V(E)])
        prog = [(abi.MULTIPLY, 4, 0, 1, 0.0), (abi.ADD, 5, 4, 2, 0.0), (abi.RELU, 6, 5, 0, 0.0),
                (abi.MULTIPLY, 7, 6, 3, 0.0)]
        ms = run(abi.fused(prog, [V(A), V(Bs.t()), V(row), V(E)], [7], [V(Y)], prepare=True))
        return {"ms": ms, "gbs": 4.0 * (3 * n * n + 2 * n) / ms / 1e6}
    if a.case in ("reduce", "log_softmax"):
        X = torch.rand(a.n, a.m or a.n, device="cuda", generator=g) * 2 - 1
        if a.case == "log_softmax":
            Y = torch.empty_like(X)
            ms = run(abi.log_softmax(V(X), 1, V(Y), prepare=True))
            return {"ms": ms, "gbs": X.numel() * 8.0 / ms / 1e6}
        op = {"sum": abi.SUM, "max": abi.MAX, "argmax": abi.ARGMAX, "lse": abi.LOGSUMEXP}[a.op]
        O = torch.empty(X.shape[1 - a.axis], device="cuda", dtype=torch.int64 if a.op == "argmax" else torch.float32)
        ms = run(abi.reduce(op, V(X), [a.axis], V(O), prepare=True))
        return {"ms": ms, "gbs": X.numel() * 4.0 / ms / 1e6}
    if a.case in ("gather", "scatter_add"):
        # row gather / scatter-add: the Int64 index column broadcast over the row width
        T = torch.randn(a.rows, a.cols, device="cuda", generator=g)
        idx = torch.randint(0, a.rows, (a.rows,), device="cuda", generator=g, dtype=torch.int64)
        O = torch.empty(a.rows, a.cols, device="cuda")
        vi = abi.View(idx, (a.rows, a.cols), (1, 0), 0)
        if a.case == "gather":
            ms = run(abi.gather(V(T), vi, 0, V(O), prepare=True))
        else:
            U = torch.floor(torch.rand(a.rows, a.cols, device="cuda", generator=g) * 16 - 8)
            ms = run(abi.gather_scatter_add(V(U), vi, 0, V(O), prepare=True))
        return {"ms": ms, "gbs": (2.0 * a.rows * a.cols * 4 + a.rows * 8) / ms / 1e6}
    if a.case == "concat":
        parts = [torch.randn(a.n, a.k, device="cuda", generator=g) for _ in range(4)]
        D = torch.empty((4 * a.n, a.k) if a.axis == 0 else (a.n, 4 * a.k), device="cuda")
        ms = run(abi.concat([V(p) for p in parts], a.axis, V(D), prepare=True))
        return {"ms": ms, "gbs": 2.0 * 4 * a.n * a.k * 4 / ms / 1e6}
    if a.case in ("uniform", "normal"):
        O = torch.empty(a.numel, device="cuda")
        fn = abi.uniform if a.case == "uniform" else abi.normal
        lo_hi = (-1.0, 1.0) if a.case == "uniform" else (0.0, 1.0)
        call = lambda: fn(V(O), *lo_hi, (a.seed, 7))
        ms = run(call)
        return {"ms": ms, "gbs": 4.0 * a.numel / ms / 1e6}
    if a.case == "adamw":
        n = a.numel
        p, gr, m = (torch.randn(n, device="cuda", generator=g) for _ in range(3))
        v = torch.rand(n, device="cuda", generator=g)
        outs = [torch.empty(n, device="cuda") for _ in range(3)]
        prog, regs = adamw_program()
        ms = run(abi.fused(prog, [V(t) for t in (p, gr, m, v)], regs, [V(t) for t in outs], prepare=True))
        return {"ms": ms, "gbs": 28.0 * n / ms / 1e6}
    if a.case == "spiral":
        from minitensor_cpp_b200.frontend import Frontend

        fe = Frontend()
        fe.set_graphs(not a.eager)
        fe.spiral_train(0, 20, loss_every=0)
        n0 = abi.launch_count()
        fe.reset_stats()
        _, secs = fe.spiral_train(0, a.spiral_steps, loss_every=0)
        st = fe.stats()
        steps = max(a.spiral_steps, 1)
        return {"ms_per_step": secs * 1e3 / steps, "samples_per_s": 300 * steps / secs,
                "launches_per_step": (abi.launch_count() - n0) / steps, "replays": st["graph_replays"],
                "evaluations": st["evaluations"], "plan_us_per_step": st["plan_ns"] / 1e3 / steps,
                "execute_us_per_step": st["execute_ns"] / 1e3 / steps}
    raise SystemExit(f"unknown case {a.case}")


def run_case(a) -> None:
    import torch

    from minitensor_cpp_b200 import abi

    if not torch.cuda.is_available():
        raise SystemExit("--case needs a CUDA device")
    torch.cuda.set_device(0)
    abi.lib()
    res = _case(a)
    abi.check_device_errors(0)
    keys = ("m", "n", "k", "batch", "at", "bt", "algo", "op", "axis", "rows", "cols", "numel", "reps", "eager")
    print(json.dumps({"case": a.case, **{k: getattr(a, k) for k in keys}, **res}))


# ------------------------------------------------------------ micro (N=1) --

def _time_ms(fn, reps=10, groups=3, warm=2) -> float:
    """Per-call device time of `fn` (a prepared ABI call): `reps` calls back to
    back between two CUDA events on the current stream, best of `groups`."""
    import torch

    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(groups):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e) / reps)
    return best


def micro_benchmarks(hbm_gbs: float, tf32_tflops: float) -> dict:
    """The elementwise/reduction, GEMM and indexing benchmarks, kernel-level
    through the C ABI on cuda:0.  Each figure is the per-call time of prepared
    calls issued back to back (best of 3 groups); every operand set is larger
    than the 126 MB L2."""
    import torch

    from minitensor_cpp_b200 import abi

    out = {}
    gbs = lambda nbytes, ms: nbytes / (ms * 1e-3) / 1e9
    V = abi.View.of
    # -- broadcast/strided chain relu(A*B^T + row)*exp(-col) and reductions on 8192^2
    n = 8192
    g = torch.Generator(device="cuda").manual_seed(SEED)
    A = torch.rand(n, n, device="cuda", generator=g) * 2 - 1
    Bs = torch.rand(n, n, device="cuda", generator=g) * 2 - 1
    row = torch.rand(1, n, device="cuda", generator=g) * 2 - 1
    col = torch.rand(n, 1, device="cuda", generator=g) * 2 - 1
    Y = torch.empty(n, n, device="cuda")
    E = torch.empty(n, 1, device="cuda")
    # the evaluator's two clusters: exp(-col) over [n,1], then relu(A*B + row) * e over [n,n]
    prog_e = [(abi.NEGATE, 1, 0, 0, 0.0), (abi.EXP, 2, 1, 0, 0.0)]
    prog = [(abi.MULTIPLY, 4, 0, 1, 0.0), (abi.ADD, 5, 4, 2, 0.0), (abi.RELU, 6, 5, 0, 0.0),
            (abi.MULTIPLY, 7, 6, 3, 0.0)]
    call_e = abi.fused(prog_e, [V(col)], [2], [V(E)], prepare=True)
    call_y = abi.fused(prog, [V(A), V(Bs.t()), V(row), V(E)], [7], [V(Y)], prepare=True)

    def chain():
        call_e()
        call_y()

    out["chain_fused_GBps"] = gbs(12 * n * n, _time_ms(chain))
    o = torch.empty(n, device="cuda")
    oi = torch.empty(n, device="cuda", dtype=torch.int64)
    for ax in (0, 1):
        for name, op, dst in (("sum", abi.SUM, o), ("max", abi.MAX, o), ("argmax", abi.ARGMAX, oi)):
            ms = _time_ms(abi.reduce(op, V(Y), [ax], V(dst), prepare=True))
            out[f"{name}_axis{ax}_GBps"] = gbs(4 * n * n, ms)
    Z = torch.empty(n, n, device="cuda")
    ms = _time_ms(abi.log_softmax(V(Y), 1, V(Z), prepare=True))
    out["log_softmax_axis1_GBps"] = gbs(8 * n * n, ms)
    # the fused AdamW update of all 150.8 M parameters: p, g, m, v read; p', m', v' written
    npar = sum(a * b + b for a, b in zip(WIDTHS[:-1], WIDTHS[1:]))
    st = [torch.randn(npar, device="cuda", generator=g) for _ in range(3)] + [torch.rand(npar, device="cuda")]
    res = [torch.empty(npar, device="cuda") for _ in range(3)]
    prog_a, regs_a = adamw_program()
    ms = _time_ms(abi.fused(prog_a, [V(t) for t in st], regs_a, [V(t) for t in res], prepare=True))
    out["adamw_fused_update_GBps"] = gbs(28 * npar, ms)
    del st, res
    hb = [v for k, v in out.items() if k.endswith("GBps")]
    out["elementwise_reduce_min_frac_of_hbm"] = min(hb) / hbm_gbs
    del A, Bs, Y, Z
    # -- GEMM sweep (3xTF32 tensor cores)
    peak3 = tf32_tflops / 3.0
    for m in (1024, 2048, 4096, 16384, 8192):
        a = torch.randn(m, m, device="cuda")
        b = torch.randn(m, m, device="cuda")
        c = torch.empty(m, m, device="cuda")
        for tag, bv in (("", V(b)), ("_bT", V(b.t()))):
            ms = _time_ms(abi.matmul(V(a), bv, V(c), abi.GEMM_3XTF32, prepare=True), reps=3)
            out[f"gemm_{m}{tag}_TFLOPs"] = 2 * m ** 3 / (ms * 1e-3) / 1e12
        if m == 4096:
            # the SIMT kernels: exact (the CPU's k-ascending rounding) and FFMA
            for tag, algo in (("exact", abi.GEMM_SIMT), ("ffma", abi.GEMM_SIMT_FFMA)):
                ms = _time_ms(abi.matmul(V(a), V(b), V(c), algo, prepare=True), reps=3)
                out[f"gemm_simt_{tag}_4096_TFLOPs"] = 2 * m ** 3 / (ms * 1e-3) / 1e12
    # the same 8192^3 GEMM under the default policy and with each kernel variant /
    # shared-memory ring forced, measured in alternating rounds (median of 4):
    # the SM clock under the power cap drifts over seconds, and measuring the
    # variants one after another once gave the last one a 15 % edge that
    # alternating runs did not reproduce
    call = abi.matmul(V(a), V(b), V(c), prepare=True)
    variants = (None, "16x4", "32x2", "pair16x6", "pair32x3")
    times = {v: [] for v in variants}
    for rnd in range(4):
        for variant in (variants if rnd % 2 == 0 else variants[::-1]):
            if variant is not None:
                os.environ["MTC_TC_PIPELINE"] = variant
            try:
                times[variant].append(_time_ms(call, reps=3, groups=1, warm=1))
            finally:
                os.environ.pop("MTC_TC_PIPELINE", None)
    for variant, ts in times.items():
        key = "gemm_8192_TFLOPs" if variant is None else f"gemm_8192_{variant}_TFLOPs"
        out[key] = 2 * 8192 ** 3 / (sorted(ts)[len(ts) // 2] * 1e-3) / 1e12
    out["gemm_8192_frac_of_3xtf32"] = out["gemm_8192_TFLOPs"] / peak3
    a = torch.randn(64, 1024, 1024, device="cuda")
    b = torch.randn(64, 1024, 1024, device="cuda")
    c = torch.empty(64, 1024, 1024, device="cuda")
    ms = _time_ms(abi.matmul(V(a), V(b), V(c), prepare=True), reps=3)
    out["gemm_batched_64x1024_TFLOPs"] = 2 * 64 * 1024 ** 3 / (ms * 1e-3) / 1e12
    a = torch.randn(65536, 1024, device="cuda")
    b = torch.randn(1024, 8192, device="cuda")
    c = torch.empty(65536, 8192, device="cuda")
    ms = _time_ms(abi.matmul(V(a), V(b), V(c), prepare=True), reps=3)
    out["gemm_skinny_65536x1024x8192_TFLOPs"] = 2 * 65536 * 1024 * 8192 / (ms * 1e-3) / 1e12
    del a, b, c
    # -- Int64 gather / scatter-add of 2^24 rows of 64 floats, concat 4 x [4096, 8192]
    rows, width = 1 << 24, 64
    table = torch.randn(rows, width, device="cuda")
    idx = torch.randint(0, rows, (rows, 1), device="cuda", dtype=torch.int64, generator=g)
    idx_b = abi.View(idx.view(-1), (rows, width), (1, 0), 0)  # broadcast_to([rows, width])
    res = torch.empty(rows, width, device="cuda")
    ms = _time_ms(abi.gather(V(table), idx_b, 0, V(res), prepare=True), reps=3)
    out["gather_rows_GBps"] = gbs(rows * 520, ms)
    upd = torch.floor(torch.rand(rows, width, device="cuda", generator=g) * 16 - 8)
    ms = _time_ms(abi.gather_scatter_add(V(upd), idx_b, 0, V(res), prepare=True), reps=3)
    out["scatter_add_rows_GBps"] = gbs(rows * 520, ms)
    del table, idx, res, upd
    parts = [torch.randn(4096, 8192, device="cuda") for _ in range(4)]
    for axis, shape in ((0, (16384, 8192)), (1, (4096, 32768))):
        dst = torch.empty(shape, device="cuda")
        ms = _time_ms(abi.concat([V(p) for p in parts], axis, V(dst), prepare=True), reps=3)
        out[f"concat_axis{axis}_GBps"] = gbs(2 * 4 * 4096 * 8192 * 4, ms)
    del parts
    torch.cuda.empty_cache()
    # -- spiral MLP (300 points, 2-64-64-3, Adam), full batch, through MiniTensor's API
    from minitensor_cpp_b200.frontend import Frontend

    fe = Frontend()
    steps = 3000  # long enough for several clock samples (200 ms apart) per leg
    # eager: every step re-planned and its kernels launched one by one
    graphs = fe.set_graphs(False)
    fe.spiral_train(0, 20, loss_every=0)  # warm-up: NVRTC programs and allocator blocks
    with ClockSampler(0) as ck:
        _, secs = fe.spiral_train(0, steps, loss_every=0)
    out["spiral_eager_samples_per_s"] = 300 * steps / secs
    out["spiral_eager_sm_mhz"] = ck.summary()["sm_mhz"] or 0.0
    # default: the repeated step plan is recorded once and replayed as a CUDA graph
    fe.set_graphs(True)
    fe.spiral_train(0, 20, loss_every=0)
    n0 = abi.launch_count()
    fe.reset_stats()
    with ClockSampler(0) as ck:
        _, secs = fe.spiral_train(0, steps, loss_every=0)
    st = fe.stats()
    fe.set_graphs(graphs)
    out["spiral_train_samples_per_s"] = 300 * steps / secs
    out["spiral_train_sm_mhz"] = ck.summary()["sm_mhz"] or 0.0
    out["spiral_host_us_per_step"] = (st["plan_ns"] + st["execute_ns"] + st["check_ns"]) / 1e3 / steps
    out["spiral_launches_per_step"] = (abi.launch_count() - n0) / steps
    out["spiral_replayed_steps_frac"] = st["graph_replays"] / max(st["evaluations"], 1)
    # -- the broadcast chain and its reductions end to end through the API: host
    #    arrays in, Y and sum(axis 0), sum(axis 1), logsumexp(axis 1) back to the host
    out["chain_api_e2e_s"] = _chain_api_seconds(fe, 0)
    return {k: round(v, 3) for k, v in out.items()}


def _chain_inputs(n: int = 8192):
    import numpy as np

    rng = np.random.default_rng(SEED)
    f = lambda *shape: rng.uniform(-1, 1, shape).astype(np.float32)
    return f(n, n), f(n, n), f(1, n), f(n, 1)


def _chain_api_seconds(fe, device: int) -> float:
    """relu(A * B^T + row) * exp(-col) on 8192^2 and its sum/sum/logsumexp
    reductions through the workload API, host arrays in and results out."""
    a, b, row, col = _chain_inputs()
    fe.chain(device, a[:64, :64], b[:64, :64], row[:, :64], col[:64], reductions=True)  # warm-up
    best = float("inf")
    for _ in range(3 if device >= 0 else 1):  # host page faults make single runs noisy
        t0 = time.perf_counter()
        fe.chain(device, a, b, row, col, reductions=True)
        best = min(best, time.perf_counter() - t0)
    return best


def cpu_micro() -> dict:
    """The other benchmark configurations on the reference CPU backend (oracle/_ref,
    one core): the spiral MLP, the chain with its reductions, a 1024^3 GEMM, a
    2^20-row sample of the row gather, and the axis-0 concat."""
    from minitensor_cpp_b200.frontend import Frontend
    from oracle import refkernels

    import numpy as np

    ref = Frontend(refkernels.LIB_PATH)
    steps = 100
    _, secs = ref.spiral_train(-1, steps, loss_every=0)
    out = {"spiral_train_samples_per_s": round(300 * steps / secs, 1),
           "chain_api_e2e_s": round(_chain_api_seconds(ref, -1), 3), "cores": 1}
    hv = refkernels.HostView
    rng = np.random.default_rng(SEED)
    # GEMM 1024^3 (contiguous operands) on the reference's CPU kernel
    n = 1024
    a = hv.of(rng.standard_normal((n, n)).astype(np.float32))
    b = hv.of(rng.standard_normal((n, n)).astype(np.float32))
    c = hv.of(np.zeros((n, n), np.float32))
    t0 = time.perf_counter()
    refkernels.matmul(a, b, c)
    out["gemm_1024_GFLOPs"] = round(2 * n ** 3 / (time.perf_counter() - t0) / 1e9, 2)
    # row gather of 2^20 rows of 64 floats (a sample of the 2^24-row benchmark)
    rows, width = 1 << 20, 64
    table = hv.of(rng.standard_normal((rows, width)).astype(np.float32))
    idx = rng.integers(0, rows, rows).astype(np.int64)
    idx_b = hv(idx, (rows, width), (1, 0), 0)
    res = hv.of(np.zeros((rows, width), np.float32))
    t0 = time.perf_counter()
    refkernels.gather(table, idx_b, 0, res)
    out["gather_rows_GBps"] = round(rows * 520 / (time.perf_counter() - t0) / 1e9, 3)
    # concat of four [4096, 8192] tensors along axis 0
    parts = [hv.of(rng.standard_normal((4096, 8192)).astype(np.float32)) for _ in range(4)]
    dst = hv.of(np.zeros((16384, 8192), np.float32))
    t0 = time.perf_counter()
    refkernels.concat(parts, 0, dst)
    out["concat_axis0_GBps"] = round(2 * 4 * 4096 * 8192 * 4 / (time.perf_counter() - t0) / 1e9, 3)
    return out


# ----------------------------------------------------------------- our arm --

def run_ours(args) -> None:
    import ctypes

    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    from minitensor_cpp_b200 import abi
    from minitensor_cpp_b200.frontend import Frontend, MlpTrainer

    fe = Frontend()
    batch = GLOBAL_BATCH // world
    tr = MlpTrainer(fe, local, WIDTHS[0], WIDTHS[1], len(WIDTHS) - 2, WIDTHS[-1], seed=SEED, lr=LR)
    comm = None
    if world > 1:
        uid = (ctypes.c_char * 128)()
        if rank == 0:
            abi.check(abi.lib().mtc_comm_unique_id(uid, 128), "nccl id")
        payload = [bytes(uid) if rank == 0 else None]
        dist.broadcast_object_list(payload, src=0)
        uid = (ctypes.c_char * 128).from_buffer_copy(payload[0])
        comm = ctypes.c_void_p()
        abi.check(abi.lib().mtc_comm_init(local, rank, world, uid, 128, ctypes.byref(comm)), "nccl init")
        tr.set_comm(comm, world)

    # BATCHES distinct batches, resident in the trainer's slots: step s of every
    # loop uses batch s mod BATCHES (the benchmark draws fresh inputs each step)
    host = [make_batch(rank, batch, k) for k in range(BATCHES)]
    for k, (xk, yk) in enumerate(host):
        tr.load_batch_slot(k, xk.data_ptr(), yk.data_ptr(), batch)
    tr.use_slot(0)
    stream = torch.cuda.ExternalStream(tr.stream(), device=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for w in range(args.warmup):
        tr.use_slot(w % BATCHES)
        tr.step_resident(read_loss=False)
    tr.synchronize()

    # ---- value: device-resident inputs
    launches0 = abi.launch_count()
    abi.profile_gemm(reset=True)
    abi.profile_enable(True)
    tr.profile(True)
    barrier()
    torch.cuda.synchronize()
    tr.synchronize()
    with ClockSampler(local) as clocks:
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for k in range(args.steps):
            tr.use_slot(k % BATCHES)
            tr.step_resident(read_loss=False)
        stop.record(stream)
        tr.synchronize()
        torch.cuda.synchronize()
    abi.profile_enable(False)
    phase_ms = tr.profile(False)
    launches = abi.launch_count() - launches0
    ms_local = start.elapsed_time(stop)
    ms = max_over_ranks(ms_local)
    barrier()
    gemm_n, gemm_ms, gemm_flops = abi.profile_gemm(reset=True)
    # device milliseconds per step on this rank: the GEMMs, and (N > 1) the
    # phases around the gradient exchange; the slowest rank's figures are kept
    phases = {"gemm": gemm_ms / args.steps, "step": phase_ms[0] / args.steps}
    if world > 1:
        phases.update({"forward_backward": phase_ms[1] / args.steps, "exposed_allreduce": phase_ms[2] / args.steps,
                       "optimizer": phase_ms[3] / args.steps})
    phases = {k: max_over_ranks(v) for k, v in phases.items()}

    # ---- e2e: host buffers through the public API, loss read back every step
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    # one untimed host step first: it sets up the input pipeline (copy stream,
    # events, the two device slots of a batch), like the warm-up steps above
    tr.step_host(host[0][0].data_ptr(), host[0][1].data_ptr(), batch)
    tr.synchronize()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    loss = 0.0
    for k in range(e2e_steps):
        xk, yk = host[k % BATCHES]
        loss = tr.step_host(xk.data_ptr(), yk.data_ptr(), batch)
    e_stop.record(stream)
    tr.synchronize()
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_stop))
    wall_e2e = time.perf_counter() - t0

    tf32 = measure_tf32_peak() if rank == 0 else None
    micro = None
    if world == 1 and not args.skip_micro:
        peaks_file = ROOT / "MEASURED_PEAKS.json"
        hbm = json.loads(peaks_file.read_text()).get("hbm_gbs", 6650.0) if peaks_file.exists() else 6650.0
        tr.close()
        micro = micro_benchmarks(hbm, tf32)
    if comm is not None:
        barrier()
        abi.lib().mtc_comm_destroy(comm)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks_path = ROOT / "MEASURED_PEAKS.json"
    peaks = json.loads(peaks_path.read_text()) if peaks_path.exists() else {}
    value = GLOBAL_BATCH * args.steps / (ms * 1e-3)
    gemm_tflops = gemm_flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None
    peak = tf32 / 3.0 if tf32 else None
    roofline = {
        "kernel": "3xTF32 tcgen05 GEMM (matmul of every Linear forward/backward)",
        "bound": "tensor",
        "achieved": gemm_tflops,
        "peak": peak,
        "unit": "TFLOP/s",
        "frac": (gemm_tflops / peak) if (gemm_tflops and peak) else None,
        "peak_source": f"measured cuBLAS TF32 {tf32:.1f} TFLOP/s / 3 (3xTF32); bf16 burst in MEASURED_PEAKS.json "
                       f"{peaks.get('bf16_tflops')}" if tf32 else None,
        "launches": gemm_n,
        "avg_launch_ms": gemm_ms / gemm_n if gemm_n else None,
        "traffic": read_traffic("gemm_3xtf32"),
    }
    cpu = None
    if world == 1 and not args.skip_cpu:
        s = cpu_reference_sample(args.cpu_batch, 1)
        cpu = {"value": s["samples"] / s["seconds"], "unit": "samples/s", "cores": 1, "host_cores": os.cpu_count(),
               "kind": "reference",
               "sample": f"1 training step at batch {args.cpu_batch} (same model, Adam) on the reference CPU "
                         f"backend, {s['seconds']:.1f} s"}
        if not args.skip_micro:
            cpu["micro"] = cpu_micro()
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "samples/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) inputs, uniform Int64 labels)",
        "config": config(world),
        "tflops": flops_per_sample() * GLOBAL_BATCH * args.steps / (ms * 1e-3) / 1e12,
        "e2e": {"value": GLOBAL_BATCH * e2e_steps / (e2e_ms * 1e-3), "unit": "samples/s",
                "steps": e2e_steps, "wall_s": wall_e2e, "last_loss": loss,
                "h2d_bytes_per_step": world * (host[0][0].numel() * 4 + host[0][1].numel() * 8),
                "d2h_bytes_per_step": world * 4},
        "gpu_launches": launches,
        "phases_ms_per_step": {k: round(v, 3) for k, v in phases.items()},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "micro": micro,
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------- reference arm --

def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import refkernels

    if not refkernels.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libmtref.so was not built"}))
        return
    import multiprocessing as mp

    cores = os.cpu_count() or 1
    try:
        avail_gb = os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE") / 2 ** 30
    except (ValueError, OSError):
        avail_gb = 64.0
    # each single-threaded reference process holds the 151M-parameter model,
    # its Adam moments and the step's intermediates (~10 GB peak)
    workers = max(1, min(cores, int(avail_gb // 12), 16, args.steps))
    batch = args.cpu_batch
    # the --steps timed steps (and one untimed step per worker when --warmup is
    # given) are shared out over the workers: a step at batch 4 takes about 12 s,
    # so the whole run stays within a couple of minutes
    shares = [args.steps // workers + (1 if k < args.steps % workers else 0) for k in range(workers)]
    warm = 1 if args.warmup > 0 else 0
    ctx = mp.get_context("spawn")
    t0 = time.perf_counter()
    with ctx.Pool(workers) as pool:
        results = pool.map(_worker, [(batch, n, warm) for n in shares])
    wall = time.perf_counter() - t0
    samples = sum(r["samples"] for r in results)
    busiest = max(r["seconds"] for r in results)
    value = samples / busiest
    steps = sum(shares)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "samples/s",
        "impl": "reference",
        "n_gpus": args.gpus,
        "steps": steps,
        "warmup": warm * workers,
        "higher_is_better": True,
        "scaling": "strong",
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) inputs, uniform Int64 labels)",
        "config": config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": workers, "host_cores": cores,
                         "kind": "reference",
                         "sample": f"{steps} training steps at batch {batch} shared over {workers} single-threaded "
                                   f"reference processes (the reference is single-threaded), each after "
                                   f"{warm} untimed step; samples / the slowest process's timed seconds; "
                                   f"wall {wall:.1f} s"},
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--e2e-steps", type=int, default=5)
    p.add_argument("--cpu-batch", type=int, default=4)
    p.add_argument("--skip-cpu", action="store_true", help="omit the CPU baseline sample")
    p.add_argument("--skip-micro", action="store_true", help="omit the kernel microbenchmarks (N=1 only)")
    c = p.add_argument_group("single-kernel cases (--case)")
    c.add_argument("--case", choices=("gemm", "chain", "reduce", "log_softmax", "gather", "scatter_add", "concat",
                                      "uniform", "normal", "adamw", "spiral"),
                   help="run one kernel alone on cuda:0 and print its time (for ncu captures)")
    c.add_argument("--m", type=int, default=0, help="gemm: rows of A (default --n); reduce: columns")
    c.add_argument("--n", type=int, default=8192)
    c.add_argument("--k", type=int, default=8192)
    c.add_argument("--batch", type=int, default=1)
    c.add_argument("--at", action="store_true", help="gemm: A is the transposed view of a [k, m] tensor")
    c.add_argument("--bt", action="store_true", help="gemm: B is the transposed view of an [n, k] tensor")
    c.add_argument("--algo", default="3xtf32", choices=("auto", "simt", "3xtf32", "simt_ffma"))
    c.add_argument("--op", default="sum", choices=("sum", "max", "argmax", "lse"))
    c.add_argument("--axis", type=int, default=0)
    c.add_argument("--rows", type=int, default=1 << 24)
    c.add_argument("--cols", type=int, default=64)
    c.add_argument("--numel", type=int, default=150823912, help="adamw / uniform / normal: element count")
    c.add_argument("--reps", type=int, default=3)
    c.add_argument("--seed", type=int, default=0)
    c.add_argument("--spiral-steps", type=int, default=500)
    c.add_argument("--eager", action="store_true", help="spiral: no plan replay")
    c.add_argument("--warm-s", type=float, default=0.3, help="untimed calls first (0 under a profiler)")
    args = p.parse_args()
    if args.case:
        run_case(args)
        return
    if args.warmup < 3:
        p.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
