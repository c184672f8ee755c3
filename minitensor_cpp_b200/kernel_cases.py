"""Single-kernel cases of the backend, for profiling and timing one kernel alone.

    python -m minitensor_cpp_b200.kernel_cases gemm --m 8192 --n 8192 --k 8192 [--bt] [--batch B]
    python -m minitensor_cpp_b200.kernel_cases chain --n 8192
    python -m minitensor_cpp_b200.kernel_cases reduce --n 8192 --op sum --axis 0
    python -m minitensor_cpp_b200.kernel_cases log_softmax --n 8192
    python -m minitensor_cpp_b200.kernel_cases gather --rows 16777216 --cols 64
    python -m minitensor_cpp_b200.kernel_cases adamw --numel 150823912
    python -m minitensor_cpp_b200.kernel_cases spiral --steps 500 [--eager]

Each case allocates its operands on cuda:0 with torch (device memory only),
calls the C ABI `--reps` times back to back (prepared calls) on the current stream, synchronises, checks
the device error word and prints one line with the mean time per call measured
with CUDA events, after --warm-s seconds of untimed calls.  Under a profiler,
pass --warm-s 0 --reps 1: the launches are then the set-up call and one timed call.
"""
from __future__ import annotations

import argparse
import json
import sys

from . import abi


WARM_S = 0.3


def _events_ms(fn, reps: int, stream) -> float:
    import torch

    import time

    fn()  # first call: NVRTC / tensor-map set-up, not timed
    torch.cuda.synchronize()
    t0 = time.perf_counter()  # then WARM_S seconds of calls so the SM clock has left idle
    while time.perf_counter() - t0 < WARM_S:
        fn()
        torch.cuda.synchronize()
    # `stream` is the current torch stream's handle, so events on it bracket the calls
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        fn()
    stop.record()
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / reps


def case_gemm(a, torch, stream):
    algo = {"auto": abi.GEMM_AUTO, "simt": abi.GEMM_SIMT, "3xtf32": abi.GEMM_3XTF32,
            "simt_ffma": abi.GEMM_SIMT_FFMA}[a.algo]
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    lead = (a.batch,) if a.batch > 1 else ()
    A = torch.randn(*lead, a.m, a.k, device="cuda", generator=g)
    B = torch.randn(*lead, a.n, a.k, device="cuda", generator=g).transpose(-1, -2) if a.bt else \
        torch.randn(*lead, a.k, a.n, device="cuda", generator=g)
    C = torch.empty(*lead, a.m, a.n, device="cuda")
    va, vb, vc = abi.View.of(A), abi.View.of(B), abi.View.of(C)
    ms = _events_ms(abi.matmul(va, vb, vc, algo, stream, prepare=True), a.reps, stream)
    flop = 2.0 * a.batch * a.m * a.n * a.k
    return {"ms": ms, "tflops": flop / ms / 1e9}


def case_chain(a, torch, stream):
    """relu(A*B + row) * e with B a transposed view and e = exp(-col) precomputed [n,1]."""
    n = a.n
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    u = lambda *s: torch.rand(*s, device="cuda", generator=g) * 2 - 1
    A, Bs, row, col = u(n, n), u(n, n), u(1, n), u(n, 1)
    E = torch.empty(n, 1, device="cuda")
    Y = torch.empty(n, n, device="cuda")
    abi.fused([(abi.NEGATE, 1, 0, 0, 0.0), (abi.EXP, 2, 1, 0, 0.0)], [abi.View.of(col)], [2], [abi.View.of(E)],
              stream)
    prog = [(abi.MULTIPLY, 4, 0, 1, 0.0), (abi.ADD, 5, 4, 2, 0.0), (abi.RELU, 6, 5, 0, 0.0),
            (abi.MULTIPLY, 7, 6, 3, 0.0)]
    ins = [abi.View.of(A), abi.View.of(Bs.t()), abi.View.of(row), abi.View.of(E)]
    vy = abi.View.of(Y)
    ms = _events_ms(abi.fused(prog, ins, [7], [vy], stream, prepare=True), a.reps, stream)
    return {"ms": ms, "gbs": 4.0 * (3 * n * n + 2 * n) / ms / 1e6}


def case_reduce(a, torch, stream):
    op = {"sum": abi.SUM, "max": abi.MAX, "argmax": abi.ARGMAX, "lse": abi.LOGSUMEXP}[a.op]
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    X = torch.rand(a.n, a.m or a.n, device="cuda", generator=g) * 2 - 1
    out_len = X.shape[1 - a.axis]
    dtype = torch.int64 if a.op == "argmax" else torch.float32
    O = torch.empty(out_len, device="cuda", dtype=dtype)
    vx, vo = abi.View.of(X), abi.View.of(O)
    ms = _events_ms(abi.reduce(op, vx, [a.axis], vo, stream, prepare=True), a.reps, stream)
    return {"ms": ms, "gbs": X.numel() * 4.0 / ms / 1e6}


def case_log_softmax(a, torch, stream):
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    X = torch.rand(a.n, a.m or a.n, device="cuda", generator=g) * 2 - 1
    Y = torch.empty_like(X)
    vx, vy = abi.View.of(X), abi.View.of(Y)
    ms = _events_ms(abi.log_softmax(vx, 1, vy, stream, prepare=True), a.reps, stream)
    return {"ms": ms, "gbs": X.numel() * 8.0 / ms / 1e6}


def case_gather(a, torch, stream):
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    T = torch.randn(a.rows, a.cols, device="cuda", generator=g)
    idx = torch.randint(0, a.rows, (a.rows,), device="cuda", generator=g, dtype=torch.int64)
    O = torch.empty(a.rows, a.cols, device="cuda")
    # row gather: the index column broadcast over the row width (stride 0)
    vt, vi, vo = abi.View.of(T), abi.View(idx, (a.rows, a.cols), (1, 0), 0), abi.View.of(O)
    ms = _events_ms(abi.gather(vt, vi, 0, vo, stream, prepare=True), a.reps, stream)
    return {"ms": ms, "gbs": (2.0 * a.rows * a.cols * 4 + a.rows * 8) / ms / 1e6}


def adamw_program(lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, c1=0.1, c2=0.001):
    """AdamW's per-parameter update as one fused program: registers 0..3 are
    p, g, m, v; outputs p', m', v' (the evaluator builds the same cluster)."""
    C, M, A, D, S = abi.CONST, abi.MULTIPLY, abi.ADD, abi.DIVIDE, abi.SUBTRACT
    prog = [(C, 4, 0, 0, b1), (M, 5, 4, 2, 0.0), (C, 6, 0, 0, 1 - b1), (M, 7, 6, 1, 0.0), (A, 8, 5, 7, 0.0),
            (C, 9, 0, 0, b2), (M, 10, 9, 3, 0.0), (C, 11, 0, 0, 1 - b2), (M, 12, 11, 1, 0.0), (M, 13, 12, 1, 0.0),
            (A, 14, 10, 13, 0.0), (C, 15, 0, 0, c1), (D, 16, 8, 15, 0.0), (C, 17, 0, 0, c2), (D, 18, 14, 17, 0.0),
            (C, 21, 0, 0, lr), (M, 22, 21, 16, 0.0), (abi.SQRT, 23, 18, 0, 0.0), (C, 24, 0, 0, eps),
            (A, 25, 23, 24, 0.0), (D, 26, 22, 25, 0.0), (S, 27, 0, 26, 0.0)]
    return prog, [27, 8, 14]


def case_adamw(a, torch, stream):
    """The fused AdamW update over --numel parameters: 4 reads + 3 writes per element."""
    n = a.numel
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    p, gr, m = (torch.randn(n, device="cuda", generator=g) for _ in range(3))
    v = torch.rand(n, device="cuda", generator=g)
    outs = [torch.empty(n, device="cuda") for _ in range(3)]
    prog, regs = adamw_program()
    call = abi.fused(prog, [abi.View.of(t) for t in (p, gr, m, v)], regs, [abi.View.of(t) for t in outs], stream,
                     prepare=True)
    ms = _events_ms(call, a.reps, stream)
    return {"ms": ms, "gbs": 28.0 * n / ms / 1e6}


def case_spiral(a, torch, stream):
    """The spiral MLP (300 points, 2-64-64-3, Adam) through MiniTensor's API:
    --warm-steps untimed steps, then --steps timed ones (host clock; the call
    returns after the final parameters are on the host).  Plans repeat from
    step to step, so they are replayed as CUDA graphs unless --eager."""
    from .frontend import Frontend

    fe = Frontend()
    fe.set_graphs(not a.eager)
    fe.spiral_train(0, a.warm_steps, loss_every=0)
    n0 = abi.launch_count()
    fe.reset_stats()
    _, secs = fe.spiral_train(0, a.steps, loss_every=0)
    st = fe.stats()
    return {"ms_per_step": secs * 1e3 / max(a.steps, 1), "samples_per_s": 300 * a.steps / secs,
            "launches_per_step": (abi.launch_count() - n0) / max(a.steps, 1),
            "replays": st["graph_replays"], "evaluations": st["evaluations"],
            "plan_us_per_step": st["plan_ns"] / 1e3 / max(a.steps, 1),
            "execute_us_per_step": st["execute_ns"] / 1e3 / max(a.steps, 1)}


CASES = {"gemm": case_gemm, "chain": case_chain, "reduce": case_reduce, "log_softmax": case_log_softmax,
         "gather": case_gather, "adamw": case_adamw, "spiral": case_spiral}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("case", choices=sorted(CASES))
    p.add_argument("--m", type=int, default=0)
    p.add_argument("--n", type=int, default=8192)
    p.add_argument("--k", type=int, default=8192)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--bt", action="store_true", help="B is the transposed view of an [n, k] tensor")
    p.add_argument("--algo", default="3xtf32")
    p.add_argument("--op", default="sum")
    p.add_argument("--axis", type=int, default=0)
    p.add_argument("--rows", type=int, default=1 << 24)
    p.add_argument("--cols", type=int, default=64)
    p.add_argument("--reps", type=int, default=3)
    p.add_argument("--numel", type=int, default=150823912, help="adamw: parameter count")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--steps", type=int, default=500, help="spiral: timed training steps")
    p.add_argument("--warm-steps", type=int, default=20, help="spiral: untimed training steps first")
    p.add_argument("--eager", action="store_true", help="spiral: no plan replay")
    p.add_argument("--warm-s", type=float, default=0.3, help="untimed calls before timing (0 under a profiler)")
    a = p.parse_args(argv)
    global WARM_S
    WARM_S = a.warm_s
    if a.case == "gemm" and a.m == 0:
        a.m = a.n
    import torch

    if not torch.cuda.is_available():
        print("kernel_cases: no CUDA device", file=sys.stderr)
        return 2
    torch.cuda.set_device(0)
    abi.lib()
    stream = torch.cuda.current_stream().cuda_stream
    res = CASES[a.case](a, torch, stream)
    abi.check_device_errors(0, stream)
    print(json.dumps({"case": a.case, **{k: v for k, v in vars(a).items() if k != "case"}, **res}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
