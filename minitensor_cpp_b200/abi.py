"""ctypes binding of libmtcuda.so, the C ABI declared in include/mtcuda.h.

This is the binding a Python caller of the B200 backend uses (and what the
GPU parity tests call through).  Operands are `View`s: a flat storage tensor
plus shape, strides and offset in elements, i.e. the reference's
`Materialization{Buffer, Layout}` (src/tensor/storage/materialization.hpp:11-22).
Errors come back as the exception type the reference would throw for the same
condition (std::invalid_argument -> ValueError, std::out_of_range -> IndexError,
std::overflow_error -> OverflowError, std::runtime_error / logic_error ->
RuntimeError).

Loading fails loudly: there is no fallback path when the library is missing.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Sequence

MAX_RANK = 8

OK, ERR_INVALID_ARGUMENT, ERR_OUT_OF_RANGE, ERR_RUNTIME, ERR_LOGIC, ERR_OVERFLOW, ERR_UNSUPPORTED = range(7)
FLOAT32, INT64 = 0, 1

# operation codes (reference PrimitiveId values; 0x..80+ are additions)
ABS, SIGN, NEGATE, EXP, LOG, SQRT, TANH, SIGMOID = range(0x0101, 0x0109)
RELU = 0x0180
ADD, SUBTRACT, MULTIPLY, DIVIDE, LOGADDEXP = range(0x0110, 0x0115)
CONST = 0x01F0
SUM, LOGSUMEXP, MAX, ARGMAX = 0x0301, 0x0302, 0x0380, 0x0381
UNARY_OPS = (ABS, SIGN, NEGATE, EXP, LOG, SQRT, TANH, SIGMOID, RELU)
BINARY_OPS = (ADD, SUBTRACT, MULTIPLY, DIVIDE, LOGADDEXP)

GEMM_AUTO, GEMM_SIMT, GEMM_3XTF32, GEMM_SIMT_FFMA = 0, 1, 2, 3

LIB_DIR = Path(__file__).resolve().parent / "lib"


class Desc(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("offset", ctypes.c_int64),
        ("capacity", ctypes.c_int64),
        ("dtype", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_RANK),
        ("strides", ctypes.c_int64 * MAX_RANK),
    ]


class Instr(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_int32),
        ("dst", ctypes.c_int16),
        ("a", ctypes.c_int16),
        ("b", ctypes.c_int16),
        ("pad", ctypes.c_int16),
        ("imm", ctypes.c_float),
    ]


def make_desc(ptr: int, capacity: int, dtype: int, shape: Sequence[int], strides: Sequence[int], offset: int) -> Desc:
    if len(shape) != len(strides) or len(shape) > MAX_RANK:
        raise ValueError("shape/strides rank mismatch or rank > 8")
    d = Desc()
    d.data = ptr
    d.offset = int(offset)
    d.capacity = int(capacity)
    d.dtype = int(dtype)
    d.rank = len(shape)
    for i, (e, s) in enumerate(zip(shape, strides)):
        d.shape[i] = int(e)
        d.strides[i] = int(s)
    return d


def contiguous_strides(shape: Sequence[int]) -> list[int]:
    """Layout::contiguous (src/tensor/storage/layout.cpp:23-48): extent-0/1 axes do not grow the stride."""
    strides = [1] * len(shape)
    run = 1
    for i in range(len(shape) - 1, -1, -1):
        strides[i] = run
        if shape[i] >= 2:
            run *= shape[i]
    return strides


@dataclass
class View:
    """A strided view of a flat storage tensor (torch tensor, on any device)."""

    storage: "object"  # torch.Tensor, 1-D
    shape: tuple
    strides: tuple
    offset: int = 0

    @staticmethod
    def of(t) -> "View":
        """View of an existing torch tensor (shares its storage)."""
        import torch

        flat = torch.empty(0, dtype=t.dtype, device=t.device).set_(t.untyped_storage())
        return View(flat, tuple(t.shape), tuple(t.stride()), t.storage_offset())

    @staticmethod
    def contiguous(storage, shape, offset: int = 0) -> "View":
        return View(storage, tuple(shape), tuple(contiguous_strides(shape)), offset)

    def desc(self) -> Desc:
        import torch

        dt = INT64 if self.storage.dtype == torch.int64 else FLOAT32
        return make_desc(self.storage.data_ptr(), self.storage.numel(), dt, self.shape, self.strides, self.offset)

    def tensor(self):
        """The same view as a torch tensor (for zero/positive strides)."""
        return self.storage.as_strided(self.shape, self.strides, self.offset)


class MtcError(RuntimeError):
    pass


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = LIB_DIR / "libmtcuda.so"
        try:  # load PyTorch first so its CUDA runtime / NCCL are the process-wide copies
            import torch  # noqa: F401
        except ImportError:
            pass
        if not path.exists():
            raise MtcError(f"libmtcuda.so is not built ({path}); run __graft_entry__.build()")
        _lib = ctypes.CDLL(str(path), mode=os.RTLD_GLOBAL if hasattr(os, "RTLD_GLOBAL") else 0)
        _declare(_lib)
    return _lib


def _declare(L):
    P = ctypes.POINTER
    c_int, c_i32, c_i64, c_f, c_vp, c_sz = ctypes.c_int, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t
    sig = {
        "mtc_last_error": ([], ctypes.c_char_p),
        "mtc_version": ([], ctypes.c_char_p),
        "mtc_device_count": ([P(c_int)], c_int),
        "mtc_device_sm_count": ([c_int, P(c_int)], c_int),
        "mtc_device_stream": ([c_int, P(c_vp)], c_int),
        "mtc_set_device": ([c_int], c_int),
        "mtc_alloc": ([c_int, c_sz, c_vp, P(c_vp)], c_int),
        "mtc_free": ([c_int, c_vp, c_vp], c_int),
        "mtc_copy_from_host": ([c_int, c_vp, c_vp, c_sz, c_vp], c_int),
        "mtc_copy_to_host": ([c_int, c_vp, c_vp, c_sz, c_vp], c_int),
        "mtc_stream_synchronize": ([c_vp], c_int),
        "mtc_pool_stats": ([c_int, P(ctypes.c_uint64), P(ctypes.c_uint64)], c_int),
        "mtc_pool_trim": ([c_int], c_int),
        "mtc_pool_take": ([c_int, c_vp, c_sz, c_vp], c_int),
        "mtc_stream_create": ([c_int, P(c_vp)], c_int),
        "mtc_stream_destroy": ([c_int, c_vp], c_int),
        "mtc_event_create": ([c_int, P(c_vp)], c_int),
        "mtc_event_destroy": ([c_int, c_vp], c_int),
        "mtc_event_record": ([c_vp, c_vp], c_int),
        "mtc_stream_wait_event": ([c_vp, c_vp], c_int),
        "mtc_event_create_timed": ([c_int, P(c_vp)], c_int),
        "mtc_event_elapsed": ([c_vp, c_vp, P(c_f)], c_int),
        "mtc_pool_protect": ([c_int, c_vp, c_i32], c_int),
        "mtc_pool_take_many": ([c_int, P(c_vp), P(c_sz), c_i32, c_vp, P(c_i32)], c_int),
        "mtc_capture_begin": ([c_int, c_vp], c_int),
        "mtc_capture_end": ([c_int, P(c_vp)], c_int),
        "mtc_capture_fused_count": ([P(c_i32)], c_int),
        "mtc_graph_launch": ([c_vp], c_int),
        "mtc_graph_set_constants": ([c_vp, c_i32, P(c_f), c_i32], c_int),
        "mtc_graph_launches": ([c_vp, P(ctypes.c_uint64)], c_int),
        "mtc_graph_destroy": ([c_vp], c_int),
        "mtc_check_device_errors": ([c_int, c_vp, P(c_i64)], c_int),
        "mtc_watch_device_errors": ([c_int, c_vp], c_int),
        "mtc_poll_device_errors": ([c_int, c_int, P(ctypes.c_int64)], c_int),
        "mtc_selftest_bounded_wait": ([c_i64, c_vp], c_int),
        "mtc_unary": ([c_i32, P(Desc), P(Desc), c_vp], c_int),
        "mtc_binary": ([c_i32, P(Desc), P(Desc), P(Desc), c_vp], c_int),
        "mtc_fused": ([P(Instr), c_i32, P(Desc), c_i32, P(c_i32), P(Desc), c_i32, c_vp], c_int),
        "mtc_copy": ([P(Desc), P(Desc), c_vp], c_int),
        "mtc_concat": ([P(Desc), c_i32, c_i64, P(Desc), c_vp], c_int),
        "mtc_index_scatter": ([P(Desc), P(Desc), P(Desc), c_vp], c_int),
        "mtc_gather": ([P(Desc), P(Desc), c_i64, P(Desc), c_vp], c_int),
        "mtc_gather_scatter_add": ([P(Desc), P(Desc), c_i64, P(Desc), c_vp], c_int),
        "mtc_gather_scatter_add_into": ([P(Desc), P(Desc), c_i64, P(Desc), c_vp], c_int),
        "mtc_reduce": ([c_i32, P(Desc), P(c_i64), c_i32, P(Desc), c_vp], c_int),
        "mtc_log_softmax": ([P(Desc), c_i64, P(Desc), c_vp], c_int),
        "mtc_matmul": ([P(Desc), P(Desc), P(Desc), c_i32, c_vp], c_int),
        "mtc_matmul_3xtf32_static": ([P(Desc), P(Desc), P(Desc), c_vp], c_int),
        "mtc_fill": ([P(Desc), c_vp, c_vp], c_int),
        "mtc_uniform": ([P(Desc), c_f, c_f, ctypes.c_uint64, ctypes.c_uint64, c_vp], c_int),
        "mtc_normal": ([P(Desc), c_f, c_f, ctypes.c_uint64, ctypes.c_uint64, c_vp], c_int),
        "mtc_launch_count": ([P(ctypes.c_uint64)], c_int),
        "mtc_profile_enable": ([c_int], c_int),
        "mtc_profile_gemm": ([P(ctypes.c_uint64), P(ctypes.c_double), P(ctypes.c_double), c_int], c_int),
        "mtc_gemm_path_counts": ([P(ctypes.c_uint64), P(ctypes.c_uint64)], c_int),
        "mtc_comm_unique_id": ([c_vp, c_sz], c_int),
        "mtc_comm_init": ([c_int, c_int, c_int, c_vp, c_sz, P(c_vp)], c_int),
        "mtc_comm_allreduce_f32": ([c_vp, P(c_vp), P(c_sz), c_i32, c_f, c_vp], c_int),
        "mtc_comm_allreduce_f32_async": ([c_vp, P(c_vp), P(c_sz), c_i32, c_f, c_vp], c_int),
        "mtc_comm_wait": ([c_vp, c_vp], c_int),
        "mtc_comm_destroy": ([c_vp], c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res


EXPORTED = (
    "mtc_last_error", "mtc_version", "mtc_device_count", "mtc_device_sm_count", "mtc_set_device", "mtc_device_stream", "mtc_alloc",
    "mtc_free", "mtc_copy_from_host", "mtc_copy_to_host", "mtc_stream_synchronize", "mtc_pool_stats", "mtc_pool_trim",
    "mtc_stream_create", "mtc_stream_destroy", "mtc_event_create", "mtc_event_destroy", "mtc_event_record",
    "mtc_stream_wait_event", "mtc_event_create_timed", "mtc_event_elapsed", "mtc_pool_take", "mtc_pool_take_many", "mtc_pool_protect", "mtc_capture_begin", "mtc_capture_end", "mtc_capture_fused_count", "mtc_graph_launch",
    "mtc_graph_set_constants", "mtc_graph_launches", "mtc_graph_destroy",
    "mtc_check_device_errors", "mtc_watch_device_errors", "mtc_poll_device_errors", "mtc_selftest_bounded_wait", "mtc_unary", "mtc_binary", "mtc_fused", "mtc_copy", "mtc_concat", "mtc_index_scatter",
    "mtc_gather", "mtc_gather_scatter_add", "mtc_gather_scatter_add_into", "mtc_reduce", "mtc_log_softmax", "mtc_matmul", "mtc_fill", "mtc_uniform",
    "mtc_normal", "mtc_launch_count", "mtc_profile_enable", "mtc_profile_gemm", "mtc_gemm_path_counts", "mtc_comm_unique_id", "mtc_comm_init", "mtc_comm_allreduce_f32", "mtc_comm_allreduce_f32_async", "mtc_comm_wait", "mtc_comm_destroy",
)


def check(rc: int, what: str = "") -> None:
    if rc == OK:
        return
    msg = lib().mtc_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if rc == ERR_INVALID_ARGUMENT:
        raise ValueError(text)
    if rc == ERR_OUT_OF_RANGE:
        raise IndexError(text)
    if rc == ERR_OVERFLOW:
        raise OverflowError(text)
    raise MtcError(f"[code {rc}] {text}")


def _stream(stream):
    if stream is None:
        import torch

        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return ctypes.c_void_p(int(stream))


# ------------------------------------------------------------------ wrappers --
# Every kernel wrapper takes `prepare=True` to return a zero-argument callable
# with its ctypes arguments converted once: repeated calls then cost one ctypes
# dispatch, so back-to-back launches keep the GPU busy in timing loops.

def _run(name: str, args: tuple, what: str, prepare: bool):
    fn = getattr(lib(), name)
    if prepare:
        def call() -> None:
            check(fn(*args), what)
        return call
    check(fn(*args), what)
    return None


def unary(op: int, x: View, out: View, stream=None, prepare: bool = False):
    return _run("mtc_unary", (op, ctypes.byref(x.desc()), ctypes.byref(out.desc()), _stream(stream)), "unary", prepare)


def binary(op: int, a: View, b: View, out: View, stream=None, prepare: bool = False):
    return _run("mtc_binary", (op, ctypes.byref(a.desc()), ctypes.byref(b.desc()), ctypes.byref(out.desc()),
                               _stream(stream)), "binary", prepare)


def fused(program: Sequence[tuple], inputs: Sequence[View], out_regs: Sequence[int], outputs: Sequence[View],
          stream=None, prepare: bool = False):
    """program: (op, dst, a, b, imm) tuples."""
    n = len(program)
    instrs = (Instr * max(n, 1))()
    for i, (op, dst, a, b, imm) in enumerate(program):
        instrs[i].op, instrs[i].dst, instrs[i].a, instrs[i].b, instrs[i].imm = op, dst, a, b, imm
    ins = (Desc * max(len(inputs), 1))(*[v.desc() for v in inputs])
    outs = (Desc * len(outputs))(*[v.desc() for v in outputs])
    regs = (ctypes.c_int32 * len(out_regs))(*out_regs)
    return _run("mtc_fused", (instrs, n, ins, len(inputs), regs, outs, len(outputs), _stream(stream)), "fused",
                prepare)


def copy(src: View, dst: View, stream=None, prepare: bool = False):
    return _run("mtc_copy", (ctypes.byref(src.desc()), ctypes.byref(dst.desc()), _stream(stream)), "copy", prepare)


def concat(inputs: Sequence[View], axis: int, out: View, stream=None, prepare: bool = False):
    arr = (Desc * len(inputs))(*[v.desc() for v in inputs])
    return _run("mtc_concat", (arr, len(inputs), axis, ctypes.byref(out.desc()), _stream(stream)), "concat", prepare)


def index_scatter(x: View, dst_view: View, out: View, stream=None, prepare: bool = False):
    return _run("mtc_index_scatter", (ctypes.byref(x.desc()), ctypes.byref(dst_view.desc()), ctypes.byref(out.desc()),
                                      _stream(stream)), "index_scatter", prepare)


def gather(src: View, idx: View, axis: int, out: View, stream=None, prepare: bool = False):
    return _run("mtc_gather", (ctypes.byref(src.desc()), ctypes.byref(idx.desc()), axis, ctypes.byref(out.desc()),
                               _stream(stream)), "gather", prepare)


def gather_scatter_add(upd: View, idx: View, axis: int, out: View, stream=None, prepare: bool = False):
    return _run("mtc_gather_scatter_add", (ctypes.byref(upd.desc()), ctypes.byref(idx.desc()), axis,
                                           ctypes.byref(out.desc()), _stream(stream)), "gather_scatter_add", prepare)


def reduce(op: int, x: View, axes: Sequence[int], out: View, stream=None, prepare: bool = False):
    ax = (ctypes.c_int64 * max(len(axes), 1))(*axes)
    return _run("mtc_reduce", (op, ctypes.byref(x.desc()), ax, len(axes), ctypes.byref(out.desc()), _stream(stream)),
                "reduce", prepare)


def log_softmax(x: View, axis: int, out: View, stream=None, prepare: bool = False):
    return _run("mtc_log_softmax", (ctypes.byref(x.desc()), axis, ctypes.byref(out.desc()), _stream(stream)),
                "log_softmax", prepare)


def matmul(a: View, b: View, out: View, algo: int = GEMM_AUTO, stream=None, prepare: bool = False):
    return _run("mtc_matmul", (ctypes.byref(a.desc()), ctypes.byref(b.desc()), ctypes.byref(out.desc()), algo,
                               _stream(stream)), "matmul", prepare)


def fill(out: View, value, stream=None) -> None:
    import torch

    if out.storage.dtype == torch.int64:
        v = ctypes.c_int64(int(value))
    else:
        v = ctypes.c_float(float(value))
    check(lib().mtc_fill(ctypes.byref(out.desc()), ctypes.byref(v), _stream(stream)), "fill")


def uniform(out: View, low: float, high: float, key: tuple, stream=None) -> None:
    check(lib().mtc_uniform(ctypes.byref(out.desc()), low, high, key[0], key[1], _stream(stream)), "uniform")


def normal(out: View, mean: float, std: float, key: tuple, stream=None) -> None:
    check(lib().mtc_normal(ctypes.byref(out.desc()), mean, std, key[0], key[1], _stream(stream)), "normal")


def launch_count() -> int:
    n = ctypes.c_uint64(0)
    check(lib().mtc_launch_count(ctypes.byref(n)))
    return n.value


def profile_enable(on: bool) -> None:
    check(lib().mtc_profile_enable(int(on)))


def profile_gemm(reset: bool = True):
    """(launches, total ms, total FLOPs) of GEMM launches since the last reset."""
    n, ms, fl = ctypes.c_uint64(0), ctypes.c_double(0.0), ctypes.c_double(0.0)
    check(lib().mtc_profile_gemm(ctypes.byref(n), ctypes.byref(ms), ctypes.byref(fl), int(reset)))
    return n.value, ms.value, fl.value


def gemm_path_counts():
    """(tensor-core calls, SIMT calls) of mtc_matmul since the process started."""
    tc, simt = ctypes.c_uint64(0), ctypes.c_uint64(0)
    check(lib().mtc_gemm_path_counts(ctypes.byref(tc), ctypes.byref(simt)))
    return tc.value, simt.value


def check_device_errors(device: int = 0, stream=None) -> None:
    detail = ctypes.c_int64(0)
    check(lib().mtc_check_device_errors(device, _stream(stream), ctypes.byref(detail)), "device error word")
