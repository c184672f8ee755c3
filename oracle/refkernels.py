"""Oracle (test infrastructure only): ctypes binding of oracle/_ref/libmtref.so.

libmtref.so is the unmodified MiniTensor reference compiled from its own
sources by oracle/Makefile, plus C shims (ref_kernels.cpp, ref_workloads.cpp)
that invoke the reference's registered CPU kernels on host buffers and run the
benchmark workloads through the reference's public API.  Operands are
`HostView`s: a flat numpy storage array plus shape/strides/offset in elements.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path
from typing import Sequence

import numpy as np

from minitensor_cpp_b200.abi import Desc, FLOAT32, INT64, make_desc, contiguous_strides

LIB_PATH = Path(__file__).resolve().parent / "_ref" / "libmtref.so"


@dataclass
class HostView:
    storage: np.ndarray  # 1-D float32 or int64
    shape: tuple
    strides: tuple
    offset: int = 0

    @staticmethod
    def contiguous(storage: np.ndarray, shape, offset: int = 0) -> "HostView":
        return HostView(storage, tuple(shape), tuple(contiguous_strides(shape)), offset)

    @staticmethod
    def of(arr: np.ndarray) -> "HostView":
        flat = np.ascontiguousarray(arr).reshape(-1).copy()
        return HostView.contiguous(flat, arr.shape)

    def desc(self) -> Desc:
        dt = INT64 if self.storage.dtype == np.int64 else FLOAT32
        return make_desc(self.storage.ctypes.data, self.storage.size, dt, self.shape, self.strides, self.offset)

    def array(self) -> np.ndarray:
        """The logical values of the view (a copy)."""
        out = np.empty(self.shape, dtype=self.storage.dtype)
        it = np.ndindex(*self.shape) if len(self.shape) else [()]
        if int(np.prod(self.shape)) == 0:
            return out
        idx = np.indices(self.shape).reshape(len(self.shape), -1) if len(self.shape) else np.zeros((0, 1), dtype=np.int64)
        offs = self.offset + sum(idx[d] * self.strides[d] for d in range(len(self.shape)))
        return self.storage[np.asarray(offs, dtype=np.int64)].reshape(self.shape)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"oracle library missing: {LIB_PATH} (run `make -C oracle`)")
        _lib = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.POINTER
        i32, i64, f, u64 = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64
        sig = {
            "mtref_last_error": ([], ctypes.c_char_p),
            "mtref_unary": ([i32, P(Desc), P(Desc)], ctypes.c_int),
            "mtref_binary": ([i32, P(Desc), P(Desc), P(Desc)], ctypes.c_int),
            "mtref_reduce": ([i32, P(Desc), P(i64), i32, i32, P(Desc)], ctypes.c_int),
            "mtref_matmul": ([P(Desc), P(Desc), P(Desc)], ctypes.c_int),
            "mtref_copy": ([P(Desc), P(Desc)], ctypes.c_int),
            "mtref_concat": ([P(Desc), i32, i64, P(Desc)], ctypes.c_int),
            "mtref_gather": ([P(Desc), P(Desc), i64, P(Desc)], ctypes.c_int),
            "mtref_gather_scatter_add": ([P(Desc), P(Desc), i64, P(Desc)], ctypes.c_int),
            "mtref_fill": ([P(Desc), ctypes.c_void_p], ctypes.c_int),
            "mtref_uniform": ([P(Desc), f, f, u64, u64], ctypes.c_int),
            "mtref_normal": ([P(Desc), f, f, u64, u64], ctypes.c_int),
            "mtref_index_scatter": ([P(Desc), P(Desc), i32, i64, i32, i64, i32, i64, i64], ctypes.c_int),
            "mtref_index_layout": ([P(Desc), i32, i64, i32, i64, i32, i64, i64, P(Desc)], ctypes.c_int),
            "mtref_key_fold_in": ([u64, u64, u64, P(u64)], None),
            "mtref_key_split": ([u64, u64, P(u64)], None),
        }
        for name, (args, res) in sig.items():
            fn = getattr(_lib, name)
            fn.argtypes = args
            fn.restype = res
    return _lib


def available() -> bool:
    return LIB_PATH.exists()


class RefError(Exception):
    pass


def _check(rc: int, what: str) -> None:
    if rc == 0:
        return
    msg = lib().mtref_last_error().decode(errors="replace")
    exc = {1: ValueError, 2: IndexError, 5: OverflowError}.get(rc, RefError)
    raise exc(f"reference {what}: {msg}")


def unary(op, x: HostView, out: HostView):
    _check(lib().mtref_unary(op, ctypes.byref(x.desc()), ctypes.byref(out.desc())), "unary")


def binary(op, a: HostView, b: HostView, out: HostView):
    _check(lib().mtref_binary(op, ctypes.byref(a.desc()), ctypes.byref(b.desc()), ctypes.byref(out.desc())), "binary")


def reduce(op, x: HostView, axes: Sequence[int], keep_dim: bool, out: HostView):
    ax = (ctypes.c_int64 * max(len(axes), 1))(*axes)
    _check(lib().mtref_reduce(op, ctypes.byref(x.desc()), ax, len(axes), int(keep_dim), ctypes.byref(out.desc())),
           "reduce")


def matmul(a: HostView, b: HostView, out: HostView):
    _check(lib().mtref_matmul(ctypes.byref(a.desc()), ctypes.byref(b.desc()), ctypes.byref(out.desc())), "matmul")


def copy(src: HostView, dst: HostView):
    _check(lib().mtref_copy(ctypes.byref(src.desc()), ctypes.byref(dst.desc())), "copy")


def concat(inputs: Sequence[HostView], axis: int, out: HostView):
    arr = (Desc * len(inputs))(*[v.desc() for v in inputs])
    _check(lib().mtref_concat(arr, len(inputs), axis, ctypes.byref(out.desc())), "concat")


def gather(src: HostView, idx: HostView, axis: int, out: HostView):
    _check(lib().mtref_gather(ctypes.byref(src.desc()), ctypes.byref(idx.desc()), axis, ctypes.byref(out.desc())),
           "gather")


def gather_scatter_add(upd: HostView, idx: HostView, axis: int, out: HostView):
    _check(lib().mtref_gather_scatter_add(ctypes.byref(upd.desc()), ctypes.byref(idx.desc()), axis,
                                          ctypes.byref(out.desc())), "gather_scatter_add")


def fill(out: HostView, value):
    v = ctypes.c_int64(int(value)) if out.storage.dtype == np.int64 else ctypes.c_float(float(value))
    _check(lib().mtref_fill(ctypes.byref(out.desc()), ctypes.byref(v)), "fill")


def uniform(out: HostView, low, high, key):
    _check(lib().mtref_uniform(ctypes.byref(out.desc()), low, high, key[0], key[1]), "uniform")


def normal(out: HostView, mean, std, key):
    _check(lib().mtref_normal(ctypes.byref(out.desc()), mean, std, key[0], key[1]), "normal")


def _index_args(select, axis, start, stop, step_or_index):
    return (int(select), axis, int(start is not None), start or 0, int(stop is not None), stop or 0, step_or_index)


def index_scatter(x: HostView, out: HostView, *, select: bool, axis: int, start=None, stop=None, step_or_index=1):
    _check(lib().mtref_index_scatter(ctypes.byref(x.desc()), ctypes.byref(out.desc()),
                                     *_index_args(select, axis, start, stop, step_or_index)), "index_scatter")


def index_layout(out: HostView, *, select: bool, axis: int, start=None, stop=None, step_or_index=1):
    """(shape, strides, offset) of the slice/select view of `out`'s layout."""
    d = Desc()
    _check(lib().mtref_index_layout(ctypes.byref(out.desc()), *_index_args(select, axis, start, stop, step_or_index),
                                    ctypes.byref(d)), "index_layout")
    return tuple(d.shape[:d.rank]), tuple(d.strides[:d.rank]), d.offset


def key_fold_in(key, data):
    out = (ctypes.c_uint64 * 2)()
    lib().mtref_key_fold_in(key[0], key[1], data, out)
    return (out[0], out[1])


def key_split(key):
    out = (ctypes.c_uint64 * 4)()
    lib().mtref_key_split(key[0], key[1], out)
    return (out[0], out[1]), (out[2], out[3])
