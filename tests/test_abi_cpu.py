"""CPU-side checks of the C ABI library: it loads, exports every entry point that
include/mtcuda.h declares, and rejects malformed descriptors on the host before
any device work (no GPU needed)."""
import ctypes
import re
from pathlib import Path

import pytest

from minitensor_cpp_b200 import abi

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "mtcuda.h").read_text()
    return sorted(set(re.findall(r"^[a-z][^;(]*?\b(mtc_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert len(syms) >= 30
    assert set(abi.EXPORTED) <= set(syms) | {"mtc_last_error", "mtc_version"}


def test_library_exports_every_declared_symbol():
    lib = abi.lib()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_version_and_device_count_without_gpu():
    lib = abi.lib()
    assert b"sm_100a" in lib.mtc_version()
    n = ctypes.c_int(-1)
    assert lib.mtc_device_count(ctypes.byref(n)) == abi.OK
    assert n.value >= 0


def _desc(shape, strides, offset, capacity, dtype=abi.FLOAT32, ptr=0x10000):
    return abi.make_desc(ptr, capacity, dtype, shape, strides, offset)


def test_out_of_bounds_view_is_rejected_on_host():
    lib = abi.lib()
    x = _desc([4, 4], [4, 1], 0, 10)  # reaches element 15 of a 10-element buffer
    out = _desc([4, 4], [4, 1], 0, 16)
    rc = lib.mtc_unary(abi.EXP, ctypes.byref(x), ctypes.byref(out), None)
    assert rc == abi.ERR_OUT_OF_RANGE
    assert b"outside buffer" in lib.mtc_last_error()
    neg = _desc([3], [-1], 1, 10)  # reaches element -1
    assert lib.mtc_unary(abi.EXP, ctypes.byref(neg), ctypes.byref(_desc([3], [1], 0, 3)), None) == abi.ERR_OUT_OF_RANGE


def test_shape_errors_map_to_invalid_argument():
    lib = abi.lib()
    a = _desc([2, 3], [3, 1], 0, 6)
    b = _desc([2, 2], [2, 1], 0, 4)
    out = _desc([2, 3], [3, 1], 0, 6)
    assert lib.mtc_binary(abi.ADD, ctypes.byref(a), ctypes.byref(b), ctypes.byref(out), None) == abi.ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        abi.check(abi.ERR_INVALID_ARGUMENT)
    bad_k = _desc([3, 5], [5, 1], 0, 15)
    assert lib.mtc_matmul(ctypes.byref(a), ctypes.byref(bad_k), ctypes.byref(out), 0, None) == abi.ERR_INVALID_ARGUMENT
    idx_f32 = _desc([2, 3], [3, 1], 0, 6)
    assert lib.mtc_gather(ctypes.byref(a), ctypes.byref(idx_f32), 1, ctypes.byref(out), None) == abi.ERR_INVALID_ARGUMENT
    axes = (ctypes.c_int64 * 2)(1, 1)
    red = _desc([2], [1], 0, 2)
    assert lib.mtc_reduce(abi.SUM, ctypes.byref(a), axes, 2, ctypes.byref(red), None) == abi.ERR_INVALID_ARGUMENT


def test_int64_is_rejected_by_float_kernels():
    lib = abi.lib()
    a = _desc([4], [1], 0, 4, abi.INT64)
    out = _desc([4], [1], 0, 4, abi.INT64)
    assert lib.mtc_unary(abi.EXP, ctypes.byref(a), ctypes.byref(out), None) == abi.ERR_LOGIC
