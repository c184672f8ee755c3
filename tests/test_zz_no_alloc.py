"""The allocation-free tensor-core GEMM (mtc_matmul_3xtf32_static).

Some callers cannot allocate device memory themselves: code whose device
memory belongs to another framework's allocator, or a latency-critical path
that must never wait on an allocation.  For them the 3xTF32 GEMM has a variant
whose split operands live in a fixed 32 MiB static device array.  This file
checks, through the C ABI, that two calls in a row give the results of the
regular entry point (mtc_matmul with MTC_GEMM_3XTF32) within the GEMM parity
bound, that the calls take nothing from the backend's memory pool, and that a
problem too large for the array is rejected.  It is collected
last so a stop-at-first-failure run has already run every other test.
"""
import ctypes

import numpy as np
import pytest

from helpers import assert_rel_sqrtk
from minitensor_cpp_b200 import abi
from oracle import mt_oracle as mo

pytestmark = pytest.mark.gpu

F = np.float32


def _desc(t, shape=None, strides=None):
    v = abi.View.of(t)
    if shape is not None:
        v = abi.View(v.storage, tuple(shape), tuple(strides), v.offset)
    return v.desc()


def _pool():
    """(reserved, used) bytes of the backend's caching allocator on device 0."""
    reserved, used = ctypes.c_uint64(0), ctypes.c_uint64(0)
    abi.check(abi.lib().mtc_pool_stats(0, ctypes.byref(reserved), ctypes.byref(used)), "pool stats")
    return reserved.value, used.value


def _both(a, b, a_view=None, b_view=None):
    """C from the static-workspace entry point and from the regular one; the
    static call must leave the pool's reserved and used bytes unchanged (it is
    made before the regular call, whose workspace comes from the pool)."""
    import torch

    A = torch.from_numpy(a).cuda()
    B = torch.from_numpy(b).cuda()
    da = _desc(A) if a_view is None else _desc(A, *a_view)
    db = _desc(B) if b_view is None else _desc(B, *b_view)
    m = a_view[0][0] if a_view else a.shape[0]
    n = b_view[0][1] if b_view else b.shape[1]
    c_static = torch.full((m, n), -1.0, device="cuda")
    c_regular = torch.full((m, n), -2.0, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lib = abi.lib()
    torch.cuda.synchronize()
    before = _pool()
    abi.check(lib.mtc_matmul_3xtf32_static(ctypes.byref(da), ctypes.byref(db), ctypes.byref(_desc(c_static)), stream),
              "static-workspace matmul")
    torch.cuda.synchronize()
    assert _pool() == before, f"the static-workspace call changed the pool: {before} -> {_pool()}"
    abi.check(lib.mtc_matmul(ctypes.byref(da), ctypes.byref(db), ctypes.byref(_desc(c_regular)), abi.GEMM_3XTF32,
                             stream), "regular matmul")
    torch.cuda.synchronize()
    abi.check_device_errors(0)
    return c_static.cpu().numpy(), c_regular.cpu().numpy()


def test_two_calls_match_the_regular_entry_point(cuda):
    rng = np.random.default_rng(91)
    # first call: contiguous operands
    a = rng.standard_normal((384, 200)).astype(F)
    b = rng.standard_normal((200, 520)).astype(F)
    got, want = _both(a, b)
    assert_rel_sqrtk(got.reshape(-1), want.reshape(-1), 200, mo.matmul(np.abs(a), np.abs(b)).reshape(-1),
                     "static vs regular, call 1")
    # second call, different shape and a transposed right operand: the shared
    # array still holds the first call's operands and must not leak into this one
    a2 = rng.standard_normal((256, 96)).astype(F)
    w2 = rng.standard_normal((300, 96)).astype(F)  # B = w2^T, a [96, 300] view with strides (1, 96)
    got2, want2 = _both(a2, w2, b_view=((96, 300), (1, 96)))
    assert_rel_sqrtk(got2.reshape(-1), want2.reshape(-1), 96, mo.matmul(np.abs(a2), np.abs(w2.T)).reshape(-1),
                     "static vs regular, call 2")
    assert_rel_sqrtk(got2.reshape(-1), mo.matmul(a2, w2.T).reshape(-1), 96,
                     mo.matmul(np.abs(a2), np.abs(w2.T)).reshape(-1), "static vs oracle, call 2")


def test_problem_beyond_the_static_workspace_is_rejected(cuda):
    import torch

    # 2 * (M + N) * K = 2 * 4096 * 2048 floats = 64 MiB > 32 MiB
    A = torch.zeros(2048, 2048, device="cuda")
    B = torch.zeros(2048, 2048, device="cuda")
    C = torch.zeros(2048, 2048, device="cuda")
    rc = abi.lib().mtc_matmul_3xtf32_static(ctypes.byref(_desc(A)), ctypes.byref(_desc(B)), ctypes.byref(_desc(C)),
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == abi.ERR_INVALID_ARGUMENT
    assert b"static workspace" in abi.lib().mtc_last_error()
