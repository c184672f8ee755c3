"""Replay of repeated evaluation plans as CUDA graphs.

The evaluator records a plan it has seen before with stream capture and
replays later evaluations of the same plan (same structure, same leaf buffers)
as one graph launch, after taking the recorded output blocks back from the
allocator.  A replay runs the very kernels an eager evaluation would, in the
same order, on the same buffers, so results must be bit-identical; the
constants that change every step (Adam's bias corrections) are patched into
the recorded fused kernels.
"""
import ctypes

import numpy as np
import pytest

from minitensor_cpp_b200 import abi

pytestmark = pytest.mark.gpu


@pytest.fixture
def fe(cuda):
    from minitensor_cpp_b200.frontend import Frontend

    f = Frontend()
    previous = f.set_graphs(True)
    f.clear_graphs()
    yield f
    f.clear_graphs()
    f.set_graphs(previous)


@pytest.mark.parametrize("loss_every", [1, 7, 0])
def test_spiral_training_replays_bit_identically(fe, loss_every):
    steps = 40
    fe.set_graphs(False)
    eager, _ = fe.spiral_train(0, steps, loss_every=loss_every if loss_every else steps - 1)
    fe.set_graphs(True)
    fe.reset_stats()
    replayed, _ = fe.spiral_train(0, steps, loss_every=loss_every if loss_every else steps - 1)
    st = fe.stats()
    np.testing.assert_array_equal(replayed.view(np.uint32), eager.view(np.uint32))
    assert st["graph_captures"] >= 1
    if loss_every == 7:
        # three plan structures recur only every 7th step: fewer steps replay
        assert st["graph_replays"] >= st["evaluations"] // 2, st
    else:
        # each structure runs eagerly once, is recorded twice (the two recordings
        # alternate their parameter blocks), and replays from then on
        assert st["graph_replays"] >= st["evaluations"] - 10, st
    assert st["graph_fallbacks"] == 0, st


def test_replays_count_their_launches(fe):
    fe.spiral_train(0, 10, loss_every=0)
    n0 = abi.launch_count()
    fe.reset_stats()
    fe.spiral_train(0, 30, loss_every=0)
    st = fe.stats()
    launches = abi.launch_count() - n0
    assert st["graph_replays"] >= 20
    # the same kernels as eager evaluation: data set-up plus about 30 per step
    # (each parameter's Adam update is one fused kernel)
    assert 30 * 24 <= launches <= 30 * 40 + 200, launches


def test_index_error_inside_a_replayed_plan_is_reported(fe):
    rng = np.random.default_rng(5)
    table = rng.standard_normal((64, 8)).astype(np.float32)
    good = rng.integers(0, 64, 32).astype(np.int64)
    fe.reset_stats()
    for _ in range(6):
        np.testing.assert_array_equal(fe.gather_rows(0, table, good), table[good])
    bad = good.copy()
    bad[17] = 64
    with pytest.raises(IndexError):
        fe.gather_rows(0, table, bad)
    np.testing.assert_array_equal(fe.gather_rows(0, table, good), table[good])
    st = fe.stats()
    assert st["graph_captures"] + st["graph_replays"] >= 1, st


def _stream():
    s = ctypes.c_void_p()
    abi.check(abi.lib().mtc_device_stream(0, ctypes.byref(s)), "stream")
    return s.value


def _alloc(nbytes, stream):
    p = ctypes.c_void_p()
    abi.check(abi.lib().mtc_alloc(0, nbytes, stream, ctypes.byref(p)), "alloc")
    return p.value


def test_pool_take_returns_exactly_the_freed_block(cuda):
    import torch

    L = abi.lib()
    s = _stream()
    a = _alloc(1 << 20, s)
    # a live block cannot be taken
    assert L.mtc_pool_take(0, ctypes.c_void_p(a), 1 << 20, ctypes.c_void_p(s)) != 0
    abi.check(L.mtc_free(0, ctypes.c_void_p(a), ctypes.c_void_p(s)), "free")
    # too large a request for the block
    assert L.mtc_pool_take(0, ctypes.c_void_p(a), 4 << 20, ctypes.c_void_p(s)) != 0
    abi.check(L.mtc_pool_take(0, ctypes.c_void_p(a), 1 << 20, ctypes.c_void_p(s)), "take")
    # taken again: it is live now
    assert L.mtc_pool_take(0, ctypes.c_void_p(a), 1 << 20, ctypes.c_void_p(s)) != 0
    # a block released on another stream is not taken for this one until that stream passed the free
    other = torch.cuda.Stream()
    abi.check(L.mtc_free(0, ctypes.c_void_p(a), ctypes.c_void_p(other.cuda_stream)), "free")
    other.synchronize()
    abi.check(L.mtc_pool_take(0, ctypes.c_void_p(a), 1 << 20, ctypes.c_void_p(s)), "take after the free completed")
    abi.check(L.mtc_free(0, ctypes.c_void_p(a), ctypes.c_void_p(s)), "free")


def test_recorded_fused_kernel_takes_new_constants(cuda):
    """mtc_capture_* / mtc_graph_set_constants directly: y = x * c0 + c1."""
    import torch

    L = abi.lib()
    s = torch.cuda.Stream()
    x = torch.arange(4096, dtype=torch.float32, device="cuda") / 7.0
    y = torch.empty_like(x)
    program = [(abi.CONST, 1, 0, 0, 3.0), (abi.MULTIPLY, 2, 0, 1, 0.0), (abi.CONST, 3, 0, 0, -1.5), (abi.ADD, 4, 2, 3, 0.0)]
    with torch.cuda.stream(s):
        abi.fused(program, [abi.View.of(x)], [4], [abi.View.of(y)], stream=s.cuda_stream)  # compile outside the recording
        s.synchronize()
        y.zero_()
        s.synchronize()
        abi.check(L.mtc_capture_begin(0, ctypes.c_void_p(s.cuda_stream)), "capture")
        n = ctypes.c_int32()
        abi.check(L.mtc_capture_fused_count(ctypes.byref(n)), "count")
        assert n.value == 0
        abi.fused(program, [abi.View.of(x)], [4], [abi.View.of(y)], stream=s.cuda_stream)
        abi.check(L.mtc_capture_fused_count(ctypes.byref(n)), "count")
        assert n.value == 1
        g = ctypes.c_void_p()
        abi.check(L.mtc_capture_end(1, ctypes.byref(g)), "end")
    try:
        s.synchronize()
        assert not y.any()  # recording runs nothing
        abi.check(L.mtc_graph_launch(g), "launch")
        s.synchronize()
        want = x.cpu().numpy() * np.float32(3.0) + np.float32(-1.5)
        np.testing.assert_array_equal(y.cpu().numpy(), want)
        imm = (ctypes.c_float * 2)(0.5, 2.0)
        abi.check(L.mtc_graph_set_constants(g, 0, imm, 2), "constants")
        abi.check(L.mtc_graph_launch(g), "launch")
        s.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy(), x.cpu().numpy() * np.float32(0.5) + np.float32(2.0))
        with pytest.raises(ValueError):
            abi.check(L.mtc_graph_set_constants(g, 1, imm, 2), "constants")
        launches = ctypes.c_uint64()
        abi.check(L.mtc_graph_launches(g, ctypes.byref(launches)), "launches")
        assert launches.value == 1
    finally:
        L.mtc_graph_destroy(g)


def test_pool_take_many_is_all_or_none(cuda):
    L = abi.lib()
    s = _stream()
    blocks = [_alloc(1 << 16, s) for _ in range(3)]
    for p in blocks[:2]:
        abi.check(L.mtc_free(0, ctypes.c_void_p(p), ctypes.c_void_p(s)), "free")
    ptrs = (ctypes.c_void_p * 3)(*blocks)
    sizes = (ctypes.c_size_t * 3)(*(1 << 16 for _ in range(3)))
    failed = ctypes.c_int32(-1)
    # the third block is still live: nothing is taken
    assert L.mtc_pool_take_many(0, ptrs, sizes, 3, ctypes.c_void_p(s), ctypes.byref(failed)) != 0
    assert failed.value == 2
    abi.check(L.mtc_pool_take_many(0, ptrs, sizes, 2, ctypes.c_void_p(s), ctypes.byref(failed)), "take two")
    for p in blocks:
        abi.check(L.mtc_free(0, ctypes.c_void_p(p), ctypes.c_void_p(s)), "free")


def test_protected_blocks_wait_for_a_take_by_address(cuda):
    L = abi.lib()
    s = _stream()
    abi.check(L.mtc_pool_trim(0), "trim")
    a = _alloc(3 << 20, s)
    abi.check(L.mtc_pool_protect(0, ctypes.c_void_p(a), 1), "protect")
    abi.check(L.mtc_free(0, ctypes.c_void_p(a), ctypes.c_void_p(s)), "free")
    b = _alloc(3 << 20, s)  # same size, same stream: a protected block is not handed out
    assert b != a
    abi.check(L.mtc_pool_take(0, ctypes.c_void_p(a), 3 << 20, ctypes.c_void_p(s)), "take the protected block")
    abi.check(L.mtc_free(0, ctypes.c_void_p(a), ctypes.c_void_p(s)), "free")
    abi.check(L.mtc_pool_protect(0, ctypes.c_void_p(a), -1), "unprotect")
    abi.check(L.mtc_free(0, ctypes.c_void_p(b), ctypes.c_void_p(s)), "free")
    c = _alloc(3 << 20, s)  # unprotected again: an ordinary cached block
    assert c in (a, b)
    abi.check(L.mtc_free(0, ctypes.c_void_p(c), ctypes.c_void_p(s)), "free")
