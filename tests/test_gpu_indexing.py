"""Row gather and the segment-sum scatter-add against the oracle, bit for bit.

Rank-2 operands along axis 0 with the Int64 index broadcast along the row (the
shape MiniTensor's gather takes for a row lookup, copy/loops.hpp:155-303) run
the row kernels: the gather with several rows in flight per half-warp, the
scatter-add as a segment sum that writes every target row once and adds each
row's updates from +0 in ascending update order.  That is the reference's own
order (zero-filled target, then += in the iteration order of the updates), so
the sums equal the oracle's (np.add.at, unbuffered and ordered) bit for bit for
any float values, not only for exactly representable sums.
"""
import numpy as np
import pytest

from helpers import assert_bits
from minitensor_cpp_b200 import abi
from oracle import mt_oracle as mo

pytestmark = pytest.mark.gpu

F = np.float32


def _view(storage, shape, strides, offset=0):
    import torch

    return abi.View(torch.from_numpy(np.ascontiguousarray(storage)).cuda(), tuple(shape), tuple(strides), offset)


def _scatter(upd, idx_col, targets, width, upd_rs=None, upd_off=0, out_rs=None, out_off=0, idx_step=1):
    """Runs mtc_gather_scatter_add on [n, width] updates stored with row stride
    upd_rs at upd_off, the index column (broadcast along the row) read every
    idx_step entries, into a [targets, width] view with row stride out_rs at
    out_off; returns (target rows as seen through the view, untouched padding)."""
    import torch

    n = len(idx_col) // idx_step
    upd_rs = upd_rs or width
    out_rs = out_rs or width
    ust = np.full(upd_off + n * upd_rs, np.nan, F)
    for i in range(n):
        ust[upd_off + i * upd_rs: upd_off + i * upd_rs + width] = upd[i]
    U = _view(ust, (n, width), (upd_rs, 1), upd_off)
    I = _view(idx_col.astype(np.int64), (n, width), (idx_step, 0), 0)
    ost = torch.full((out_off + targets * out_rs,), -5.0, device="cuda")
    O = abi.View(ost, (targets, width), (out_rs, 1), out_off)
    abi.gather_scatter_add(U, I, 0, O)
    abi.check_device_errors(0)
    flat = ost.cpu().numpy()
    rows = np.stack([flat[out_off + t * out_rs: out_off + t * out_rs + width] for t in range(targets)]) \
        if targets else np.zeros((0, width), F)
    pad = np.concatenate([flat[:out_off]] + [flat[out_off + t * out_rs + width: out_off + (t + 1) * out_rs]
                                             for t in range(targets)])
    return rows, pad


def _want(upd, idx, targets, width):
    return mo.gather_scatter_add(upd, np.broadcast_to(idx[:, None], upd.shape), 0, (targets, width))


@pytest.mark.parametrize("n, targets", [(5000, 300), (40000, 2500), (7, 100), (20000, 20000), (50000, 20000)])
def test_segment_scatter_add_is_ordered_bit_exact(cuda, n, targets):
    """Non-integer N(0,1) updates with many duplicates: only the reference's
    summation order reproduces the oracle's bits.  Dense cases put more than 16
    updates in every group of 8 target rows (segments sorted beforehand); about
    one update per row (20000 / 20000) orders nearly every group in registers."""
    rng = np.random.default_rng(n)
    width = 64
    upd = rng.standard_normal((n, width)).astype(F)
    idx = rng.integers(0, targets, n)
    got, _ = _scatter(upd, idx, targets, width)
    assert_bits(got, _want(upd, idx, targets, width), f"segment scatter-add n={n} targets={targets}")


def test_long_segments_are_sorted(cuda):
    """Segments of 33 to 4096 updates are ordered by a shared-memory sort."""
    rng = np.random.default_rng(7)
    width = 8
    idx = np.concatenate([np.full(c, t) for t, c in enumerate((33, 100, 1000, 4096, 1))])
    rng.shuffle(idx)
    upd = rng.standard_normal((len(idx), width)).astype(F)
    got, _ = _scatter(upd, idx, 6, width)
    assert_bits(got, _want(upd, idx, 6, width), "long segments")


def test_segment_longer_than_the_sort_keeps_exact_integer_sums(cuda):
    """A segment above 4096 updates is summed in fill order: still exact for
    integer-valued updates (every partial sum representable)."""
    rng = np.random.default_rng(8)
    width = 4
    idx = np.zeros(6000, dtype=np.int64)
    idx[::7] = 1
    upd = np.floor(rng.uniform(-8, 8, (len(idx), width))).astype(F)
    got, _ = _scatter(upd, idx, 3, width)
    assert_bits(got, _want(upd, idx, 3, width), "segment above the sort limit")


def test_strided_offset_views_and_padding(cuda):
    """Padded update and target rows, element offsets and an index column read
    every other entry: the padding stays untouched."""
    rng = np.random.default_rng(9)
    width, n, targets = 16, 3000, 200
    upd = rng.standard_normal((n, width)).astype(F)
    idx_full = rng.integers(0, targets, 2 * n)
    got, pad = _scatter(upd, idx_full, targets, width, upd_rs=24, upd_off=8, out_rs=20, out_off=4, idx_step=2)
    assert_bits(got, _want(upd, idx_full[::2], targets, width), "strided views")
    assert (pad == -5.0).all(), "wrote outside the target view"


@pytest.mark.parametrize("width", [8, 64])
def test_bucketed_prelude_for_large_targets(cuda, width):
    """From 2^22 target rows the segments are built by a two-level counting sort
    with shared-memory counters (buckets of 2^13 rows, chunks of 2^14 updates):
    a partial last bucket, duplicates, a 3000-update segment (the long sort), a
    bucket holding more updates than its shared-memory stage (placed and sorted
    in global memory), non-integer values, and the same bits as the oracle."""
    rng = np.random.default_rng(31)
    targets = (1 << 22) + 12345
    n = 3_000_000 if width == 8 else 600_000
    idx = rng.integers(0, targets, n)
    picked = rng.choice(n, 23000, replace=False)
    idx[picked[:3000]] = targets - 1  # long segment in the last bucket
    idx[picked[3000:]] = 7 * 8192 + rng.integers(0, 100, 20000)  # 20000 updates in bucket 7
    upd = rng.standard_normal((n, width)).astype(F)
    got, _ = _scatter_fast(upd, idx, targets, width)
    want = np.zeros((targets, width), F)
    np.add.at(want, idx, upd)
    assert_bits(got, want, f"bucketed scatter-add width {width}")


def test_bucketed_prelude_reports_out_of_range(cuda):
    rng = np.random.default_rng(32)
    targets = 1 << 22
    idx = rng.integers(0, targets, 50_000)
    idx[777] = targets
    upd = rng.standard_normal((len(idx), 4)).astype(F)
    with pytest.raises(IndexError):
        _scatter_fast(upd, idx, targets, 4)
    idx[777] = 5
    got, _ = _scatter_fast(upd, idx, targets, 4)
    want = np.zeros((targets, 4), F)
    np.add.at(want, idx, upd)
    assert_bits(got, want, "bucketed scatter-add after an index error")


def _scatter_fast(upd, idx, targets, width):
    """_scatter for large contiguous cases (no padding, no per-row host loop)."""
    import torch

    U = abi.View(torch.from_numpy(np.ascontiguousarray(upd)).cuda(), (len(idx), width), (width, 1), 0)
    I = abi.View(torch.from_numpy(idx.astype(np.int64)).cuda(), (len(idx), width), (1, 0), 0)
    O = abi.View(torch.full((targets * width,), -5.0, device="cuda"), (targets, width), (width, 1), 0)
    abi.gather_scatter_add(U, I, 0, O)
    abi.check_device_errors(0)
    return O.storage.cpu().numpy().reshape(targets, width), None


def test_out_of_range_index_is_reported(cuda):
    rng = np.random.default_rng(10)
    upd = rng.standard_normal((64, 8)).astype(F)
    idx = rng.integers(0, 50, 64)
    idx[17] = 50
    with pytest.raises(IndexError):
        _scatter(upd, idx, 50, 8)
    # the next call on the device is unaffected
    idx[17] = 3
    got, _ = _scatter(upd, idx, 50, 8)
    assert_bits(got, _want(upd, idx, 50, 8), "after an index error")


@pytest.mark.parametrize("idx_step, off", [(1, 0), (3, 4)])
def test_row_gather_views_and_errors(cuda, idx_step, off):
    import torch

    rng = np.random.default_rng(11 + idx_step)
    rows, width, n = 1000, 32, 4097
    table = rng.standard_normal(off + rows * (width + 4)).astype(F)
    T = _view(table, (rows, width), (width + 4, 1), off)
    tv = mo.view(table, (rows, width), (width + 4, 1), off)
    idx = rng.integers(0, rows, n * idx_step)
    I = _view(idx.astype(np.int64), (n, width), (idx_step, 0), 0)
    O = abi.View(torch.full((n * width,), -1.0, device="cuda"), (n, width), (width, 1), 0)
    abi.gather(T, I, 0, O)
    abi.check_device_errors(0)
    assert_bits(O.storage.cpu().numpy().reshape(n, width), tv[idx[::idx_step]], "row gather")
    idx[5 * idx_step] = -1
    I = _view(idx.astype(np.int64), (n, width), (idx_step, 0), 0)
    abi.gather(T, I, 0, O)
    with pytest.raises(IndexError):
        abi.check_device_errors(0)


def _into(upd, idx_view, axis, base):
    import ctypes
    import torch

    U = _view(upd.reshape(-1), upd.shape, abi.contiguous_strides(list(upd.shape)))
    O = _view(base.reshape(-1).copy(), base.shape, abi.contiguous_strides(list(base.shape)))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    abi.check(abi.lib().mtc_gather_scatter_add_into(ctypes.byref(U.desc()), ctypes.byref(idx_view.desc()), axis,
                                                    ctypes.byref(O.desc()), stream), "scatter-add into")
    abi.check_device_errors(0)
    return O.storage.cpu().numpy().reshape(base.shape)


def test_scatter_add_into_existing_values(cuda):
    """mtc_gather_scatter_add_into adds to the target's values instead of
    clearing it: rows (a row index broadcast along the row, 128-bit reductions)
    and one index per row along axis 1 (the cross-entropy gradient's shape)."""
    rng = np.random.default_rng(12)
    base = rng.standard_normal((300, 64)).astype(F)
    upd = rng.standard_normal((200, 64)).astype(F)
    idx = rng.choice(300, 200, replace=False)  # distinct rows: one update per element
    got = _into(upd, _view(idx.astype(np.int64), (200, 64), (1, 0)), 0, base)
    want = base.copy()
    want[idx] = (want[idx] + upd).astype(F)
    assert_bits(got, want, "row scatter-add into")
    logits_grad = rng.standard_normal((128, 1000)).astype(F)
    g = rng.standard_normal((128, 1)).astype(F)
    t = rng.integers(0, 1000, 128)
    got = _into(g, _view(t.astype(np.int64), (128, 1), (1, 1)), 1, logits_grad)
    want = logits_grad.copy()
    want[np.arange(128), t] = (want[np.arange(128), t] + g[:, 0]).astype(F)
    assert_bits(got, want, "axis-1 scatter-add into")
