"""The backend's stream-ordered caching allocator (mtc_alloc / mtc_free).

Blocks freed on their own stream are reused by the next request on that stream;
a block freed on another stream is reused only after that stream has passed
the free; requests are rounded (512 B up to 1 MiB, 2 MiB above); trimming
returns every unused block to the driver.  Data written through a reused block
is checked with the fill kernel and a device-to-host copy.
"""
import ctypes

import numpy as np
import pytest

from minitensor_cpp_b200 import abi

pytestmark = pytest.mark.gpu


def _alloc(nbytes, stream):
    p = ctypes.c_void_p()
    abi.check(abi.lib().mtc_alloc(0, nbytes, stream, ctypes.byref(p)), "alloc")
    return p.value


def _free(ptr, stream):
    abi.check(abi.lib().mtc_free(0, ptr, stream), "free")


def _stats():
    r, u = ctypes.c_uint64(), ctypes.c_uint64()
    abi.check(abi.lib().mtc_pool_stats(0, ctypes.byref(r), ctypes.byref(u)), "pool stats")
    return r.value, u.value


def _stream():
    s = ctypes.c_void_p()
    abi.check(abi.lib().mtc_device_stream(0, ctypes.byref(s)), "stream")
    return s.value


def _fill_and_read(ptr, n, value, stream):
    d = abi.make_desc(ptr, n, abi.FLOAT32, [n], [1], 0)
    v = ctypes.c_float(value)
    abi.check(abi.lib().mtc_fill(ctypes.byref(d), ctypes.byref(v), stream), "fill")
    out = np.empty(n, np.float32)
    abi.check(abi.lib().mtc_copy_to_host(0, out.ctypes.data, ptr, n * 4, stream), "copy")
    return out


def test_same_stream_reuse_rounding_and_trim(cuda):
    s = _stream()
    abi.check(abi.lib().mtc_pool_trim(0), "trim")
    r0, u0 = _stats()
    a = _alloc(3 << 20, s)  # 3 MiB -> one 4 MiB block
    r1, u1 = _stats()
    assert r1 - r0 == 4 << 20 and u1 - u0 == 4 << 20
    assert _fill_and_read(a, (3 << 20) // 4, 1.5, s).min() == 1.5
    _free(a, s)
    assert _stats() == (r1, u0)
    b = _alloc(3 << 20, s)  # same stream: the cached block comes back, nothing new reserved
    assert b == a and _stats() == (r1, u1)
    assert (_fill_and_read(b, 1000, -2.0, s) == -2.0).all()
    _free(b, s)
    small = _alloc(1000, s)  # 1000 B -> a 1024-byte block
    assert _stats()[1] - u0 == 1024
    _free(small, s)
    abi.check(abi.lib().mtc_pool_trim(0), "trim")
    assert _stats() == (r0, u0)


def test_cross_stream_free_waits_for_the_freeing_stream(cuda):
    import torch

    s = _stream()
    other = torch.cuda.Stream()
    abi.check(abi.lib().mtc_pool_trim(0), "trim")  # no cached block of the stream competes
    a = _alloc(8 << 20, s)
    _free(a, other.cuda_stream)
    other.synchronize()
    b = _alloc(8 << 20, s)  # the free has completed: the block is reusable by any stream
    assert b == a
    _free(b, s)


def test_large_blocks_are_not_handed_out_for_small_requests(cuda):
    s = _stream()
    abi.check(abi.lib().mtc_pool_trim(0), "trim")
    big = _alloc(64 << 20, s)
    _free(big, s)
    small = _alloc(4 << 20, s)  # a 64 MiB block is more than 1/8 too large for 4 MiB
    assert small != big
    _free(small, s)
    again = _alloc(64 << 20, s)
    assert again == big
    _free(again, s)


def test_freeing_an_unknown_pointer_is_an_error(cuda):
    s = _stream()
    a = _alloc(4096, s)
    with pytest.raises(ValueError):
        _free(a + 512, s)
    _free(a, s)
