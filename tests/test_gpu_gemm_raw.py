"""The tensor core reads a TF32 operand from the upper 19 bits of each fp32 word.

The 3xTF32 GEMM relies on this when it reads a K-contiguous operand raw: the raw
tile serves as hi and the kernel computes lo = x - trunc(x) in shared memory.
The split pack instead stores hi = x with the low 13 mantissa bits cleared. If
the hardware truncates, both routes feed the tensor core the same bits, so the
products must be bit-identical.
"""
import numpy as np
import pytest

from minitensor_cpp_b200 import abi

pytestmark = pytest.mark.gpu


def _gemm(monkeypatch, direct, a, bt):
    import torch

    monkeypatch.setenv("MTC_TC_PIPELINE", "16x4")
    monkeypatch.setenv("MTC_TC_DIRECT", direct)
    A = torch.from_numpy(a).cuda()
    B = torch.from_numpy(bt).cuda().t()  # K-contiguous B view
    C = torch.empty(a.shape[0], bt.shape[0], device="cuda")
    abi.matmul(abi.View.of(A), abi.View.of(B), abi.View.of(C), abi.GEMM_3XTF32)
    torch.cuda.synchronize()
    return C.cpu().numpy()


def test_raw_and_split_operands_give_identical_bits(cuda, monkeypatch):
    rng = np.random.default_rng(12)
    # values with all mantissa bits in use, including subnormal-adjacent magnitudes
    a = (rng.standard_normal((384, 200)) * np.exp2(rng.integers(-20, 20, (384, 200)))).astype(np.float32)
    bt = (rng.standard_normal((320, 200)) * np.exp2(rng.integers(-20, 20, (320, 200)))).astype(np.float32)
    split = _gemm(monkeypatch, "0", a, bt)
    for direct in ("a", "b", "ab"):
        raw = _gemm(monkeypatch, direct, a, bt)
        assert np.array_equal(raw.view(np.uint32), split.view(np.uint32)), f"raw operands {direct!r} differ"
