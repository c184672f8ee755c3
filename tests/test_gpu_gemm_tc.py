"""Parity of the tcgen05 3xTF32 tensor-core GEMM (forced, no SIMT fallback)
against the float32 oracle: |C - C_ref| <= 1e-5 * sqrt(K) * (|A| |B|)_ij, the
normwise per-element form of the 1e-5*sqrt(K) relative bound.  Every case runs
with each kernel variant and shared-memory ring, under both work-unit schedules."""
import numpy as np
import pytest

from helpers import assert_rel_sqrtk
from minitensor_cpp_b200 import abi
from oracle import mt_oracle as mo

pytestmark = pytest.mark.gpu

F = np.float32


@pytest.fixture(autouse=True, params=["auto", "16x4", "16x4-0", "16x4-ab", "32x2", "pair16x6", "pair32x3"])
def pipeline(request, monkeypatch):
    """Every kernel and ring: the single-CTA kernel with 4 stages of BK=16 (64-byte
    swizzle) or 2 of BK=32 (128-byte swizzle), reading a K-contiguous A raw (lo
    computed in shared memory; the default), splitting every operand first
    ("-0"), or reading both K-contiguous operands raw ("-ab"); the CTA-pair
    kernel (split operands) with 6 stages of BK=16 or 3 of BK=32; and the
    default choice between them ("auto")."""
    name = request.param
    pipe, _, direct = name.partition("-")
    if pipe != "auto":
        monkeypatch.setenv("MTC_TC_PIPELINE", pipe)
    else:
        monkeypatch.delenv("MTC_TC_PIPELINE", raising=False)
    if direct:
        monkeypatch.setenv("MTC_TC_DIRECT", direct)
    else:
        monkeypatch.delenv("MTC_TC_DIRECT", raising=False)
    return name


@pytest.fixture(autouse=True, params=["static", "dynamic"])
def schedule(request, monkeypatch):
    """Work units round-robin (the default of a process without a communicator)
    or handed out at run time from a per-launch counter (the default once NCCL
    is in use): the same tiles, so the same results."""
    monkeypatch.setenv("MTC_TC_SCHEDULE", request.param)
    return request.param


def _run(a_st, a_shape, a_strides, b_st, b_shape, b_strides, out_offset=0, algo=abi.GEMM_3XTF32):
    import torch

    av = mo.view(a_st, a_shape, a_strides, 0)
    bv = mo.view(b_st, b_shape, b_strides, 0)
    exp = mo.matmul(av, bv)
    A = abi.View(torch.from_numpy(a_st).cuda(), tuple(a_shape), tuple(a_strides), 0)
    B = abi.View(torch.from_numpy(b_st).cuda(), tuple(b_shape), tuple(b_strides), 0)
    out_st = torch.full((exp.size + out_offset,), -3.0, device="cuda")
    C = abi.View(out_st, exp.shape, tuple(abi.contiguous_strides(list(exp.shape))), out_offset)
    abi.matmul(A, B, C, algo)
    torch.cuda.synchronize()
    abi.check_device_errors(0)
    got = out_st.cpu().numpy()
    assert (got[:out_offset] == -3.0).all(), "wrote before the output offset"
    scale = mo.matmul(np.abs(av), np.abs(bv))
    assert_rel_sqrtk(got[out_offset:], exp.reshape(-1), av.shape[-1], scale.reshape(-1),
                     f"3xTF32 {a_shape}x{b_shape}")
    return got[out_offset:].reshape(exp.shape), exp


def test_tile_aligned_contiguous(cuda):
    rng = np.random.default_rng(1)
    M, N, K = 256, 512, 64
    _run(rng.standard_normal(M * K).astype(F), [M, K], [K, 1], rng.standard_normal(K * N).astype(F), [K, N], [N, 1])


def test_ragged_edges_and_k_tail(cuda):
    rng = np.random.default_rng(2)
    for M, N, K in ((300, 520, 100), (129, 257, 35), (1000, 700, 513)):
        _run(rng.standard_normal(M * K).astype(F), [M, K], [K, 1], rng.standard_normal(K * N).astype(F), [K, N],
             [N, 1], out_offset=3)


def test_transposed_operands(cuda):
    rng = np.random.default_rng(3)
    M, N, K = 384, 320, 200
    a = rng.standard_normal(M * K).astype(F)
    b = rng.standard_normal(N * K).astype(F)
    _run(a, [M, K], [K, 1], b, [K, N], [1, K])   # x @ W^T (Linear forward)
    _run(a, [M, K], [1, M], b, [K, N], [N, 1])   # A^T @ B (weight gradient)
    _run(a, [M, K], [1, M], b, [K, N], [1, K])   # both transposed


def test_batched_with_broadcast(cuda):
    rng = np.random.default_rng(4)
    a = rng.standard_normal(3 * 2 * 130 * 70).astype(F)
    b = rng.standard_normal(2 * 70 * 260).astype(F)
    _run(a, [3, 2, 130, 70], [2 * 130 * 70, 130 * 70, 70, 1], b, [2, 70, 260], [70 * 260, 260, 1])


def test_batched_aligned_operands_take_the_vector_packs(cuda):
    """K, M and N multiples of 4 and 16-byte aligned views: the float4 split packs
    (K-contiguous rows, and the 64x64 swizzled transpose) with a K tail inside a
    64-wide tile, partial row tiles and a batch axis, for both operand layouts."""
    rng = np.random.default_rng(8)
    bt, M, N, K = 3, 132, 200, 100
    a = rng.standard_normal(bt * M * K).astype(F)
    b = rng.standard_normal(bt * K * N).astype(F)
    _run(a, [bt, M, K], [M * K, K, 1], b, [bt, K, N], [K * N, N, 1])         # rows pack for A, transpose for B
    _run(a, [bt, M, K], [M * K, 1, M], b, [bt, K, N], [K * N, 1, K])         # transpose for A, rows pack for B


def test_padded_row_pitch_and_offset_views(cuda):
    """K-contiguous operands whose rows are further apart than K (a column slice of
    a wider matrix) and start at an element offset: still 16-byte aligned, so
    they are read raw; an unaligned offset falls back to the split pack."""
    rng = np.random.default_rng(9)
    M, N, K, pad = 200, 260, 96, 12
    a = rng.standard_normal(M * (K + pad) + 8).astype(F)
    b = rng.standard_normal(N * (K + pad) + 8).astype(F)
    for off in (0, 4, 1):
        import torch

        av = mo.view(a, [M, K], [K + pad, 1], off)
        bv = mo.view(b, [K, N], [1, K + pad], off)
        exp = mo.matmul(av, bv)
        A = abi.View(torch.from_numpy(a).cuda(), (M, K), (K + pad, 1), off)
        B = abi.View(torch.from_numpy(b).cuda(), (K, N), (1, K + pad), off)
        C = abi.View(torch.empty(M * N, device="cuda"), (M, N), (N, 1), 0)
        abi.matmul(A, B, C, abi.GEMM_3XTF32)
        torch.cuda.synchronize()
        assert_rel_sqrtk(C.tensor().cpu().numpy().reshape(-1), exp.reshape(-1), K,
                         mo.matmul(np.abs(av), np.abs(bv)).reshape(-1), f"padded rows, offset {off}")


def test_split_k_when_tiles_do_not_fill_the_gpu(cuda):
    """Few output tiles and a long K: the single-CTA kernel splits K (partial tiles
    summed in split order), batched, with ragged edges and an output offset."""
    rng = np.random.default_rng(13)
    bt, M, N, K = 2, 200, 300, 1000
    a = rng.standard_normal(bt * M * K).astype(F)
    b = rng.standard_normal(bt * K * N).astype(F)
    _run(a, [bt, M, K], [M * K, K, 1], b, [bt, K, N], [K * N, N, 1], out_offset=5)  # element-wise reduction
    _run(a, [bt, M, K], [M * K, K, 1], b, [bt, K, N], [K * N, N, 1], out_offset=4)  # 128-bit reduction
    _run(a[: M * K], [M, K], [K, 1], b[: K * N], [K, N], [1, K])  # one tile column, transposed B


def test_large_values_and_specials_stay_finite(cuda):
    rng = np.random.default_rng(5)
    M, N, K = 128, 256, 64
    a = (rng.standard_normal(M * K) * 1e18).astype(F)
    b = (rng.standard_normal(K * N) * 1e-18).astype(F)
    _run(a, [M, K], [K, 1], b, [K, N], [N, 1])


def test_auto_uses_tensor_cores_for_large_problems(cuda):
    """MTC_GEMM_AUTO takes the tcgen05 path at 1024 x 512 x 512 (M*N*K = 2^28,
    the threshold) and the exact SIMT kernel below it; the path counters show
    which kernel family ran each call."""
    rng = np.random.default_rng(6)
    M, N, K = 1024, 512, 512
    tc0, simt0 = abi.gemm_path_counts()
    got, exp = _run(rng.standard_normal(M * K).astype(F), [M, K], [K, 1], rng.standard_normal(K * N).astype(F),
                    [K, N], [N, 1], algo=abi.GEMM_AUTO)
    tc1, simt1 = abi.gemm_path_counts()
    assert (tc1 - tc0, simt1 - simt0) == (1, 0), (tc1 - tc0, simt1 - simt0)
    _run(rng.standard_normal(M * K).astype(F), [M, K], [K, 1], rng.standard_normal(K * N).astype(F), [K, N],
         [N, 1], algo=abi.GEMM_SIMT)
    tc2, simt2 = abi.gemm_path_counts()
    assert (tc2 - tc1, simt2 - simt1) == (0, 1), (tc2 - tc1, simt2 - simt1)
    # below 2^28 multiply-adds AUTO keeps the exact SIMT kernel
    _run(rng.standard_normal(256 * 256).astype(F), [256, 256], [256, 1], rng.standard_normal(256 * 256).astype(F),
         [256, 256], [256, 1], algo=abi.GEMM_AUTO)
    tc3, simt3 = abi.gemm_path_counts()
    assert (tc3 - tc2, simt3 - simt2) == (0, 1), (tc3 - tc2, simt3 - simt2)


def test_many_tiles_per_cluster(cuda):
    """Enough 256x256 tiles that the default picks the CTA pair and each pair
    runs several tiles (both TMEM accumulators, every ring phase), with ragged
    row tiles and a K tail."""
    rng = np.random.default_rng(14)
    M, N, K = 2600, 2560, 300
    _run(rng.standard_normal(M * K).astype(F), [M, K], [K, 1], rng.standard_normal(K * N).astype(F), [K, N],
         [N, 1], out_offset=2)
