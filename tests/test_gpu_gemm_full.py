"""The tcgen05 3xTF32 GEMM at the sizes the benchmark measures, against the oracle.

Shapes of the GEMM sweep and of the wide-MLP training step:
  8192^3 with a contiguous B and with a transposed-view B, 16384^3,
  the weight-gradient shape 8192 x 8192 x 65536 (A = G^T, a transposed view, as
  the matmul VJP forms it, src/tensor/autograd/rules/linalg.cpp:16-54),
  batched [64,1024,1024] x [64,1024,1024], skinny [65536,1024] x [1024,8192].
Each shape runs under the default kernel policy and with the CTA-pair kernel
forced (MTC_TC_PIPELINE=pair16x6), on the same N(0,1) inputs.

Bound (the 1e-5*sqrt(K) relative bound, normwise per element):
  |C - C_ref|_ij <= 1e-5 * sqrt(K) * (|A| |B|)_ij.
What is compared, at sizes where the sequential float32 oracle cannot run on
every element:
  - 64 sampled rows (4 sampled batches x 16 rows when batched) against the exact
    product of those rows in float64;
  - 4 of those rows against the oracle itself (mo.matmul, the reference's
    k-ascending float32 loop, linalg/loops.hpp:198-286);
  - every element through two checksums: the column sums of C against
    (1^T A) B and the row sums against A (B 1), both in float64, each within
    the sum of the per-element bounds it covers (1e-5*sqrt(K) * (1^T|A|)|B| and
    |A|(|B| 1)).  A wrong tile, a skipped K block or a misplaced store breaks them.
"""
import os

import numpy as np
import pytest

from helpers import assert_rel_sqrtk
from minitensor_cpp_b200 import abi
from oracle import mt_oracle as mo

pytestmark = pytest.mark.gpu

# kernel choice ("MTC_TC_PIPELINE") and, after "/", the work-unit schedule
POLICIES = (None, "pair16x6", "/dynamic", "pair16x6/dynamic")
ROWS = 64
ORACLE_ROWS = 4


def _normal(shape, seed):
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(shape, device="cuda", generator=g)


def _run_policy(A, B, C, policy):
    import torch

    old = os.environ.pop("MTC_TC_PIPELINE", None)
    pipe, _, sched = (policy or "").partition("/")
    if pipe:
        os.environ["MTC_TC_PIPELINE"] = pipe
    if sched:
        os.environ["MTC_TC_SCHEDULE"] = sched
    try:
        tc0, _ = abi.gemm_path_counts()
        abi.matmul(A, B, C, abi.GEMM_AUTO)
        torch.cuda.synchronize()
        abi.check_device_errors(0)
        tc1, _ = abi.gemm_path_counts()
    finally:
        os.environ.pop("MTC_TC_PIPELINE", None)
        os.environ.pop("MTC_TC_SCHEDULE", None)
        if old is not None:
            os.environ["MTC_TC_PIPELINE"] = old
    assert tc1 - tc0 == 1, "the problem did not run on the tensor-core path"


def _check_matrix(a_host, b_host, c_host, rows, what):
    """a_host [M, K], b_host [K, N], c_host [M, N] (float32 host arrays)."""
    K = a_host.shape[1]
    b64 = b_host.astype(np.float64)
    babs = np.abs(b64)
    ar = a_host[rows].astype(np.float64)
    exact = ar @ b64
    scale = np.abs(ar) @ babs
    assert_rel_sqrtk(c_host[rows], exact, K, scale, f"{what}: sampled rows vs exact")
    orows = rows[:ORACLE_ROWS]
    want = mo.matmul(a_host[orows], b_host)
    assert_rel_sqrtk(c_host[orows], want, K, np.abs(a_host[orows].astype(np.float64)) @ babs,
                     f"{what}: rows vs the oracle")
    # column checksum: 1^T C = (1^T A) B
    col_a = a_host.sum(axis=0, dtype=np.float64)
    col_abs = np.abs(a_host).sum(axis=0, dtype=np.float64)
    got = c_host.sum(axis=0, dtype=np.float64)
    assert_rel_sqrtk(got, col_a @ b64, K, col_abs @ babs, f"{what}: column checksum")
    # row checksum: C 1 = A (B 1)
    b1 = b64.sum(axis=1)
    babs1 = babs.sum(axis=1)
    want_r = np.empty(a_host.shape[0])
    scale_r = np.empty(a_host.shape[0])
    for s in range(0, a_host.shape[0], 4096):
        blk = a_host[s:s + 4096].astype(np.float64)
        want_r[s:s + 4096] = blk @ b1
        scale_r[s:s + 4096] = np.abs(blk) @ babs1
    assert_rel_sqrtk(c_host.sum(axis=1, dtype=np.float64), want_r, K, scale_r, f"{what}: row checksum")


def _sample_rows(m, seed):
    rng = np.random.default_rng(seed)
    picked = rng.choice(m, ROWS, replace=False)
    # always include the first and last row tiles' edges
    picked[:2] = [0, m - 1]
    return np.sort(picked)


SHAPES = {
    # name: (A shape, A is a transposed view, B shape, B is a transposed view)
    "8192^3": ((8192, 8192), False, (8192, 8192), False),
    "8192^3 B^T view": ((8192, 8192), False, (8192, 8192), True),
    "16384^3": ((16384, 16384), False, (16384, 16384), False),
    "weight gradient 8192x8192x65536": ((8192, 65536), True, (65536, 8192), False),
    "skinny 65536x1024x8192": ((65536, 1024), False, (1024, 8192), False),
}


@pytest.mark.parametrize("name", list(SHAPES))
def test_gemm_at_benchmark_size(cuda, name):
    import torch

    (m, k), a_t, (k2, n), b_t = SHAPES[name]
    assert k == k2
    # a transposed view is the transpose of a contiguous [cols, rows] tensor
    a_store = _normal((k, m) if a_t else (m, k), 11)
    b_store = _normal((n, k) if b_t else (k, n), 12)
    a = a_store.t() if a_t else a_store
    b = b_store.t() if b_t else b_store
    A, B = abi.View.of(a), abi.View.of(b)
    a_host = a.cpu().numpy()  # logical [M, K] values (the transpose copied out)
    b_host = np.ascontiguousarray(b.cpu().numpy())
    a_host = np.ascontiguousarray(a_host)
    rows = _sample_rows(m, 5)
    for policy in POLICIES:
        c = torch.full((m, n), float("nan"), device="cuda")
        _run_policy(A, B, abi.View.of(c), policy)
        c_host = c.cpu().numpy()
        assert np.isfinite(c_host).all(), f"{name} [{policy}]: unwritten or non-finite outputs"
        _check_matrix(a_host, b_host, c_host, rows, f"{name} [{policy or 'default'}]")
        del c, c_host
    del a_store, b_store
    torch.cuda.empty_cache()


def test_batched_gemm_at_benchmark_size(cuda):
    """[64,1024,1024] x [64,1024,1024]: 4 sampled batches checked like a matrix."""
    import torch

    bt, m = 64, 1024
    a = _normal((bt, m, m), 21)
    b = _normal((bt, m, m), 22)
    a_host, b_host = a.cpu().numpy(), b.cpu().numpy()
    batches = [0, 17, 40, 63]
    for policy in POLICIES:
        c = torch.full((bt, m, m), float("nan"), device="cuda")
        _run_policy(abi.View.of(a), abi.View.of(b), abi.View.of(c), policy)
        c_host = c.cpu().numpy()
        assert np.isfinite(c_host).all()
        for i in batches:
            rows = _sample_rows(m, 100 + i)[:16]
            _check_matrix(a_host[i], b_host[i], c_host[i], rows, f"batch {i} [{policy or 'default'}]")


@pytest.mark.parametrize("k", [1024, 4096])
@pytest.mark.parametrize("policy", [None, "16x4", "32x2", "pair16x6", "pair32x3"])
def test_accuracy_against_the_exact_product(cuda, k, policy):
    """Every kernel variant's error against the exact (float64) product, relative
    to (|A||B|)_ij, stays within the measured envelope of the 3xTF32 product with
    float32 accumulation in TMEM: median <= 1e-8*sqrt(K), maximum <= 1e-7*sqrt(K)
    (measured on B200: median 2.4e-7 and maximum 2.0e-6 at K = 1024 without
    split-K, 4.7e-7 and 2.9e-6 at K = 4096).  A dropped lo term (error ~2^-11)
    or a single-TF32 product would exceed it a hundredfold; the 1e-5*sqrt(K)
    parity bound alone would not notice either."""
    import torch

    m, n = 512, 768
    a = _normal((m, k), 31)
    bs = _normal((n, k), 32)  # B = bs^T, as a Linear layer's weight
    A, B = abi.View.of(a), abi.View.of(bs.t())
    c = torch.full((m, n), float("nan"), device="cuda")
    _run_policy(A, B, abi.View.of(c), policy)
    a64 = a.cpu().numpy().astype(np.float64)
    b64 = bs.cpu().numpy().astype(np.float64).T
    rel = np.abs(c.cpu().numpy() - a64 @ b64) / (np.abs(a64) @ np.abs(b64))
    med, worst = float(np.median(rel)), float(rel.max())
    assert med <= 1e-8 * np.sqrt(k) and worst <= 1e-7 * np.sqrt(k), (policy, k, med, worst)
