"""Shared helpers of the parity tests."""
from __future__ import annotations

import numpy as np

F32 = np.float32


def ordered(x: np.ndarray) -> np.ndarray:
    """Maps float32 bit patterns onto a monotone int64 line (ulp distance = difference)."""
    i = np.asarray(x, dtype=F32).view(np.int32).astype(np.int64)
    return np.where(i < 0, -(i & 0x7FFFFFFF), i)


def ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """ulp distance of two float32 arrays; NaN==NaN counts as 0, NaN vs number as huge."""
    a = np.asarray(a, dtype=F32)
    b = np.asarray(b, dtype=F32)
    d = np.abs(ordered(a) - ordered(b))
    both_nan = np.isnan(a) & np.isnan(b)
    one_nan = np.isnan(a) ^ np.isnan(b)
    d = np.where(both_nan, 0, d)
    return np.where(one_nan, np.iinfo(np.int64).max, d)


def assert_ulp(actual, expected, max_ulp: int, what: str = ""):
    d = ulp_diff(actual, expected)
    worst = int(d.max()) if d.size else 0
    assert worst <= max_ulp, f"{what}: {worst} ulp > {max_ulp} (first bad at {np.argmax(d.reshape(-1))})"


def assert_bits(actual, expected, what: str = ""):
    a = np.asarray(actual)
    e = np.asarray(expected)
    assert a.shape == e.shape, f"{what}: shape {a.shape} != {e.shape}"
    if a.dtype == np.float32:
        ok = (a.view(np.int32) == e.view(np.int32)) | (np.isnan(a) & np.isnan(e))
    else:
        ok = a == e
    assert ok.all(), f"{what}: {int((~ok).sum())} of {ok.size} elements differ; first at {np.argmax(~ok.reshape(-1))}"


def assert_rel_sqrtk(actual, expected, k: int, scale=None, what: str = ""):
    """Reduction / GEMM parity bound: |a - e| <= 1e-5 * sqrt(K) * scale (scale = |e| when None,
    floored at 1e-30); NaN/inf positions must agree exactly."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    finite = np.isfinite(e)
    assert (np.isnan(a) == np.isnan(e)).all(), f"{what}: NaN positions differ"
    assert (a[~finite & ~np.isnan(e)] == e[~finite & ~np.isnan(e)]).all(), f"{what}: infinities differ"
    s = np.abs(e) if scale is None else np.asarray(scale, dtype=np.float64)
    tol = 1e-5 * np.sqrt(max(k, 1)) * np.maximum(s, 1e-30)
    with np.errstate(invalid="ignore"):  # inf - inf at the infinities checked above
        err = np.abs(a - e)
    bad = finite & (err > tol)
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements exceed 1e-5*sqrt({k}); worst ratio "
                           f"{float(np.max(np.where(finite, err / tol, 0))):.3g}")


def check_added_ops(fe, device: int, x: np.ndarray, axis: int):
    """relu, max, argmax and log-softmax through the front-end's added operations
    against the oracle: relu bit for bit against max(x, 0) (NaN propagated) and
    its gradient against the step [x > 0] (NaN where x is NaN), max and argmax
    bit for bit, log-softmax within the logsumexp bound (1e-5*sqrt(K) of |lse|)."""
    from oracle import mt_oracle as mo

    relu, mx, am, lsm, grad = fe.added_ops(device, x, axis)
    assert_bits(relu, mo.unary(mo.RELU, x), f"relu device {device}")
    assert_bits(relu, np.where(np.isnan(x), x, np.maximum(x, F32(0))) + F32(0), f"relu vs maximum, device {device}")
    step = np.where(np.isnan(x), F32(np.nan), (x > 0).astype(F32))
    assert_bits(grad, step, f"relu gradient device {device}")
    assert_bits(mx, mo.reduce_max(x, [axis]), f"max axis {axis} device {device}")
    assert_bits(am, mo.reduce_argmax(x, axis), f"argmax axis {axis} device {device}")
    lse = mo.reduce_logsumexp(x, [axis], keep_dim=True)
    scale = np.broadcast_to(np.abs(lse), x.shape)
    assert_rel_sqrtk(lsm, mo.log_softmax(x, axis), x.shape[axis], scale, f"log_softmax axis {axis} device {device}")


def added_ops_input(rows: int, cols: int, seed: int) -> np.ndarray:
    """Uniform values with a tie, a NaN, a row of -inf, a -0, 0 and values beyond
    FLT_MAX / 2 planted."""
    rng = np.random.default_rng(seed)
    x = rng.uniform(-10, 10, (rows, cols)).astype(F32)
    x[1, 2] = x[1, 5] = F32(50)  # a tie along axis 1
    x[3, 4] = F32(np.nan)
    x[5, :] = F32(-np.inf)
    x[2, 0] = F32(-0.0)
    x[2, 1] = F32(0.0)
    x[4, 3] = F32(3e38)  # x + x overflows: a composite (x + |x|) / 2 would give inf
    x[6, 1] = F32(-3e38)
    return x
