"""Oracle (test infrastructure only): a numpy restatement of the MiniTensor
reference CPU backend's arithmetic for every kernel on the hot path.

Each function names the reference code it follows.  The restatement is pinned
two ways (tests/test_oracle.py): against the known-answer vectors of the
reference's own test suite (tests/golden/known_answers.json, transcribed with
file:line) and against the compiled reference itself (oracle/_ref/libmtref.so,
built from the unmodified sources by oracle/Makefile; fixtures in
tests/golden/*.npz made by tests/golden/make_golden.py).

Conventions: float32 throughout like the reference; transcendental functions
are evaluated in float64 and rounded once to float32 (a correctly rounded
stand-in for libm's expf/logf/...).  Sequential float32 accumulation orders
are reproduced exactly (cumulative sums), so sums, matmuls and scatter-adds
match the reference bit for bit.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import it.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32

# op codes (match include/mtcuda.h)
ABS, SIGN, NEGATE, EXP, LOG, SQRT, TANH, SIGMOID = range(0x0101, 0x0109)
RELU = 0x0180
ADD, SUBTRACT, MULTIPLY, DIVIDE, LOGADDEXP = range(0x0110, 0x0115)


def _f64(fn, x):
    with np.errstate(all="ignore"):
        return fn(np.asarray(x, dtype=np.float64)).astype(F32)


# ---------------------------------------------------------------- views --

def view(storage: np.ndarray, shape, strides, offset: int) -> np.ndarray:
    """Values of a strided view, Layout{strides, offset} (src/tensor/storage/layout.hpp:18-42)."""
    shape = tuple(int(s) for s in shape)
    if int(np.prod(shape)) == 0:
        return np.empty(shape, dtype=storage.dtype)
    if not shape:
        return np.array(storage[offset], dtype=storage.dtype)
    idx = np.indices(shape).reshape(len(shape), -1)
    offs = offset + sum(idx[d] * int(strides[d]) for d in range(len(shape)))
    return storage[offs.astype(np.int64)].reshape(shape)


# ----------------------------------------------------------- elementwise --

def unary(op: int, x: np.ndarray) -> np.ndarray:
    """elementwise/kernels.cpp:58-125."""
    x = np.asarray(x, dtype=F32)
    with np.errstate(all="ignore"):
        if op == NEGATE:
            return -x
        if op == EXP:
            return _f64(np.exp, x)
        if op == LOG:
            return _f64(np.log, x)
        if op == SQRT:
            return np.sqrt(x)  # IEEE correctly rounded, like std::sqrt
        if op == TANH:
            return _f64(np.tanh, x)
        if op == ABS:
            return np.abs(x)
        if op == SIGN:
            # kernels.cpp:96-107: +-1, otherwise the input itself (keeps +-0 and NaN)
            return np.where(x > 0, F32(1), np.where(x < 0, F32(-1), x)).astype(F32)
        if op == SIGMOID:
            # kernels.cpp:113-124: branch on the sign to stay finite
            e_neg = _f64(np.exp, -x)
            e_pos = _f64(np.exp, x)
            pos = F32(1) / (F32(1) + e_neg)
            neg = e_pos / (F32(1) + e_pos)
            return np.where(x >= 0, pos, neg).astype(F32)
        if op == RELU:
            # new op: max(x, 0) with NaN propagated and -0 -> +0
            return np.where(x > 0, x, np.where(np.isnan(x), x, F32(0))).astype(F32)
    raise ValueError(f"unknown unary op {op:#x}")


def binary(op: int, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """elementwise/kernels.cpp:127-167, with right-aligned broadcasting (layout.cpp:105-143)."""
    a = np.asarray(a, dtype=F32)
    b = np.asarray(b, dtype=F32)
    with np.errstate(all="ignore"):
        if op == ADD:
            return a + b
        if op == SUBTRACT:
            return a - b
        if op == MULTIPLY:
            return a * b
        if op == DIVIDE:
            return a / b
        if op == LOGADDEXP:
            a, b = np.broadcast_arrays(a, b)
            nan = np.isnan(a) | np.isnan(b)
            m = np.where(a < b, b, a)  # std::max(a, b)
            tail = _f64(np.log1p, _f64(np.exp, -np.abs(a - b)))
            out = np.where(np.isinf(m), m, m + tail)
            return np.where(nan, a + b, out).astype(F32)
    raise ValueError(f"unknown binary op {op:#x}")


# ------------------------------------------------------------ reductions --

def _move_reduced_last(x: np.ndarray, axes) -> tuple[np.ndarray, tuple]:
    axes = sorted(int(a) for a in axes)
    kept = [d for d in range(x.ndim) if d not in axes]
    y = np.transpose(x, kept + axes)
    kept_shape = tuple(x.shape[d] for d in kept)
    r = int(np.prod([x.shape[d] for d in axes])) if axes else 1
    return y.reshape(kept_shape + (r,)), kept_shape


def _keep(out: np.ndarray, x: np.ndarray, axes, keep_dim: bool) -> np.ndarray:
    if not keep_dim:
        return out
    shape = tuple(1 if d in set(int(a) for a in axes) else x.shape[d] for d in range(x.ndim))
    return out.reshape(shape)


def reduce_sum(x: np.ndarray, axes, keep_dim: bool = False) -> np.ndarray:
    """reduce_values with + (reduction/loops.hpp:21-57): sequential float32 accumulation
    in row-major order of the reduced axes (ReductionPlan, iteration/reduction.cpp:14-121)."""
    x = np.asarray(x, dtype=F32)
    y, kept = _move_reduced_last(x, axes)
    if y.shape[-1] == 0:
        out = np.zeros(kept, dtype=F32)
    else:
        out = np.cumsum(y, axis=-1, dtype=F32)[..., -1]
    return _keep(np.asarray(out, dtype=F32), x, axes, keep_dim)


def reduce_logsumexp(x: np.ndarray, axes, keep_dim: bool = False) -> np.ndarray:
    """reduce_logsumexp (reduction/loops.hpp:59-136): NaN-ignoring max, NaN -> NaN,
    infinite max -> max, else max + log(sequential sum of exp(x - max))."""
    x = np.asarray(x, dtype=F32)
    y, kept = _move_reduced_last(x, axes)
    with np.errstate(all="ignore"):
        has_nan = np.isnan(y).any(axis=-1)
        ym = np.where(np.isnan(y), -np.inf, y).astype(F32)
        mx = ym.max(axis=-1, initial=-np.inf).astype(F32)
        shifted = (y - mx[..., None]).astype(F32)
        e = _f64(np.exp, shifted)
        s = np.cumsum(e, axis=-1, dtype=F32)[..., -1] if y.shape[-1] else np.zeros(kept, F32)
        res = (mx + _f64(np.log, s)).astype(F32)
        res = np.where(np.isinf(mx), mx, res)
        res = np.where(has_nan, F32(np.nan), res).astype(F32)
    return _keep(res, x, axes, keep_dim)


def reduce_max(x: np.ndarray, axes, keep_dim: bool = False) -> np.ndarray:
    """New op (no reference counterpart): maximum, NaN propagates, empty -> -inf."""
    x = np.asarray(x, dtype=F32)
    y, kept = _move_reduced_last(x, axes)
    with np.errstate(all="ignore"):
        mx = np.where(np.isnan(y), -np.inf, y).max(axis=-1, initial=-np.inf).astype(F32)
        mx = np.where(np.isnan(y).any(axis=-1), F32(np.nan), mx).astype(F32)
    return _keep(mx, x, axes, keep_dim)


def reduce_argmax(x: np.ndarray, axis: int, keep_dim: bool = False) -> np.ndarray:
    """New op: index (Int64) of the first maximum along `axis`; a NaN counts as the maximum."""
    x = np.asarray(x, dtype=F32)
    y, kept = _move_reduced_last(x, [axis])
    nan = np.isnan(y)
    first_nan = np.argmax(nan, axis=-1)
    plain = np.argmax(np.where(nan, -np.inf, y), axis=-1)
    out = np.where(nan.any(axis=-1), first_nan, plain).astype(np.int64)
    return _keep(out, x, [axis], keep_dim)


def log_softmax(x: np.ndarray, axis: int) -> np.ndarray:
    """x - logsumexp(x, {axis}, keep_dim=true): the reference composite (Subtract of LogSumExp)."""
    x = np.asarray(x, dtype=F32)
    with np.errstate(invalid="ignore"):  # a row of -inf (or +inf) gives NaN, as in IEEE arithmetic
        return (x - reduce_logsumexp(x, [axis], keep_dim=True)).astype(F32)


# ------------------------------------------------------------------ matmul --

def matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """matmul_dispatch (linalg/loops.hpp:288-324): every output element is the
    sequential float32 sum over k of the float32 products, k ascending (dot,
    gemv, vector_matrix and both gemm paths accumulate in that order); batch
    axes broadcast (primitives/linalg/matmul.cpp:18-52)."""
    a = np.asarray(a, dtype=F32)
    b = np.asarray(b, dtype=F32)
    av, bv = a.ndim == 1, b.ndim == 1
    A = a[None, :] if av else a
    B = b[:, None] if bv else b
    K = A.shape[-1]
    if B.shape[-2] != K:
        raise ValueError("matmul contraction extents differ")
    batch = np.broadcast_shapes(A.shape[:-2], B.shape[:-2])
    A = np.broadcast_to(A, batch + A.shape[-2:])
    B = np.broadcast_to(B, batch + B.shape[-2:])
    acc = np.zeros(batch + (A.shape[-2], B.shape[-1]), dtype=F32)
    for k in range(K):
        acc = (acc + (A[..., :, k:k + 1] * B[..., k:k + 1, :]).astype(F32)).astype(F32)
    if av:
        acc = acc[..., 0, :]
    if bv:
        acc = acc[..., 0]
    return acc


# --------------------------------------------------------------- indexing --

def gather(src: np.ndarray, axis: int, idx: np.ndarray) -> np.ndarray:
    """gather_copy (copy/loops.hpp:155-220): take-along-axis, out_of_range on a bad index."""
    idx = np.asarray(idx, dtype=np.int64)
    if idx.size and (idx.min() < 0 or idx.max() >= src.shape[axis]):
        raise IndexError("gather index is out of range")
    return np.take_along_axis(np.asarray(src), idx, axis=axis)


def gather_scatter_add(upd: np.ndarray, idx: np.ndarray, axis: int, target_shape) -> np.ndarray:
    """gather_scatter_add (copy/loops.hpp:222-303): zero target, then += in the
    row-major iteration order of the updates (np.add.at is unbuffered and ordered)."""
    upd = np.asarray(upd, dtype=F32)
    idx = np.asarray(idx, dtype=np.int64)
    if idx.size and (idx.min() < 0 or idx.max() >= target_shape[axis]):
        raise IndexError("gather scatter add index is out of range")
    out = np.zeros(target_shape, dtype=F32)
    coords = list(np.indices(idx.shape))
    coords[axis] = idx
    np.add.at(out, tuple(coords), upd)
    return out


def concatenate(inputs, axis: int) -> np.ndarray:
    """concatenate_copy (copy/loops.hpp:90-127)."""
    return np.concatenate([np.asarray(x) for x in inputs], axis=axis)


# ------------------------------------------------------------------ random --

_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox_blocks(key0: int, key1: int, n_blocks: int) -> np.ndarray:
    """Philox-4x32-10 blocks 0..n-1 (detail/random_engine.cpp:14-52): [n, 4] uint32."""
    b = np.arange(n_blocks, dtype=np.uint64)
    c0 = (b & _MASK32).astype(np.uint64)
    c1 = (b >> np.uint64(32)).astype(np.uint64)
    c2 = np.full(n_blocks, np.uint64(key1) & _MASK32, dtype=np.uint64)
    c3 = np.full(n_blocks, np.uint64(key1) >> np.uint64(32), dtype=np.uint64)
    k0 = np.uint32(key0 & 0xFFFFFFFF)
    k1 = np.uint32(key0 >> 32)
    for rnd in range(10):
        p0 = _M0 * c0
        p1 = _M1 * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK32
        c0, c1, c2, c3 = (hi1 ^ c1 ^ np.uint64(k0)), lo1, (hi0 ^ c3 ^ np.uint64(k1)), lo0
        if rnd != 9:
            k0 = np.uint32((int(k0) + int(_W0)) & 0xFFFFFFFF)
            k1 = np.uint32((int(k1) + int(_W1)) & 0xFFFFFFFF)
    return np.stack([c0, c1, c2, c3], axis=1).astype(np.uint32)


def uniform(n: int, low: float, high: float, key) -> np.ndarray:
    """uniform (creation/loops.hpp:39-86): 24-bit unit in float, double affine map, clamp below high."""
    low, high = F32(low), F32(high)
    if low == high:
        return np.full(n, low, dtype=F32)
    words = philox_blocks(key[0], key[1], (n + 3) // 4).reshape(-1)[:n]
    unit = ((words >> np.uint32(8)).astype(F32) * F32(2.0 ** -24)).astype(np.float64)
    v = (np.float64(low) + (np.float64(high) - np.float64(low)) * unit).astype(F32)
    return np.where(v >= high, np.nextafter(high, low, dtype=F32), v).astype(F32)


def normal(n: int, mean: float, std: float, key) -> np.ndarray:
    """normal (creation/loops.hpp:88-141): double Box-Muller on open-unit uniforms."""
    mean, std = F32(mean), F32(std)
    if std == 0:
        return np.full(n, mean, dtype=F32)
    w = philox_blocks(key[0], key[1], (n + 3) // 4).astype(np.float64)
    u = (w + 0.5) * 2.0 ** -32
    r0 = np.sqrt(-2.0 * np.log(u[:, 0]))
    r1 = np.sqrt(-2.0 * np.log(u[:, 2]))
    a0 = 2.0 * np.pi * u[:, 1]
    a1 = 2.0 * np.pi * u[:, 3]
    z = np.stack([r0 * np.cos(a0), r0 * np.sin(a0), r1 * np.cos(a1), r1 * np.sin(a1)], axis=1).reshape(-1)[:n]
    return (np.float64(mean) + np.float64(std) * z).astype(F32)


_GOLDEN = 0x9E3779B97F4A7C15
_SPLIT_TAG = 0xD2B74407B1CE6E93
_M64 = (1 << 64) - 1


def _mix(v: int) -> int:
    """splitmix-style finaliser (src/tensor/random.cpp:13-21)."""
    v = (v + _GOLDEN) & _M64
    v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & _M64
    return v ^ (v >> 31)


def key_fold_in(key, data: int):
    """fold_in (src/tensor/random.cpp:28-32)."""
    return (_mix(key[0] ^ _mix(data)), _mix(key[1] ^ _mix(data ^ _GOLDEN)))


def key_split(key):
    """split (src/tensor/random.cpp:23-26)."""
    return key_fold_in(key, _SPLIT_TAG), key_fold_in(key, _SPLIT_TAG + 1)


def random_key(seed: int):
    """RandomKey{seed} = words {seed, 0} (include/minitensor/random.hpp:22-24)."""
    return (seed & _M64, 0)


# ----------------------------------------------------------------- nn ------

def cross_entropy(logits: np.ndarray, targets: np.ndarray) -> F32:
    """categorical_cross_entropy_with_logits (src/nn/loss.cpp:41-57) on the last axis:
    mean(logsumexp(logits, {-1}, true) - gather(logits, -1, unsqueeze(targets)))."""
    lse = reduce_logsumexp(logits, [logits.ndim - 1], keep_dim=True)
    sel = gather(logits, logits.ndim - 1, np.asarray(targets, dtype=np.int64)[..., None])
    d = (lse - sel).astype(F32)
    return (reduce_sum(d, list(range(d.ndim))) / F32(d.size)).astype(F32)


def adamw_coefficients(lr: float, wd: float, beta1: float, beta2: float, step: int):
    """AdamW::step_coefficients (src/nn/optimizers/adamw.cpp:53-65) for the update after `step` steps."""
    t = float(step + 1)
    decay = F32(1.0) - F32(lr) * F32(wd)
    c1 = F32(1.0) - F32(np.power(np.float64(F32(beta1)), t))
    c2 = F32(1.0) - F32(np.power(np.float64(F32(beta2)), t))
    return decay, c1, c2


def adamw_update(p, g, m, v, lr, wd, beta1, beta2, eps, step):
    """AdamW::update_parameter (src/nn/optimizers/adamw.cpp:67-97), op for op in float32."""
    p, g, m, v = (np.asarray(x, dtype=F32) for x in (p, g, m, v))
    lr, wd, beta1, beta2, eps = (F32(x) for x in (lr, wd, beta1, beta2, eps))
    decay, c1, c2 = adamw_coefficients(lr, wd, beta1, beta2, step)
    m2 = (beta1 * m + (F32(1) - beta1) * g).astype(F32)
    v2 = (beta2 * v + ((F32(1) - beta2) * g) * g).astype(F32)
    mhat = (m2 / c1).astype(F32)
    vhat = (v2 / c2).astype(F32)
    upd = ((lr * mhat) / (np.sqrt(vhat) + eps)).astype(F32)
    return (decay * p - upd).astype(F32), m2, v2
