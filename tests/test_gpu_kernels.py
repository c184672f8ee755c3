"""GPU parity of every libmtcuda kernel family against the reference CPU kernels.

Each case runs the compiled reference (oracle/_ref/libmtref.so: the unmodified
MiniTensor CPU kernels) or the pinned numpy oracle on the same seeded host
inputs, and the CUDA kernel through the C ABI (minitensor_cpp_b200.abi).
Bars: bit-exact for data movement, indexing, +,-,*,/ and Philox uniform;
<= 2 ulp for transcendental elementwise ops; |err| <= 1e-5*sqrt(K)*scale for
reductions and GEMM (scale = sum|x| or |A||B|, stated per test).
"""
import json
from pathlib import Path

import numpy as np
import pytest

from helpers import assert_bits, assert_rel_sqrtk, assert_ulp
from minitensor_cpp_b200 import abi
from oracle import mt_oracle as mo
from oracle import refkernels as rk

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
F = np.float32


def gpu(hv: rk.HostView) -> abi.View:
    import torch

    return abi.View(torch.from_numpy(hv.storage.copy()).cuda(), hv.shape, hv.strides, hv.offset)


def host(v: abi.View) -> np.ndarray:
    import torch

    torch.cuda.synchronize()
    return v.storage.cpu().numpy()


def hv(storage, shape, strides=None, offset=0):
    storage = np.ascontiguousarray(storage).reshape(-1)
    if strides is None:
        strides = abi.contiguous_strides(list(shape))
    return rk.HostView(storage, tuple(shape), tuple(strides), offset)


def out_like(shape, dtype=F, fill=-7.0, offset=0):
    n = int(np.prod(shape)) + offset
    return hv(np.full(max(n, 1), fill, dtype=dtype), shape, None, offset)


# ------------------------------------------------------------- known answers --

KA = json.loads((GOLDEN / "known_answers.json").read_text())


def _ka_view(spec):
    dt = np.int64 if spec.get("dtype") == "int64" else F
    return hv(np.asarray(spec["storage"], dtype=dt), spec["shape"], spec["strides"], spec["offset"])


@pytest.mark.parametrize("name", [k for k in sorted(KA) if KA[k]["op"] in
                                  ("add", "sum", "matmul", "copy", "concat", "gather", "fill", "index_scatter")])
def test_known_answers_on_gpu(cuda, name):
    case = KA[name]
    op = case["op"]
    out = gpu(_ka_view(case["out"]))
    if op == "add":
        abi.binary(abi.ADD, gpu(_ka_view(case["lhs"])), gpu(_ka_view(case["rhs"])), out)
    elif op == "sum":
        abi.reduce(abi.SUM, gpu(_ka_view(case["in"])), case["axes"], out)
    elif op == "matmul":
        abi.matmul(gpu(_ka_view(case["lhs"])), gpu(_ka_view(case["rhs"])), out)
    elif op == "copy":
        abi.copy(gpu(_ka_view(case["in"])), out)
    elif op == "concat":
        ins = [_ka_view(s) for s in case["inputs"]]
        for i, s in enumerate(ins):
            if s.storage.size == 0:
                ins[i] = hv(np.zeros(1, F), s.shape, s.strides, 0)
        abi.concat([gpu(s) for s in ins], case["axis"], out)
    elif op == "gather":
        abi.gather(gpu(_ka_view(case["src"])), gpu(_ka_view(case["idx"])), case["axis"], out)
    elif op == "fill":
        abi.fill(out, case["value"])
    elif op == "index_scatter":
        outv = _ka_view(case["out"])
        shape, strides, offset = rk.index_layout(outv, select=case["select"], axis=case["axis"], start=case["start"],
                                                 stop=case["stop"], step_or_index=case["step_or_index"])
        dst = abi.View(out.storage, shape, strides, offset)
        abi.index_scatter(gpu(_ka_view(case["in"])), dst, out)
    assert_bits(host(out), np.asarray(case["expected"], dtype=F), name)


# ----------------------------------------------------------------- elementwise --

SPECIAL = np.array([0.0, -0.0, 1.0, -1.0, 1e-30, -1e-30, 0.5, -0.5, 88.0, -88.0, 89.0, -104.0, 1000.0, -1000.0,
                    np.inf, -np.inf, np.nan, 3.4e38, -3.4e38, 1e-45], dtype=F)
UNARY_ULP = {abi.ABS: 0, abi.SIGN: 0, abi.NEGATE: 0, abi.SQRT: 0, abi.EXP: 2, abi.LOG: 2, abi.TANH: 2,
             abi.SIGMOID: 2}


def _unary_layouts(rng, kind):
    base = rng.uniform(0.01, 20, 5000) if kind == "positive" else rng.uniform(-40, 40, 5000)
    st = np.concatenate([SPECIAL, base.astype(F)])
    big = (rng.uniform(0.01, 20, 400 * 330) if kind == "positive" else rng.uniform(-40, 40, 400 * 330)).astype(F)
    return [
        hv(st, [st.size]),                                   # contiguous, 128-bit path
        hv(st, [50, 40], [40, 1], 3),                        # misaligned offset -> scalar flat path
        hv(st, [40, 50], [1, 40], 0),                        # small transposed view -> strided path
        hv(big, [400, 330], [1, 400], 0),                    # transposed view of 42 tiles -> tiled path
        hv(st, [20, 30], [-60, 2], 19 * 60),                 # negative + stride-2 -> generic strided path
    ]


@pytest.mark.parametrize("op", sorted(UNARY_ULP))
def test_unary_vs_reference(cuda, op):
    rng = np.random.default_rng(op)
    kind = "positive" if op in (abi.LOG, abi.SQRT) else "wide"
    for x in _unary_layouts(rng, kind):
        ref = out_like(x.shape)
        rk.unary(op, x, ref)
        out = gpu(out_like(x.shape))
        abi.unary(op, gpu(x), out)
        assert_ulp(host(out), ref.storage, UNARY_ULP[op], f"unary {op:#x} {x.shape}/{x.strides}")


def test_relu_vs_oracle(cuda):
    x = hv(np.concatenate([SPECIAL, np.random.default_rng(1).standard_normal(999).astype(F)]), [SPECIAL.size + 999])
    out = gpu(out_like(x.shape))
    abi.unary(abi.RELU, gpu(x), out)
    assert_bits(host(out), mo.unary(mo.RELU, x.storage), "relu")
    # equals the reference composite (x + |x|) * 0.5 used by the training workloads
    comp = mo.binary(mo.MULTIPLY, mo.binary(mo.ADD, x.storage, mo.unary(mo.ABS, x.storage)), F(0.5))
    finite = np.isfinite(x.storage) & (np.abs(x.storage) < 1e38)
    assert_bits(host(out)[finite], comp[finite], "relu == composite")


BINARY_ULP = {abi.ADD: 0, abi.SUBTRACT: 0, abi.MULTIPLY: 0, abi.DIVIDE: 0, abi.LOGADDEXP: 2}


def _check_binary(op, got, exp, a, b, what):
    if op != abi.LOGADDEXP:
        assert_ulp(np.asarray(got).reshape(-1)[: exp.size], exp.reshape(-1), BINARY_ULP[op], what)
        return
    # logaddexp = max + log1p(exp(-|a-b|)): when max ~ -log(2) the sum cancels, so
    # its error is bounded by 2 ulp of the larger summand, not of the result
    av = np.broadcast_to(mo.view(a.storage, a.shape, a.strides, a.offset), exp.shape).reshape(-1)
    bv = np.broadcast_to(mo.view(b.storage, b.shape, b.strides, b.offset), exp.shape).reshape(-1)
    mag = np.maximum(np.maximum(np.abs(av), np.abs(bv)), F(0.6931472)).astype(F)
    e = exp.reshape(-1)
    g = np.asarray(got).reshape(-1)[: e.size]
    assert (np.isnan(g) == np.isnan(e)).all(), what
    assert (g[np.isinf(e)] == e[np.isinf(e)]).all(), what
    finite = np.isfinite(e) & np.isfinite(mag)
    tol = 2 * np.spacing(mag[finite])
    err = np.abs(g[finite].astype(np.float64) - e[finite].astype(np.float64))
    assert (err <= tol).all(), f"{what}: worst {float(np.max(err / tol)):.2f} x (2 ulp of max(|a|,|b|))"


@pytest.mark.parametrize("op", sorted(BINARY_ULP))
def test_binary_vs_reference(cuda, op):
    rng = np.random.default_rng(op)
    a_st = rng.uniform(-50, 50, 200 * 301).astype(F)
    b_st = rng.uniform(-50, 50, 200 * 301).astype(F)
    row = rng.uniform(-5, 5, 301).astype(F)
    col = rng.uniform(-5, 5, 200).astype(F)
    big_a = rng.uniform(-50, 50, 300 * 401).astype(F)
    big_b = rng.uniform(-50, 50, 300 * 401).astype(F)
    cases = [
        (hv(a_st, [200, 301]), hv(b_st, [200, 301])),                      # same shape, contiguous
        (hv(a_st, [200, 301]), hv(row, [1, 301])),                          # row broadcast
        (hv(a_st, [200, 301]), hv(col, [200, 1])),                          # column broadcast
        (hv(a_st, [200, 301]), hv(b_st, [200, 301], [1, 200])),             # transposed rhs, 20 tiles (strided)
        (hv(big_a, [300, 401]), hv(big_b, [300, 401], [1, 300])),           # transposed rhs, 35 tiles (tiled)
        (hv(big_b, [300, 401], [1, 300]), hv(big_a, [300, 401], [1, 300])), # both transposed (tiled)
        (hv(np.array([2.5], F), []), hv(a_st, [200, 301])),                 # scalar lhs
        (hv(a_st, [100, 301], [-602, 1], 199 * 301), hv(row, [301])),       # negative stride, rank-1 rhs
    ]
    for a, b in cases:
        shape = np.broadcast_shapes(a.shape, b.shape)
        ref = out_like(shape)
        rk.binary(op, a, b, ref)
        out = gpu(out_like(shape))
        abi.binary(op, gpu(a), gpu(b), out)
        _check_binary(op, host(out), ref.storage.reshape(shape), a, b, f"binary {op:#x} {a.strides}/{b.strides}")
    sa, sb = np.meshgrid(SPECIAL, SPECIAL)
    a, b = hv(sa.copy(), [sa.size]), hv(sb.copy(), [sb.size])
    ref = out_like([sa.size])
    rk.binary(op, a, b, ref)
    out = gpu(out_like([sa.size]))
    abi.binary(op, gpu(a), gpu(b), out)
    _check_binary(op, host(out), ref.storage, a, b, f"binary special {op:#x}")


def test_fused_chain_equals_unfused_chain(cuda):
    """relu(A*B^T + row) * exp(-col): one fused kernel vs the reference's five materialised ops."""
    rng = np.random.default_rng(7)
    n, m = 192, 320
    A = hv(rng.uniform(-1, 1, n * m).astype(F), [n, m])
    B = hv(rng.uniform(-1, 1, n * m).astype(F), [n, m], [1, n])  # transposed view
    row = hv(rng.uniform(-1, 1, m).astype(F), [1, m])
    col = hv(rng.uniform(-1, 1, n).astype(F), [n, 1])
    # reference, op by op on the CPU backend
    t1, t2, t3, c1, c2, y = (out_like(s) for s in ([n, m], [n, m], [n, m], [n, 1], [n, 1], [n, m]))
    rk.binary(abi.MULTIPLY, A, B, t1)
    rk.binary(abi.ADD, t1, row, t2)
    relu = mo.unary(mo.RELU, t2.storage)
    t3 = hv(relu, [n, m])
    rk.unary(abi.NEGATE, col, c1)
    rk.unary(abi.EXP, c1, c2)
    rk.binary(abi.MULTIPLY, t3, c2, y)
    # fused: registers 0..3 = A, B, row, col
    prog = [(abi.MULTIPLY, 4, 0, 1, 0.0), (abi.ADD, 5, 4, 2, 0.0), (abi.RELU, 6, 5, 0, 0.0),
            (abi.NEGATE, 7, 3, 0, 0.0), (abi.EXP, 8, 7, 0, 0.0), (abi.MULTIPLY, 9, 6, 8, 0.0)]
    out = gpu(out_like([n, m]))
    abi.fused(prog, [gpu(A), gpu(B), gpu(row), gpu(col)], [9], [out])
    assert_ulp(host(out), y.storage, 2, "fused chain")


@pytest.mark.parametrize("offset", [0, 4, 1])
def test_fused_tiled_transposes_batched_two_outputs(cuda, offset):
    """Two transposed inputs, a contiguous one and a column broadcast in a batched
    space with partial 64x64 tiles; two outputs.  Offsets 0 and 4 keep every
    operand 16-byte aligned (the float4 tile kernel), offset 1 does not (the
    scalar tile kernel).  Only +, * and relu: bit-exact against numpy."""
    rng = np.random.default_rng(21)
    b, n, m = 3, 200, 260  # 4 x 5 tiles per batch entry, partial at both edges
    st = lambda: rng.uniform(-1, 1, b * n * m + offset).astype(F)
    P, Q, R = st(), st(), st()
    colv = rng.uniform(-1, 1, b * n).astype(F)
    tr = [n * m, 1, n]  # element (i, r, c) at i*n*m + c*n + r
    Pt = hv(P, [b, n, m], tr, offset)
    Qt = hv(Q, [b, n, m], tr, offset)
    Rc = hv(R, [b, n, m], None, offset)
    Cb = hv(colv, [b, n, 1])
    pv = mo.view(P, [b, n, m], tr, offset)
    qv = mo.view(Q, [b, n, m], tr, offset)
    rv = mo.view(R, [b, n, m], abi.contiguous_strides([b, n, m]), offset)
    cv = colv.reshape(b, n, 1)
    e0 = mo.unary(mo.RELU, (pv * qv + rv).astype(F)) * cv
    e1 = (pv + cv) * rv
    prog = [(abi.MULTIPLY, 4, 0, 1, 0.0), (abi.ADD, 5, 4, 2, 0.0), (abi.RELU, 6, 5, 0, 0.0),
            (abi.MULTIPLY, 7, 6, 3, 0.0), (abi.ADD, 8, 0, 3, 0.0), (abi.MULTIPLY, 9, 8, 2, 0.0)]
    outs = [gpu(out_like([b, n, m], offset=offset)) for _ in range(2)]
    abi.fused(prog, [gpu(Pt), gpu(Qt), gpu(Rc), gpu(Cb)], [7, 9], outs)
    for o, e, name in zip(outs, (e0, e1), ("relu(p*q + r) * c", "(p + c) * r")):
        got = host(o)
        assert (got[:offset] == -7.0).all(), "wrote before the output offset"
        assert_bits(got[offset:], e.astype(F).reshape(-1), name)


def test_fused_multi_output_adamw_program(cuda):
    """AdamW's update graph as one fused program with three outputs (p', m', v')."""
    rng = np.random.default_rng(11)
    n = 4097
    p, g, m, v = (rng.standard_normal(n).astype(F) for _ in range(4))
    v = np.abs(v)
    lr, wd, b1, b2, eps, step = 1e-3, 0.01, 0.9, 0.999, 1e-8, 4
    decay, c1, c2 = mo.adamw_coefficients(lr, wd, b1, b2, step)
    exp_p, exp_m, exp_v = mo.adamw_update(p, g, m, v, lr, wd, b1, b2, eps, step)
    C = abi.CONST
    prog = [
        (C, 4, 0, 0, b1), (abi.MULTIPLY, 5, 4, 2, 0.0), (C, 6, 0, 0, float(F(1) - F(b1))), (abi.MULTIPLY, 7, 6, 1, 0.0),
        (abi.ADD, 8, 5, 7, 0.0),                                        # m'
        (C, 9, 0, 0, b2), (abi.MULTIPLY, 10, 9, 3, 0.0), (C, 11, 0, 0, float(F(1) - F(b2))),
        (abi.MULTIPLY, 12, 11, 1, 0.0), (abi.MULTIPLY, 13, 12, 1, 0.0), (abi.ADD, 14, 10, 13, 0.0),  # v'
        (C, 15, 0, 0, float(c1)), (abi.DIVIDE, 16, 8, 15, 0.0), (C, 17, 0, 0, float(c2)), (abi.DIVIDE, 18, 14, 17, 0.0),
        (C, 19, 0, 0, float(decay)), (abi.MULTIPLY, 20, 19, 0, 0.0), (C, 21, 0, 0, lr), (abi.MULTIPLY, 22, 21, 16, 0.0),
        (abi.SQRT, 23, 18, 0, 0.0), (C, 24, 0, 0, eps), (abi.ADD, 25, 23, 24, 0.0), (abi.DIVIDE, 26, 22, 25, 0.0),
        (abi.SUBTRACT, 27, 20, 26, 0.0),                                # p'
    ]
    outs = [gpu(out_like([n])) for _ in range(3)]
    abi.fused(prog, [gpu(hv(x, [n])) for x in (p, g, m, v)], [27, 8, 14], outs)
    assert_bits(host(outs[0]), exp_p, "p'")
    assert_bits(host(outs[1]), exp_m, "m'")
    assert_bits(host(outs[2]), exp_v, "v'")


# ------------------------------------------------------------------- reductions --

def _red_cases(rng):
    big = rng.standard_normal(64 * 3000).astype(F)
    x3 = rng.standard_normal(6 * 7 * 300).astype(F)
    return [
        (hv(big, [64, 3000]), [1]),            # long rows -> CTA per row
        (hv(big, [3000, 64]), [1]),            # short rows -> warp per row
        (hv(big, [3000, 64]), [0]),            # column reduction, chunked
        (hv(big, [64, 3000], [1, 64]), [0]),   # transposed view, reduce the contiguous axis
        (hv(x3, [6, 7, 300]), [0, 2]),         # non-adjacent axes
        (hv(x3, [6, 7, 300]), [0, 1, 2]),      # full reduction
        (hv(x3, [6, 7, 300], [-2100, 300, 1], 5 * 2100), [2]),  # negative stride
        (hv(big, [4, 0, 3]), [1]),             # empty reduction
    ]


@pytest.mark.parametrize("op", [abi.SUM, abi.LOGSUMEXP])
def test_sum_logsumexp_vs_reference(cuda, op):
    rng = np.random.default_rng(3)
    for x, axes in _red_cases(rng):
        kept = [e for d, e in enumerate(x.shape) if d not in axes]
        ref = out_like(kept)
        rk.reduce(op, x, axes, False, ref)
        out = gpu(out_like(kept))
        abi.reduce(op, gpu(x), axes, out)
        R = int(np.prod([x.shape[d] for d in axes]))
        xa = mo.view(x.storage, x.shape, x.strides, x.offset)
        scale = mo.reduce_sum(np.abs(xa), axes) if op == abi.SUM else None
        assert_rel_sqrtk(host(out)[:max(int(np.prod(kept)), 1)], ref.storage[:max(int(np.prod(kept)), 1)], R,
                         None if scale is None else scale.reshape(-1), f"op {op:#x} {x.shape} {axes}")


def test_logsumexp_special_rows(cuda):
    x = hv(np.array([[0, 1, 2], [-np.inf, -np.inf, -np.inf], [np.inf, 0, 1], [np.nan, 0, 1],
                     [1000, 1000, -1000], [np.inf, np.nan, 0]], dtype=F), [6, 3])
    ref = out_like([6])
    rk.reduce(abi.LOGSUMEXP, x, [1], False, ref)
    out = gpu(out_like([6]))
    abi.reduce(abi.LOGSUMEXP, gpu(x), [1], out)
    assert_ulp(host(out), ref.storage, 2, "lse special")


def test_max_argmax_vs_oracle(cuda):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((300, 257)).astype(F)
    x[3, 7] = np.nan
    x[5, :] = -np.inf
    x[9, 4] = x[9, 200] = 50.0  # tie: first index wins
    for axis in (0, 1):
        for layout in (hv(x, x.shape), hv(np.ascontiguousarray(x.T), x.shape, [1, 300])):
            kept = [x.shape[1 - axis]]
            out = gpu(out_like(kept))
            abi.reduce(abi.MAX, gpu(layout), [axis], out)
            assert_bits(host(out), mo.reduce_max(x, [axis]), f"max axis {axis}")
            oi = gpu(out_like(kept, dtype=np.int64, fill=-1))
            abi.reduce(abi.ARGMAX, gpu(layout), [axis], oi)
            assert_bits(host(oi), mo.reduce_argmax(x, axis), f"argmax axis {axis}")


@pytest.mark.parametrize("op", [abi.SUM, abi.LOGSUMEXP, abi.MAX, abi.ARGMAX])
def test_column_reductions_beyond_the_exact_regime(cuda, op):
    """Reductions of a strided axis with a contiguous kept axis, large enough to
    leave the small exact path: [6000, 516] over axis 0 (a partial 128-column
    group, chunked) and [3, 2000, 388] over axis 1 (batched).  NaN, an all -inf
    row and a tie are planted for max/argmax.  A second call must give the same
    bits (deterministic merge order; the last-CTA merge counters re-arm)."""
    rng = np.random.default_rng(17)
    a = rng.standard_normal((6000, 516)).astype(F)
    b = rng.standard_normal((3, 2000, 388)).astype(F)
    if op in (abi.MAX, abi.ARGMAX):
        a[4000, 7] = np.nan
        a[17, :] = -np.inf
        a[100, 9] = a[5000, 9] = 60.0  # tie: the first index wins
        b[1, 1500, 3] = np.nan
        b[2, 10, 5] = b[2, 1999, 5] = 70.0
    for x, axis in ((a, 0), (b, 1)):
        kept = [e for d, e in enumerate(x.shape) if d != axis]
        view = hv(x, x.shape)
        if op == abi.ARGMAX:
            oi = gpu(out_like(kept, dtype=np.int64, fill=-1))
            abi.reduce(op, gpu(view), [axis], oi)
            assert_bits(host(oi), mo.reduce_argmax(x, axis).reshape(-1), f"argmax {x.shape} axis {axis}")
            continue
        out = gpu(out_like(kept))
        xv = gpu(view)
        abi.reduce(op, xv, [axis], out)
        again = gpu(out_like(kept))
        abi.reduce(op, xv, [axis], again)  # the chunk-merge counters re-arm: same bits again
        assert_bits(host(again), host(out), f"repeat {x.shape} axis {axis}")
        if op == abi.MAX:
            assert_bits(host(out), mo.reduce_max(x, [axis]).reshape(-1), f"max {x.shape} axis {axis}")
            continue
        ref = out_like(kept)
        rk.reduce(op, view, [axis], False, ref)
        scale = mo.reduce_sum(np.abs(x), [axis]).reshape(-1) if op == abi.SUM else None
        assert_rel_sqrtk(host(out), ref.storage, x.shape[axis], scale, f"op {op:#x} {x.shape} axis {axis}")


def test_log_softmax_vs_oracle(cuda):
    rng = np.random.default_rng(9)
    for shape, strides in (([37, 1000], None), ([512, 8192], None), ([100, 64], [1, 100])):
        x = hv(rng.uniform(-10, 10, int(np.prod(shape))).astype(F), shape, strides)
        xa = mo.view(x.storage, x.shape, x.strides, x.offset)
        out = gpu(out_like(shape))
        abi.log_softmax(gpu(x), 1, out)
        exp = mo.log_softmax(xa, 1).reshape(-1)
        # error of x - lse is that of lse (rel 1e-5*sqrt(K)) measured against |lse|
        lse = mo.reduce_logsumexp(xa, [1], keep_dim=True)
        scale = np.broadcast_to(np.abs(lse), xa.shape).reshape(-1)
        assert_rel_sqrtk(host(out), exp, shape[1], scale, f"log_softmax {shape}")


# ------------------------------------------------------------------------ GEMM --

def _gemm_check(a: rk.HostView, b: rk.HostView, algo):
    av = mo.view(a.storage, a.shape, a.strides, a.offset)
    bv = mo.view(b.storage, b.shape, b.strides, b.offset)
    exp = mo.matmul(av, bv)
    out = gpu(out_like(exp.shape))
    abi.matmul(gpu(a), gpu(b), out, algo)
    got = host(out)[: max(exp.size, 1)][: exp.size]
    scale = mo.matmul(np.abs(av), np.abs(bv)).reshape(-1)
    assert_rel_sqrtk(got, exp.reshape(-1), av.shape[-1], scale, f"matmul {a.shape}x{b.shape} algo {algo}")


@pytest.mark.parametrize("algo", [abi.GEMM_SIMT, abi.GEMM_AUTO])
def test_matmul_forms(cuda, algo):
    rng = np.random.default_rng(13)
    forms = [([7], [7]), ([33, 70], [70]), ([70], [70, 45]), ([129, 257], [257, 131]), ([3, 65, 40], [40, 33]),
             ([2, 1, 17, 19], [4, 19, 23]), ([5, 0], [0, 3]), ([0, 4], [4, 6])]
    for sa, sb in forms:
        a = hv(rng.standard_normal(int(np.prod(sa))).astype(F), sa)
        b = hv(rng.standard_normal(int(np.prod(sb))).astype(F), sb)
        if int(np.prod(sa)) == 0 or int(np.prod(sb)) == 0:
            exp = mo.matmul(np.zeros(sa, F), np.zeros(sb, F))
            out = gpu(out_like(exp.shape, fill=5.0))
            za = hv(np.zeros(max(int(np.prod(sa)), 1), F), sa)
            zb = hv(np.zeros(max(int(np.prod(sb)), 1), F), sb)
            abi.matmul(gpu(za), gpu(zb), out, algo)
            assert_bits(host(out)[: exp.size], exp.reshape(-1), f"empty matmul {sa}x{sb}")
            continue
        _gemm_check(a, b, algo)


@pytest.mark.parametrize("algo", [abi.GEMM_SIMT, abi.GEMM_AUTO])
def test_matmul_strided_operands(cuda, algo):
    rng = np.random.default_rng(17)
    M, N, K = 300, 260, 520
    a_st = rng.standard_normal(M * K + 3).astype(F)
    b_st = rng.standard_normal(N * K + 5).astype(F)
    _gemm_check(hv(a_st, [M, K], [K, 1], 3), hv(b_st, [K, N], [1, K], 5), algo)       # Linear: x @ W^T
    _gemm_check(hv(a_st, [M, K], [1, M], 0), hv(b_st, [K, N], [N, 1], 0), algo)       # A^T @ B (dW)
    _gemm_check(hv(a_st, [M, K], [1, M], 0), hv(b_st, [K, N], [1, K], 0), algo)       # both transposed


def test_matmul_matches_reference_kernel(cuda):
    """Same inputs through the compiled reference matmul kernel (not only the oracle)."""
    rng = np.random.default_rng(19)
    a = hv(rng.standard_normal(64 * 96).astype(F), [64, 96])
    b = hv(rng.standard_normal(96 * 80).astype(F), [96, 80], [1, 96])
    ref = out_like([64, 80])
    rk.matmul(a, b, ref)
    out = gpu(out_like([64, 80]))
    abi.matmul(gpu(a), gpu(b), out)
    scale = mo.matmul(np.abs(mo.view(a.storage, a.shape, a.strides, 0)), np.abs(mo.view(b.storage, b.shape, b.strides, 0)))
    assert_rel_sqrtk(host(out), ref.storage, 96, scale.reshape(-1), "matmul vs reference kernel")


# ---------------------------------------------------------- indexing and copies --

def test_row_gather_and_scatter_add_bit_exact(cuda):
    """The config-4 shape at small size: Int64 row indices broadcast along the row."""
    rng = np.random.default_rng(23)
    rows, width = 4096, 64
    table = rng.standard_normal(rows * width).astype(F)
    idx_col = rng.integers(0, rows, rows).astype(np.int64)
    idx = hv(idx_col, [rows, width], [1, 0])  # broadcast_to([rows, width]) of an [rows, 1] tensor
    ref = out_like([rows, width])
    rk.gather(hv(table, [rows, width]), idx, 0, ref)
    out = gpu(out_like([rows, width]))
    abi.gather(gpu(hv(table, [rows, width])), gpu(idx), 0, out)
    assert_bits(host(out), ref.storage, "row gather")
    upd = np.floor(rng.uniform(-8, 8, rows * width)).astype(F)
    ref = out_like([rows, width])
    rk.gather_scatter_add(hv(upd, [rows, width]), idx, 0, ref)
    out = gpu(out_like([rows, width]))
    abi.gather_scatter_add(gpu(hv(upd, [rows, width])), gpu(idx), 0, out)
    assert_bits(host(out), ref.storage, "row scatter-add (duplicate indices)")


def test_generic_gather_scatter_and_int64(cuda):
    rng = np.random.default_rng(29)
    src = rng.standard_normal(6 * 5 * 4).astype(F)
    idx = rng.integers(0, 5, 6 * 7 * 4).astype(np.int64)
    ref = out_like([6, 7, 4])
    rk.gather(hv(src, [6, 5, 4]), hv(idx, [6, 7, 4]), 1, ref)
    out = gpu(out_like([6, 7, 4]))
    abi.gather(gpu(hv(src, [6, 5, 4])), gpu(hv(idx, [6, 7, 4])), 1, out)
    assert_bits(host(out), ref.storage, "gather axis 1")
    src_i = rng.integers(-1000, 1000, 30).astype(np.int64)
    idx_i = rng.integers(0, 6, 8 * 5).astype(np.int64)
    ref = out_like([8, 5], dtype=np.int64, fill=-1)
    rk.gather(hv(src_i, [6, 5]), hv(idx_i, [8, 5]), 0, ref)
    out = gpu(out_like([8, 5], dtype=np.int64, fill=-1))
    abi.gather(gpu(hv(src_i, [6, 5])), gpu(hv(idx_i, [8, 5])), 0, out)
    assert_bits(host(out), ref.storage, "int64 gather")
    upd = np.floor(rng.uniform(-8, 8, 6 * 7 * 4)).astype(F)
    ref = out_like([6, 5, 4])
    rk.gather_scatter_add(hv(upd, [6, 7, 4]), hv(idx, [6, 7, 4]), 1, ref)
    out = gpu(out_like([6, 5, 4]))
    abi.gather_scatter_add(gpu(hv(upd, [6, 7, 4])), gpu(hv(idx, [6, 7, 4])), 1, out)
    assert_bits(host(out), ref.storage, "scatter-add axis 1")


def test_gather_out_of_range_sets_error_word(cuda):
    src = hv(np.arange(6, dtype=F), [2, 3])
    idx = hv(np.array([0, 3, 1, 1], dtype=np.int64), [2, 2])
    with pytest.raises(IndexError):
        rk.gather(src, idx, 1, out_like([2, 2]))
    out = gpu(out_like([2, 2]))
    abi.gather(gpu(src), gpu(idx), 1, out)
    with pytest.raises(IndexError):
        abi.check_device_errors(0)
    abi.check_device_errors(0)  # cleared after the report


def test_copies_and_concat(cuda):
    rng = np.random.default_rng(31)
    st = rng.standard_normal(130 * 70 + 9).astype(F)
    for src in (hv(st, [130, 70], [1, 130], 0), hv(st, [65, 70], [-140, 2], 64 * 140), hv(st, [130, 70], [70, 1], 9)):
        ref = out_like(src.shape, offset=1)
        rk.copy(src, ref)
        out = gpu(out_like(src.shape, offset=1))
        abi.copy(gpu(src), out)
        assert_bits(host(out), ref.storage, f"copy {src.strides}")
    ist = rng.integers(-9, 9, 40 * 30).astype(np.int64)
    src = hv(ist, [40, 30], [1, 40])
    ref = out_like([40, 30], dtype=np.int64, fill=0)
    rk.copy(src, ref)
    out = gpu(out_like([40, 30], dtype=np.int64, fill=0))
    abi.copy(gpu(src), out)
    assert_bits(host(out), ref.storage, "int64 transposed copy")
    parts = [hv(rng.standard_normal(64 * 96).astype(F), [64, 96]) for _ in range(4)]
    for axis in (0, 1):
        shape = [64 * 4, 96] if axis == 0 else [64, 96 * 4]
        ref = out_like(shape)
        rk.concat(parts, axis, ref)
        out = gpu(out_like(shape))
        abi.concat([gpu(p) for p in parts], axis, out)
        assert_bits(host(out), ref.storage, f"concat axis {axis}")


def test_index_scatter_slice_and_select(cuda):
    rng = np.random.default_rng(37)
    for select, axis, start, stop, step, in_shape, out_shape in (
        (False, 1, 1, None, 3, [4, 5], [4, 15]),
        (False, 0, None, None, -1, [6, 3], [6, 3]),
        (True, 2, None, None, 2, [3, 4], [3, 4, 5]),
    ):
        x = hv(rng.standard_normal(int(np.prod(in_shape))).astype(F), in_shape)
        ref = out_like(out_shape, offset=2)
        rk.index_scatter(x, ref, select=select, axis=axis, start=start, stop=stop, step_or_index=step)
        o = out_like(out_shape, offset=2)
        shape, strides, offset = rk.index_layout(o, select=select, axis=axis, start=start, stop=stop,
                                                 step_or_index=step)
        out = gpu(o)
        abi.index_scatter(gpu(x), abi.View(out.storage, shape, strides, offset), out)
        assert_bits(host(out), ref.storage, f"index scatter {select} {axis} {step}")


# ---------------------------------------------------------------------- creation --

def test_fill_and_random_vs_reference(cuda):
    o = out_like([3, 5], offset=1)
    abi.fill(gpu(o), 2.5)
    out = gpu(out_like([3, 5], offset=1))
    abi.fill(out, 2.5)
    ref = out_like([3, 5], offset=1)
    rk.fill(ref, 2.5)
    assert_bits(host(out), ref.storage, "fill f32")
    out = gpu(out_like([7], dtype=np.int64, fill=0))
    abi.fill(out, -(2 ** 40) - 3)
    assert_bits(host(out), np.full(7, -(2 ** 40) - 3, dtype=np.int64), "fill i64")
    key = mo.key_split(mo.key_fold_in(mo.random_key(2026), 3))
    for n in (1, 7, 4096, 1 << 20):
        for which in ("uniform", "normal"):
            ref = out_like([n], fill=0.0)
            out = gpu(out_like([n], fill=0.0))
            if which == "uniform":
                rk.uniform(ref, -1.0, 1.0, key[0])
                abi.uniform(out, -1.0, 1.0, key[0])
                assert_bits(host(out), ref.storage, f"uniform {n}")
            else:
                rk.normal(ref, 0.0, 1.0, key[1])
                abi.normal(out, 0.0, 1.0, key[1])
                assert_ulp(host(out), ref.storage, 1, f"normal {n}")


def test_descriptor_validation_rejects_out_of_bounds_views(cuda):
    import torch

    st = torch.zeros(10, device="cuda")
    with pytest.raises(IndexError):
        abi.unary(abi.EXP, abi.View(st, (4, 4), (4, 1), 0), abi.View(torch.zeros(16, device="cuda"), (4, 4), (4, 1), 0))
    with pytest.raises(ValueError):
        abi.binary(abi.ADD, abi.View(st, (2, 3), (3, 1), 0), abi.View(st, (2, 2), (2, 1), 0),
                   abi.View(torch.zeros(6, device="cuda"), (2, 3), (3, 1), 0))


def test_exact_simt_gemm_is_bit_identical_to_reference(cuda):
    """MTC_GEMM_SIMT rounds like the CPU (float product, float sum, k ascending)."""
    rng = np.random.default_rng(41)
    # (lhs shape, rhs shape, lhs transposed view, rhs transposed view); the small
    # ones take the shared-memory staged kernel (K >= 32, a warp of outputs per
    # tile), the spiral model's weight gradients among them (xT . G, K = 300)
    cases = (([33, 70], [70, 45], False, False), ([129, 257], [257, 131], False, True), ([7], [7, 3], False, False),
             ([2, 3, 17, 19], [19, 23], False, False), ([64, 300], [300, 64], True, False),
             ([300, 64], [64, 64], False, True), ([2, 300], [300, 64], True, False), ([8, 1000], [1000, 8], False, True),
             ([3, 40, 300], [300, 24], False, False))
    for sa, sb, at, bt in cases:
        if at:
            a = hv(rng.standard_normal(int(np.prod(sa))).astype(F), sa, [1, sa[0]])
        else:
            a = hv(rng.standard_normal(int(np.prod(sa))).astype(F), sa)
        if bt:
            b = hv(rng.standard_normal(int(np.prod(sb))).astype(F), sb, [1, sb[0]])
        else:
            b = hv(rng.standard_normal(int(np.prod(sb))).astype(F), sb)
        exp = mo.matmul(mo.view(a.storage, a.shape, a.strides, 0), mo.view(b.storage, b.shape, b.strides, 0))
        out = gpu(out_like(exp.shape))
        abi.matmul(gpu(a), gpu(b), out, abi.GEMM_SIMT)
        assert_bits(host(out)[: exp.size], exp.reshape(-1), f"exact SIMT {sa}x{sb}")


def test_small_sums_are_bit_identical_to_reference(cuda):
    rng = np.random.default_rng(43)
    # reductions of at most 8192 elements per output and 2^21 in all take the
    # reference's sequential order (the spiral model's bias gradients and loss mean)
    cases = [(hv(rng.standard_normal(60 * 64).astype(F), [60, 64]), axes) for axes in ([0], [1], [0, 1])]
    cases += [
        (hv(rng.standard_normal(300 * 64).astype(F), [300, 64]), [0]),          # bias gradient, staged
        (hv(rng.standard_normal(300 * 3).astype(F), [300, 3]), [0]),            # three long columns
        (hv(rng.standard_normal(300).astype(F), [300]), [0]),                   # a loss mean's sum
        (hv(rng.standard_normal(64 * 300).astype(F), [300, 64], [1, 300]), [0]),  # transposed storage
        (hv(rng.standard_normal(6 * 50 * 8).astype(F), [6, 50, 8]), [0, 2]),     # two reduced axes
        (hv(rng.standard_normal(300 * 10).astype(F), [300, 10]), [1]),          # short rows: per-thread kernel
    ]
    for x, axes in cases:
        kept = [e for d, e in enumerate(x.shape) if d not in axes]
        ref = out_like(kept)
        rk.reduce(abi.SUM, x, axes, False, ref)
        out = gpu(out_like(kept))
        abi.reduce(abi.SUM, gpu(x), axes, out)
        assert_bits(host(out)[: ref.storage.size], ref.storage, f"small sum {x.shape} {axes}")
