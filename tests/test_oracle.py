"""Pins the numpy oracle (oracle/mt_oracle.py) to the reference: its known-answer
tests (tests/golden/known_answers.json) and the compiled reference's outputs on
seeded cases (tests/golden/ref_cases.npz, made by tests/golden/make_golden.py).
CPU only."""
import json
from pathlib import Path

import numpy as np
import pytest

from helpers import assert_bits, assert_ulp
from oracle import mt_oracle as mo

GOLDEN = Path(__file__).resolve().parent / "golden"
KA = json.loads((GOLDEN / "known_answers.json").read_text())
CASES = np.load(GOLDEN / "ref_cases.npz")

F = np.float32


def _view(spec, dtype=F):
    st = np.asarray(spec["storage"], dtype=np.int64 if spec.get("dtype") == "int64" else dtype)
    return st, mo.view(st, spec["shape"], spec["strides"], spec["offset"])


def _write(out_spec, values):
    st = np.asarray(out_spec["storage"], dtype=F).copy()
    shape = out_spec["shape"]
    idx = np.indices(shape).reshape(len(shape), -1)
    offs = out_spec["offset"] + sum(idx[d] * out_spec["strides"][d] for d in range(len(shape)))
    st[offs] = np.asarray(values, dtype=F).reshape(-1)
    return st


@pytest.mark.parametrize("name", sorted(KA))
def test_known_answers(name):
    case = KA[name]
    op = case["op"]
    if op == "add":
        _, a = _view(case["lhs"])
        _, b = _view(case["rhs"])
        got = _write(case["out"], mo.binary(mo.ADD, a, b))
    elif op == "sum":
        _, x = _view(case["in"])
        got = _write(case["out"], mo.reduce_sum(x, case["axes"]))
    elif op == "matmul":
        _, a = _view(case["lhs"])
        _, b = _view(case["rhs"])
        got = _write(case["out"], mo.matmul(a, b))
    elif op == "copy":
        _, x = _view(case["in"])
        got = _write(case["out"], x)
    elif op == "concat":
        parts = [_view(s)[1] for s in case["inputs"]]
        got = _write(case["out"], mo.concatenate(parts, case["axis"]))
    elif op == "gather":
        _, src = _view(case["src"])
        _, idx = _view(case["idx"])
        got = _write(case["out"], mo.gather(src, case["axis"], idx))
    elif op == "fill":
        got = _write(case["out"], np.full(case["out"]["shape"], case["value"], dtype=F))
    elif op == "index_scatter":
        _, x = _view(case["in"])
        out = np.zeros(case["out"]["shape"], dtype=F)
        sl = [slice(None)] * out.ndim
        if case["select"]:
            sl[case["axis"]] = case["step_or_index"]
        else:
            sl[case["axis"]] = slice(case["start"], case["stop"], case["step_or_index"])
        out[tuple(sl)] = x
        got = _write(case["out"], out)
    elif op == "cross_entropy":
        logits = np.asarray(case["logits"], dtype=F)
        targets = np.asarray(case["targets"], dtype=np.int64)
        ax = case["class_axis"]
        moved = np.moveaxis(logits, ax, -1)
        loss = mo.cross_entropy(moved, targets)
        assert abs(float(loss) - case["expected_loss"]) <= case["tolerance"]
        # analytic gradient of the mean CE: (softmax - onehot) / N along the class axis
        sm = np.exp(moved - mo.reduce_logsumexp(moved, [moved.ndim - 1], keep_dim=True))
        onehot = np.eye(moved.shape[-1], dtype=F)[targets]
        grad = np.moveaxis((sm - onehot) / targets.size, -1, ax)
        np.testing.assert_allclose(grad.reshape(-1), case["expected_gradient"], atol=1e-6, rtol=1e-5)
        return
    elif op == "adamw":
        p = np.asarray(case["params"], dtype=F)
        g = np.asarray(case["grads"], dtype=F)
        z = np.zeros_like(p)
        new_p, _, _ = mo.adamw_update(p, g, z, z, case["lr"], case["weight_decay"], case["beta1"], case["beta2"],
                                      case["eps"], 0)
        np.testing.assert_allclose(new_p, case["expected"], atol=case["tolerance"])
        return
    elif op == "adamw2":
        p = np.asarray([case["param"]], dtype=F)
        m = v = np.zeros(1, dtype=F)
        for step, g in enumerate(case["grads"]):
            p, m, v = mo.adamw_update(p, np.asarray([g], dtype=F), m, v, case["lr"], case["weight_decay"],
                                      case["beta1"], case["beta2"], case["eps"], step)
        np.testing.assert_allclose(p[0], case["expected"], atol=case["tolerance"])
        return
    else:
        pytest.fail(f"unhandled known answer {op}")
    assert_bits(got, np.asarray(case["expected"], dtype=F), name)


UNARY_ULP = {mo.ABS: 0, mo.SIGN: 0, mo.NEGATE: 0, mo.SQRT: 0, mo.EXP: 1, mo.LOG: 1, mo.TANH: 2, mo.SIGMOID: 2}


@pytest.mark.parametrize("op", sorted(UNARY_ULP))
def test_unary_matches_reference(op):
    c = lambda k: CASES[f"unary_{op:#x}/{k}"]
    x = mo.view(c("x_storage"), c("x_shape"), c("x_strides"), int(c("x_offset")))
    expected = c("out_storage")[1:17].reshape(4, 4)
    assert_ulp(mo.unary(op, x), expected, UNARY_ULP[op], f"unary {op:#x}")
    s = lambda k: CASES[f"unary_special_{op:#x}/{k}"]
    assert_ulp(mo.unary(op, s("x")), s("out"), UNARY_ULP[op], f"unary special {op:#x}")


BINARY_ULP = {mo.ADD: 0, mo.SUBTRACT: 0, mo.MULTIPLY: 0, mo.DIVIDE: 0, mo.LOGADDEXP: 1}


@pytest.mark.parametrize("op", sorted(BINARY_ULP))
def test_binary_matches_reference(op):
    c = lambda k: CASES[f"binary_{op:#x}/{k}"]
    a = mo.view(c("a_storage"), [5, 6], [1, 10], 2)
    b = mo.view(c("b_storage"), [1, 6], [6, 1], 0)
    assert_ulp(mo.binary(op, a, b).reshape(-1), c("out"), BINARY_ULP[op], f"binary {op:#x}")
    s = lambda k: CASES[f"binary_special_{op:#x}/{k}"]
    assert_ulp(mo.binary(op, s("a"), s("b")), s("out"), BINARY_ULP[op], f"binary special {op:#x}")


@pytest.mark.parametrize("axes", [[0], [1], [2], [0, 2], [0, 1, 2]])
def test_reductions_match_reference(axes):
    key = "_".join(map(str, axes))
    x = mo.view(CASES[f"reduce_sum_{key}/x_storage"], [4, 5, 6], [60, 1, 5], 7)
    assert_bits(mo.reduce_sum(x, axes).reshape(-1), CASES[f"reduce_sum_{key}/out"], f"sum {axes}")
    assert_ulp(mo.reduce_logsumexp(x, axes).reshape(-1), CASES[f"reduce_lse_{key}/out"], 2, f"lse {axes}")


def test_logsumexp_special_rows():
    x = CASES["reduce_lse_special/x"].reshape(5, 3)
    assert_ulp(mo.reduce_logsumexp(x, [1]), CASES["reduce_lse_special/out"], 1, "lse special")


@pytest.mark.parametrize("i", range(6))
def test_matmul_forms_bit_exact(i):
    a, b, out = (CASES[f"matmul_{i}/{k}"] for k in ("a", "b", "out"))
    assert_bits(mo.matmul(a, b), out, f"matmul form {i}")


def test_matmul_transposed_rhs_bit_exact():
    a = CASES["matmul_transposed_rhs/a"]
    b = mo.view(CASES["matmul_transposed_rhs/b_storage"], [7, 4], [1, 7], 0)
    assert_bits(mo.matmul(a, b).reshape(-1), CASES["matmul_transposed_rhs/out"], "matmul B^T")


def test_gather_and_scatter_add_bit_exact():
    src, idx = CASES["gather_axis0/src"], CASES["gather_axis0/idx"]
    assert_bits(mo.gather(src, 0, idx).reshape(-1), CASES["gather_axis0/out"], "gather axis 0")
    idx1 = CASES["gather_axis1/idx"]
    assert_bits(mo.gather(src, 1, idx1).reshape(-1), CASES["gather_axis1/out"], "gather axis 1")
    upd = CASES["scatter_add_axis0/upd"]
    assert_bits(mo.gather_scatter_add(upd, idx, 0, (6, 5)).reshape(-1), CASES["scatter_add_axis0/out"], "scatter")


def test_gather_rejects_out_of_range():
    with pytest.raises(IndexError):
        mo.gather(np.zeros((2, 2), F), 0, np.array([[0, 2]]))


@pytest.mark.parametrize("axis", [0, 1])
def test_concat_bit_exact(axis):
    parts = [CASES[f"concat_axis{axis}/p{i}"] for i in range(3)]
    assert_bits(mo.concatenate(parts, axis).reshape(-1), CASES[f"concat_axis{axis}/out"], f"concat {axis}")


def test_key_derivation_matches_reference():
    base = tuple(int(x) for x in CASES["keys/base"])
    fold = mo.key_fold_in(base, 7)
    assert fold == tuple(int(x) for x in CASES["keys/fold7"])
    split = mo.key_split(fold)
    assert [tuple(k) for k in split] == [tuple(int(x) for x in row) for row in CASES["keys/split"]]


@pytest.mark.parametrize("n", [1, 5, 4099])
def test_random_creation_matches_reference(n):
    ukey = tuple(int(x) for x in CASES[f"random_{n}/ukey"])
    nkey = tuple(int(x) for x in CASES[f"random_{n}/nkey"])
    assert_bits(mo.uniform(n, -2.0, 3.0, ukey), CASES[f"random_{n}/uniform"], "uniform")
    assert_ulp(mo.normal(n, 0.5, 2.0, nkey), CASES[f"random_{n}/normal"], 1, "normal")


# ---- ops with no reference kernel (max, argmax, log-softmax): hand answers ----

NINF = F(-np.inf)


def test_max_known_answers():
    x = np.array([[1, 3, 2], [NINF, -5, NINF], [7, np.nan, 9]], dtype=F)
    assert_bits(mo.reduce_max(x, [1]), np.array([3, -5, np.nan], dtype=F), "max axis 1")
    assert_bits(mo.reduce_max(x, [0]), np.array([7, np.nan, 9], dtype=F), "max axis 0")
    assert mo.reduce_max(x, [1], keep_dim=True).shape == (3, 1)
    assert_bits(mo.reduce_max(np.zeros((2, 0), F), [1]), np.array([NINF, NINF], dtype=F), "empty axis")
    assert_bits(mo.reduce_max(x[:2], [0, 1]), np.array(3, dtype=F), "all axes")


def test_argmax_known_answers():
    x = np.array([[2, 5, 5, 1], [1, np.nan, 9, np.nan], [NINF, NINF, NINF, NINF]], dtype=F)
    # first maximum wins a tie; the first NaN is the maximum; an all -inf row gives 0
    assert_bits(mo.reduce_argmax(x, 1), np.array([1, 1, 0], dtype=np.int64), "argmax axis 1")
    assert_bits(mo.reduce_argmax(x, 0), np.array([0, 1, 1, 1], dtype=np.int64), "argmax axis 0")
    assert mo.reduce_argmax(x, 0, keep_dim=True).shape == (1, 4)


def test_log_softmax_known_answers():
    # softmax of [0, ln 2, ln 3] is [1/6, 2/6, 3/6]
    x = np.array([[0, np.log(2), np.log(3)], [NINF, 0, NINF]], dtype=F)
    want = np.array([np.log([1 / 6, 1 / 3, 1 / 2]), [-np.inf, 0, -np.inf]], dtype=F)
    assert_ulp(mo.log_softmax(x, 1), want, 2, "log_softmax")
    # large equal logits stay finite; the composite x - logsumexp(x) rounds
    # logsumexp near 1001, so the error is one spacing there, not ulps of ln 3
    big = mo.log_softmax(np.full((1, 3), 1000, F), 1)
    assert np.all(np.abs(big.astype(np.float64) + np.log(3)) <= np.spacing(F(1001)))
    # the composite: x - logsumexp(x) with the reference's logsumexp, bit for bit
    y = CASES["reduce_lse_special/x"].reshape(5, 3)
    with np.errstate(invalid="ignore"):
        composite = (y - mo.reduce_logsumexp(y, [1], keep_dim=True)).astype(F)
    assert_bits(mo.log_softmax(y, 1), composite, "composite")
