"""Generates the golden fixtures of the parity tests.

known_answers.json  Known-answer vectors of the MiniTensor reference's own test
                    suite, transcribed with the file:line they come from.
ref_cases.npz       Seeded small cases for every kernel family, evaluated by the
                    compiled reference (oracle/_ref/libmtref.so, built from the
                    unmodified sources by oracle/Makefile).

Run from the repository root after `make -C oracle`:
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import refkernels as rk  # noqa: E402
from oracle import mt_oracle as mo  # noqa: E402

OUT = Path(__file__).resolve().parent

F = np.float32


def known_answers() -> dict:
    seq = [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
    return {
        "elementwise_add_broadcast_negative_stride": {
            "source": "tests/tensor/backend/cpu/kernels/elementwise_test.cpp:17-42",
            "op": "add",
            "lhs": {"storage": seq, "shape": [2, 3], "strides": [-3, 1], "offset": 3},
            "rhs": {"storage": [10.0, 20.0, 30.0], "shape": [1, 3], "strides": [3, 1], "offset": 0},
            "out": {"storage": [-1.0] * 7, "shape": [2, 3], "strides": [3, 1], "offset": 1},
            "expected": [-1.0, 14.0, 25.0, 36.0, 11.0, 22.0, 33.0],
        },
        "sum_negative_stride_output_offset": {
            "source": "tests/tensor/backend/cpu/kernels/reduction_test.cpp:17-37",
            "op": "sum",
            "axes": [1],
            "in": {"storage": seq, "shape": [2, 3], "strides": [-3, 1], "offset": 3},
            "out": {"storage": [-1.0] * 4, "shape": [2], "strides": [1], "offset": 1},
            "expected": [-1.0, 15.0, 6.0, -1.0],
        },
        "matmul_output_offset": {
            "source": "tests/tensor/backend/cpu/kernels/linalg_test.cpp:17-42",
            "op": "matmul",
            "lhs": {"storage": seq, "shape": [2, 3], "strides": [3, 1], "offset": 0},
            "rhs": {"storage": [7.0, 8.0, 9.0, 10.0, 11.0, 12.0], "shape": [3, 2], "strides": [2, 1], "offset": 0},
            "out": {"storage": [-1.0] * 6, "shape": [2, 2], "strides": [2, 1], "offset": 1},
            "expected": [-1.0, 58.0, 64.0, 139.0, 154.0, -1.0],
        },
        "reshape_copy_negative_stride": {
            "source": "tests/tensor/backend/cpu/kernels/copy_test.cpp:22-42",
            "op": "copy",
            "in": {"storage": seq, "shape": [2, 3], "strides": [-3, 1], "offset": 3},
            "out": {"storage": [-1.0] * 7, "shape": [2, 3], "strides": [3, 1], "offset": 1},
            "expected": [-1.0, 4.0, 5.0, 6.0, 1.0, 2.0, 3.0],
        },
        "concat_strided_and_empty_sections": {
            "source": "tests/tensor/backend/cpu/kernels/copy_test.cpp:44-72",
            "op": "concat",
            "axis": 1,
            "inputs": [
                {"storage": [1.0, 4.0], "shape": [2, 1], "strides": [1, 1], "offset": 0},
                {"storage": [], "shape": [2, 0], "strides": [1, 1], "offset": 0},
                {"storage": [2.0, 5.0, 3.0, 6.0], "shape": [2, 2], "strides": [1, 2], "offset": 0},
            ],
            "out": {"storage": [-1.0] * 7, "shape": [2, 3], "strides": [3, 1], "offset": 1},
            "expected": [-1.0, 1.0, 2.0, 3.0, 4.0, 5.0, 6.0],
        },
        "index_scatter_slice_negative_step": {
            "source": "tests/tensor/backend/cpu/kernels/copy_test.cpp:74-95",
            "op": "index_scatter",
            "select": False, "axis": 1, "start": None, "stop": None, "step_or_index": -2,
            "in": {"storage": seq, "shape": [2, 3], "strides": [3, 1], "offset": 0},
            "out": {"storage": [-1.0] * 11, "shape": [2, 5], "strides": [5, 1], "offset": 1},
            "expected": [-1.0, 3.0, 0.0, 2.0, 0.0, 1.0, 6.0, 0.0, 5.0, 0.0, 4.0],
        },
        "index_scatter_select": {
            "source": "tests/tensor/backend/cpu/kernels/copy_test.cpp:97-117",
            "op": "index_scatter",
            "select": True, "axis": 1, "start": None, "stop": None, "step_or_index": 1,
            "in": {"storage": [1.0, 2.0, 3.0, 4.0], "shape": [2, 2], "strides": [2, 1], "offset": 0},
            "out": {"storage": [-1.0] * 13, "shape": [2, 3, 2], "strides": [6, 2, 1], "offset": 1},
            "expected": [-1.0, 0.0, 0.0, 1.0, 2.0, 0.0, 0.0, 0.0, 0.0, 3.0, 4.0, 0.0, 0.0],
        },
        "gather_negative_stride_output_offset": {
            "source": "tests/tensor/backend/cpu/kernels/copy_test.cpp:119-143",
            "op": "gather",
            "axis": 1,
            "src": {"storage": seq, "shape": [2, 3], "strides": [-3, 1], "offset": 3},
            "idx": {"storage": [2, 0, 1, 1], "shape": [2, 2], "strides": [2, 1], "offset": 0, "dtype": "int64"},
            "out": {"storage": [-1.0] * 6, "shape": [2, 2], "strides": [2, 1], "offset": 1},
            "expected": [-1.0, 6.0, 4.0, 2.0, 2.0, -1.0],
        },
        "full_output_offset": {
            "source": "tests/tensor/backend/cpu/kernels/creation_test.cpp:20-40",
            "op": "fill",
            "value": 2.5,
            "out": {"storage": [-10.0] * 7, "shape": [2, 3], "strides": [3, 1], "offset": 1},
            "expected": [-10.0, 2.5, 2.5, 2.5, 2.5, 2.5, 2.5],
        },
        "cross_entropy_class_axis_0": {
            "source": "tests/nn/public/loss_test.cpp:66-78",
            "op": "cross_entropy",
            "logits": [[2.0, 0.0], [1.0, 1.0], [0.0, 2.0]],
            "targets": [0, 1],
            "class_axis": 0,
            "expected_loss": 0.9076060,
            "expected_gradient": [-0.1673795, 0.0450153, 0.1223642, -0.3776358, 0.0450153, 0.3326205],
            "tolerance": 1e-6,
        },
        "adamw_one_step": {
            "source": "tests/nn/public/adamw_test.cpp:43-61",
            "op": "adamw",
            "params": [1.0, -2.0], "grads": [2.0, -4.0],
            "lr": 0.1, "weight_decay": 0.2, "beta1": 0.5, "beta2": 0.25, "eps": 0.01,
            "expected": [float(F(1.0) - F(0.1) * F(0.2)) * 1.0 - 0.1 * 2.0 / 2.01,
                         float(F(1.0) - F(0.1) * F(0.2)) * -2.0 + 0.1 * 4.0 / 4.01],
            "tolerance": 1e-6,
        },
        "adamw_two_steps": {
            "source": "tests/nn/public/adamw_test.cpp:63-95",
            "op": "adamw2",
            "param": 1.0, "grads": [2.0, 1.0],
            "lr": 0.1, "weight_decay": 0.2, "beta1": 0.5, "beta2": 0.25, "eps": 0.01,
            "expected": 0.98 * (0.98 - 0.1 * 2.0 / 2.01) - 0.1 * (1.0 / 0.75) / (np.sqrt(1.5 / 0.9375) + 0.01),
            "tolerance": 1e-6,
        },
    }


def _storage(rng, n, dtype=np.float32, kind="normal"):
    if dtype == np.int64:
        return rng.integers(0, 5, size=n).astype(np.int64)
    if kind == "wide":
        return rng.uniform(-30, 30, size=n).astype(F)
    if kind == "positive":
        return rng.uniform(0.01, 10, size=n).astype(F)
    return rng.standard_normal(n).astype(F)


def _hv(storage, shape, strides, offset):
    return rk.HostView(storage, tuple(shape), tuple(strides), offset)


def _pack(cases: dict, name: str, **arrays):
    for k, v in arrays.items():
        cases[f"{name}/{k}"] = np.asarray(v)


def ref_cases() -> dict:
    rng = np.random.default_rng(20261201)
    cases: dict = {}
    special = np.array([0.0, -0.0, 1.0, -1.0, 1e-30, -1e-30, 88.0, -88.0, 1000.0, -1000.0, np.inf, -np.inf, np.nan],
                       dtype=F)
    # unary: contiguous special values + a strided random view
    for op in (mo.ABS, mo.SIGN, mo.NEGATE, mo.EXP, mo.LOG, mo.SQRT, mo.TANH, mo.SIGMOID):
        kind = "positive" if op in (mo.LOG, mo.SQRT) else "wide"
        st = np.concatenate([special, _storage(rng, 51, kind=kind)])
        x = _hv(st, [4, 4], [-16, 3], 48)  # reversed rows, stride-3 columns
        out_st = np.full(17, -7.0, dtype=F)
        out = _hv(out_st, [4, 4], [4, 1], 1)
        rk.unary(op, x, out)
        _pack(cases, f"unary_{op:#x}", x_storage=st, out_storage=out_st, x_shape=x.shape, x_strides=x.strides,
              x_offset=x.offset)
        xs = _hv(special.copy(), [13], [1], 0)
        o2 = np.zeros(13, dtype=F)
        rk.unary(op, xs, _hv(o2, [13], [1], 0))
        _pack(cases, f"unary_special_{op:#x}", x=special, out=o2)
    # binary with broadcasting (row and column operands) and a transposed view
    for op in (mo.ADD, mo.SUBTRACT, mo.MULTIPLY, mo.DIVIDE, mo.LOGADDEXP):
        a_st = _storage(rng, 60, kind="wide")
        b_st = _storage(rng, 6, kind="wide")
        a = _hv(a_st, [5, 6], [1, 10], 2)  # transposed view
        b = _hv(b_st, [1, 6], [6, 1], 0)
        out_st = np.zeros(30, dtype=F)
        rk.binary(op, a, b, _hv(out_st, [5, 6], [6, 1], 0))
        _pack(cases, f"binary_{op:#x}", a_storage=a_st, b_storage=b_st, out=out_st)
        sa, sb = np.meshgrid(special, special)
        sa, sb = sa.reshape(-1).copy(), sb.reshape(-1).copy()
        o2 = np.zeros(sa.size, dtype=F)
        rk.binary(op, _hv(sa, [sa.size], [1], 0), _hv(sb, [sb.size], [1], 0), _hv(o2, [sa.size], [1], 0))
        _pack(cases, f"binary_special_{op:#x}", a=sa, b=sb, out=o2)
    # reductions over several axis sets of a strided 3-D view
    x_st = _storage(rng, 400)
    for op, name in ((0x0301, "sum"), (0x0302, "lse")):
        for axes in ([0], [1], [2], [0, 2], [0, 1, 2]):
            x = _hv(x_st, [4, 5, 6], [60, 1, 5], 7)
            kept = [e for d, e in enumerate(x.shape) if d not in axes]
            out_st = np.zeros(max(int(np.prod(kept)), 1), dtype=F)
            rk.reduce(op, x, axes, False, _hv(out_st, kept, mo_strides(kept), 0))
            _pack(cases, f"reduce_{name}_{'_'.join(map(str, axes))}", x_storage=x_st, out=out_st)
    lse_special = np.array([[0, 1, 2], [-np.inf, -np.inf, -np.inf], [np.inf, 0, 1], [np.nan, 0, 1],
                            [1000, 1000, -1000]], dtype=F).reshape(-1)
    out_st = np.zeros(5, dtype=F)
    rk.reduce(0x0302, _hv(lse_special, [5, 3], [3, 1], 0), [1], False, _hv(out_st, [5], [1], 0))
    _pack(cases, "reduce_lse_special", x=lse_special, out=out_st)
    # matmul: all vector/matrix forms, batch broadcast, transposed operands
    forms = [
        ([7], [7]), ([3, 7], [7]), ([7], [7, 4]), ([3, 7], [7, 4]), ([2, 3, 7], [7, 4]), ([2, 1, 3, 7], [5, 7, 4]),
    ]
    for i, (sa, sb) in enumerate(forms):
        a = rng.standard_normal(sa).astype(F)
        b = rng.standard_normal(sb).astype(F)
        out = mo.matmul(a, b)
        out_st = np.zeros(max(out.size, 1), dtype=F)
        rk.matmul(rk.HostView.of(a), rk.HostView.of(b), _hv(out_st, out.shape, mo_strides(out.shape), 0))
        _pack(cases, f"matmul_{i}", a=a, b=b, out=out_st.reshape(out.shape) if out.size else out)
    bt_st = rng.standard_normal(7 * 4).astype(F)
    a = rng.standard_normal((3, 7)).astype(F)
    out_st = np.zeros(12, dtype=F)
    rk.matmul(rk.HostView.of(a), _hv(bt_st, [7, 4], [1, 7], 0), _hv(out_st, [3, 4], [4, 1], 0))
    _pack(cases, "matmul_transposed_rhs", a=a, b_storage=bt_st, out=out_st)
    # gather / scatter-add with duplicate indices, integer-valued updates
    src = rng.standard_normal((6, 5)).astype(F)
    idx = rng.integers(0, 6, size=(9, 5)).astype(np.int64)
    out_st = np.zeros(45, dtype=F)
    rk.gather(rk.HostView.of(src), rk.HostView.of(idx), 0, _hv(out_st, [9, 5], [5, 1], 0))
    _pack(cases, "gather_axis0", src=src, idx=idx, out=out_st)
    upd = np.floor(rng.uniform(-8, 8, size=(9, 5))).astype(F)
    out_st = np.zeros(30, dtype=F)
    rk.gather_scatter_add(rk.HostView.of(upd), rk.HostView.of(idx), 0, _hv(out_st, [6, 5], [5, 1], 0))
    _pack(cases, "scatter_add_axis0", upd=upd, idx=idx, out=out_st)
    idx1 = rng.integers(0, 5, size=(6, 8)).astype(np.int64)
    out_st = np.zeros(48, dtype=F)
    rk.gather(rk.HostView.of(src), rk.HostView.of(idx1), 1, _hv(out_st, [6, 8], [8, 1], 0))
    _pack(cases, "gather_axis1", src=src, idx=idx1, out=out_st)
    # concatenate along both axes
    parts = [rng.standard_normal((3, 4)).astype(F) for _ in range(3)]
    for axis in (0, 1):
        shape = list(parts[0].shape)
        shape[axis] *= 3
        out_st = np.zeros(36, dtype=F)
        rk.concat([rk.HostView.of(p) for p in parts], axis, _hv(out_st, shape, mo_strides(shape), 0))
        _pack(cases, f"concat_axis{axis}", p0=parts[0], p1=parts[1], p2=parts[2], out=out_st)
    # random creation and key derivation
    key = (12345, 0)
    k2 = rk.key_fold_in(key, 7)
    ks = rk.key_split(k2)
    _pack(cases, "keys", base=np.array(key, dtype=np.uint64), fold7=np.array(k2, dtype=np.uint64),
          split=np.array(ks, dtype=np.uint64))
    for n in (1, 5, 4099):
        u = np.zeros(n, dtype=F)
        rk.uniform(_hv(u, [n], [1], 0), -2.0, 3.0, ks[0])
        z = np.zeros(n, dtype=F)
        rk.normal(_hv(z, [n], [1], 0), 0.5, 2.0, ks[1])
        _pack(cases, f"random_{n}", uniform=u, normal=z, ukey=np.array(ks[0], dtype=np.uint64),
              nkey=np.array(ks[1], dtype=np.uint64))
    return cases


def mo_strides(shape):
    from minitensor_cpp_b200.abi import contiguous_strides

    return contiguous_strides(list(shape))


def main():
    (OUT / "known_answers.json").write_text(json.dumps(known_answers(), indent=1))
    cases = ref_cases()
    np.savez_compressed(OUT / "ref_cases.npz", **cases)
    print(f"wrote {len(cases)} arrays")


if __name__ == "__main__":
    main()
