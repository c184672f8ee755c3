"""Parity of the CUDA path at the benchmark configurations, against the oracle.

- Tensor-core training: the wide-MLP trainer at widths where MTC_GEMM_AUTO runs
  every GEMM on the tcgen05 path, against the same trainer on the reference CPU
  backend (oracle/_ref): loss, every layer's weight and bias gradient, and two
  Adam steps.  The trainer runs MiniTensor's own Linear
  (src/nn/modules/linear.cpp:65-83) and matmul VJP
  (src/tensor/autograd/rules/linalg.cpp:16-54) on both devices.
- The nn known answers of the reference's tests (cross entropy, AdamW, SGD) on
  the CUDA device, and AdamW / SGD updates of 2^20 parameters bit for bit
  against the reference CPU backend.
- Config 2 at 8192^2: the lazily evaluated chain relu(A*B^T + row)*exp(-col)
  through the API, then sum / max / argmax along both axes and log-softmax.
- Config 4 at 2^24 rows: row gather and scatter-add bit-exact, and the two
  concatenations of four [4096, 8192] tensors.
"""
import numpy as np
import pytest

from helpers import assert_bits, assert_rel_sqrtk, assert_ulp
from minitensor_cpp_b200 import abi
from minitensor_cpp_b200.frontend import Frontend, MlpTrainer
from oracle import mt_oracle as mo
from oracle import refkernels as rk

pytestmark = pytest.mark.gpu

F = np.float32
F64 = np.float64


@pytest.fixture(scope="module")
def fe(cuda):
    return Frontend()


@pytest.fixture(scope="module")
def ref():
    return Frontend(rk.LIB_PATH)


# ------------------------------------------------------ tensor-core training --

def _layers(vec, widths):
    """(W [out, in], b [out]) per layer from the trainer's parameter order."""
    out, pos = [], 0
    for i, o in zip(widths[:-1], widths[1:]):
        W = vec[pos:pos + o * i].reshape(o, i)
        pos += o * i
        out.append((W, vec[pos:pos + o]))
        pos += o
    assert pos == vec.size
    return out


def _backward_f64(layers, x, y):
    """Exact (float64) forward and backward pass of the MLP with ReLU and mean
    softmax cross entropy: inputs h_l of every layer, pre-activations z_l and the
    gradients G_l = dLoss/dz_l."""
    hs, zs = [x.astype(F64)], []
    for li, (W, b) in enumerate(layers):
        z = hs[-1] @ W.T.astype(F64) + b.astype(F64)
        zs.append(z)
        if li + 1 < len(layers):
            hs.append(np.maximum(z, 0.0))
    logits = zs[-1]
    p = np.exp(logits - logits.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    G = p.copy()
    G[np.arange(len(y)), y] -= 1.0
    G /= len(y)
    Gs = [None] * len(layers)
    Gs[-1] = G
    for li in range(len(layers) - 1, 0, -1):
        Gs[li - 1] = (Gs[li] @ layers[li][0].astype(F64)) * (zs[li - 1] > 0)
    return hs, zs, Gs


def _near_zero_rows(layers, x, margin=1e-5):
    """Rows of x with a hidden pre-activation within margin * (|h| |W|^T + |b|)
    of 0 (exact float64 pass): there the two backends' roundings could send the
    ReLU derivative to different sides."""
    h = x.astype(F64)
    bad = np.zeros(len(x), dtype=bool)
    for W, b in layers[:-1]:
        W64, b64 = W.T.astype(F64), b.astype(F64)
        z = h @ W64 + b64
        env = np.abs(h) @ np.abs(W64) + np.abs(b64)
        bad |= (np.abs(z) < margin * env).any(axis=1)
        h = np.maximum(z, 0.0)
    return bad


def _clean_batch(layers, rng, batch, fin):
    """N(0,1) rows, redrawn until no hidden pre-activation is within 1e-5 of its
    rounding envelope of 0, so both backends take the same ReLU branch
    everywhere (a 1e-5 margin is ~100x the float32 rounding of a 1024-term sum)."""
    x = rng.standard_normal((batch, fin)).astype(F)
    for _ in range(50):
        bad = _near_zero_rows(layers, x)
        if not bad.any():
            return x
        x[bad] = rng.standard_normal((int(bad.sum()), fin)).astype(F)
    raise AssertionError("could not draw a batch away from the ReLU kinks")


def _envelopes(layers, hs, zs, Gs):
    """One-level rounding envelopes of the weight and bias gradients: each term
    is the magnitude sum of one product the backends compute in float32,
      dW_l:  |G_l|^T (|h_l| + F_l) + D_l^T |h_l|,   db_l: sum_s (|G_l| + D_l)
    with F_l = (|h_(l-1)| |W_(l-1)|^T + |b_(l-1)|) * [z_(l-1) > 0] (the layer
    input's own product, 0 for the data), D_l = (|G_(l+1)| |W_(l+1)|) * [z_l > 0]
    (G_l's own product) and, on the logits, D = 2 p / B * max_c of the logits'
    envelope (the softmax gradient moves by at most 2 p / B per unit of logit
    error)."""
    L = len(layers)
    env = []
    for li in range(L):
        W, b = layers[li]
        if li == 0:
            F_l = np.zeros_like(hs[0])
        else:
            Wp, bp = layers[li - 1]
            F_l = (np.abs(hs[li - 1]) @ np.abs(Wp.T.astype(F64)) + np.abs(bp.astype(F64))) * (zs[li - 1] > 0)
        if li + 1 < L:
            D = (np.abs(Gs[li + 1]) @ np.abs(layers[li + 1][0].astype(F64))) * (zs[li] > 0)
        else:
            zenv = np.abs(hs[li]) @ np.abs(W.T.astype(F64)) + np.abs(b.astype(F64))
            logits = zs[li]
            prob = np.exp(logits - logits.max(axis=1, keepdims=True))
            prob /= prob.sum(axis=1, keepdims=True)
            D = 2.0 * prob / len(hs[0]) * zenv.max(axis=1, keepdims=True)
        G = np.abs(Gs[li])
        env.append((G.T @ (np.abs(hs[li]) + F_l) + D.T @ np.abs(hs[li]), (G + D).sum(axis=0)))
    return env


def _check_gradients(got, want, params, widths, x, y):
    """Weight and bias gradients of two backends within
      (2L + 1) * 1e-5 * sqrt(K) * envelope
    with K the longest contraction on the path and one 1e-5*sqrt(K) term for
    each of the 2L + 1 GEMMs whose rounding reaches a weight gradient (L forward,
    L - 1 input gradients, the weight gradient); envelope of _envelopes from an
    exact float64 pass.  The batch must keep every pre-activation away from the
    ReLU kink (_clean_batch)."""
    layers = _layers(params, widths)
    assert not _near_zero_rows(layers, x).any()
    hs, zs, Gs = _backward_f64(layers, x, y)
    env = _envelopes(layers, hs, zs, Gs)
    L = len(layers)
    k = (2 * L + 1) * 1e-5 * np.sqrt(max(max(widths), len(y)))
    for li, ((gW, gb), (cW, cb)) in enumerate(zip(_layers(got, widths), _layers(want, widths))):
        for g, c, scale, what in ((gW, cW, env[li][0], "dW"), (gb, cb, env[li][1], "db")):
            err = np.abs(g.astype(F64) - c)
            tol = k * scale
            bad = err > tol
            assert not bad.any(), (f"layer {li} {what}: {int(bad.sum())} of {err.size} beyond the bound "
                                   f"(worst ratio {float((err / np.maximum(tol, 1e-30)).max()):.3g})")


@pytest.mark.parametrize("pipeline", [None, "pair16x6"])
def test_tensor_core_training_matches_reference(fe, ref, pipeline, monkeypatch):
    """MLP 1024 -> 1024 -> 1024 -> 1024 at batch 256: every GEMM of the forward and
    backward pass has M*N*K = 2^28, so MTC_GEMM_AUTO runs them all on the
    tcgen05 3xTF32 kernels (default policy, then the CTA pair forced).

    Gradients within the componentwise bound of _check_gradients; the loss within
    1e-5*sqrt(K) relative; after two Adam steps the parameters within Adam's
    sign-flip bound."""
    if pipeline:
        monkeypatch.setenv("MTC_TC_PIPELINE", pipeline)
    else:
        monkeypatch.delenv("MTC_TC_PIPELINE", raising=False)
    rng = np.random.default_rng(41)
    batch, fin, hid, cls = 256, 1024, 1024, 1024
    widths = [fin, hid, hid, cls]
    y = rng.integers(0, cls, batch).astype(np.int64)
    g = MlpTrainer(fe, 0, fin, hid, 2, cls, seed=9, lr=1e-3)
    c = MlpTrainer(ref, -1, fin, hid, 2, cls, seed=9, lr=1e-3)
    p0 = c.parameters()
    np.testing.assert_array_equal(g.parameters(), p0)  # identical Philox initialisation
    x = _clean_batch(_layers(p0, widths), rng, batch, fin)
    g.load_batch(x.ctypes.data, y.ctypes.data, batch)
    c.load_batch(x.ctypes.data, y.ctypes.data, batch)

    tc0, simt0 = abi.gemm_path_counts()
    lg, gg = g.gradients()
    tc1, simt1 = abi.gemm_path_counts()
    assert tc1 - tc0 >= 8 and simt1 == simt0, (tc1 - tc0, simt1 - simt0)
    lc, gc = c.gradients()

    assert abs(lg - lc) <= 1e-5 * np.sqrt(hid) * abs(lc), (lg, lc)
    _check_gradients(gg, gc, p0, widths, x, y)

    # two Adam steps on both devices.  Each GPU step must equal the oracle's
    # AdamW update (src/nn/optimizers/adamw.cpp:67-97, lr 1e-3, no decay) of
    # the GPU's own parameters and gradients bit for bit, and the losses stay
    # within the bound.  (The gradient bound above is checked at the initial
    # parameters only: the batch keeps its pre-activations away from the ReLU
    # kink for those parameters, not for the updated ones.)
    m = v = np.zeros_like(p0)
    for step in range(2):
        p_gpu = g.parameters()
        lg, gg = g.gradients()
        lc, _ = c.gradients()
        assert abs(lg - lc) <= 1e-5 * np.sqrt(hid) * abs(lc), (step, lg, lc)
        tc0, _ = abi.gemm_path_counts()
        g.step_resident()
        assert abi.gemm_path_counts()[0] - tc0 >= 8
        c.step_resident()
        want, m, v = mo.adamw_update(p_gpu, gg, m, v, 1e-3, 0.0, 0.9, 0.999, 1e-8, step)
        assert_bits(g.parameters(), want, f"Adam step {step} on the GPU")
    # Adam moves each parameter by about lr * sign(gradient) per step
    assert np.abs(g.parameters() - c.parameters()).max() <= 2 * 2 * 1e-3 + 1e-6
    g.close()
    c.close()


# --------------------------------------------------------- nn known answers --

def test_cross_entropy_known_answer_on_cuda(fe):
    """loss_test.cpp:66-78: logits [3, 2] with classes along axis 0."""
    logits = np.array([[2.0, 0.0], [1.0, 1.0], [0.0, 2.0]], dtype=F)
    loss, grad = fe.cross_entropy(0, logits, np.array([0, 1]), class_axis=0)
    assert abs(loss - 0.9076060) <= 1e-6
    want = [-0.1673795, 0.0450153, 0.1223642, -0.3776358, 0.0450153, 0.3326205]
    np.testing.assert_allclose(grad.reshape(-1), want, atol=1e-6)


def test_cross_entropy_matches_reference_at_training_shape(fe, ref):
    """[2048, 1000] logits (the wide MLP's classes): loss within 1e-5*sqrt(C)
    relative, gradient within 1e-5*sqrt(C) of its magnitude plus 2 ulp."""
    rng = np.random.default_rng(43)
    x = (rng.standard_normal((2048, 1000)) * 3).astype(F)
    t = rng.integers(0, 1000, 2048)
    lg, gg = fe.cross_entropy(0, x, t)
    lc, gc = ref.cross_entropy(-1, x, t)
    assert abs(lg - lc) <= 1e-5 * np.sqrt(1000) * abs(lc), (lg, lc)
    assert_rel_sqrtk(gg, gc, 1000, np.abs(gc) + np.abs(gc).max() * 1e-3, "cross-entropy gradient")


def test_adamw_and_sgd_known_answers_on_cuda(fe):
    """adamw_test.cpp:43-61 and :63-95, sgd_test.cpp:84-98, on the CUDA device."""
    got = fe.optimizer_steps(0, "adamw", np.array([1.0, -2.0]), np.array([[2.0, -4.0]]), 0.1, 0.2, 0.5, 0.25, 0.01)
    decay = F(1.0) - F(0.1) * F(0.2)
    np.testing.assert_allclose(got, [decay * 1.0 - 0.1 * 2.0 / 2.01, decay * -2.0 + 0.1 * 4.0 / 4.01], atol=1e-6)
    got = fe.optimizer_steps(0, "adamw", np.array([1.0]), np.array([[2.0], [1.0]]), 0.1, 0.2, 0.5, 0.25, 0.01)
    first = 0.98 - 0.1 * 2.0 / 2.01
    want = 0.98 * first - 0.1 * (1.0 / 0.75) / (np.sqrt(1.5 / 0.9375) + 0.01)
    assert abs(got[0] - want) <= 1e-6, (got, want)
    got = fe.optimizer_steps(0, "sgd", np.array([1.0, 2.0]), np.array([[0.5, 1.0]]), 0.5)
    assert got.tolist() == [0.75, 1.5]


@pytest.mark.parametrize("kind", ["adamw", "sgd"])
def test_optimizer_updates_bit_exact_against_reference(fe, ref, kind):
    """Three steps on 2^20 parameters through the API: the fused update kernel
    rounds every operation like the reference's unfused CPU ops, so the results
    are identical bit for bit (AdamW with weight decay; SGD p - lr * g)."""
    rng = np.random.default_rng(47)
    n = 1 << 20
    p = rng.standard_normal(n).astype(F)
    gs = (rng.standard_normal((3, n)) * rng.uniform(1e-4, 10, (3, 1))).astype(F)
    args = (1e-3, 0.01, 0.9, 0.999, 1e-8) if kind == "adamw" else (0.05,)
    got = fe.optimizer_steps(0, kind, p, gs, *args)
    want = ref.optimizer_steps(-1, kind, p, gs, *args)
    assert_bits(got, want, f"{kind} update")
    if kind == "sgd":
        exp = p
        for s in range(3):
            exp = (exp - F(0.05) * gs[s]).astype(F)
        assert_bits(got, exp, "sgd update vs p - lr*g")


def test_sgd_training_step_on_cuda(fe, ref):
    """The trainer with SGD(0.05) instead of Adam on the GPU: its gradients against
    the reference CPU backend's (the bound of _check_gradients), and its update
    equal to p - lr * g of its own gradients bit for bit, as on the reference."""
    rng = np.random.default_rng(53)
    batch, fin, hid, cls = 128, 64, 96, 10
    widths = [fin, hid, hid, cls]
    y = rng.integers(0, cls, batch).astype(np.int64)
    g = MlpTrainer(fe, 0, fin, hid, 2, cls, seed=5, lr=1e-3)
    c = MlpTrainer(ref, -1, fin, hid, 2, cls, seed=5, lr=1e-3)
    p0 = c.parameters()
    x = _clean_batch(_layers(p0, widths), rng, batch, fin)
    for t in (g, c):
        t.use_sgd(0.05)
        t.load_batch(x.ctypes.data, y.ctypes.data, batch)
    _, gg = g.gradients()
    _, gc = c.gradients()
    _check_gradients(gg, gc, p0, widths, x, y)
    g.step_resident()
    c.step_resident()
    assert_bits(c.parameters(), (p0 - F(0.05) * gc).astype(F), "reference SGD step = p - lr*g")
    assert_bits(g.parameters(), (p0 - F(0.05) * gg).astype(F), "GPU SGD step = p - lr*g")
    g.close()
    c.close()


# ------------------------------------------------------- config 2 at 8192^2 --

def test_chain_and_reductions_at_8192(fe, cuda):
    """relu(A * B^T + row) * exp(-col) through the API on 8192^2 (the evaluator
    fuses it), against the oracle within the composed per-operation bound (exp
    within 2 ulp, every other operation rounded like the oracle); then, on that Y, sum / max /
    argmax along both axes and log-softmax along axis 1 on the CUDA kernels:
    max and argmax bit-exact, sums within 1e-5*sqrt(K)*sum|y| of the exact sum,
    log-softmax within 1e-5*sqrt(K)*|logsumexp|."""
    import torch

    n = 8192
    rng = np.random.default_rng(2026)
    u = lambda *shape: rng.uniform(-1, 1, shape).astype(F)
    a, bs, row, col = u(n, n), u(n, n), u(1, n), u(n, 1)
    y, s0, s1, l1 = fe.chain(0, a, bs, row, col, reductions=True)
    pre = mo.binary(mo.ADD, mo.binary(mo.MULTIPLY, a, bs.T), row)
    relu = ((pre + np.abs(pre)) * F(0.5)).astype(F)
    e = mo.unary(mo.EXP, mo.unary(mo.NEGATE, col))
    want = mo.binary(mo.MULTIPLY, relu, e)
    # per-operation bounds composed: the product, sum and relu round exactly like
    # the oracle; exp is within 2 ulp of exact on the GPU and within 0.5 ulp in
    # the oracle, and the final product is rounded once on each side
    tol = np.abs(relu).astype(F64) * (2.5 * np.spacing(np.abs(e)).astype(F64)) + np.spacing(np.abs(want)).astype(F64)
    err = np.abs(y.astype(F64) - want)
    bad = err > tol
    assert not bad.any(), f"chain at 8192^2: {int(bad.sum())} elements beyond the composed bound"
    assert_ulp(y[want == 0], want[want == 0], 0, "chain zeros")
    del pre, relu, a, bs, err, tol
    y64 = y.astype(F64)
    yabs = np.abs(y64)
    assert_rel_sqrtk(s0, y64.sum(axis=0), n, yabs.sum(axis=0), "sum axis 0 (API)")
    assert_rel_sqrtk(s1, y64.sum(axis=1), n, yabs.sum(axis=1), "sum axis 1 (API)")
    lse = mo.reduce_logsumexp(y, [1])
    assert_rel_sqrtk(l1, lse, n, np.abs(lse), "logsumexp axis 1 (API)")
    Y = torch.from_numpy(y).cuda()
    V = abi.View.of
    for ax in (0, 1):
        o = torch.empty(n, device="cuda")
        oi = torch.empty(n, device="cuda", dtype=torch.int64)
        abi.reduce(abi.SUM, V(Y), [ax], V(o))
        assert_rel_sqrtk(o.cpu().numpy(), y64.sum(axis=ax), n, yabs.sum(axis=ax), f"sum axis {ax}")
        abi.reduce(abi.MAX, V(Y), [ax], V(o))
        assert_bits(o.cpu().numpy(), y.max(axis=ax), f"max axis {ax}")
        abi.reduce(abi.ARGMAX, V(Y), [ax], V(oi))
        assert_bits(oi.cpu().numpy(), y.argmax(axis=ax).astype(np.int64), f"argmax axis {ax}")
    Z = torch.empty(n, n, device="cuda")
    abi.log_softmax(V(Y), 1, V(Z))
    abi.check_device_errors(0)
    lse_k = np.broadcast_to(np.abs(lse)[:, None], (n, n))
    assert_rel_sqrtk(Z.cpu().numpy(), (y64 - lse.astype(F64)[:, None]), n, lse_k, "log-softmax axis 1")


# -------------------------------------------------------- config 4 at 2^24 --

def test_gather_and_scatter_add_at_2_24_rows(cuda):
    """Row gather of a [2^24, 64] table with 2^24 uniform Int64 indices
    (broadcast along the row, as the API's gather needs), and the backward
    scatter-add of integer-valued updates with duplicate indices: both bit-exact
    against the oracle (table[idx], and the per-row sums of np.add.at, which are
    exact because every partial sum is an integer below 2^24)."""
    import torch

    rows, width = 1 << 24, 64
    g = torch.Generator(device="cuda").manual_seed(4)
    table = torch.randn(rows, width, device="cuda", generator=g)
    idx = torch.randint(0, rows, (rows, 1), device="cuda", dtype=torch.int64, generator=g)
    idx_b = abi.View(idx.view(-1), (rows, width), (1, 0), 0)
    out = torch.full((rows, width), float("nan"), device="cuda")
    abi.gather(abi.View.of(table), idx_b, 0, abi.View.of(out))
    abi.check_device_errors(0)
    ih = idx.view(-1).cpu().numpy()
    th = table.cpu().numpy()
    assert_bits(out.cpu().numpy(), th[ih], "row gather 2^24 x 64")
    del th, table
    upd = torch.floor(torch.rand(rows, width, device="cuda", generator=g) * 16 - 8)
    abi.gather_scatter_add(abi.View.of(upd), idx_b, 0, abi.View.of(out))
    abi.check_device_errors(0)
    got = out.cpu().numpy()
    del out
    uh = upd.cpu().numpy()
    del upd
    order = np.argsort(ih, kind="stable")
    keys = ih[order]
    starts = np.flatnonzero(np.r_[True, keys[1:] != keys[:-1]])
    sums = np.add.reduceat(uh[order], starts, axis=0)
    del uh
    want = np.zeros((rows, width), dtype=F)
    want[keys[starts]] = sums
    dup = int((np.diff(starts, append=rows) > 1).sum())
    assert dup > 1000, "the index draw should repeat rows"
    assert_bits(got, want, f"scatter-add 2^24 x 64 ({dup} rows hit more than once)")


def test_concat_at_benchmark_size(cuda):
    """Four [4096, 8192] tensors concatenated along axis 0 and along axis 1, bit-exact."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(6)
    parts = [torch.randn(4096, 8192, device="cuda", generator=g) for _ in range(4)]
    host = [p.cpu().numpy() for p in parts]
    for axis, shape in ((0, (16384, 8192)), (1, (4096, 32768))):
        dst = torch.full(shape, float("nan"), device="cuda")
        abi.concat([abi.View.of(p) for p in parts], axis, abi.View.of(dst))
        torch.cuda.synchronize()
        assert_bits(dst.cpu().numpy(), mo.concatenate(host, axis), f"concat axis {axis}")
