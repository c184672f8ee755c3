"""End-to-end parity through MiniTensor's own API with the CUDA backend.

The workloads (minitensor_cpp_b200/host/workloads.cpp) run once on cuda:0
through libminitensor_b200.so and once on the CPU through the oracle library
(the unmodified reference compiled from its sources).  Tolerances: loss curves
within 1e-3 relative (1e-5 at step 0), fused elementwise results within 2 ulp,
parameters after a training step within 1e-5*sqrt(K) of their magnitude.
"""
import numpy as np
import pytest

from helpers import assert_rel_sqrtk, assert_ulp
from minitensor_cpp_b200.frontend import Frontend, MlpTrainer
from oracle import mt_oracle as mo
from oracle import refkernels as rk

pytestmark = pytest.mark.gpu

F = np.float32


@pytest.fixture(scope="module")
def fe(cuda):
    return Frontend()


@pytest.fixture(scope="module")
def ref():
    return Frontend(rk.LIB_PATH)


def test_spiral_loss_curve_matches_reference(fe, ref):
    """Config 1: spiral MLP 2-64-64-3, ReLU, Adam(1e-2), full batch, 2000 steps."""
    steps = 2000
    gpu_losses, _ = fe.spiral_train(0, steps, loss_every=1)
    cpu_losses, _ = ref.spiral_train(-1, steps, loss_every=1)
    # The reference's own sensitivity: the same CPU run with the learning rate
    # moved by one float32 ulp.  Adam amplifies last-bit differences (a gradient
    # within rounding of zero flips sign and moves its parameter by 2*lr), so the
    # GPU curve is required to stay within 3x of that noise floor.
    lr_ulp = float(np.nextafter(np.float32(1e-2), np.float32(1)))
    cpu_perturbed, _ = ref.spiral_train(-1, steps, lr=lr_ulp, loss_every=1)
    noise = np.abs(cpu_perturbed.astype(np.float64) - cpu_losses) / np.abs(cpu_losses)
    assert np.isfinite(gpu_losses).all()
    rel = np.abs(gpu_losses.astype(np.float64) - cpu_losses) / np.abs(cpu_losses)
    assert rel[0] <= 1e-6, rel[0]
    assert rel[:200].max() <= 3 * noise[:200].max() + 1e-6, (float(rel[:200].max()), float(noise[:200].max()))
    assert rel[-1] <= max(1e-2, 3 * noise[-1]), (float(rel[-1]), float(noise[-1]))
    assert gpu_losses[-1] < 0.05 * gpu_losses[0]


def test_fused_chain_through_api(fe, ref):
    """Config 2's chain relu(A*B^T + row)*exp(-col): one fused launch on the GPU."""
    rng = np.random.default_rng(3)
    n, m = 300, 420
    a = rng.uniform(-1, 1, (n, m)).astype(F)
    bs = rng.uniform(-1, 1, (m, n)).astype(F)
    row = rng.uniform(-1, 1, m).astype(F)
    col = rng.uniform(-1, 1, n).astype(F)
    fe.reset_stats()
    y_gpu, s0, s1, l1 = fe.chain(0, a, bs, row, col, reductions=True)
    stats = fe.stats()
    y_cpu, r0, r1, rl = ref.chain(-1, a, bs, row, col, reductions=True)
    assert_ulp(y_gpu, y_cpu, 2, "chain")
    assert stats["fused_launches"] >= 1 and stats["fused_nodes"] >= 6, stats
    scale0 = mo.reduce_sum(np.abs(y_cpu), [0])
    assert_rel_sqrtk(s0, r0, n, scale0, "sum axis 0")
    assert_rel_sqrtk(s1, r1, m, mo.reduce_sum(np.abs(y_cpu), [1]), "sum axis 1")
    assert_rel_sqrtk(l1, rl, m, None, "logsumexp axis 1")


def test_mlp_training_steps_match_reference(fe, ref):
    """Config 5's trainer at reduced width: losses and parameters after 3 steps."""
    rng = np.random.default_rng(5)
    batch, fin, hid, cls = 256, 96, 160, 10
    x = rng.standard_normal((batch, fin)).astype(F)
    y = rng.integers(0, cls, batch).astype(np.int64)
    g = MlpTrainer(fe, 0, fin, hid, 3, cls, seed=7, lr=1e-3)
    c = MlpTrainer(ref, -1, fin, hid, 3, cls, seed=7, lr=1e-3)
    np.testing.assert_array_equal(g.parameters(), c.parameters())  # identical Philox init
    g.load_batch(x.ctypes.data, y.ctypes.data, batch)
    c.load_batch(x.ctypes.data, y.ctypes.data, batch)
    for step in range(3):
        lg = g.step_resident(read_loss=True)
        lc = c.step_resident(read_loss=True)
        assert abs(lg - lc) <= 1e-5 * abs(lc) * np.sqrt(hid), (step, lg, lc)
    pg, pc = g.parameters(), c.parameters()
    # Adam's first steps move every parameter by ~lr * sign(gradient), so a
    # gradient within rounding of 0 may flip sign between backends: such
    # elements differ by up to 2*lr per step, all others agree to rounding.
    diff = np.abs(pg - pc)
    assert diff.max() <= 3 * 2 * 1e-3 + 1e-6, float(diff.max())
    assert np.mean(diff > 1e-5) < 1e-3, float(np.mean(diff > 1e-5))
    lh = g.step_host(x.ctypes.data, y.ctypes.data, batch)
    lc = c.step_host(x.ctypes.data, y.ctypes.data, batch)
    assert abs(lh - lc) <= 1e-4 * abs(lc), (lh, lc)
    g.close()
    c.close()


def test_gather_index_error_through_the_api(fe, ref):
    """An index outside the table raises IndexError through MiniTensor's API on the
    GPU as on the reference CPU backend (on the GPU at the read that follows the
    evaluation), and the next evaluation on the device is unaffected."""
    rng = np.random.default_rng(31)
    table = rng.standard_normal((1000, 64)).astype(F)
    bad = np.array([3, 999, 1000, 7], dtype=np.int64)
    good = rng.integers(0, 1000, 4096).astype(np.int64)
    for lib in (ref, fe):
        dev = -1 if lib is ref else 0
        with pytest.raises(IndexError):
            lib.gather_rows(dev, table, bad)
        out = lib.gather_rows(dev, table, good)
        np.testing.assert_array_equal(out, table[good])


def test_synchronous_index_check_installs_no_storage(fe):
    """MTB_INDEX_CHECKS=sync (here switched on at run time): an out-of-range
    gather index throws out_of_range from the evaluation itself and the gather
    stays unmaterialised, as the reference's evaluator guarantees
    (evaluator_test.cpp:199-216).  In the default deferred mode the evaluation
    installs the value and the next read raises."""
    rng = np.random.default_rng(37)
    table = rng.standard_normal((1000, 64)).astype(F)
    bad = np.array([3, 999, 1000, 7], dtype=np.int64)
    good = rng.integers(0, 1000, 4096).astype(np.int64)
    previous = fe.set_index_checks("sync")
    try:
        assert fe.gather_eval_probe(0, table, bad) == (True, False)
        np.testing.assert_array_equal(fe.gather_rows(0, table, good), table[good])
    finally:
        fe.set_index_checks(previous)
    assert previous == "deferred"
    with pytest.raises(IndexError):
        fe.gather_eval_probe(0, table, bad)
    np.testing.assert_array_equal(fe.gather_rows(0, table, good), table[good])


@pytest.mark.parametrize("class_axis", [1, 0])
def test_cross_entropy_gradient_defers_its_scatter(fe, ref, class_axis):
    """The gradient of categorical cross entropy (src/nn/loss.cpp:41-57) sums the
    logsumexp VJP's g * exp(x - lse) and the gather VJP's scatter-add.  The
    evaluator adds the scatter's updates into that sum's output instead of
    materialising a zero-filled [B, C] tensor: bit for bit the same gradient as
    the unfused evaluation, and within 1e-5*sqrt(C) of the reference's."""
    from helpers import assert_bits

    rng = np.random.default_rng(59 + class_axis)
    x = (rng.standard_normal((2048, 1000)) * 3).astype(F)
    t = rng.integers(0, 1000 if class_axis == 1 else 2048, x.shape[1 - class_axis])
    fe.reset_stats()
    lf, gf = fe.cross_entropy(0, x, t, class_axis)
    assert fe.stats()["scatters_deferred"] >= 1
    previous = fe.set_fusion(False)
    try:
        lu, gu = fe.cross_entropy(0, x, t, class_axis)
    finally:
        fe.set_fusion(previous)
    assert np.float32(lf).view(np.uint32) == np.float32(lu).view(np.uint32)
    assert_bits(gf, gu, "deferred vs unfused scatter")
    lc, gc = ref.cross_entropy(-1, x, t, class_axis)
    classes = x.shape[class_axis]
    assert abs(lf - lc) <= 1e-5 * np.sqrt(classes) * abs(lc)
    assert_rel_sqrtk(gf, gc, classes, np.abs(gc) + np.abs(gc).max() * 1e-3, "cross-entropy gradient")


def test_pipelined_host_steps_match_resident_steps(fe):
    """step_host copies each batch into one of two device slots on a copy
    stream and reads the loss as soon as the forward pass has computed it.
    Losses and parameters must equal those of steps on the same batches loaded
    synchronously (load_batch + step_resident), bit for bit, including when
    the batch size changes (the slots are reallocated)."""
    rng = np.random.default_rng(17)
    fin, hid, cls = 96, 160, 10
    batches = []
    for n in (256, 256, 256, 128, 128):
        batches.append((rng.standard_normal((n, fin)).astype(F), rng.integers(0, cls, n).astype(np.int64)))
    a = MlpTrainer(fe, 0, fin, hid, 3, cls, seed=11, lr=1e-3)
    b = MlpTrainer(fe, 0, fin, hid, 3, cls, seed=11, lr=1e-3)
    for x, y in batches:
        a.load_batch(x.ctypes.data, y.ctypes.data, x.shape[0])
        la = a.step_resident(read_loss=True)
        lb = b.step_host(x.ctypes.data, y.ctypes.data, x.shape[0])
        assert np.float32(la).view(np.uint32) == np.float32(lb).view(np.uint32), (la, lb)
    np.testing.assert_array_equal(a.parameters().view(np.uint32), b.parameters().view(np.uint32))
    a.close()
    b.close()


@pytest.mark.parametrize("axis", [0, 1])
@pytest.mark.parametrize("rows, cols", [(9, 13), (1024, 3000)])
def test_added_operations_on_the_cuda_device(fe, axis, rows, cols):
    """relu, max, argmax and log-softmax through MiniTensor's API on the GPU (the
    evaluator fuses relu; the reductions run the CUDA kernels), against the oracle."""
    from helpers import added_ops_input, check_added_ops

    check_added_ops(fe, 0, added_ops_input(rows, cols, seed=5), axis)


def test_checkpoint_between_devices(fe, ref, tmp_path):
    """Parameters saved on the GPU load bit for bit into the reference CPU trainer
    and back; a step from the loaded parameters gives the same loss on both
    (within 1e-5*sqrt(K)).  The reference build cannot hold Adam's moments
    (version-1 checkpoint), so here both trainers start them from zero."""
    rng = np.random.default_rng(61)
    batch, fin, hid, cls = 256, 96, 160, 10
    x = rng.standard_normal((batch, fin)).astype(F)
    y = rng.integers(0, cls, batch).astype(np.int64)
    g = MlpTrainer(fe, 0, fin, hid, 2, cls, seed=13, lr=1e-3)
    g.load_batch(x.ctypes.data, y.ctypes.data, batch)
    for _ in range(3):
        g.step_resident()
    g.save(tmp_path / "gpu.ckpt")
    c = MlpTrainer(ref, -1, fin, hid, 2, cls, seed=77, lr=1e-3)
    c.load(tmp_path / "gpu.ckpt")
    np.testing.assert_array_equal(c.parameters().view(np.uint32), g.parameters().view(np.uint32))
    c.save(tmp_path / "cpu.ckpt")
    g2 = MlpTrainer(fe, 0, fin, hid, 2, cls, seed=78, lr=1e-3)
    g2.load(tmp_path / "cpu.ckpt")
    np.testing.assert_array_equal(g2.parameters().view(np.uint32), g.parameters().view(np.uint32))
    g2.load_batch(x.ctypes.data, y.ctypes.data, batch)
    c.load_batch(x.ctypes.data, y.ctypes.data, batch)
    lg, lc = g2.step_resident(read_loss=True), c.step_resident(read_loss=True)
    assert abs(lg - lc) <= 1e-5 * np.sqrt(hid) * abs(lc), (lg, lc)
    for t in (g, g2, c):
        t.close()


def test_resume_from_checkpoint_on_cuda(fe, tmp_path):
    """Adam's step count and moments travel with the parameters (version-2
    checkpoint): three steps, save, load into a fresh GPU trainer, two more
    steps equal five uninterrupted steps bit for bit."""
    rng = np.random.default_rng(67)
    batch, fin, hid, cls = 256, 96, 160, 10
    x = rng.standard_normal((batch, fin)).astype(F)
    y = rng.integers(0, cls, batch).astype(np.int64)
    full = MlpTrainer(fe, 0, fin, hid, 2, cls, seed=21, lr=1e-3)
    part = MlpTrainer(fe, 0, fin, hid, 2, cls, seed=21, lr=1e-3)
    for t in (full, part):
        t.load_batch(x.ctypes.data, y.ctypes.data, batch)
    for _ in range(5):
        full.step_resident()
    for _ in range(3):
        part.step_resident()
    part.save(tmp_path / "step3.ckpt")
    resumed = MlpTrainer(fe, 0, fin, hid, 2, cls, seed=22, lr=1e-3)
    resumed.load(tmp_path / "step3.ckpt")
    resumed.load_batch(x.ctypes.data, y.ctypes.data, batch)
    for _ in range(2):
        resumed.step_resident()
    np.testing.assert_array_equal(resumed.parameters().view(np.uint32), full.parameters().view(np.uint32))
    for t in (full, part, resumed):
        t.close()
