"""The MiniTensor front-end built with the backend behaves exactly like the
unmodified reference on the CPU device (same graphs, same kernels, same bits),
and a CUDA device without a GPU is reported the reference's way. CPU only."""
import numpy as np
import pytest

from minitensor_cpp_b200.frontend import Frontend, MlpTrainer
from oracle import refkernels as rk

F = np.float32


@pytest.fixture(scope="module")
def fe():
    return Frontend()


@pytest.fixture(scope="module")
def ref():
    return Frontend(rk.LIB_PATH)


def test_cpu_device_is_bit_identical_to_reference(fe, ref):
    a, _ = fe.spiral_train(-1, 30)
    b, _ = ref.spiral_train(-1, 30)
    assert np.array_equal(a.view(np.int32), b.view(np.int32))
    rng = np.random.default_rng(1)
    args = (rng.uniform(-1, 1, (20, 30)).astype(F), rng.uniform(-1, 1, (30, 20)).astype(F),
            rng.uniform(-1, 1, 30).astype(F), rng.uniform(-1, 1, 20).astype(F))
    assert np.array_equal(fe.chain(-1, *args), ref.chain(-1, *args))


def test_mlp_trainer_cpu_identical(fe, ref):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((32, 12)).astype(F)
    y = rng.integers(0, 5, 32).astype(np.int64)
    t1 = MlpTrainer(fe, -1, 12, 16, 2, 5, seed=3, lr=1e-2)
    t2 = MlpTrainer(ref, -1, 12, 16, 2, 5, seed=3, lr=1e-2)
    t1.load_batch(x.ctypes.data, y.ctypes.data, 32)
    t2.load_batch(x.ctypes.data, y.ctypes.data, 32)
    for _ in range(2):
        assert t1.step_resident(True) == t2.step_resident(True)
    assert np.array_equal(t1.parameters(), t2.parameters())


def test_cuda_device_without_gpu_raises_runtime_error(fe):
    import ctypes

    n = ctypes.c_int(0)
    from minitensor_cpp_b200 import abi

    abi.lib().mtc_device_count(ctypes.byref(n))
    if n.value > 0:
        pytest.skip("a GPU is visible")
    with pytest.raises(RuntimeError, match="no runtime is registered"):
        fe.spiral_train(0, 1)


def test_gather_rows_and_index_error_on_the_cpu_device():
    """The row-gather workload on the CPU device of both libraries: same rows, and
    an index outside the table raises IndexError (copy/loops.hpp:206-209)."""
    from minitensor_cpp_b200.frontend import Frontend
    from oracle import refkernels as rk

    table = np.arange(60, dtype=np.float32).reshape(15, 4)
    idx = np.array([14, 0, 7, 7], dtype=np.int64)
    for fe in (Frontend(), Frontend(rk.LIB_PATH)):
        np.testing.assert_array_equal(fe.gather_rows(-1, table, idx), table[idx])
        with pytest.raises(IndexError):
            fe.gather_rows(-1, table, np.array([15], dtype=np.int64))


@pytest.mark.parametrize("axis", [0, 1])
def test_added_operations_on_the_cpu_device(fe, axis):
    """relu, max, argmax and log-softmax (the operations this backend adds, with
    their CPU kernels) through MiniTensor's API, against the oracle."""
    from helpers import added_ops_input, check_added_ops

    check_added_ops(fe, -1, added_ops_input(9, 13, seed=4), axis)
    with pytest.raises(ValueError):
        fe.added_ops(-1, np.zeros((2, 2), F), 2)


def _checkpoint_names(path):
    """Format version and parameter paths of a checkpoint of MlpTrainer.save
    (version 2 carries Adam's step count and moments after the parameters)."""
    import struct

    data = path.read_bytes()
    assert data[:7] == b"MTBCKPT" and data[7:8] in (b"1", b"2")
    version = int(data[7:8])
    (count,) = struct.unpack_from("<I", data, 8)
    pos, names, sizes = 12, [], []
    for _ in range(count):
        (n,) = struct.unpack_from("<I", data, pos)
        names.append(data[pos + 4:pos + 4 + n].decode())
        pos += 4 + n
        (rank,) = struct.unpack_from("<I", data, pos)
        extents = struct.unpack_from(f"<{rank}q", data, pos + 4)
        sizes.append(int(np.prod(extents)))
        pos += 4 + 8 * rank + 4 * sizes[-1]
    if version == 2:
        pos += 8 + 2 * 4 * sum(sizes)
    assert pos == len(data)
    return version, names


def test_checkpoint_round_trip_between_builds(fe, ref, tmp_path):
    """Parameters saved under their tree paths (for_each_named_parameter,
    parameter_tree.hpp:179-190) by one build load bit for bit into the other;
    a model of another shape is refused.  The backend build adds Adam's state
    (version 2); the build against the unmodified reference writes version 1."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((16, 12)).astype(F)
    y = rng.integers(0, 5, 16).astype(np.int64)
    a = MlpTrainer(fe, -1, 12, 16, 2, 5, seed=3, lr=1e-2)
    a.load_batch(x.ctypes.data, y.ctypes.data, 16)
    for _ in range(2):
        a.step_resident()
    path = tmp_path / "mlp.ckpt"
    a.save(path)
    assert _checkpoint_names(path) == (2, ["layer0.weight", "layer0.bias", "layer1.weight", "layer1.bias",
                                           "layer2.weight", "layer2.bias"])
    b = MlpTrainer(ref, -1, 12, 16, 2, 5, seed=99, lr=1e-2)
    assert not np.array_equal(b.parameters(), a.parameters())
    b.load(path)
    np.testing.assert_array_equal(b.parameters().view(np.uint32), a.parameters().view(np.uint32))
    b.save(tmp_path / "again.ckpt")
    assert _checkpoint_names(tmp_path / "again.ckpt")[0] == 1
    c = MlpTrainer(fe, -1, 12, 16, 2, 5, seed=98, lr=1e-2)
    c.load(tmp_path / "again.ckpt")
    np.testing.assert_array_equal(c.parameters().view(np.uint32), a.parameters().view(np.uint32))
    other = MlpTrainer(fe, -1, 12, 24, 2, 5, seed=3, lr=1e-2)
    with pytest.raises(ValueError):
        other.load(path)
    for t in (a, b, c, other):
        t.close()


def test_resume_from_checkpoint_is_bit_identical(fe, tmp_path):
    """With Adam's step count and moments in the checkpoint (version 2), three
    steps, a save, a load into a fresh trainer and two more steps give the
    parameters of five uninterrupted steps bit for bit."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((16, 12)).astype(F)
    y = rng.integers(0, 5, 16).astype(np.int64)
    full = MlpTrainer(fe, -1, 12, 16, 2, 5, seed=3, lr=1e-2)
    part = MlpTrainer(fe, -1, 12, 16, 2, 5, seed=3, lr=1e-2)
    for t in (full, part):
        t.load_batch(x.ctypes.data, y.ctypes.data, 16)
    for _ in range(5):
        full.step_resident()
    for _ in range(3):
        part.step_resident()
    part.save(tmp_path / "step3.ckpt")
    resumed = MlpTrainer(fe, -1, 12, 16, 2, 5, seed=7, lr=1e-2)
    resumed.load(tmp_path / "step3.ckpt")
    resumed.load_batch(x.ctypes.data, y.ctypes.data, 16)
    for _ in range(2):
        resumed.step_resident()
    np.testing.assert_array_equal(resumed.parameters().view(np.uint32), full.parameters().view(np.uint32))
    for t in (full, part, resumed):
        t.close()
