"""Data-parallel training on two GPUs over NCCL (skipped with fewer than two).

Each rank trains the wide-MLP trainer of host/workloads.cpp on its half of the
batch.  The trainer evaluates the gradients layer by layer and queues each
layer's NCCL all-reduce on the communicator's own stream while the next layer's
backward kernels run.  The result must match one GPU training on the full
batch: both ranks hold identical parameters, the mean of the two half-batch
losses equals the full-batch loss, and the parameters agree within the
sign-flip bound of Adam.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F = np.float32
WIDTHS = (64, 256, 2, 40)  # in, hidden, hidden layers, classes
BATCH = 512
STEPS = 3
LR = 1e-3


def _data():
    rng = np.random.default_rng(23)
    x = rng.standard_normal((BATCH, WIDTHS[0])).astype(F)
    y = rng.integers(0, WIDTHS[-1], BATCH).astype(np.int64)
    return x, y


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_path):
    import ctypes
    import sys
    from datetime import timedelta

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist

    from minitensor_cpp_b200 import abi
    from minitensor_cpp_b200.frontend import Frontend, MlpTrainer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    comm = ctypes.c_void_p()
    try:
        uid = (ctypes.c_char * 128)()
        if rank == 0:
            abi.check(abi.lib().mtc_comm_unique_id(uid, 128), "nccl id")
        payload = [bytes(uid) if rank == 0 else None]
        dist.broadcast_object_list(payload, src=0)
        uid = (ctypes.c_char * 128).from_buffer_copy(payload[0])
        abi.check(abi.lib().mtc_comm_init(rank, rank, world, uid, 128, ctypes.byref(comm)), "nccl init")
        fe = Frontend()
        tr = MlpTrainer(fe, rank, WIDTHS[0], WIDTHS[1], WIDTHS[2], WIDTHS[3], seed=9, lr=LR)
        tr.set_comm(comm, world)
        x, y = _data()
        shard = BATCH // world
        xs = np.ascontiguousarray(x[rank * shard:(rank + 1) * shard])
        ys = np.ascontiguousarray(y[rank * shard:(rank + 1) * shard])
        tr.load_batch(xs.ctypes.data, ys.ctypes.data, shard)
        losses = [tr.step_resident(read_loss=True) for _ in range(STEPS)]
        # one more step from host memory: the input pipeline, with the loss read
        # right after the first layer of the gradient exchange
        losses.append(tr.step_host(xs.ctypes.data, ys.ctypes.data, shard))
        np.savez(out_path, losses=np.array(losses, dtype=np.float64), params=tr.parameters())
        tr.close()
        dist.barrier()
    finally:
        if comm:
            abi.lib().mtc_comm_destroy(comm)
        dist.destroy_process_group()


def test_two_gpu_training_matches_one_gpu(cuda, tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from minitensor_cpp_b200.frontend import Frontend, MlpTrainer

    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(tmp_path / f"rank{r}.npz"))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    r0 = np.load(tmp_path / "rank0.npz")
    r1 = np.load(tmp_path / "rank1.npz")
    np.testing.assert_array_equal(r0["params"], r1["params"])

    fe = Frontend()
    single = MlpTrainer(fe, 0, WIDTHS[0], WIDTHS[1], WIDTHS[2], WIDTHS[3], seed=9, lr=LR)
    x, y = _data()
    single.load_batch(x.ctypes.data, y.ctypes.data, BATCH)
    losses = [single.step_resident(read_loss=True) for _ in range(STEPS)]
    losses = np.array(losses + [single.step_host(x.ctypes.data, y.ctypes.data, BATCH)])
    mean_rank_loss = (r0["losses"] + r1["losses"]) / 2
    np.testing.assert_allclose(mean_rank_loss, losses, rtol=1e-5, atol=1e-6)
    diff = np.abs(single.parameters() - r0["params"])
    # Adam may flip the sign of an update whose gradient is within rounding of zero (moves 2*lr)
    assert diff.max() <= (STEPS + 1) * 2 * LR + 1e-6
    assert np.mean(diff > 1e-5) < 0.02, float(np.mean(diff > 1e-5))
    single.close()
