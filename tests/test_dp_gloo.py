"""Data-parallel training path at world size 2 on CPU (gloo process group).

Each rank trains the MLP trainer of host/workloads.cpp on its half of the
batch; the trainer's gradient exchange (materialise gradients, locate their
dense storage, sum over ranks, scale by 1/world, then the unchanged AdamW
step) runs with a gloo all-reduce as the host callback.  The result must equal
single-process training on the full batch: the mean of the two half-batch
losses equals the full-batch loss, so the averaged gradients agree to rounding.
"""
import os
import socket

import numpy as np
import pytest

F = np.float32
WIDTHS = (12, 16, 5)
BATCH = 64
STEPS = 3
LR = 1e-2


def _data():
    rng = np.random.default_rng(17)
    x = rng.standard_normal((BATCH, WIDTHS[0])).astype(F)
    y = rng.integers(0, WIDTHS[-1], BATCH).astype(np.int64)
    return x, y


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_path):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist

    from minitensor_cpp_b200.frontend import Frontend, MlpTrainer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fe = Frontend()
        tr = MlpTrainer(fe, -1, WIDTHS[0], WIDTHS[1], 1, WIDTHS[-1], seed=5, lr=LR)

        def sum_in_place(arr):
            t = torch.from_numpy(arr)
            dist.all_reduce(t, op=dist.ReduceOp.SUM)

        tr.set_host_allreduce(sum_in_place, world)
        x, y = _data()
        shard = BATCH // world
        xs = np.ascontiguousarray(x[rank * shard:(rank + 1) * shard])
        ys = np.ascontiguousarray(y[rank * shard:(rank + 1) * shard])
        tr.load_batch(xs.ctypes.data, ys.ctypes.data, shard)
        losses = [tr.step_resident(read_loss=True) for _ in range(STEPS)]
        np.savez(out_path, losses=np.array(losses, dtype=np.float64), params=tr.parameters())
        tr.close()
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_training_matches_single_process(tmp_path):
    import torch.multiprocessing as mp

    from minitensor_cpp_b200.frontend import Frontend, MlpTrainer

    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = []
    for r in range(2):
        p = ctx.Process(target=_rank_main, args=(r, 2, port, str(tmp_path / f"rank{r}.npz")))
        p.start()
        procs.append(p)
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    r0 = np.load(tmp_path / "rank0.npz")
    r1 = np.load(tmp_path / "rank1.npz")
    # both ranks hold identical parameters after every exchange
    np.testing.assert_array_equal(r0["params"], r1["params"])

    fe = Frontend()
    single = MlpTrainer(fe, -1, WIDTHS[0], WIDTHS[1], 1, WIDTHS[-1], seed=5, lr=LR)
    x, y = _data()
    single.load_batch(x.ctypes.data, y.ctypes.data, BATCH)
    losses = np.array([single.step_resident(read_loss=True) for _ in range(STEPS)])
    mean_rank_loss = (r0["losses"] + r1["losses"]) / 2
    np.testing.assert_allclose(mean_rank_loss, losses, rtol=1e-5, atol=1e-6)
    diff = np.abs(single.parameters() - r0["params"])
    # Adam may flip the sign of a gradient within rounding of zero (moves 2*lr)
    assert diff.max() <= STEPS * 2 * LR + 1e-6
    assert np.mean(diff > 1e-5) < 0.02, float(np.mean(diff > 1e-5))
    single.close()


def _rank_fails_main(rank, world, port, out_path):
    """Rank 1 leaves before the gradient exchange; rank 0 must see the exchange
    fail (an exception from its step, within the process-group timeout) rather
    than hang."""
    import sys
    from datetime import timedelta

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist

    from minitensor_cpp_b200.frontend import Frontend, MlpTrainer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    if rank == 1:
        os._exit(3)  # the failure: this rank is gone before any collective
    fe = Frontend()
    tr = MlpTrainer(fe, -1, WIDTHS[0], WIDTHS[1], 1, WIDTHS[-1], seed=5, lr=LR)

    def sum_in_place(arr):
        t = torch.from_numpy(arr)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)

    tr.set_host_allreduce(sum_in_place, world)
    x, y = _data()
    tr.load_batch(x.ctypes.data, y.ctypes.data, BATCH // world)
    try:
        tr.step_resident(read_loss=True)
        outcome = "completed"
    except RuntimeError as e:
        outcome = f"failed: {e}"
    with open(out_path, "w") as f:
        f.write(outcome)
    os._exit(0)


def test_a_rank_that_leaves_makes_the_exchange_fail_not_hang(tmp_path):
    import torch.multiprocessing as mp

    port = _free_port()
    ctx = mp.get_context("spawn")
    out = tmp_path / "rank0.txt"
    procs = [ctx.Process(target=_rank_fails_main, args=(r, 2, port, str(out))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0
    text = out.read_text()
    assert text.startswith("failed:") and "all-reduce" in text, text
