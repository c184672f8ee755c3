"""ctypes binding of the workload entry points (host/workloads.hpp).

`Frontend()` loads libminitensor_b200.so: MiniTensor's own C++ front-end
(Tensor / lazy graph / autograd / nn / AdamW) built with the CUDA backend, so a
workload placed on `device >= 0` runs on cuda:device through the backend and
`device = -1` runs the reference CPU kernels.  The same API is exported by the
oracle library (oracle/_ref/libmtref.so, CPU only) for baselines and parity.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "lib" / "libminitensor_b200.so"

# int sum_in_place(void *buffer, size_t count): sums a float buffer over all ranks
HOST_ALLREDUCE = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t)


class Frontend:
    def __init__(self, path: Path | str = LIB):
        path = Path(path)
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built; run __graft_entry__.build()")
        try:  # PyTorch's CUDA runtime and NCCL first, so one copy of each serves the process
            import torch  # noqa: F401
        except ImportError:
            pass
        # RTLD_LOCAL: the backend library and the oracle define the same MiniTensor
        # symbols; each must bind to its own copy (both are linked -Bsymbolic)
        self.lib = ctypes.CDLL(str(path), mode=os.RTLD_LOCAL)
        L = self.lib
        P = ctypes.POINTER
        vp, i32, i64, u64, f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float
        sigs = {
            "mtb_last_error": ([], ctypes.c_char_p),
            "mtb_has_cuda": ([], ctypes.c_int),
            "mtb_spiral_train": ([ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, u64, f32, ctypes.c_int,
                                  P(f32), P(ctypes.c_double)], ctypes.c_int),
            "mtb_mlp_create": ([ctypes.c_int, i64, i64, i32, i64, u64, f32, P(vp)], ctypes.c_int),
            "mtb_mlp_destroy": ([vp], None),
            "mtb_mlp_set_comm": ([vp, vp, i32], ctypes.c_int),
            "mtb_mlp_set_host_allreduce": ([vp, HOST_ALLREDUCE, i32], ctypes.c_int),
            "mtb_mlp_load_batch": ([vp, vp, vp, i64], ctypes.c_int),
            "mtb_mlp_load_batch_slot": ([vp, i32, vp, vp, i64], ctypes.c_int),
            "mtb_mlp_use_slot": ([vp, i32], ctypes.c_int),
            "mtb_mlp_step_resident": ([vp, i32, P(f32)], ctypes.c_int),
            "mtb_mlp_step_host": ([vp, vp, vp, i64, P(f32)], ctypes.c_int),
            "mtb_mlp_parameters": ([vp, P(f32), i64], ctypes.c_int),
            "mtb_mlp_parameter_count": ([vp], i64),
            "mtb_mlp_gradients": ([vp, P(f32), P(f32), i64], ctypes.c_int),
            "mtb_mlp_use_sgd": ([vp, f32], ctypes.c_int),
            "mtb_mlp_set_parameters": ([vp, P(f32), i64], ctypes.c_int),
            "mtb_mlp_profile": ([vp, i32, P(ctypes.c_double)], ctypes.c_int),
            "mtb_mlp_save": ([vp, ctypes.c_char_p], ctypes.c_int),
            "mtb_mlp_load": ([vp, ctypes.c_char_p], ctypes.c_int),
            "mtb_cross_entropy": ([ctypes.c_int, i64, i64, P(f32), i32, P(i64), P(f32), P(f32)], ctypes.c_int),
            "mtb_optimizer_steps": ([ctypes.c_int, i32, i64, P(f32), i32, P(f32), f32, f32, f32, f32, f32, P(f32)],
                                    ctypes.c_int),
            "mtb_mlp_synchronize": ([vp], ctypes.c_int),
            "mtb_mlp_materialize": ([vp], ctypes.c_int),
            "mtb_mlp_stream": ([vp], vp),
            "mtb_chain": ([ctypes.c_int, i64, i64, P(f32), P(f32), P(f32), P(f32), P(f32), P(f32)], ctypes.c_int),
            "mtb_gather_rows": ([ctypes.c_int, i64, i64, P(f32), i64, P(i64), P(f32)], ctypes.c_int),
            "mtb_evaluator_stats": ([P(u64)], None),
            "mtb_evaluator_reset_stats": ([], None),
            "mtb_graph_cache_clear": ([], None),
            "mtb_set_graphs": ([ctypes.c_int], ctypes.c_int),
            "mtb_set_fusion": ([ctypes.c_int], ctypes.c_int),
        }
        for name, (args, res) in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        # only the backend library has the operations it adds to MiniTensor
        if hasattr(L, "mtb_gather_eval_probe"):
            L.mtb_gather_eval_probe.argtypes = [ctypes.c_int, i64, i64, P(f32), i64, P(i64), P(i32), P(i32)]
            L.mtb_gather_eval_probe.restype = ctypes.c_int
            L.mtb_set_index_checks.argtypes = [ctypes.c_int]
            L.mtb_set_index_checks.restype = ctypes.c_int
        if hasattr(L, "mtb_added_ops"):
            L.mtb_added_ops.argtypes = [ctypes.c_int, i64, i64, P(f32), i32, P(f32), P(f32), P(i64), P(f32), P(f32)]
            L.mtb_added_ops.restype = ctypes.c_int

    def _check(self, rc: int, what: str):
        if rc == 0:
            return
        msg = self.lib.mtb_last_error().decode(errors="replace")
        exc = {1: ValueError, 2: IndexError, 5: OverflowError}.get(rc, RuntimeError)
        raise exc(f"{what}: {msg}")

    @property
    def has_cuda(self) -> bool:
        return bool(self.lib.mtb_has_cuda())

    def spiral_train(self, device: int, steps: int, points: int = 100, hidden: int = 64, seed: int = 0,
                     lr: float = 1e-2, loss_every: int = 1):
        losses = np.full(max(steps, 1), np.nan, dtype=np.float32)
        secs = ctypes.c_double(0.0)
        self._check(self.lib.mtb_spiral_train(device, steps, points, hidden, seed, lr, loss_every,
                                              losses.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                              ctypes.byref(secs)), "spiral_train")
        return losses[:steps], secs.value

    def chain(self, device: int, a, b_storage, row, col, reductions: bool = False):
        n, m = a.shape
        out = np.empty((n, m), dtype=np.float32)
        red = np.empty(m + 2 * n, dtype=np.float32) if reductions else None
        f = lambda x: np.ascontiguousarray(x, dtype=np.float32).ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        keep = [np.ascontiguousarray(x, dtype=np.float32) for x in (a, b_storage, row, col)]
        self._check(self.lib.mtb_chain(device, n, m, *[k.ctypes.data_as(ctypes.POINTER(ctypes.c_float)) for k in keep],
                                       out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                       red.ctypes.data_as(ctypes.POINTER(ctypes.c_float)) if red is not None else None),
                    "chain")
        if red is None:
            return out
        return out, red[:m], red[m:m + n], red[m + n:]

    def gather_rows(self, device: int, table: np.ndarray, index: np.ndarray) -> np.ndarray:
        """table[index, :] through MiniTensor's gather (IndexError for an index out of range)."""
        t = np.ascontiguousarray(table, dtype=np.float32)
        i = np.ascontiguousarray(index, dtype=np.int64)
        out = np.empty((i.size, t.shape[1]), dtype=np.float32)
        P = ctypes.POINTER
        self._check(self.lib.mtb_gather_rows(device, t.shape[0], t.shape[1], t.ctypes.data_as(P(ctypes.c_float)),
                                             i.size, i.ctypes.data_as(P(ctypes.c_int64)),
                                             out.ctypes.data_as(P(ctypes.c_float))), "gather_rows")
        return out

    def added_ops(self, device: int, x: np.ndarray, axis: int):
        """relu(x), and max, argmax and log-softmax of x along `axis`, and the
        gradient of sum(relu(x)), through the operations this backend adds to
        MiniTensor's API."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, cols = x.shape
        relu = np.empty_like(x)
        lsm = np.empty_like(x)
        grad = np.empty_like(x)
        reduced = cols if axis == 0 else rows
        mx = np.empty(reduced, dtype=np.float32)
        am = np.empty(reduced, dtype=np.int64)
        P = ctypes.POINTER
        f = lambda a: a.ctypes.data_as(P(ctypes.c_float))
        self._check(self.lib.mtb_added_ops(device, rows, cols, f(x), axis, f(relu), f(mx),
                                           am.ctypes.data_as(P(ctypes.c_int64)), f(lsm), f(grad)), "added_ops")
        return relu, mx, am, lsm, grad

    def gather_eval_probe(self, device: int, table: np.ndarray, index: np.ndarray):
        """(threw, materialized) of evaluating a row gather with mt::eval (see
        workloads.hpp); a deferred index error raises IndexError from the read
        that follows."""
        t = np.ascontiguousarray(table, dtype=np.float32)
        i = np.ascontiguousarray(index, dtype=np.int64)
        threw, mat = ctypes.c_int32(0), ctypes.c_int32(0)
        P = ctypes.POINTER
        self._check(self.lib.mtb_gather_eval_probe(device, t.shape[0], t.shape[1], t.ctypes.data_as(P(ctypes.c_float)),
                                                   i.size, i.ctypes.data_as(P(ctypes.c_int64)), ctypes.byref(threw),
                                                   ctypes.byref(mat)), "gather_eval_probe")
        return bool(threw.value), bool(mat.value)

    def set_index_checks(self, mode: str) -> str:
        """"off", "deferred" (default) or "sync"; returns the previous mode."""
        names = ("off", "deferred", "sync")
        return names[self.lib.mtb_set_index_checks(names.index(mode))]

    def cross_entropy(self, device: int, logits: np.ndarray, targets: np.ndarray, class_axis: int = 1):
        """(loss, d loss / d logits) of categorical_cross_entropy_with_logits on a
        [rows, cols] matrix through the API."""
        x = np.ascontiguousarray(logits, dtype=np.float32)
        t = np.ascontiguousarray(targets, dtype=np.int64)
        loss = ctypes.c_float(0.0)
        grad = np.empty_like(x)
        P = ctypes.POINTER
        self._check(self.lib.mtb_cross_entropy(device, x.shape[0], x.shape[1], x.ctypes.data_as(P(ctypes.c_float)),
                                               class_axis, t.ctypes.data_as(P(ctypes.c_int64)), ctypes.byref(loss),
                                               grad.ctypes.data_as(P(ctypes.c_float))), "cross_entropy")
        return loss.value, grad

    def optimizer_steps(self, device: int, kind: str, params: np.ndarray, grads: np.ndarray, lr: float,
                        weight_decay: float = 0.0, beta1: float = 0.9, beta2: float = 0.999,
                        eps: float = 1e-8) -> np.ndarray:
        """Parameters after len(grads) steps of AdamW ("adamw") or SGD ("sgd") on one
        parameter vector through the API; grads is [steps, n]."""
        p = np.ascontiguousarray(params, dtype=np.float32).reshape(-1)
        g = np.ascontiguousarray(grads, dtype=np.float32).reshape(-1, p.size)
        out = np.empty_like(p)
        P = ctypes.POINTER
        f = lambda a: a.ctypes.data_as(P(ctypes.c_float))
        self._check(self.lib.mtb_optimizer_steps(device, {"adamw": 0, "sgd": 1}[kind], p.size, f(p), g.shape[0], f(g),
                                                 lr, weight_decay, beta1, beta2, eps, f(out)), "optimizer_steps")
        return out

    def stats(self) -> dict:
        buf = (ctypes.c_uint64 * 13)()
        self.lib.mtb_evaluator_stats(buf)
        keys = ("kernel_steps", "fused_launches", "fused_nodes", "folded_constants", "view_steps", "evaluations",
                "plan_ns", "execute_ns", "check_ns", "graph_captures", "graph_replays", "graph_fallbacks",
                "scatters_deferred")
        return dict(zip(keys, list(buf)))

    def reset_stats(self):
        self.lib.mtb_evaluator_reset_stats()

    def set_fusion(self, on: bool) -> bool:
        """Turns elementwise fusion on or off; returns the previous setting."""
        return bool(self.lib.mtb_set_fusion(1 if on else 0))

    def set_graphs(self, on: bool) -> bool:
        """Turns the replay of repeated evaluation plans on or off; returns the previous setting."""
        return bool(self.lib.mtb_set_graphs(1 if on else 0))

    def clear_graphs(self):
        """Destroys every plan recorded for replay."""
        self.lib.mtb_graph_cache_clear()


class MlpTrainer:
    """The wide-MLP trainer of host/workloads.cpp on one device."""

    def __init__(self, fe: Frontend, device: int, in_features: int, hidden: int, hidden_layers: int, classes: int,
                 seed: int, lr: float):
        self.fe = fe
        self.in_features = in_features
        self.h = ctypes.c_void_p()
        fe._check(fe.lib.mtb_mlp_create(device, in_features, hidden, hidden_layers, classes, seed, lr,
                                        ctypes.byref(self.h)), "mlp_create")

    def close(self):
        if self.h:
            self.fe.lib.mtb_mlp_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_comm(self, comm, world: int):
        self.fe._check(self.fe.lib.mtb_mlp_set_comm(self.h, comm, world), "mlp_set_comm")

    def set_host_allreduce(self, sum_in_place, world: int):
        """CPU-device data parallelism: sum_in_place(ndarray) sums a float32 view over the ranks in place."""
        import numpy as np

        def _cb(ptr, count):
            try:
                arr = np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctypes.c_float)), shape=(count,))
                sum_in_place(arr)
                return 0
            except Exception:  # reported to C++ as a failed exchange
                return 1

        self._host_cb = HOST_ALLREDUCE(_cb)  # keep alive while attached
        self.fe._check(self.fe.lib.mtb_mlp_set_host_allreduce(self.h, self._host_cb, world), "mlp_set_host_allreduce")

    def load_batch(self, x_ptr: int, y_ptr: int, batch: int):
        self.fe._check(self.fe.lib.mtb_mlp_load_batch(self.h, x_ptr, y_ptr, batch), "mlp_load_batch")

    def load_batch_slot(self, slot: int, x_ptr: int, y_ptr: int, batch: int):
        """Uploads a batch into resident slot `slot` (not made current)."""
        self.fe._check(self.fe.lib.mtb_mlp_load_batch_slot(self.h, slot, x_ptr, y_ptr, batch), "mlp_load_batch_slot")

    def use_slot(self, slot: int):
        """Makes resident slot `slot` the batch of the following steps (no copy)."""
        self.fe._check(self.fe.lib.mtb_mlp_use_slot(self.h, slot), "mlp_use_slot")

    def step_resident(self, read_loss: bool = False) -> float:
        loss = ctypes.c_float(0.0)
        self.fe._check(self.fe.lib.mtb_mlp_step_resident(self.h, int(read_loss), ctypes.byref(loss)), "mlp_step")
        return loss.value

    def step_host(self, x_ptr: int, y_ptr: int, batch: int) -> float:
        loss = ctypes.c_float(0.0)
        self.fe._check(self.fe.lib.mtb_mlp_step_host(self.h, x_ptr, y_ptr, batch, ctypes.byref(loss)), "mlp_step_host")
        return loss.value

    def parameters(self) -> np.ndarray:
        n = self.fe.lib.mtb_mlp_parameter_count(self.h)
        out = np.empty(n, dtype=np.float32)
        self.fe._check(self.fe.lib.mtb_mlp_parameters(self.h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n),
                       "mlp_parameters")
        return out

    def gradients(self):
        """(loss, gradients) on the resident batch at the current parameters, without an
        update; gradients in the order of parameters()."""
        n = self.fe.lib.mtb_mlp_parameter_count(self.h)
        out = np.empty(n, dtype=np.float32)
        loss = ctypes.c_float(0.0)
        self.fe._check(self.fe.lib.mtb_mlp_gradients(self.h, ctypes.byref(loss),
                                                     out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n),
                       "mlp_gradients")
        return loss.value, out

    def save(self, path) -> None:
        """Writes the parameters under their tree paths to `path`."""
        self.fe._check(self.fe.lib.mtb_mlp_save(self.h, os.fsencode(path)), "mlp_save")

    def load(self, path) -> None:
        """Replaces the parameters with those saved at `path` (matched by path)."""
        self.fe._check(self.fe.lib.mtb_mlp_load(self.h, os.fsencode(path)), "mlp_load")

    def profile(self, on: bool):
        """Switches the device-time phase profile on or off; returns the
        milliseconds summed since the last call: (steps, forward + backward,
        exposed gradient exchange, optimizer)."""
        ms = (ctypes.c_double * 4)()
        self.fe._check(self.fe.lib.mtb_mlp_profile(self.h, int(on), ms), "mlp_profile")
        return tuple(ms)

    def set_parameters(self, values: np.ndarray):
        """Replaces the parameters with `values` (the order of parameters())."""
        v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        self.fe._check(self.fe.lib.mtb_mlp_set_parameters(self.h, v.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                                          v.size), "mlp_set_parameters")

    def use_sgd(self, lr: float):
        """SGD(lr) replaces Adam for the following steps."""
        self.fe._check(self.fe.lib.mtb_mlp_use_sgd(self.h, lr), "mlp_use_sgd")

    def synchronize(self):
        self.fe._check(self.fe.lib.mtb_mlp_synchronize(self.h), "mlp_synchronize")

    def materialize(self):
        self.fe._check(self.fe.lib.mtb_mlp_materialize(self.h), "mlp_materialize")

    def stream(self) -> int:
        return self.fe.lib.mtb_mlp_stream(self.h) or 0
