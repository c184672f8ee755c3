// Benchmark and parity workloads written against MiniTensor's unchanged public
// API (the way a user program such as demo.cpp is written).  The same source is
// compiled into libminitensor_b200.so (any device) and, with MTB_CPU_ONLY, into
// the oracle library built from the unmodified reference (CPU device only), so
// both sides run exactly the same graphs.  C ABI for the Python drivers.
#pragma once

#include <cstddef>
#include <cstdint>

#ifdef __cplusplus
extern "C" {
#endif

// Thread-local message of the last failing call.
const char *mtb_last_error(void);
// Status codes follow include/mtcuda.h (0 = ok).

// Spiral classification (3 classes x `points` points, seed 0 keys split as in
// demo.cpp:163-164), MLP 2 -> hidden -> hidden -> 3 with ReLU, softmax cross
// entropy, Adam (AdamW(lr, 0)), full batch.  device < 0 = CPU, else cuda:device.
// losses[s] receives the loss of step s when (s % loss_every == 0), or NaN.
int mtb_spiral_train(int device, int steps, int points, int hidden, uint64_t seed, float lr, int loss_every,
                     float *losses, double *seconds);

// Wide MLP trainer: in -> hidden (x layers) -> classes, ReLU, softmax cross
// entropy, Adam(lr).  Parameters initialised from `seed` (identical on every rank).
int mtb_mlp_create(int device, int64_t in_features, int64_t hidden, int32_t hidden_layers, int64_t classes,
                   uint64_t seed, float lr, void **handle);
void mtb_mlp_destroy(void *handle);
// Attach a data-parallel communicator (from mtc_comm_init) of `world` ranks:
// gradients are summed over ranks and scaled by 1/world before the update.
int mtb_mlp_set_comm(void *handle, void *comm, int32_t world);
// CPU-device data parallelism: `sum_in_place(buffer, count)` must sum the float
// buffer over all ranks in place (0 = ok); gradients are then scaled by 1/world.
int mtb_mlp_set_host_allreduce(void *handle, int (*sum_in_place)(void *, size_t), int32_t world);
// Upload one batch (host memory; copied to the device) that mtb_mlp_step_resident reuses.
int mtb_mlp_load_batch(void *handle, const float *x, const int64_t *labels, int64_t batch);
// Upload a batch into resident slot `slot` (0..64) without making it current;
// mtb_mlp_use_slot makes a slot the resident batch (no copy), so a timed loop
// can cycle through several device-resident batches.
int mtb_mlp_load_batch_slot(void *handle, int32_t slot, const float *x, const int64_t *labels, int64_t batch);
int mtb_mlp_use_slot(void *handle, int32_t slot);
// One training step on the resident batch; *loss receives the step's loss when read_loss != 0.
int mtb_mlp_step_resident(void *handle, int32_t read_loss, float *loss);
// One end-to-end training step from host buffers: the batch is copied host -> device,
// the step runs, and the loss is read back to the host.
int mtb_mlp_step_host(void *handle, const float *x, const int64_t *labels, int64_t batch, float *loss);
// Copies the current parameters (layer by layer: weight [out, in] then bias [out]) to host.
int mtb_mlp_parameters(void *handle, float *out, int64_t capacity);
// Gradients of the loss on the resident batch at the current parameters, without
// an update (nn::parameter_gradients): *loss receives the loss, `out` the
// gradients in the order of mtb_mlp_parameters.
int mtb_mlp_gradients(void *handle, float *loss, float *out, int64_t capacity);
// Device-time profile of the training steps (CUDA device): ms4 (may be NULL)
// receives the milliseconds summed over the steps profiled since the last call
// -- [0] whole steps, [1] forward + backward up to the wait for the gradient
// exchange, [2] the exchange's exposed part, [3] the optimizer -- and the
// profile is then switched on or off.  With one rank only [0] is measured.
int mtb_mlp_profile(void *handle, int32_t on, double *ms4);
// Checkpoint of the parameters under their tree paths (nn::for_each_named_parameter,
// include/minitensor/nn/parameters/parameter_tree.hpp:179-190: "layer0.weight",
// "layer0.bias", ...).  File format, little-endian: "MTBCKPT1" or "MTBCKPT2",
// u32 count, then per parameter u32 path length, path, u32 rank, i64 extents,
// float32 values.  Version 2 (the backend build with Adam) continues with the
// u64 step count and each parameter's first and second moments (float32, in
// the parameters' order); the build against the unmodified reference cannot
// reach AdamW::State's private moments and writes version 1.
int mtb_mlp_save(void *handle, const char *path);
// Loads a checkpoint of mtb_mlp_save onto the trainer's device, matched by path;
// every parameter of the model must be present with its shape.  A version-2
// file also restores Adam's step count and moments (backend build), so the
// following steps equal those of an uninterrupted run bit for bit.
int mtb_mlp_load(void *handle, const char *path);
// Replaces the parameters' values with `count` host values in the order of
// mtb_mlp_parameters (the optimizer state is kept).
int mtb_mlp_set_parameters(void *handle, const float *values, int64_t count);
// Replaces the trainer's Adam with SGD(lr) (include/minitensor/nn/optimizers/sgd.hpp)
// for the following steps.
int mtb_mlp_use_sgd(void *handle, float lr);
int64_t mtb_mlp_parameter_count(void *handle);
// Evaluates the (lazily initialised) parameters and optimizer state.
int mtb_mlp_materialize(void *handle);
// Blocks until the device finished all work of this trainer.
int mtb_mlp_synchronize(void *handle);
// The CUDA stream the trainer's kernels run on (NULL on the CPU).
void *mtb_mlp_stream(void *handle);

// relu(A * B^T + row) * exp(-col) through the API on `device` (inputs uploaded
// from host; B given as the [n, m] storage whose transpose view is used), result
// copied to `out` [n, m].  reductions (optional, may be NULL) receive
// sum(Y, 0) [m], sum(Y, 1) [n] and logsumexp(Y, 1) [n].
int mtb_chain(int device, int64_t n, int64_t m, const float *a, const float *b_storage, const float *row,
              const float *col, float *out, float *reductions);

// Row gather through the public API: out[r, :] = table[index[r], :] for n rows
// (gather along axis 0 with the index column broadcast over the row width).  An
// index outside [0, rows) raises out_of_range (MTC_ERR_OUT_OF_RANGE).
int mtb_gather_rows(int device, int64_t rows, int64_t cols, const float *table, int64_t n, const int64_t *index,
                    float *out);

// gather(table, 0, index broadcast along the row) evaluated with mt::eval and
// not read back: *threw = 1 when that evaluation itself raised out_of_range,
// *materialized = 1 when the result holds storage afterwards.  Without a throw
// the result is then read (to_vector), which raises a deferred index error
// (MTC_ERR_OUT_OF_RANGE).  Not in the CPU-only build.
int mtb_gather_eval_probe(int device, int64_t rows, int64_t cols, const float *table, int64_t n, const int64_t *index,
                          int32_t *threw, int32_t *materialized);
// How the CUDA evaluator checks gather / scatter-add indices: 0 = not at all,
// 1 = deferred to the next evaluation or read (default), 2 = synchronously
// before the kernel's output is installed (as MTB_INDEX_CHECKS=sync).  Returns
// the previous mode.  Not in the CPU-only build.
int mtb_set_index_checks(int mode);

// The operations this backend adds (relu, max, argmax, log-softmax) on a
// [rows, cols] matrix through the public API; the reductions run along `axis`
// (0 or 1).  relu_out, log_softmax_out and relu_grad_out (the gradient of
// sum(relu(x)) through relu's VJP rule; may be NULL) hold rows * cols values,
// max_out and argmax_out the extent of the other axis.  Not in the CPU-only
// build: the unmodified reference has none of these operations.
int mtb_added_ops(int device, int64_t rows, int64_t cols, const float *x, int32_t axis, float *relu_out,
                  float *max_out, int64_t *argmax_out, float *log_softmax_out, float *relu_grad_out);

// categorical_cross_entropy_with_logits (src/nn/loss.cpp:41-57) of a [rows, cols]
// logits matrix whose classes run along `class_axis` (0 or 1), with Int64
// targets (one per row for axis 1, one per column for axis 0), through the API
// on `device`: *loss receives the mean loss, grad (rows * cols, may be NULL)
// its gradient with respect to the logits (autograd `grad`).
int mtb_cross_entropy(int device, int64_t rows, int64_t cols, const float *logits, int32_t class_axis,
                      const int64_t *targets, float *loss, float *grad);

// `steps` optimizer steps on one parameter vector of n values through the API on
// `device`: kind 0 = AdamW(lr, weight_decay, beta1, beta2, eps)
// (src/nn/optimizers/adamw.cpp:53-97), kind 1 = SGD(lr) (sgd.hpp:30-39).
// grads holds steps * n values (step s uses grads[s * n ...]); out receives the
// parameters after the last step.  The parameters and the optimizer state are
// leafified after every step, as a training loop does.
int mtb_optimizer_steps(int device, int32_t kind, int64_t n, const float *params, int32_t steps, const float *grads,
                        float lr, float weight_decay, float beta1, float beta2, float eps, float *out);

// Counters of the fusing evaluator (zeros in the CPU-only build):
// kernel_steps, fused_launches, fused_nodes, folded_constants, view_steps, evaluations,
// host nanoseconds spent planning, issuing kernels and in the index-error check,
// graph_captures, graph_replays, graph_fallbacks, scatters_deferred.
void mtb_evaluator_stats(uint64_t *out13);
void mtb_evaluator_reset_stats(void);
// Destroys every plan recorded for replay.
void mtb_graph_cache_clear(void);
// Turns the replay of repeated plans on or off; returns the previous setting.
int mtb_set_graphs(int on);
// Turns elementwise fusion (and the scatter-add deferral) on or off; returns
// the previous setting.
int mtb_set_fusion(int on);
// 1 when the library has the CUDA backend, 0 for the CPU-only build.
int mtb_has_cuda(void);

#ifdef __cplusplus
}
#endif
