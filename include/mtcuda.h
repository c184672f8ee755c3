/*
 * mtcuda.h — C ABI of the B200 (sm_100a) CUDA backend for MiniTensor.
 *
 * Every entry point here replaces one CPU kernel (a `KernelFn` registered under
 * `KernelKey{PrimitiveId, DeviceType}`, src/tensor/dispatch/kernel_registry.hpp:15-16)
 * or one `DeviceRuntime` method (src/tensor/backend/device_runtime.hpp:13-29) of the
 * MiniTensor reference.  The C++ adapter that registers these under
 * `DeviceType::Cuda` lives in minitensor_cpp_b200/host/; any other host language
 * can bind the same symbols (ctypes, cgo, JNI) because the signatures carry only
 * plain pointers, integers and the POD descriptor below.
 *
 * Conventions
 *  - A tensor operand is an `mtc_desc`: base pointer of the device buffer, plus
 *    shape, strides and offset counted in ELEMENTS, exactly like the reference
 *    `Layout{strides, offset}` (src/tensor/storage/layout.hpp:18-42).  Strides may be
 *    zero (broadcast views) or negative (reversed slices); offsets are >= 0.
 *  - `capacity` is the buffer size in elements.  Every entry point checks on the
 *    host that every reachable element of every view lies inside [0, capacity),
 *    like `Materialization::validate` (src/tensor/storage/materialization.cpp:77-129),
 *    and returns MTC_ERR_OUT_OF_RANGE otherwise; no kernel is launched then.
 *  - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default stream)
 *    and returns without synchronising.  Data-dependent failures that can only be
 *    seen on the device (a gather index outside its axis) are recorded in a
 *    per-device error word and reported by mtc_check_device_errors().
 *  - Return value: MTC_OK or one of the MTC_ERR_* codes; mtc_last_error() gives a
 *    thread-local message.  No C++ exception crosses this boundary.  The codes map
 *    one-to-one onto the reference's exception types (invalid_argument,
 *    out_of_range, runtime_error, logic_error, overflow_error).
 */
#ifndef MTCUDA_H
#define MTCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MTC_MAX_RANK 8
#define MTC_MAX_FUSED_OPERANDS 12
#define MTC_MAX_FUSED_OUTPUTS 4
#define MTC_MAX_FUSED_INSTRUCTIONS 96
#define MTC_MAX_CONCAT_INPUTS 64

/* Status codes (reference exception type in brackets). */
enum {
    MTC_OK = 0,
    MTC_ERR_INVALID_ARGUMENT = 1, /* std::invalid_argument */
    MTC_ERR_OUT_OF_RANGE = 2,     /* std::out_of_range      */
    MTC_ERR_RUNTIME = 3,          /* std::runtime_error (CUDA / NCCL failure) */
    MTC_ERR_LOGIC = 4,            /* std::logic_error       */
    MTC_ERR_OVERFLOW = 5,         /* std::overflow_error    */
    MTC_ERR_UNSUPPORTED = 6       /* no kernel for this case (std::runtime_error) */
};

/* Element types: the numbering of minitensor::DType (include/minitensor/types.hpp:55-59). */
enum { MTC_FLOAT32 = 0, MTC_INT64 = 1 };

/* Operation codes.  Codes of reference primitives equal their PrimitiveId value
 * (src/tensor/primitives/<family>/<op>.hpp: `static constexpr PrimitiveId ID{...}`);
 * codes >= 0x..80 within a family are additions of this backend. */
enum {
    /* unary elementwise, src/tensor/backend/cpu/kernels/elementwise/kernels.cpp:58-125 */
    MTC_OP_ABS = 0x0101,
    MTC_OP_SIGN = 0x0102,
    MTC_OP_NEGATE = 0x0103,
    MTC_OP_EXP = 0x0104,
    MTC_OP_LOG = 0x0105,
    MTC_OP_SQRT = 0x0106,
    MTC_OP_TANH = 0x0107,
    MTC_OP_SIGMOID = 0x0108,
    MTC_OP_RELU = 0x0180, /* new: max(x, 0), NaN propagates */
    /* binary elementwise, elementwise/kernels.cpp:127-167 */
    MTC_OP_ADD = 0x0110,
    MTC_OP_SUBTRACT = 0x0111,
    MTC_OP_MULTIPLY = 0x0112,
    MTC_OP_DIVIDE = 0x0113,
    MTC_OP_LOGADDEXP = 0x0114,
    /* fused-program pseudo ops */
    MTC_OP_CONST = 0x01F0, /* dst = imm */
    /* reductions, src/tensor/backend/cpu/kernels/reduction/kernels.cpp:22-42 */
    MTC_OP_SUM = 0x0301,
    MTC_OP_LOGSUMEXP = 0x0302,
    MTC_OP_MAX = 0x0380,    /* new: NaN propagates, empty -> -inf */
    MTC_OP_ARGMAX = 0x0381  /* new: Int64 output, first maximum; a NaN counts as the maximum */
};

/* Strided view of a device buffer (reference TensorView, src/tensor/dispatch/tensor_view.hpp:15-45). */
typedef struct mtc_desc {
    void *data;       /* base address of the buffer (element 0 of the storage) */
    int64_t offset;   /* Layout::offset(), in elements, >= 0 */
    int64_t capacity; /* buffer size in elements */
    int32_t dtype;    /* MTC_FLOAT32 / MTC_INT64 */
    int32_t rank;     /* 0..MTC_MAX_RANK */
    int64_t shape[MTC_MAX_RANK];
    int64_t strides[MTC_MAX_RANK]; /* Layout::strides(), in elements */
} mtc_desc;

/* One instruction of a fused elementwise program (see mtc_fused). */
typedef struct mtc_instr {
    int32_t op;  /* MTC_OP_* unary/binary code, or MTC_OP_CONST */
    int16_t dst; /* destination register */
    int16_t a;   /* first source register */
    int16_t b;   /* second source register (binary ops) */
    int16_t pad;
    float imm;   /* MTC_OP_CONST value */
} mtc_instr;

/* ---------------------------------------------------------------- library -- */

/* Thread-local text of the last failure on this thread ("" when none). */
const char *mtc_last_error(void);
/* Version string of the library and the architecture it was compiled for. */
const char *mtc_version(void);
/* Number of visible CUDA devices (0 when no driver/GPU is present). */
int mtc_device_count(int *count);
/* Streaming-multiprocessor count of `device` (grid sizing; 148 on B200). */
int mtc_device_sm_count(int device, int *count);
/* Makes `device` current for the calling thread (kernels launch on the current device). */
int mtc_set_device(int device);

/* ------------------------------------------------------ DeviceRuntime (A2) --
 * Replaces CpuRuntime/CpuBuffer (src/tensor/backend/cpu/cpu_runtime.cpp:31-87,
 * cpu_buffer.cpp:13-32).  Memory comes from a per-device caching allocator whose
 * blocks are reused in stream order, so freed blocks serve later work on the
 * same stream without a device synchronisation. */

/* Per-device work stream created on first use (non-blocking w.r.t. the legacy stream). */
int mtc_device_stream(int device, void **stream);
/* Stream-ordered allocation of `bytes` on `device` from the backend's caching
 * allocator (cached blocks are reused in stream order; cudaMalloc only when
 * nothing fits); *ptr = NULL for 0 bytes (the reference hands out a valid
 * empty buffer, runtime_test.cpp:85-94). */
int mtc_alloc(int device, size_t bytes, void *stream, void **ptr);
/* Stream-ordered release of a block from mtc_alloc: reusable at once by later
 * work on `stream`, by other streams once `stream` has passed this point. */
int mtc_free(int device, void *ptr, void *stream);
/* Host -> device copy, ordered on `stream`; `src` must stay valid until the
 * stream reaches the copy (pageable sources are staged by the driver before return). */
int mtc_copy_from_host(int device, void *dst, const void *src, size_t bytes, void *stream);
/* Device -> host copy; returns after the data is in `dst` (synchronises `stream`). */
int mtc_copy_to_host(int device, void *dst, const void *src, size_t bytes, void *stream);
/* Wait for all work queued on `stream`. */
int mtc_stream_synchronize(void *stream);
/* Streams and events for callers that overlap their own host transfers with
 * work queued on the device stream (an input pipeline: the next batch's copy
 * runs while the current step computes).  No reference counterpart: the
 * reference copies and evaluates synchronously on one host thread.
 * mtc_stream_create makes a stream that does not synchronise with the legacy
 * default stream; mtc_event_create an event without timing.  A wait on an
 * event that was never recorded returns at once. */
int mtc_stream_create(int device, void **stream);
int mtc_stream_destroy(int device, void *stream);
int mtc_event_create(int device, void **event);
int mtc_event_destroy(int device, void *event);
int mtc_event_record(void *event, void *stream);
int mtc_stream_wait_event(void *stream, void *event);
/* Events that record a time stamp, for measuring phases of work on a stream;
 * mtc_event_elapsed waits for `stop` and gives the milliseconds between the two
 * recordings.  No reference counterpart. */
int mtc_event_create_timed(int device, void **event);
int mtc_event_elapsed(void *start, void *stop, float *milliseconds);
/* Bytes held from the driver by / handed out from the caching allocator. */
int mtc_pool_stats(int device, uint64_t *reserved_bytes, uint64_t *used_bytes);
/* Return cached-but-unused blocks to the driver (synchronises the device).
 * Blocks protected for recorded graphs (mtc_pool_protect) stay. */
int mtc_pool_trim(int device);

/* Device-side error word: synchronises `stream`, then returns MTC_ERR_OUT_OF_RANGE
 * (and the offending index in *detail) if a gather/scatter kernel met an index
 * outside its axis since the last check, MTC_OK otherwise; the word is cleared. */
int mtc_check_device_errors(int device, void *stream, int64_t *detail);
/* Asynchronous form of the same check, for evaluators that must not
 * synchronise: mtc_watch_device_errors queues a copy of the error word to
 * pinned host memory on `stream` behind the work queued so far;
 * mtc_poll_device_errors returns MTC_ERR_OUT_OF_RANGE (index in *detail) when
 * the latest such copy, once it has arrived (wait = 0) or after waiting for it
 * (wait = 1), shows an error, and clears the word.  No reference counterpart:
 * the reference's CPU loop throws out_of_range inline (copy/loops.hpp:206-209);
 * here the throw comes at the next evaluation or device-to-host read. */
int mtc_watch_device_errors(int device, void *stream);
int mtc_poll_device_errors(int device, int wait, int64_t *detail);
/* Failure-path self-test: a one-thread kernel waits on a shared-memory barrier
 * that nothing completes, gives up after `spins` polls (1 .. 2^24) exactly like
 * the GEMM's bounded waits, and records MTC_ERR_RUNTIME in the device error
 * word; mtc_check_device_errors then reports it and clears the word.  Tests the
 * give-up path of a bounded wait without a fault or a hang.  No reference
 * counterpart. */
int mtc_selftest_bounded_wait(int64_t spins, void *stream);

/* --------------------------------------------------- elementwise (A4, A5) -- */

/* out = f(in), Negate/Exp/Log/Sqrt/Tanh/Abs/Sign/Sigmoid (+ReLU);
 * replaces unary_elementwise (elementwise/loops.hpp:19-67).  Float32 only;
 * in.shape == out.shape. */
int mtc_unary(int32_t op, const mtc_desc *in, const mtc_desc *out, void *stream);

/* out = g(lhs, rhs) with right-aligned broadcasting of lhs/rhs to out.shape,
 * Add/Subtract/Multiply/Divide/LogAddExp; replaces binary_elementwise
 * (elementwise/loops.hpp:69-153).  Float32 only. */
int mtc_binary(int32_t op, const mtc_desc *lhs, const mtc_desc *rhs, const mtc_desc *out, void *stream);

/* Fused elementwise program over one index space (the shape of every output).
 * Registers 0..n_inputs-1 hold the inputs (each broadcast to the output shape);
 * instruction k writes register `dst`; outputs[j] receives register out_regs[j].
 * Every instruction rounds to float32 exactly as the unfused op does (no FMA
 * contraction across instructions), so a fused chain equals the chain of single
 * kernels bit for bit.  The kernel for a new program is generated and compiled
 * for sm_100a on first use and cached for the life of the process. */
int mtc_fused(const mtc_instr *program, int32_t n_instr, const mtc_desc *inputs, int32_t n_inputs,
              const int32_t *out_regs, const mtc_desc *outputs, int32_t n_outputs, void *stream);

/* ---------------------------------------------------------- copies (A7, A13) -- */

/* dst[i] = src[i] over src.shape; dst is any same-shape view (Contiguous 0x0201 and
 * Reshape 0x0202, copy/loops.hpp:22-88).  Float32 and Int64. */
int mtc_copy(const mtc_desc *src, const mtc_desc *dst, void *stream);

/* out = concatenate(inputs, axis) (Concatenate 0x0205, copy/loops.hpp:90-127). */
int mtc_concat(const mtc_desc *inputs, int32_t n_inputs, int64_t axis, const mtc_desc *out, void *stream);

/* out = 0, then the view `dst_view` of out's buffer receives `in`
 * (BasicIndexScatter 0x0207, copy/loops.hpp:129-153). */
int mtc_index_scatter(const mtc_desc *in, const mtc_desc *dst_view, const mtc_desc *out, void *stream);

/* --------------------------------------------------- Int64 indexing (A11, A12) -- */

/* take-along-axis: out[..i..] = src[..idx[..i..]..] (Gather 0x0208, copy/loops.hpp:155-220).
 * idx.shape == out.shape, same rank as src.  An index outside [0, src.shape[axis])
 * writes nothing for that element and sets the device error word. */
int mtc_gather(const mtc_desc *src, const mtc_desc *idx, int64_t axis, const mtc_desc *out, void *stream);

/* out = 0; out[..idx[..i..]..] += upd[..i..] (GatherScatterAdd 0x0209,
 * copy/loops.hpp:222-303).  Duplicate indices accumulate with float32 atomics:
 * bit-exact against the sequential CPU loop whenever the partial sums are exact
 * (integer-valued updates below 2^24), otherwise equal up to summation order. */
int mtc_gather_scatter_add(const mtc_desc *upd, const mtc_desc *idx, int64_t axis, const mtc_desc *out,
                           void *stream);

/* out[..idx[..i..]..] += upd[..i..] WITHOUT clearing out first: the updates are
 * added to the values already there (float32 atomics, so duplicate indices
 * accumulate in an unspecified order).  No reference counterpart: the fusing
 * evaluator uses it for the gather VJP's scatter-add (rules/manipulation.cpp:81-91)
 * when its only consumer is an elementwise Add that becomes the scatter's
 * target, so the [B, C] zero fill and its read-back disappear. */
int mtc_gather_scatter_add_into(const mtc_desc *upd, const mtc_desc *idx, int64_t axis, const mtc_desc *out,
                                void *stream);

/* -------------------------------------------------------- reductions (A8, A9) -- */

/* Reduce `in` over `axes` (normalised, distinct).  `out` is contiguous and holds the
 * kept dimensions in order (keep_dim only changes out.shape).  SUM (0x0301,
 * reduce_values, reduction/loops.hpp:21-57), LOGSUMEXP (0x0302, reduce_logsumexp,
 * reduction/loops.hpp:59-136), MAX, ARGMAX (one axis, Int64 out). */
int mtc_reduce(int32_t op, const mtc_desc *in, const int64_t *axes, int32_t n_axes, const mtc_desc *out,
               void *stream);

/* out = in - logsumexp(in, {axis}, keep_dim=true), one pass over HBM per row
 * (the composite of reduce_logsumexp and Subtract). */
int mtc_log_softmax(const mtc_desc *in, int64_t axis, const mtc_desc *out, void *stream);

/* ---------------------------------------------------------------- GEMM (A10) -- */

enum {
    MTC_GEMM_AUTO = 0,      /* 3xTF32 tensor cores for large problems (M, N >= 128, K >= 64,
                               M*N*K >= 2^28), the exact SIMT kernel otherwise */
    MTC_GEMM_SIMT = 1,      /* exact SIMT kernel: float product then float sum per k, k ascending,
                               the CPU reference's rounding and order (bit-identical results) */
    MTC_GEMM_3XTF32 = 2,    /* tcgen05/TMEM kernel, split-float32 (hi+lo) operands */
    MTC_GEMM_SIMT_FFMA = 3  /* SIMT kernel with one fused multiply-add per k */
};

/* matmul with the reference's full semantics (Matmul 0x0401, matmul_dispatch,
 * linalg/loops.hpp:288-324; shape rules src/tensor/primitives/linalg/matmul.cpp:18-52):
 * 1-D x 1-D dot, matrix x vector, vector x matrix, batched matrices with broadcast
 * batch dimensions and arbitrary strides.  Float32 in, float32 accumulate. */
int mtc_matmul(const mtc_desc *lhs, const mtc_desc *rhs, const mtc_desc *out, int32_t algo, void *stream);

/* The MTC_GEMM_3XTF32 matmul for callers that cannot allocate device memory:
 * code whose memory is owned by another framework's allocator, or a latency
 * path that must never wait on an allocation.  No reference counterpart (the
 * reference allocates only through DeviceRuntime::allocate).  Nothing is
 * allocated: the split hi/lo operands (2*batch*(M+N)*round_up(K,4) floats) go
 * to one fixed 32 MiB device array, so larger problems are rejected with
 * MTC_ERR_INVALID_ARGUMENT, and problems too small for the tensor-core path with
 * MTC_ERR_UNSUPPORTED.  The array exists on every GPU that loads the library,
 * until the process exits.  The first call on a device looks up its device
 * address (cudaGetSymbolAddress); make that first call before any stream
 * capture.  All calls share the array: calls that overlap on the GPU race, so
 * serialise them (one stream, or events between streams). */
int mtc_matmul_3xtf32_static(const mtc_desc *lhs, const mtc_desc *rhs, const mtc_desc *out, void *stream);

/* --------------------------------------------------------- creation (A14) -- */

/* out[...] = value; `value` points at 4 bytes (Float32) or 8 bytes (Int64)
 * (Full 0x0001, creation/loops.hpp:21-37). */
int mtc_fill(const mtc_desc *out, const void *value, void *stream);

/* Philox-4x32-10 counter RNG keyed by RandomKey words {key0, key1}
 * (src/tensor/backend/cpu/detail/random_engine.cpp:14-64).  Uniform
 * (creation/loops.hpp:39-86) is bit-exact; Normal (creation/loops.hpp:88-141)
 * uses double Box-Muller like the CPU and matches it to float32 rounding. */
int mtc_uniform(const mtc_desc *out, float low, float high, uint64_t key0, uint64_t key1, void *stream);
int mtc_normal(const mtc_desc *out, float mean, float std_dev, uint64_t key0, uint64_t key1, void *stream);

/* ------------------------------------------------------ graph replay (plan cache) --
 * The evaluator of a repeated plan (a training step) records the plan's launches
 * once with stream capture and replays them as one CUDA graph.  The reference
 * re-plans and re-dispatches every node on every evaluation
 * (src/tensor/execution/evaluator.cpp:196-206); the README lists reusable
 * compiled graphs as future work (README.md:35). */

typedef struct mtc_graph mtc_graph;

/* Starts recording the calling thread's launches on `stream` (relaxed stream
 * capture: nothing runs until mtc_graph_launch).  While recording, blocks that
 * mtc_free / the kernels' workspaces release on `device` stay allocated and
 * belong to the graph, because its replays use them again. */
int mtc_capture_begin(int device, void *stream);
/* Ends the recording.  keep != 0: instantiates it into *graph (MTC_OK), which
 * owns the retained blocks.  keep == 0 (or a failed capture): discards it,
 * returns the retained blocks to the pool and sets *graph = NULL. */
int mtc_capture_end(int keep, mtc_graph **graph);
/* Number of mtc_fused calls recorded so far by the calling thread's capture. */
int mtc_capture_fused_count(int32_t *count);
/* Runs the recorded launches on the stream they were recorded on. */
int mtc_graph_launch(mtc_graph *graph);
/* Replaces the constants (MTC_OP_CONST immediates, in program order) of the
 * `index`-th recorded mtc_fused launch for the following replays. */
int mtc_graph_set_constants(mtc_graph *graph, int32_t index, const float *imm, int32_t n_imm);
/* Kernels one replay launches (counted by mtc_launch_count at each replay). */
int mtc_graph_launches(const mtc_graph *graph, uint64_t *count);
/* Frees the graph; its retained blocks return to the pool in stream order. */
int mtc_graph_destroy(mtc_graph *graph);
/* Takes the cached free block that starts at `ptr` (a block an earlier
 * mtc_alloc returned and mtc_free released) for `bytes` on `stream`, as
 * mtc_alloc would.  MTC_OK when it was free, reusable on `stream` and large
 * enough; MTC_ERR_UNSUPPORTED (nothing changes) otherwise. */
int mtc_pool_take(int device, void *ptr, size_t bytes, void *stream);
/* mtc_pool_take for `n` blocks at once, under one lock: all are taken
 * (MTC_OK) or none (MTC_ERR_UNSUPPORTED; *failed = the first that was not free). */
int mtc_pool_take_many(int device, void *const *ptrs, const size_t *bytes, int32_t n, void *stream, int32_t *failed);
/* Adds `delta` to the protection count of the pool block at `ptr`.  While the
 * count is positive the block, once released, is kept for mtc_pool_take
 * (the replays of the graphs that use it) instead of being handed to other
 * requests; at zero it becomes an ordinary cached block again. */
int mtc_pool_protect(int device, void *ptr, int32_t delta);

/* ------------------------------------------------------------ instrumentation -- */

/* Number of kernels this library has launched in this process (all devices). */
int mtc_launch_count(uint64_t *count);
/* While enabled, every GEMM launch is bracketed by CUDA events on its stream. */
int mtc_profile_enable(int on);
/* Totals since the last reset for GEMM launches: launch count, summed device
 * time (ms, from the events; synchronises them) and algorithmic FLOPs (2*M*N*K
 * per batch entry).  reset != 0 clears the totals afterwards. */
int mtc_profile_gemm(uint64_t *launches, double *milliseconds, double *flops, int reset);

/* Matmul calls since process start by the kernel family that ran them:
 * *tensor_core counts calls served by the tcgen05 3xTF32 kernels, *simt those
 * served by the SIMT kernels (exact or FFMA).  Lets a caller confirm which path
 * MTC_GEMM_AUTO took.  No reference counterpart (the reference has one CPU loop). */
int mtc_gemm_path_counts(uint64_t *tensor_core, uint64_t *simt);

/* -------------------------------------------------- data parallel (config 5) --
 * Gradient all-reduce between the ranks of a data-parallel job, one process per
 * GPU; NCCL over NVLink/NVSwitch.  No reference counterpart: the reference is
 * single-process (it has no collective at all). */

/* Writes NCCL_UNIQUE_ID_BYTES (128) bytes of a fresh communicator id into `id`. */
int mtc_comm_unique_id(void *id, size_t id_bytes);
int mtc_comm_init(int device, int rank, int n_ranks, const void *id, size_t id_bytes, void **comm);
/* In-place sum all-reduce of `n` float32 buffers, then scale by `scale`, all on `stream`. */
int mtc_comm_allreduce_f32(void *comm, void *const *buffers, const size_t *counts, int32_t n, float scale,
                           void *stream);
/* The same reduction queued on the communicator's own stream behind the work
 * already queued on `stream` (the gradients), so it overlaps later work on
 * `stream`.  The buffers must not be touched by other streams until
 * mtc_comm_wait.  No reference counterpart (the reference has no collective). */
int mtc_comm_allreduce_f32_async(void *comm, void *const *buffers, const size_t *counts, int32_t n, float scale,
                                 void *stream);
/* Makes `stream` wait for every reduction queued by mtc_comm_allreduce_f32_async. */
int mtc_comm_wait(void *comm, void *stream);
int mtc_comm_destroy(void *comm);

#ifdef __cplusplus
}
#endif

#endif /* MTCUDA_H */
