// CUDA device backend of MiniTensor: the pieces that plug into the reference's
// seams.  `CudaRuntime` implements DeviceRuntime
// (src/tensor/backend/device_runtime.hpp:13-29), `CudaBuffer` implements Buffer
// (src/tensor/storage/buffer.hpp:13-27), `register_cuda_kernels` fills the
// KernelRegistry (src/tensor/dispatch/kernel_registry.hpp:15-27) under
// DeviceType::Cuda with adapters that call the C ABI of include/mtcuda.h, and
// `evaluate_fused` is the graph evaluator used for graphs with CUDA work.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <span>
#include <string>

#include <minitensor/types.hpp>

#include "mtcuda.h"
#include "tensor/backend/device_runtime.hpp"
#include "tensor/dispatch/kernel_registry.hpp"
#include "tensor/dispatch/tensor_view.hpp"
#include "tensor/execution/runtime_registry.hpp"
#include "tensor/graph/fwd.hpp"
#include "tensor/storage/buffer.hpp"

namespace minitensor::detail::cuda {

// Throws the reference's exception type for an mtcuda status code.
void check(int rc, const char *what);

class CudaBuffer final : public Buffer {
  public:
    CudaBuffer(Device device, void *data, std::size_t size_bytes, void *stream) noexcept;
    ~CudaBuffer() override;

    [[nodiscard]] Device device() const noexcept override { return device_; }
    [[nodiscard]] std::size_t size_bytes() const noexcept override { return size_bytes_; }
    [[nodiscard]] void *data() const noexcept { return data_; }

  private:
    Device device_;
    void *data_;
    std::size_t size_bytes_;
    void *stream_;
};

class CudaRuntime final : public DeviceRuntime {
  public:
    explicit CudaRuntime(Device device);

    [[nodiscard]] Device device() const noexcept override { return device_; }
    [[nodiscard]] BufferRef allocate(std::size_t size_bytes) override;
    // A buffer over a block already taken from the allocator (mtc_pool_take).
    [[nodiscard]] BufferRef adopt(void *data, std::size_t size_bytes);
    void copy_from_host(Buffer &destination, std::size_t destination_offset_bytes,
                        std::span<const std::byte> source) override;
    void copy_to_host(std::span<std::byte> destination, const Buffer &source, std::size_t source_offset_bytes) override;

    [[nodiscard]] int index() const noexcept { return static_cast<int>(device_.index()); }
    // The device's work stream (created lazily on first use).
    [[nodiscard]] void *stream();
    // Makes this device current on the calling thread.
    void activate() const;

  private:
    Device device_;
    void *stream_ = nullptr;
};

// Number of CUDA devices the driver reports (0 without a GPU).
[[nodiscard]] int device_count() noexcept;

// Operand descriptor of a materialised view on a CUDA buffer.
[[nodiscard]] mtc_desc make_desc(const TensorView &view);
[[nodiscard]] mtc_desc make_desc(const MutableTensorView &view);

void register_cuda_kernels(KernelRegistry &registry);

// Evaluates `roots` with elementwise fusion, stream-ordered allocation and
// deferred device error checks when any pending value lives on a CUDA device.
// Returns false (and does nothing) when the graph has no CUDA work.
bool evaluate_fused(const RuntimeRegistry &runtimes, const KernelRegistry &kernels, std::span<const ValueRef> roots);

// Process-wide switches: environment MTB_FUSION=0 disables elementwise fusion,
// MTB_GRAPHS=0 the replay of repeated plans, MTB_GRAPH_MAX_BYTES (default 64 MiB)
// bounds the output bytes of a plan that is recorded for replay.
struct EvaluatorOptions {
    bool fusion = true;
    bool check_index_errors = true;
    // MTB_INDEX_CHECKS=sync: every gather / scatter-add kernel is checked before
    // its output is installed (the stream is synchronised there), so an index
    // outside its axis throws std::out_of_range with the node unmaterialised,
    // as the reference's CPU kernel does (copy/loops.hpp:206-209).  Plans with
    // index kernels are then not recorded for replay.
    bool sync_index_checks = false;
    bool graphs = true;
    std::size_t graph_max_bytes = std::size_t(64) << 20;
};
EvaluatorOptions &evaluator_options();

// Counters of work issued by the evaluator (for benchmarks and tests).
struct EvaluatorStats {
    std::uint64_t kernel_steps = 0;    // non-fused kernel launches through KernelFns
    std::uint64_t fused_launches = 0;  // fused elementwise launches
    std::uint64_t fused_nodes = 0;     // elementwise nodes computed inside fused launches
    std::uint64_t folded_constants = 0;
    std::uint64_t view_steps = 0;
    std::uint64_t evaluations = 0;
    std::uint64_t plan_ns = 0;     // host time planning and clustering
    std::uint64_t execute_ns = 0;  // host time issuing kernels (allocation and launch calls)
    std::uint64_t check_ns = 0;    // host time queueing the deferred index-error check
    std::uint64_t graph_captures = 0;  // plans recorded for replay
    std::uint64_t graph_replays = 0;   // evaluations run as one replay of a recorded plan
    std::uint64_t graph_fallbacks = 0; // recorded plans whose output blocks were in use (run eagerly)
    std::uint64_t scatters_deferred = 0;  // scatter-adds added into their consumer's cluster output
};
EvaluatorStats &evaluator_stats();

// Destroys every recorded plan (their workspaces return to the allocator).
void clear_graph_cache();

// Throws std::out_of_range when an index kernel on `device` recorded an index
// outside its axis (a snapshot of the device error word queued after an
// evaluation); wait = true waits for the latest snapshot first.
void raise_device_errors(int device, bool wait);

}  // namespace minitensor::detail::cuda
