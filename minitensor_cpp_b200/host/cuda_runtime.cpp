// CudaRuntime / CudaBuffer: the device-memory side of the backend.
// Same contract and checks as CpuRuntime (src/tensor/backend/cpu/cpu_runtime.cpp:31-87):
// wrong buffer kind or device -> invalid_argument, copies outside the buffer ->
// out_of_range, zero-byte allocations give a valid empty buffer.
#include <stdexcept>
#include <string>

#include "cuda_backend.hpp"

namespace minitensor::detail::cuda {

void check(int rc, const char *what) {
    if (rc == MTC_OK) return;
    std::string msg = std::string(what) + ": " + mtc_last_error();
    switch (rc) {
    case MTC_ERR_INVALID_ARGUMENT: throw std::invalid_argument{msg};
    case MTC_ERR_OUT_OF_RANGE: throw std::out_of_range{msg};
    case MTC_ERR_OVERFLOW: throw std::overflow_error{msg};
    case MTC_ERR_LOGIC: throw std::logic_error{msg};
    default: throw std::runtime_error{msg};
    }
}

int device_count() noexcept {
    int n = 0;
    mtc_device_count(&n);
    return n;
}

CudaBuffer::CudaBuffer(Device device, void *data, std::size_t size_bytes, void *stream) noexcept
    : device_{device}, data_{data}, size_bytes_{size_bytes}, stream_{stream} {}

CudaBuffer::~CudaBuffer() {
    if (data_ != nullptr) {
        // Stream-ordered: the block returns to the pool once the stream has run
        // every kernel enqueued so far, so no host synchronisation is needed.
        (void)mtc_free(static_cast<int>(device_.index()), data_, stream_);
    }
}

CudaRuntime::CudaRuntime(Device device) : device_{device} {
    if (device_.type() != DeviceType::Cuda) {
        throw std::invalid_argument{"CudaRuntime requires a CUDA device"};
    }
}

void *CudaRuntime::stream() {
    if (stream_ == nullptr) {
        check(mtc_device_stream(index(), &stream_), "device stream");
    }
    return stream_;
}

void CudaRuntime::activate() const { check(mtc_set_device(static_cast<int>(device_.index())), "set device"); }

BufferRef CudaRuntime::allocate(std::size_t size_bytes) {
    void *s = stream();
    void *ptr = nullptr;
    check(mtc_alloc(index(), size_bytes, s, &ptr), "device allocation");
    return std::make_shared<CudaBuffer>(device_, ptr, size_bytes, s);
}

BufferRef CudaRuntime::adopt(void *data, std::size_t size_bytes) {
    return std::make_shared<CudaBuffer>(device_, data, size_bytes, stream());
}

void CudaRuntime::copy_from_host(Buffer &destination, std::size_t destination_offset_bytes,
                                 std::span<const std::byte> source) {
    auto *buffer = dynamic_cast<CudaBuffer *>(&destination);
    if (!buffer) throw std::invalid_argument{"CudaRuntime requires a CudaBuffer destination"};
    if (buffer->device() != device()) throw std::invalid_argument{"destination buffer belongs to a different device"};
    const std::size_t size = buffer->size_bytes();
    if (destination_offset_bytes > size || source.size() > size - destination_offset_bytes) {
        throw std::out_of_range{"host-to-device copy exceeds destination buffer"};
    }
    if (source.empty()) return;
    check(mtc_copy_from_host(index(), static_cast<std::byte *>(buffer->data()) + destination_offset_bytes,
                             source.data(), source.size(), stream()),
          "host-to-device copy");
}

void CudaRuntime::copy_to_host(std::span<std::byte> destination, const Buffer &source,
                               std::size_t source_offset_bytes) {
    const auto *buffer = dynamic_cast<const CudaBuffer *>(&source);
    if (!buffer) throw std::invalid_argument{"CudaRuntime requires a CudaBuffer source"};
    if (buffer->device() != device()) throw std::invalid_argument{"source buffer belongs to a different device"};
    const std::size_t size = buffer->size_bytes();
    if (source_offset_bytes > size || destination.size() > size - source_offset_bytes) {
        throw std::out_of_range{"device-to-host copy exceeds source buffer"};
    }
    if (destination.empty()) return;
    check(mtc_copy_to_host(index(), destination.data(),
                           static_cast<const std::byte *>(buffer->data()) + source_offset_bytes, destination.size(),
                           stream()),
          "device-to-host copy");
    // the copy synchronised the stream: every queued error-word snapshot has arrived
    raise_device_errors(static_cast<int>(index()), true);
}

void raise_device_errors(int device, bool wait) {
    int64_t detail = 0;
    const int rc = mtc_poll_device_errors(device, wait ? 1 : 0, &detail);
    if (rc == MTC_ERR_OUT_OF_RANGE) throw std::out_of_range{"gather index is out of range"};
    check(rc, "device error check");
}

}  // namespace minitensor::detail::cuda
