// libmtcuda runtime: status strings, device pools and streams, host<->device
// copies and the device error word.  Replaces CpuRuntime / CpuBuffer
// (src/tensor/backend/cpu/cpu_runtime.cpp:31-87, cpu_buffer.cpp:13-32).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace mtc {

namespace {
thread_local std::string t_last_error;

struct DeviceState {
    bool ready = false;
    cudaStream_t stream = nullptr;
    int sms = 0;
};

std::mutex g_mutex;
std::vector<DeviceState> g_devices;

int ensure_device(int device, DeviceState **out) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(MTC_ERR_RUNTIME, "no CUDA device available: %s", cudaGetErrorString(e));
    }
    if (device < 0 || device >= count) {
        return fail(MTC_ERR_INVALID_ARGUMENT, "CUDA device %d does not exist (%d visible)", device, count);
    }
    std::lock_guard<std::mutex> lock(g_mutex);
    if (g_devices.size() < static_cast<size_t>(count)) g_devices.resize(count);
    DeviceState &st = g_devices[device];
    if (!st.ready) {
        int prev = 0;
        MTC_CUDA_TRY(cudaGetDevice(&prev));
        MTC_CUDA_TRY(cudaSetDevice(device));
        MTC_CUDA_TRY(cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking));
        MTC_CUDA_TRY(cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, device));
        // Keep freed blocks cached in the default pool: the evaluator allocates
        // one buffer per graph node, so returning memory to the driver on every
        // synchronisation would make each step pay cudaMalloc again.
        cudaMemPool_t pool;
        MTC_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, device));
        uint64_t threshold = UINT64_MAX;
        MTC_CUDA_TRY(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold));
        MTC_CUDA_TRY(cudaSetDevice(prev));
        st.ready = true;
    }
    *out = &st;
    return MTC_OK;
}

// Makes `device` current for the lifetime of the guard.
struct DeviceGuard {
    int prev = -1;
    int rc = MTC_OK;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != device) {
            if (cudaSetDevice(device) != cudaSuccess) rc = fail(MTC_ERR_RUNTIME, "cudaSetDevice(%d) failed", device);
        }
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};
}  // namespace

int fail(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

void clear_error() { t_last_error.clear(); }

std::atomic<uint64_t> g_launches{0};

int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MTC_ERR_RUNTIME, "launch of %s failed: %s", what, cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return MTC_OK;
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// ------------------------------------------------------------ GEMM profile --

namespace {
struct GemmSample {
    cudaEvent_t start, stop;
    double flops;
};
std::mutex g_profile_mutex;
std::vector<GemmSample> g_profile_samples;
std::vector<cudaEvent_t> g_event_pool;
bool g_profile_on = false;
uint64_t g_profile_launches = 0;
double g_profile_ms = 0.0, g_profile_flops = 0.0;

cudaEvent_t take_event() {
    if (!g_event_pool.empty()) {
        cudaEvent_t e = g_event_pool.back();
        g_event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void drain_samples() {
    for (GemmSample &s : g_profile_samples) {
        float ms = 0.0f;
        if (cudaEventSynchronize(s.stop) == cudaSuccess && cudaEventElapsedTime(&ms, s.start, s.stop) == cudaSuccess) {
            g_profile_ms += ms;
            g_profile_flops += s.flops;
            ++g_profile_launches;
        }
        g_event_pool.push_back(s.start);
        g_event_pool.push_back(s.stop);
    }
    g_profile_samples.clear();
}
}  // namespace

bool profiling() { return g_profile_on; }

void *profile_begin(cudaStream_t stream) {
    std::lock_guard<std::mutex> lock(g_profile_mutex);
    cudaEvent_t e = take_event();
    cudaEventRecord(e, stream);
    return e;
}

void profile_end(void *begin, cudaStream_t stream, double flops) {
    std::lock_guard<std::mutex> lock(g_profile_mutex);
    cudaEvent_t e = take_event();
    cudaEventRecord(e, stream);
    g_profile_samples.push_back(GemmSample{static_cast<cudaEvent_t>(begin), e, flops});
    if (g_profile_samples.size() > 4096) drain_samples();
}

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

int sm_count(int device) {
    DeviceState *st = nullptr;
    if (ensure_device(device, &st) != MTC_OK) return 148;
    return st->sms;
}

int scratch_alloc(size_t bytes, cudaStream_t stream, void **ptr) {
    *ptr = nullptr;
    if (bytes == 0) return MTC_OK;
    MTC_CUDA_TRY(cudaMallocAsync(ptr, bytes, stream));
    return MTC_OK;
}

void scratch_free(void *ptr, cudaStream_t stream) {
    if (ptr) cudaFreeAsync(ptr, stream);
}

int validate(const mtc_desc *d, const char *name) {
    if (d == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "%s: null descriptor", name);
    if (d->rank < 0 || d->rank > MTC_MAX_RANK)
        return fail(MTC_ERR_INVALID_ARGUMENT, "%s: rank %d outside [0, %d]", name, d->rank, MTC_MAX_RANK);
    if (d->dtype != MTC_FLOAT32 && d->dtype != MTC_INT64)
        return fail(MTC_ERR_INVALID_ARGUMENT, "%s: unknown dtype %d", name, d->dtype);
    if (d->offset < 0) return fail(MTC_ERR_INVALID_ARGUMENT, "%s: negative offset", name);
    int64_t numel = 1;
    for (int i = 0; i < d->rank; ++i) {
        if (d->shape[i] < 0) return fail(MTC_ERR_INVALID_ARGUMENT, "%s: negative extent", name);
        if (d->shape[i] != 0 && numel > INT64_MAX / d->shape[i])
            return fail(MTC_ERR_OVERFLOW, "%s: element count overflows int64", name);
        numel *= d->shape[i];
    }
    if (numel == 0) return MTC_OK;
    __int128 lo = d->offset, hi = d->offset;
    for (int i = 0; i < d->rank; ++i) {
        __int128 span = static_cast<__int128>(d->strides[i]) * (d->shape[i] - 1);
        if (span < 0) lo += span; else hi += span;
    }
    if (lo < 0 || hi >= d->capacity)
        return fail(MTC_ERR_OUT_OF_RANGE, "%s: view reaches elements [%lld, %lld] outside buffer of %lld", name,
                    static_cast<long long>(lo), static_cast<long long>(hi), static_cast<long long>(d->capacity));
    if (d->data == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "%s: null data for non-empty view", name);
    return MTC_OK;
}

int broadcast_strides(const mtc_desc &d, const int64_t *shape, int rank, int64_t *strides_out) {
    if (d.rank > rank) return fail(MTC_ERR_INVALID_ARGUMENT, "operand rank %d exceeds result rank %d", d.rank, rank);
    const int lead = rank - d.rank;
    for (int i = 0; i < rank; ++i) {
        if (i < lead) {
            strides_out[i] = 0;
            continue;
        }
        const int64_t e = d.shape[i - lead];
        if (e == shape[i]) {
            strides_out[i] = (e == 1) ? 0 : d.strides[i - lead];
        } else if (e == 1) {
            strides_out[i] = 0;
        } else {
            return fail(MTC_ERR_INVALID_ARGUMENT, "operand extent %lld does not broadcast to %lld",
                        static_cast<long long>(e), static_cast<long long>(shape[i]));
        }
    }
    return MTC_OK;
}

void simplify(IterSpace &s) {
    s.numel = 1;
    for (int i = 0; i < s.rank; ++i) s.numel *= s.shape[i];
    // Drop extent-1 axes.
    int r = 0;
    for (int i = 0; i < s.rank; ++i) {
        if (s.shape[i] == 1) continue;
        s.shape[r] = s.shape[i];
        for (int k = 0; k < s.nops; ++k) s.stride[k][r] = s.stride[k][i];
        ++r;
    }
    s.rank = r;
    // Merge axis i into axis i+1 (outer into inner) when strides chain for every operand.
    if (s.rank > 1) {
        int out = s.rank - 1;  // walk from the innermost axis outwards
        int64_t shape[MTC_MAX_RANK];
        int64_t stride[kMaxOps][MTC_MAX_RANK];
        int w = MTC_MAX_RANK - 1;
        shape[w] = s.shape[out];
        for (int k = 0; k < s.nops; ++k) stride[k][w] = s.stride[k][out];
        for (int i = out - 1; i >= 0; --i) {
            bool chain = true;
            for (int k = 0; k < s.nops && chain; ++k) chain = (s.stride[k][i] == stride[k][w] * shape[w]);
            if (chain) {
                shape[w] *= s.shape[i];
            } else {
                --w;
                shape[w] = s.shape[i];
                for (int k = 0; k < s.nops; ++k) stride[k][w] = s.stride[k][i];
            }
        }
        s.rank = MTC_MAX_RANK - w;
        for (int i = 0; i < s.rank; ++i) {
            s.shape[i] = shape[w + i];
            for (int k = 0; k < s.nops; ++k) s.stride[k][i] = stride[k][w + i];
        }
    }
    if (s.rank == 0) {
        s.rank = 1;
        s.shape[0] = 1;
        for (int k = 0; k < s.nops; ++k) s.stride[k][0] = 0;
    }
}

}  // namespace mtc

using namespace mtc;

extern "C" {

const char *mtc_last_error(void) { return t_last_error.c_str(); }

const char *mtc_version(void) { return "mtcuda 0.1 sm_100a"; }

int mtc_device_count(int *count) {
    *count = 0;
    cudaError_t e = cudaGetDeviceCount(count);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *count = 0;
    }
    return MTC_OK;
}

int mtc_device_sm_count(int device, int *count) {
    DeviceState *st = nullptr;
    MTC_TRY(ensure_device(device, &st));
    *count = st->sms;
    return MTC_OK;
}

int mtc_launch_count(uint64_t *count) {
    *count = g_launches.load(std::memory_order_relaxed);
    return MTC_OK;
}

int mtc_profile_enable(int on) {
    std::lock_guard<std::mutex> lock(g_profile_mutex);
    g_profile_on = on != 0;
    return MTC_OK;
}

int mtc_profile_gemm(uint64_t *launches, double *milliseconds, double *flops, int reset) {
    std::lock_guard<std::mutex> lock(g_profile_mutex);
    drain_samples();
    if (launches) *launches = g_profile_launches;
    if (milliseconds) *milliseconds = g_profile_ms;
    if (flops) *flops = g_profile_flops;
    if (reset) {
        g_profile_launches = 0;
        g_profile_ms = 0.0;
        g_profile_flops = 0.0;
    }
    return MTC_OK;
}

int mtc_set_device(int device) {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur == device) return MTC_OK;
    MTC_CUDA_TRY(cudaSetDevice(device));
    return MTC_OK;
}

int mtc_device_stream(int device, void **stream) {
    DeviceState *st = nullptr;
    MTC_TRY(ensure_device(device, &st));
    *stream = st->stream;
    return MTC_OK;
}

int mtc_alloc(int device, size_t bytes, void *stream, void **ptr) {
    *ptr = nullptr;
    if (bytes == 0) return MTC_OK;
    DeviceState *st = nullptr;
    MTC_TRY(ensure_device(device, &st));
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    // 256-byte granularity keeps every buffer aligned for 128-bit and TMA access.
    const size_t rounded = (bytes + 255) & ~static_cast<size_t>(255);
    cudaError_t e = cudaMallocAsync(ptr, rounded, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        cudaGetLastError();
        *ptr = nullptr;
        return fail(MTC_ERR_RUNTIME, "device %d: allocation of %zu bytes failed: %s", device, bytes,
                    cudaGetErrorString(e));
    }
    return MTC_OK;
}

int mtc_free(int device, void *ptr, void *stream) {
    if (ptr == nullptr) return MTC_OK;
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    MTC_CUDA_TRY(cudaFreeAsync(ptr, static_cast<cudaStream_t>(stream)));
    return MTC_OK;
}

int mtc_copy_from_host(int device, void *dst, const void *src, size_t bytes, void *stream) {
    if (bytes == 0) return MTC_OK;
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    MTC_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)));
    return MTC_OK;
}

int mtc_copy_to_host(int device, void *dst, const void *src, size_t bytes, void *stream) {
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    if (bytes != 0) {
        MTC_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)));
    }
    MTC_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    return MTC_OK;
}

int mtc_stream_synchronize(void *stream) {
    MTC_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    return MTC_OK;
}

int mtc_pool_stats(int device, uint64_t *reserved_bytes, uint64_t *used_bytes) {
    cudaMemPool_t pool;
    MTC_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, device));
    MTC_CUDA_TRY(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, reserved_bytes));
    MTC_CUDA_TRY(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemCurrent, used_bytes));
    return MTC_OK;
}

int mtc_pool_trim(int device) {
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    MTC_CUDA_TRY(cudaDeviceSynchronize());
    cudaMemPool_t pool;
    MTC_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, device));
    MTC_CUDA_TRY(cudaMemPoolTrimTo(pool, 0));
    return MTC_OK;
}

}  // extern "C"
