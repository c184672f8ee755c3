// libmtcuda runtime: status strings, device pools and streams, host<->device
// copies and the device error word.  Replaces CpuRuntime / CpuBuffer
// (src/tensor/backend/cpu/cpu_runtime.cpp:31-87, cpu_buffer.cpp:13-32).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <unordered_map>
#include <string>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "graph.cuh"

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

// ------------------------------------------------------ caching allocator --
// Device memory for graph buffers and kernel workspaces.  The evaluator
// allocates one buffer per materialised node and the GEMM one workspace per
// call, gigabytes per training step, so blocks are cached and reused in stream
// order instead of going to the driver: a block freed on stream S is handed to
// the next request on S at once (everything that used it is queued before
// anything that will), and a block freed on another stream becomes reusable by
// every stream when an event recorded at the free has completed.  Requests of
// 1 MiB or less are rounded to 512 bytes, larger ones to 2 MiB; the best fit
// whose size is within 1/8 (at least 2 MiB) of the request is reused whole.
// cudaMalloc is called only when nothing fits; when it fails, the unused cached
// blocks are released (after a device synchronisation) and it is retried once.

struct Block {
    void *ptr = nullptr;
    size_t size = 0;
    cudaStream_t stream = nullptr;  // stream of the last owner
};

struct PendingFree {
    Block block;
    cudaEvent_t done = nullptr;
};

struct DevicePool {
    using FreeList = std::multimap<size_t, Block>;
    std::mutex mu;
    // free blocks reusable by one stream (stream order) or, key nullptr, by any stream
    std::vector<std::pair<cudaStream_t, std::unique_ptr<FreeList>>> free_lists;
    // every free block by address, for taking one back by address (graph replay)
    std::unordered_map<void *, std::pair<FreeList *, FreeList::iterator>> free_at;
    std::vector<PendingFree> pending;
    std::unordered_map<void *, Block> live;
    // blocks recorded graphs use (reference counts): when free they are parked
    // in `parked`, where only a take by address (a replay) finds them
    std::unordered_map<void *, int> protect;
    FreeList parked;
    std::vector<cudaEvent_t> spare_events;
    uint64_t reserved = 0;
    uint64_t cached = 0;

    FreeList &list_for(cudaStream_t s) {
        for (auto &fl : free_lists)
            if (fl.first == s) return *fl.second;
        free_lists.emplace_back(s, std::make_unique<FreeList>());
        return *free_lists.back().second;
    }

    void put_free(cudaStream_t s, const Block &b) {
        FreeList &fl = protect.count(b.ptr) ? parked : list_for(s);
        free_at[b.ptr] = {&fl, fl.emplace(b.size, b)};
    }

    void erase_free(FreeList &fl, FreeList::iterator it) {
        free_at.erase(it->second.ptr);
        fl.erase(it);
    }
};

std::mutex g_pool_mutex;
std::vector<std::unique_ptr<DevicePool>> g_pools;

DevicePool &pool_of(int device) {
    std::lock_guard<std::mutex> lock(g_pool_mutex);
    if (static_cast<int>(g_pools.size()) <= device) g_pools.resize(device + 1);
    if (!g_pools[device]) g_pools[device] = std::make_unique<DevicePool>();
    return *g_pools[device];
}

size_t round_request(size_t bytes) {
    constexpr size_t kSmall = size_t(1) << 20, kLarge = size_t(2) << 20;
    if (bytes <= kSmall) return (bytes + 511) & ~size_t(511);
    return (bytes + kLarge - 1) / kLarge * kLarge;
}

bool take_fit(DevicePool &pool, cudaStream_t s, size_t want, Block &out) {
    DevicePool::FreeList &fl = pool.list_for(s);
    auto it = fl.lower_bound(want);
    if (it == fl.end()) return false;
    const size_t slack = std::max(want / 8, size_t(2) << 20);
    if (it->first > want + slack) return false;
    out = it->second;
    pool.erase_free(fl, it);
    return true;
}

// Moves blocks whose cross-stream free has completed to the any-stream list.
void collect_pending(DevicePool &pool) {
    for (size_t i = 0; i < pool.pending.size();) {
        PendingFree &pf = pool.pending[i];
        if (cudaEventQuery(pf.done) == cudaSuccess) {
            Block b = pf.block;
            b.stream = nullptr;
            pool.put_free(nullptr, b);
            pool.spare_events.push_back(pf.done);
            pool.pending[i] = pool.pending.back();
            pool.pending.pop_back();
        } else {
            cudaGetLastError();  // cudaErrorNotReady is not an error here
            ++i;
        }
    }
}

// Returns every cached (unused) block to the driver; the caller holds pool.mu.
int release_cached(DevicePool &pool) {
    MTC_CUDA_TRY(cudaDeviceSynchronize());
    collect_pending(pool);
    for (auto &fl : pool.free_lists) {
        for (auto &kv : *fl.second) {
            cudaFree(kv.second.ptr);
            pool.reserved -= kv.second.size;
            pool.cached -= kv.second.size;
        }
        fl.second->clear();
    }
    // parked blocks stay: recorded graphs replay into them
    pool.free_at.clear();
    for (auto it = pool.parked.begin(); it != pool.parked.end(); ++it) pool.free_at[it->second.ptr] = {&pool.parked, it};
    return MTC_OK;
}

int pool_alloc(int device, size_t bytes, cudaStream_t stream, void **ptr) {
    *ptr = nullptr;
    if (bytes == 0) return MTC_OK;
    DevicePool &pool = pool_of(device);
    const size_t want = round_request(bytes);
    std::lock_guard<std::mutex> lock(pool.mu);
    if (!pool.pending.empty()) collect_pending(pool);
    Block b;
    bool hit = take_fit(pool, stream, want, b);
    if (!hit) hit = take_fit(pool, nullptr, want, b);
    if (hit) {
        pool.cached -= b.size;
    } else {
        void *p = nullptr;
        cudaError_t e = cudaMalloc(&p, want);
        if (e != cudaSuccess) {
            cudaGetLastError();
            MTC_TRY(release_cached(pool));
            e = cudaMalloc(&p, want);
        }
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(MTC_ERR_RUNTIME, "device %d: allocation of %zu bytes failed: %s", device, bytes,
                        cudaGetErrorString(e));
        }
        b.ptr = p;
        b.size = want;
        pool.reserved += want;
    }
    b.stream = stream;
    pool.live.emplace(b.ptr, b);
    *ptr = b.ptr;
    return MTC_OK;
}

int pool_free(int device, void *ptr, cudaStream_t stream) {
    if (ptr == nullptr) return MTC_OK;
    if (Capture *c = active_capture(); c != nullptr && c->device == device) {
        // recording: the graph's replays use this block again, so it stays
        // allocated until the graph is destroyed
        DevicePool &pool = pool_of(device);
        std::lock_guard<std::mutex> lock(pool.mu);
        if (pool.live.count(ptr) == 0)
            return fail(MTC_ERR_INVALID_ARGUMENT, "device %d: %p is not a live block", device, ptr);
        c->retained.push_back(ptr);
        return MTC_OK;
    }
    return release_block(device, ptr, stream);
}

// Takes the free block at `ptr` back for a request of `bytes` on `stream`.
// Changes the protection count of the block at `ptr`; a block whose count
// drops to zero while parked returns to its stream's free list.
int pool_protect(int device, void *ptr, int delta) {
    DevicePool &pool = pool_of(device);
    std::lock_guard<std::mutex> lock(pool.mu);
    const bool known = pool.live.count(ptr) || pool.free_at.count(ptr);
    if (!known) return fail(MTC_ERR_INVALID_ARGUMENT, "device %d: %p is not a block of the pool", device, ptr);
    int &n = pool.protect[ptr];
    n += delta;
    if (n > 0) return MTC_OK;
    pool.protect.erase(ptr);
    auto f = pool.free_at.find(ptr);
    if (f != pool.free_at.end() && f->second.first == &pool.parked) {
        const Block b = f->second.second->second;
        pool.erase_free(pool.parked, f->second.second);
        pool.put_free(b.stream, b);
    }
    return MTC_OK;
}

// Takes the free block at `ptr` back for a request of `bytes` on `stream`;
// the caller holds pool.mu.
int take_locked(DevicePool &pool, int device, void *ptr, size_t bytes, cudaStream_t stream) {
    const size_t want = round_request(bytes);
    auto f = pool.free_at.find(ptr);
    if (f == pool.free_at.end()) return fail(MTC_ERR_UNSUPPORTED, "device %d: %p is not a free block", device, ptr);
    DevicePool::FreeList *fl = f->second.first;
    auto it = f->second.second;
    const bool usable = fl == &pool.list_for(stream) || fl == &pool.list_for(nullptr) ||
                        (fl == &pool.parked && (it->second.stream == stream || it->second.stream == nullptr));
    if (!usable) return fail(MTC_ERR_UNSUPPORTED, "device %d: %p was released on another stream", device, ptr);
    Block b = it->second;
    if (b.size < want) return fail(MTC_ERR_UNSUPPORTED, "device %d: the block at %p is too small", device, ptr);
    pool.erase_free(*fl, it);
    pool.cached -= b.size;
    b.stream = stream;
    pool.live.emplace(b.ptr, b);
    return MTC_OK;
}

int pool_take(int device, void *ptr, size_t bytes, cudaStream_t stream) {
    DevicePool &pool = pool_of(device);
    std::lock_guard<std::mutex> lock(pool.mu);
    if (!pool.pending.empty()) collect_pending(pool);
    return take_locked(pool, device, ptr, bytes, stream);
}

// Takes all of `n` blocks or none.
int pool_take_many(int device, void *const *ptrs, const size_t *bytes, int n, cudaStream_t stream, int *failed) {
    DevicePool &pool = pool_of(device);
    std::lock_guard<std::mutex> lock(pool.mu);
    if (!pool.pending.empty()) collect_pending(pool);
    for (int i = 0; i < n; ++i) {
        const int rc = take_locked(pool, device, ptrs[i], bytes[i], stream);
        if (rc == MTC_OK) continue;
        *failed = i;
        // hand back what was taken, to this stream's free list (or parked)
        for (int j = 0; j < i; ++j) {
            auto it = pool.live.find(ptrs[j]);
            Block b = it->second;
            pool.live.erase(it);
            pool.cached += b.size;
            pool.put_free(stream, b);
        }
        return rc;
    }
    return MTC_OK;
}

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

int release_block(int device, void *ptr, cudaStream_t stream) {
    if (ptr == nullptr) return MTC_OK;
    DevicePool &pool = pool_of(device);
    std::lock_guard<std::mutex> lock(pool.mu);
    auto it = pool.live.find(ptr);
    if (it == pool.live.end()) return fail(MTC_ERR_INVALID_ARGUMENT, "device %d: %p is not a live block", device, ptr);
    Block b = it->second;
    pool.live.erase(it);
    pool.cached += b.size;
    if (stream == b.stream) {
        pool.put_free(stream, b);
        return MTC_OK;
    }
    // freed on another stream: reusable once that stream has passed this point
    cudaEvent_t ev = nullptr;
    if (!pool.spare_events.empty()) {
        ev = pool.spare_events.back();
        pool.spare_events.pop_back();
    } else {
        MTC_CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    }
    MTC_CUDA_TRY(cudaEventRecord(ev, stream));
    pool.pending.push_back(PendingFree{b, ev});
    return MTC_OK;
}

namespace {
thread_local Capture *t_capture = nullptr;
}  // namespace

Capture *active_capture() { return t_capture; }
void set_active_capture(Capture *c) { t_capture = c; }

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

uint64_t launches_so_far() { return g_launches.load(std::memory_order_relaxed); }

void count_launches(int64_t n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }

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

bool host_trace() {
    static const bool on = std::getenv("MTB_TRACE") != nullptr;
    return on;
}

static double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

HostSpan::HostSpan(const char *l) : label{l}, t0{host_trace() ? now_ms() : 0.0} {}

HostSpan::~HostSpan() {
    if (!host_trace()) return;
    const double ms = now_ms() - t0;
    if (ms >= 5.0) std::fprintf(stderr, "mtc slow host call: %s %.1f ms\n", label, ms);
}

int scratch_alloc(size_t bytes, cudaStream_t stream, void **ptr) {
    int device = 0;
    MTC_CUDA_TRY(cudaGetDevice(&device));
    return pool_alloc(device, bytes, stream, ptr);
}

void scratch_free(void *ptr, cudaStream_t stream) {
    if (ptr == nullptr) return;
    int device = 0;
    if (cudaGetDevice(&device) == cudaSuccess) (void)pool_free(device, ptr, stream);
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
    // cudaMalloc blocks are 512-byte aligned: every buffer suits 128-bit and TMA access
    HostSpan span("buffer allocation");
    return pool_alloc(device, bytes, static_cast<cudaStream_t>(stream), ptr);
}

int mtc_free(int device, void *ptr, void *stream) {
    if (ptr == nullptr) return MTC_OK;
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    return pool_free(device, ptr, static_cast<cudaStream_t>(stream));
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
    clear_error();
    if (device < 0) return fail(MTC_ERR_INVALID_ARGUMENT, "negative device index");
    DevicePool &pool = pool_of(device);
    std::lock_guard<std::mutex> lock(pool.mu);
    if (reserved_bytes) *reserved_bytes = pool.reserved;
    if (used_bytes) *used_bytes = pool.reserved - pool.cached;
    return MTC_OK;
}

int mtc_stream_create(int device, void **stream) {
    clear_error();
    if (stream == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null stream slot");
    DeviceState *st = nullptr;
    MTC_TRY(ensure_device(device, &st));
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    cudaStream_t s = nullptr;
    MTC_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    *stream = s;
    return MTC_OK;
}

int mtc_stream_destroy(int device, void *stream) {
    if (stream == nullptr) return MTC_OK;
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    MTC_CUDA_TRY(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
    return MTC_OK;
}

int mtc_event_create(int device, void **event) {
    clear_error();
    if (event == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null event slot");
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    cudaEvent_t e = nullptr;
    MTC_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    *event = e;
    return MTC_OK;
}

int mtc_event_create_timed(int device, void **event) {
    clear_error();
    if (event == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null event slot");
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    cudaEvent_t e = nullptr;
    MTC_CUDA_TRY(cudaEventCreate(&e));
    *event = e;
    return MTC_OK;
}

int mtc_event_elapsed(void *start, void *stop, float *milliseconds) {
    clear_error();
    if (start == nullptr || stop == nullptr || milliseconds == nullptr)
        return fail(MTC_ERR_INVALID_ARGUMENT, "null event or result");
    MTC_CUDA_TRY(cudaEventSynchronize(static_cast<cudaEvent_t>(stop)));
    MTC_CUDA_TRY(cudaEventElapsedTime(milliseconds, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(stop)));
    return MTC_OK;
}

int mtc_event_destroy(int device, void *event) {
    if (event == nullptr) return MTC_OK;
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    MTC_CUDA_TRY(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
    return MTC_OK;
}

int mtc_event_record(void *event, void *stream) {
    clear_error();
    if (event == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null event");
    MTC_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)));
    return MTC_OK;
}

int mtc_stream_wait_event(void *stream, void *event) {
    clear_error();
    if (event == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null event");
    MTC_CUDA_TRY(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0));
    return MTC_OK;
}

int mtc_pool_take(int device, void *ptr, size_t bytes, void *stream) {
    clear_error();
    if (device < 0) return fail(MTC_ERR_INVALID_ARGUMENT, "negative device index");
    if (ptr == nullptr || bytes == 0) return fail(MTC_ERR_INVALID_ARGUMENT, "nothing to take");
    return pool_take(device, ptr, bytes, static_cast<cudaStream_t>(stream));
}

int mtc_pool_take_many(int device, void *const *ptrs, const size_t *bytes, int32_t n, void *stream, int32_t *failed) {
    clear_error();
    if (device < 0 || n < 0 || (n > 0 && (ptrs == nullptr || bytes == nullptr)))
        return fail(MTC_ERR_INVALID_ARGUMENT, "bad block list");
    int bad = -1;
    const int rc = pool_take_many(device, ptrs, bytes, n, static_cast<cudaStream_t>(stream), &bad);
    if (failed) *failed = bad;
    return rc;
}

int mtc_pool_protect(int device, void *ptr, int32_t delta) {
    clear_error();
    if (device < 0 || ptr == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "no block to protect");
    return pool_protect(device, ptr, delta);
}

int mtc_pool_trim(int device) {
    DeviceGuard guard(device);
    MTC_TRY(guard.rc);
    DevicePool &pool = pool_of(device);
    std::lock_guard<std::mutex> lock(pool.mu);
    return release_cached(pool);
}

}  // extern "C"
