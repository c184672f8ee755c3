// Data-parallel gradient all-reduce over NCCL (NVLink / NVSwitch on one node).
// No reference counterpart: the reference has no collective.  One process per
// GPU; the communicator id is produced by rank 0 and shared by the caller's own
// rendezvous (torch.distributed in the Python driver).
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"

namespace mtc {
namespace {

// NCCL is resolved at first use with dlopen("libnccl.so.2") instead of being
// linked: inside a process that already loaded PyTorch this returns the NCCL
// PyTorch brought (one copy per process), elsewhere the system library.
struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
};

NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (h == nullptr) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(dlsym(h, "ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(dlsym(h, "ncclGroupEnd"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.group_start && api.group_end &&
                 api.comm_destroy && api.error_string;
    });
    return api;
}

int need_nccl() {
    if (!nccl().ok) return fail(MTC_ERR_RUNTIME, "NCCL (libnccl.so.2) could not be loaded");
    return MTC_OK;
}

struct Comm {
    ncclComm_t comm = nullptr;
    int device = 0;
    int rank = 0;
    int n_ranks = 1;
    cudaStream_t side = nullptr;  // the communicator's own stream (asynchronous reductions)
    cudaEvent_t ready = nullptr;  // recorded on the caller's stream: the gradients are queued
    cudaEvent_t done = nullptr;   // recorded on `side` after the latest reduction
};

__global__ void k_scale(float *p, long long n, float s) {
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        p[i] *= s;
}

#define MTC_NCCL_TRY(expr)                                                                      \
    do {                                                                                        \
        ncclResult_t r__ = (expr);                                                              \
        if (r__ != ncclSuccess) return fail(MTC_ERR_RUNTIME, "%s failed: %s", #expr, nccl().error_string(r__)); \
    } while (0)

// Grouped in-place sum of the buffers over the ranks on stream `s`, then x scale.
// A scale of 1 / ranks with a power-of-two rank count is folded into the
// reduction as ncclAvg (NCCL multiplies each contribution by 1 / ranks before
// summing floats; with a power of two that multiplication is exact outside
// the subnormal range, so the result equals the sum scaled afterwards bit for
// bit) and no scale kernel runs.
int allreduce_on(Comm *c, void *const *buffers, const size_t *counts, int32_t n, float scale, cudaStream_t s) {
    const bool pow2 = c->n_ranks > 1 && (c->n_ranks & (c->n_ranks - 1)) == 0;
    const bool avg = pow2 && scale == 1.0f / static_cast<float>(c->n_ranks);
    if (avg) scale = 1.0f;
    MTC_NCCL_TRY(nccl().group_start());
    for (int i = 0; i < n; ++i) {
        if (counts[i] == 0) continue;
        ncclResult_t r = nccl().all_reduce(buffers[i], buffers[i], counts[i], ncclFloat32, avg ? ncclAvg : ncclSum,
                                           c->comm, s);
        if (r != ncclSuccess) {
            nccl().group_end();
            return fail(MTC_ERR_RUNTIME, "ncclAllReduce failed: %s", nccl().error_string(r));
        }
    }
    MTC_NCCL_TRY(nccl().group_end());
    if (scale != 1.0f) {
        const int sms = sm_count(c->device);
        for (int i = 0; i < n; ++i) {
            if (counts[i] == 0) continue;
            long long blocks = (static_cast<long long>(counts[i]) + 255) / 256;
            if (blocks > sms * 4) blocks = sms * 4;
            k_scale<<<static_cast<unsigned>(blocks), 256, 0, s>>>(static_cast<float *>(buffers[i]),
                                                                   static_cast<long long>(counts[i]), scale);
        }
        MTC_TRY(check_launch("gradient scale"));
    }
    return MTC_OK;
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" {

int mtc_comm_unique_id(void *id, size_t id_bytes) {
    clear_error();
    if (id == nullptr || id_bytes < sizeof(ncclUniqueId)) return fail(MTC_ERR_INVALID_ARGUMENT, "id buffer too small");
    MTC_TRY(need_nccl());
    ncclUniqueId uid;
    MTC_NCCL_TRY(nccl().get_unique_id(&uid));
    std::memcpy(id, &uid, sizeof(uid));
    return MTC_OK;
}

int mtc_comm_init(int device, int rank, int n_ranks, const void *id, size_t id_bytes, void **comm) {
    clear_error();
    if (id == nullptr || id_bytes < sizeof(ncclUniqueId) || comm == nullptr)
        return fail(MTC_ERR_INVALID_ARGUMENT, "bad communicator arguments");
    if (rank < 0 || rank >= n_ranks) return fail(MTC_ERR_INVALID_ARGUMENT, "rank outside the communicator");
    MTC_TRY(need_nccl());
    MTC_CUDA_TRY(cudaSetDevice(device));
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    Comm *c = new Comm;
    c->device = device;
    c->rank = rank;
    c->n_ranks = n_ranks;
    ncclResult_t r = nccl().comm_init_rank(&c->comm, n_ranks, uid, rank);
    if (r != ncclSuccess) {
        delete c;
        return fail(MTC_ERR_RUNTIME, "ncclCommInitRank failed: %s", nccl().error_string(r));
    }
    *comm = c;
    gemm_note_collectives();
    return MTC_OK;
}

int mtc_comm_allreduce_f32(void *comm, void *const *buffers, const size_t *counts, int32_t n, float scale, void *stream) {
    clear_error();
    Comm *c = static_cast<Comm *>(comm);
    if (c == nullptr || (n > 0 && (buffers == nullptr || counts == nullptr)))
        return fail(MTC_ERR_INVALID_ARGUMENT, "bad all-reduce arguments");
    MTC_TRY(need_nccl());
    return allreduce_on(c, buffers, counts, n, scale, static_cast<cudaStream_t>(stream));
}

int mtc_comm_allreduce_f32_async(void *comm, void *const *buffers, const size_t *counts, int32_t n, float scale,
                                 void *stream) {
    clear_error();
    Comm *c = static_cast<Comm *>(comm);
    if (c == nullptr || (n > 0 && (buffers == nullptr || counts == nullptr)))
        return fail(MTC_ERR_INVALID_ARGUMENT, "bad all-reduce arguments");
    MTC_TRY(need_nccl());
    if (c->side == nullptr) {
        MTC_CUDA_TRY(cudaSetDevice(c->device));
        // The reductions run at the device's highest stream priority: when a
        // layer's gradients are done, its all-reduce and the next GEMM become
        // ready together, and the block scheduler then seats the reduction's
        // CTAs first instead of leaving them behind a GEMM that fills every SM.
        // MTC_COMM_PRIORITY=normal keeps the default priority (measurements).
        int least = 0, greatest = 0;
        MTC_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&least, &greatest));
        const char *pr = std::getenv("MTC_COMM_PRIORITY");
        const bool high = pr == nullptr || std::strcmp(pr, "normal") != 0;
        MTC_CUDA_TRY(cudaStreamCreateWithPriority(&c->side, cudaStreamNonBlocking, high ? greatest : least));
        MTC_CUDA_TRY(cudaEventCreateWithFlags(&c->ready, cudaEventDisableTiming));
        MTC_CUDA_TRY(cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming));
    }
    MTC_CUDA_TRY(cudaEventRecord(c->ready, static_cast<cudaStream_t>(stream)));
    MTC_CUDA_TRY(cudaStreamWaitEvent(c->side, c->ready, 0));
    MTC_TRY(allreduce_on(c, buffers, counts, n, scale, c->side));
    MTC_CUDA_TRY(cudaEventRecord(c->done, c->side));
    return MTC_OK;
}

int mtc_comm_wait(void *comm, void *stream) {
    clear_error();
    Comm *c = static_cast<Comm *>(comm);
    if (c == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null communicator");
    if (c->done == nullptr) return MTC_OK;  // nothing was queued asynchronously
    MTC_CUDA_TRY(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), c->done, 0));
    return MTC_OK;
}


int mtc_comm_destroy(void *comm) {
    Comm *c = static_cast<Comm *>(comm);
    if (c == nullptr) return MTC_OK;
    if (c->side != nullptr) {
        cudaStreamSynchronize(c->side);
        cudaEventDestroy(c->ready);
        cudaEventDestroy(c->done);
        cudaStreamDestroy(c->side);
    }
    if (c->comm && nccl().ok) nccl().comm_destroy(c->comm);
    delete c;
    return MTC_OK;
}

}  // extern "C"
