// Shared host/device utilities of libmtcuda: status reporting, descriptor
// validation and the iteration-space simplification every kernel family uses.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "mtcuda.h"

namespace mtc {

// ----------------------------------------------------------------- status --

// Records `message` as this thread's last error and returns `code`.
int fail(int code, const char *fmt, ...);
// Clears this thread's last error.
void clear_error();

#define MTC_CUDA_TRY(expr)                                                                   \
    do {                                                                                     \
        cudaError_t mtc_err__ = (expr);                                                      \
        if (mtc_err__ != cudaSuccess) {                                                      \
            return ::mtc::fail(MTC_ERR_RUNTIME, "%s failed: %s (%s:%d)", #expr,              \
                               cudaGetErrorString(mtc_err__), __FILE__, __LINE__);           \
        }                                                                                    \
    } while (0)

#define MTC_TRY(expr)                                                                        \
    do {                                                                                     \
        int mtc_rc__ = (expr);                                                               \
        if (mtc_rc__ != MTC_OK) return mtc_rc__;                                             \
    } while (0)

// Checks the launch that was just enqueued (and counts it).
int check_launch(const char *what);
// Counts a launch made through the driver API.
void count_launch();
// GEMM launch profiling (CUDA events around each launch while enabled).
bool profiling();
void *profile_begin(cudaStream_t stream);
void profile_end(void *begin, cudaStream_t stream, double flops);

inline size_t dtype_size(int32_t dtype) { return dtype == MTC_INT64 ? 8 : 4; }

inline int64_t numel_of(const mtc_desc &d) {
    int64_t n = 1;
    for (int i = 0; i < d.rank; ++i) n *= d.shape[i];
    return n;
}

// Validates rank, dtype, extents and that every reachable element lies inside
// [0, capacity), the check Materialization::validate performs on the CPU side
// (src/tensor/storage/materialization.cpp:77-129).
int validate(const mtc_desc *d, const char *name);

// ------------------------------------------------------- iteration spaces --

constexpr int kMaxOps = MTC_MAX_FUSED_OPERANDS + MTC_MAX_FUSED_OUTPUTS;

// A set of operands walked over one common logical shape.  Operand k reads or
// writes element (i_0..i_{r-1}) at offset[k] + sum_d i_d * stride[k][d].
struct IterSpace {
    int rank = 0;
    int nops = 0;
    int64_t shape[MTC_MAX_RANK];
    int64_t stride[kMaxOps][MTC_MAX_RANK];
    int64_t offset[kMaxOps];
    int64_t numel = 1;
};

// Right-aligned broadcast of operand `d` to `shape` (reference
// Layout::broadcasted_to, src/tensor/storage/layout.cpp:105-143): missing or
// extent-1 axes get stride 0.  Fails on incompatible extents.
int broadcast_strides(const mtc_desc &d, const int64_t *shape, int rank, int64_t *strides_out);

// Drops extent-1 axes and merges neighbouring axes whose strides chain for all
// operands (the same folding ElementwisePlan does on the CPU,
// src/tensor/backend/cpu/iteration/elementwise.cpp:13-59).  A rank-0 space
// becomes rank 1 with extent 1.
void simplify(IterSpace &s);

// ------------------------------------------------------------ device side --

// Unsigned 32-bit division by a runtime-invariant divisor with a precomputed
// multiplier (Granlund-Montgomery round-up method).
struct FastDiv {
    uint32_t d;
    uint32_t mul;
    uint32_t shift;
};

inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f{d, 0, 0};
    if (d <= 1) return f;
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;  // l = ceil(log2 d)
    uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
    f.mul = static_cast<uint32_t>(m);
    f.shift = l;
    return f;
}

#ifdef __CUDACC__
// Asynchronous 4-byte global -> shared copy (sm_80+ cp.async): a thread issues
// any number of them back to back and waits once, so staging loops do not
// pay one memory latency per element.
__device__ __forceinline__ void cp_async4(float *smem, const float *gmem) {
    const unsigned int dst = static_cast<unsigned int>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(gmem) : "memory");
}
// Waits for every cp.async the calling thread issued.
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

__device__ __forceinline__ uint32_t fastdiv(uint32_t n, const FastDiv &f) {
    if (f.d <= 1) return n;
    uint32_t t = __umulhi(n, f.mul);
    return (t + ((n - t) >> 1)) >> (f.shift - 1);
}
#endif


// Number of SMs on the current device (cached per device).
int sm_count(int device);
int current_device();

// Stream-ordered scratch allocation for kernels that need workspace.
// MTB_TRACE set: host calls of the library that take 5 ms or more are reported
// on stderr with a label (allocation, packing, launch), to find host stalls.
bool host_trace();
struct HostSpan {
    const char *label;
    double t0;
    explicit HostSpan(const char *l);
    ~HostSpan();
};

int scratch_alloc(size_t bytes, cudaStream_t stream, void **ptr);
void scratch_free(void *ptr, cudaStream_t stream);

}  // namespace mtc
