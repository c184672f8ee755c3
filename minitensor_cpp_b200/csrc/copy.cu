// Data movement kernels: strided copy (Contiguous/Reshape), concatenation,
// basic-index scatter, Int64 gather and gather-scatter-add, fill.
// Reference: src/tensor/backend/cpu/kernels/copy/loops.hpp:22-303 and
// creation/loops.hpp:21-37.
#include <climits>
#include <cstdlib>
#include <atomic>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace mtc {

__device__ unsigned long long g_device_error[2];

__device__ __forceinline__ void record_device_error(int code, long long detail) {
    if (atomicCAS(&g_device_error[0], 0ull, static_cast<unsigned long long>(code)) == 0ull) {
        atomicExch(&g_device_error[1], static_cast<unsigned long long>(detail));
    }
}

// Device address of the error word on the current device (kernels in other
// files receive it as an argument), looked up once per device.  MTC_OK, or
// MTC_ERR_RUNTIME (and *out = nullptr) when the address cannot be had: callers
// then refuse to launch, because a kernel that gives up a bounded wait writes
// through this pointer.
int device_error_word(unsigned long long **out) {
    static std::mutex mu;
    static unsigned long long *words[64] = {};
    *out = nullptr;
    const int dev = current_device();
    if (dev < 0 || dev >= 64) return fail(MTC_ERR_RUNTIME, "device index %d outside the supported range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (words[dev] == nullptr) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_device_error);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            return fail(MTC_ERR_RUNTIME, "cudaGetSymbolAddress of the device error word failed: %s",
                        cudaGetErrorString(e));
        }
        words[dev] = static_cast<unsigned long long *>(p);
    }
    *out = words[dev];
    return MTC_OK;
}

namespace {

constexpr int kOps = 3;

struct MoveArgs {
    long long numel;
    int rank;
    unsigned int shape[MTC_MAX_RANK];
    FastDiv div[MTC_MAX_RANK];
    char *ptr[kOps];  // 0 = destination, 1 = source / updates, 2 = indices
    long long off[kOps];
    long long str[kOps][MTC_MAX_RANK];
    long long axis_extent;  // gather / scatter: extent of the indexed axis
    long long axis_stride;  // gather / scatter: stride of the indexed axis in the indexed tensor
};

// Coordinates of linear index i over the simplified shape -> per-operand offsets.
template <int NOPS>
__device__ __forceinline__ void offsets_of(const MoveArgs &a, unsigned int i, long long (&o)[NOPS]) {
#pragma unroll
    for (int k = 0; k < NOPS; ++k) o[k] = a.off[k];
    unsigned int rem = i;
#pragma unroll
    for (int d = MTC_MAX_RANK - 1; d >= 1; --d) {
        if (d < a.rank) {
            const unsigned int q = fastdiv(rem, a.div[d]);
            const long long c = static_cast<long long>(rem - q * a.shape[d]);
            rem = q;
#pragma unroll
            for (int k = 0; k < NOPS; ++k) o[k] += c * a.str[k][d];
        }
    }
#pragma unroll
    for (int k = 0; k < NOPS; ++k) o[k] += static_cast<long long>(rem) * a.str[k][0];
}

template <typename T>
__global__ void __launch_bounds__(256) k_copy_strided(const MoveArgs a) {
    const unsigned int n = static_cast<unsigned int>(a.numel);
    for (unsigned int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        long long o[2];
        offsets_of<2>(a, i, o);
        reinterpret_cast<T *>(a.ptr[0])[o[0]] = reinterpret_cast<const T *>(a.ptr[1])[o[1]];
    }
}

// Transposing copy through a 64x64 shared-memory tile: the destination is
// contiguous along the last axis, the source along the second-to-last one.
template <typename T>
__global__ void __launch_bounds__(256) k_copy_tiled(const MoveArgs a) {
    constexpr int TT = 64;
    __shared__ T tile[TT][TT + 1];
    const int r = a.rank;
    const unsigned int rows = a.shape[r - 2], cols = a.shape[r - 1];
    const unsigned int r0 = blockIdx.y * TT, c0 = blockIdx.x * TT;
    long long ob = a.off[0], ib = a.off[1];
    unsigned int rem = blockIdx.z;
    for (int d = r - 3; d >= 0; --d) {
        const unsigned int c = rem % a.shape[d];
        rem /= a.shape[d];
        ob += static_cast<long long>(c) * a.str[0][d];
        ib += static_cast<long long>(c) * a.str[1][d];
    }
    const T *src = reinterpret_cast<const T *>(a.ptr[1]);
    T *dst = reinterpret_cast<T *>(a.ptr[0]);
    const int tx = threadIdx.x % TT, ty = threadIdx.x / TT;
#pragma unroll 4
    for (int s = 0; s < 16; ++s) {
        const unsigned int lr = tx, lc = ty + s * 4;
        if (r0 + lr < rows && c0 + lc < cols)
            tile[lc][lr] = src[ib + static_cast<long long>(r0 + lr) * a.str[1][r - 2] +
                               static_cast<long long>(c0 + lc) * a.str[1][r - 1]];
    }
    __syncthreads();
#pragma unroll 4
    for (int s = 0; s < 16; ++s) {
        const unsigned int lc = tx, lr = ty + s * 4;
        if (r0 + lr < rows && c0 + lc < cols)
            dst[ob + static_cast<long long>(r0 + lr) * a.str[0][r - 2] + static_cast<long long>(c0 + lc) * a.str[0][r - 1]] =
                tile[lc][lr];
    }
}

// Row copy: rank-2 space whose inner axis is contiguous for both operands and a
// multiple of 16 bytes; one 128-bit lane per 16 bytes.
__global__ void __launch_bounds__(256) k_copy_rows16(const MoveArgs a, long long row_vec) {
    const long long total = static_cast<long long>(a.shape[0]) * row_vec;
    for (long long v = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
         v += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long row = v / row_vec, col = v - row * row_vec;
        const uint4 *s = reinterpret_cast<const uint4 *>(a.ptr[1] + (a.off[1] + row * a.str[1][0]) * 4) + col;
        uint4 *d = reinterpret_cast<uint4 *>(a.ptr[0] + (a.off[0] + row * a.str[0][0]) * 4) + col;
        *d = __ldg(s);
    }
}

template <typename T>
__global__ void __launch_bounds__(256) k_fill_flat(T *out, long long n, T value) {
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        out[i] = value;
}

template <typename T>
__global__ void __launch_bounds__(256) k_fill_strided(const MoveArgs a, T value) {
    const unsigned int n = static_cast<unsigned int>(a.numel);
    for (unsigned int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        long long o[1];
        offsets_of<1>(a, i, o);
        reinterpret_cast<T *>(a.ptr[0])[o[0]] = value;
    }
}

// take-along-axis gather, one element per thread.  Operand 0 = out, 1 = source
// base (indexed axis stride zeroed), 2 = indices.
template <typename T>
__global__ void __launch_bounds__(256) k_gather(const MoveArgs a) {
    const unsigned int n = static_cast<unsigned int>(a.numel);
    const long long *idx = reinterpret_cast<const long long *>(a.ptr[2]);
    for (unsigned int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        long long o[3];
        offsets_of<3>(a, i, o);
        const long long j = idx[o[2]];
        if (j < 0 || j >= a.axis_extent) {
            record_device_error(MTC_ERR_OUT_OF_RANGE, j);
            continue;
        }
        reinterpret_cast<T *>(a.ptr[0])[o[0]] = reinterpret_cast<const T *>(a.ptr[1])[o[1] + j * a.axis_stride];
    }
}

// Row gather: the innermost axis is contiguous in out and source and broadcast
// (stride 0) in the indices, so every index selects a whole row of `row_vec`
// 16-byte vectors.  One index load per row; 128-bit copies.
__global__ void __launch_bounds__(256) k_gather_rows16(const MoveArgs a, long long rows, long long row_vec) {
    const long long *idx = reinterpret_cast<const long long *>(a.ptr[2]);
    const long long total = rows * row_vec;
    for (long long v = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
         v += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long row = v / row_vec, col = v - row * row_vec;
        // outer coordinates of this row (all axes but the innermost)
        long long o[3];
        offsets_of<3>(a, static_cast<unsigned int>(row * a.shape[a.rank - 1]), o);
        const long long j = __ldg(idx + o[2]);
        if (j < 0 || j >= a.axis_extent) {
            if (col == 0) record_device_error(MTC_ERR_OUT_OF_RANGE, j);
            continue;
        }
        const uint4 *s = reinterpret_cast<const uint4 *>(a.ptr[1] + (o[1] + j * a.axis_stride) * 4) + col;
        uint4 *d = reinterpret_cast<uint4 *>(a.ptr[0] + o[0] * 4) + col;
        *d = __ldg(s);
    }
}

// Scatter-add: operand 0 = target base (indexed axis stride zeroed), 1 = updates, 2 = indices.
__global__ void __launch_bounds__(256) k_scatter_add(const MoveArgs a) {
    const unsigned int n = static_cast<unsigned int>(a.numel);
    const long long *idx = reinterpret_cast<const long long *>(a.ptr[2]);
    for (unsigned int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        long long o[3];
        offsets_of<3>(a, i, o);
        const long long j = idx[o[2]];
        if (j < 0 || j >= a.axis_extent) {
            record_device_error(MTC_ERR_OUT_OF_RANGE, j);
            continue;
        }
        atomicAdd(reinterpret_cast<float *>(a.ptr[0]) + o[0] + j * a.axis_stride,
                  reinterpret_cast<const float *>(a.ptr[1])[o[1]]);
    }
}

// Row scatter-add with 128-bit vector reductions into L2 (sm_90+ red.v4.f32).
__global__ void __launch_bounds__(256) k_scatter_add_rows16(const MoveArgs a, long long rows, long long row_vec) {
    const long long *idx = reinterpret_cast<const long long *>(a.ptr[2]);
    const long long total = rows * row_vec;
    for (long long v = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
         v += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long row = v / row_vec, col = v - row * row_vec;
        long long o[3];
        offsets_of<3>(a, static_cast<unsigned int>(row * a.shape[a.rank - 1]), o);
        const long long j = __ldg(idx + o[2]);
        if (j < 0 || j >= a.axis_extent) {
            if (col == 0) record_device_error(MTC_ERR_OUT_OF_RANGE, j);
            continue;
        }
        const float4 u = __ldg(reinterpret_cast<const float4 *>(a.ptr[1] + o[1] * 4) + col);
        float4 *t = reinterpret_cast<float4 *>(a.ptr[0] + (o[0] + j * a.axis_stride) * 4) + col;
        atomicAdd(t, u);
    }
}

// ------------------------------------------------ rank-2 row gather / scatter --
// The iteration space [rows, W] after simplification: the inner axis contiguous
// in the table / target and the updates / output, the Int64 index broadcast
// along it (stride 0), so index j of row r selects a whole row of `row_vec`
// 16-byte vectors.  A half-warp (16 lanes) owns ROWS_PER_HALF rows per step and
// issues all of their loads before any store, so every lane keeps several
// 16-byte loads in flight (Little's law at ~6.5 TB/s needs tens of KB in flight
// per SM for random 256-byte rows).

constexpr int kRowsPerHalf = 4;

// Rank-2 row operands from their own descriptors (logical row order kept):
// `rows` rows of row_vec 16-byte vectors; element offsets and row strides.
struct RowArgs {
    char *out;                // gather: output; scatter: target
    const char *in;           // gather: table; scatter: updates
    const long long *idx;
    long long out_off, out_rs, in_off, in_rs, idx_off, idx_rs;
    long long rows;           // gather: output rows; scatter: update rows
    long long extent;         // gather: table rows; scatter: target rows
    int row_vec;
};

__device__ __forceinline__ const uint4 *row_in(const RowArgs &a, long long r, int c) {
    return reinterpret_cast<const uint4 *>(a.in + (a.in_off + r * a.in_rs) * 4) + c;
}
__device__ __forceinline__ uint4 *row_out(const RowArgs &a, long long r, int c) {
    return reinterpret_cast<uint4 *>(a.out + (a.out_off + r * a.out_rs) * 4) + c;
}

__global__ void __launch_bounds__(256) k_gather_rows2(const RowArgs a) {
    const int lane = threadIdx.x & 15;
    const long long half = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 4;
    const long long halves = (static_cast<long long>(gridDim.x) * blockDim.x) >> 4;
    for (long long r0 = half * kRowsPerHalf; r0 < a.rows; r0 += halves * kRowsPerHalf) {
        long long j[kRowsPerHalf];
        bool ok[kRowsPerHalf];
#pragma unroll
        for (int u = 0; u < kRowsPerHalf; ++u) {
            const long long r = r0 + u;
            j[u] = r < a.rows ? __ldg(a.idx + a.idx_off + r * a.idx_rs) : 0;
            ok[u] = r < a.rows && j[u] >= 0 && j[u] < a.extent;
            if (r < a.rows && !ok[u] && lane == 0) record_device_error(MTC_ERR_OUT_OF_RANGE, j[u]);
        }
        for (int c = lane; c < a.row_vec; c += 16) {
            uint4 v[kRowsPerHalf];
#pragma unroll
            for (int u = 0; u < kRowsPerHalf; ++u)
                if (ok[u]) v[u] = __ldg(row_in(a, j[u], c));
#pragma unroll
            for (int u = 0; u < kRowsPerHalf; ++u)
                if (ok[u]) __stcs(row_out(a, r0 + u, c), v[u]);
        }
    }
}

// Row scatter-add with 128-bit reductions into L2 (red.global.add.v4.f32) into
// the values already in the target (mtc_gather_scatter_add_into): the loop of
// k_gather_rows2 with the roles swapped.  As the clearing scatter-add it
// measured 2.68 ms at 2^24 rows of 64 floats (with the zero fill), against
// 2.77 ms for the ordered segment sum, which is kept there for its order.
__global__ void __launch_bounds__(256) k_scatter_rows2(const RowArgs a) {
    const int lane = threadIdx.x & 15;
    const long long half = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 4;
    const long long halves = (static_cast<long long>(gridDim.x) * blockDim.x) >> 4;
    for (long long r0 = half * kRowsPerHalf; r0 < a.rows; r0 += halves * kRowsPerHalf) {
        long long j[kRowsPerHalf];
        bool ok[kRowsPerHalf];
#pragma unroll
        for (int u = 0; u < kRowsPerHalf; ++u) {
            const long long r = r0 + u;
            j[u] = r < a.rows ? __ldg(a.idx + a.idx_off + r * a.idx_rs) : 0;
            ok[u] = r < a.rows && j[u] >= 0 && j[u] < a.extent;
            if (r < a.rows && !ok[u] && lane == 0) record_device_error(MTC_ERR_OUT_OF_RANGE, j[u]);
        }
        for (int c = lane; c < a.row_vec; c += 16) {
            float4 v[kRowsPerHalf];
#pragma unroll
            for (int u = 0; u < kRowsPerHalf; ++u)
                if (ok[u]) v[u] = __ldg(reinterpret_cast<const float4 *>(row_in(a, r0 + u, c)));
#pragma unroll
            for (int u = 0; u < kRowsPerHalf; ++u)
                if (ok[u]) atomicAdd(reinterpret_cast<float4 *>(row_out(a, j[u], c)), v[u]);
        }
    }
}

// Scatter-add as a segment sum.  out[t] = sum of upd[i] over the rows i with
// idx[i] = t, added in ascending i starting from +0 -- the reference's order
// (zero-filled target, then += in the iteration order of the updates), so the
// result is the reference's bit for bit whatever the values.  Steps:
//   count  : counts[t] = number of rows i with idx[i] = t, and rank[i] = the
//            slot row i took (returning atomics on the L2-resident counts)
//   scan   : block-local exclusive prefix sums of the counts in place, and
//            the scanned block totals; start(t) = starts[t] + sums[t / kScanBlock]
//   fill   : perm[start(idx[i]) + rank[i]] = i (plain stores)
//   sort   : each segment sorted ascending (in-thread up to 32 rows; a CTA
//            bitonic sort in shared memory up to kLongSegment rows)
//   sum    : every target row written once (zeros for rows no index names),
//            so the target needs no zero fill and is never read back.
// Scratch: counts / starts (T + 1), rank and perm (n each), block sums, the long-segment list.

constexpr int kScanItems = 8;                       // per thread
constexpr int kScanBlock = 256 * kScanItems;        // counts per scan block
constexpr int kLongSegment = 4096;                  // longest segment sorted in shared memory

// counts[j] += 1 for every update row i with idx[i] = j; rank[i] = the slot i
// took within its target's segment (a returning atomic on the L2-resident
// counts), -1 for an index outside the target.  rank may be null (no slots).
// (Counting in slices of the targets, so that each launch's counts stay in
// L2, measured no faster at 2^24 rows: the returning atomics bound it.)
__global__ void __launch_bounds__(256) k_seg_count(const RowArgs a, int *counts, int *rank) {
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.rows;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long j = __ldg(a.idx + a.idx_off + i * a.idx_rs);
        if (j < 0 || j >= a.extent) {
            record_device_error(MTC_ERR_OUT_OF_RANGE, j);
            if (rank != nullptr) rank[i] = -1;
            continue;
        }
        const int r = atomicAdd(counts + j, 1);
        if (rank != nullptr) rank[i] = r;
    }
}

// Block-local exclusive scan of kScanBlock counts; block totals to `sums`.
__global__ void __launch_bounds__(256) k_scan_blocks(const int *in, int *out, long long len, int *sums) {
    __shared__ int warp_tot[8];
    const long long base = static_cast<long long>(blockIdx.x) * kScanBlock + threadIdx.x * kScanItems;
    int v[kScanItems];
    int run = 0;
#pragma unroll
    for (int q = 0; q < kScanItems; ++q) {
        v[q] = base + q < len ? in[base + q] : 0;
        const int t = v[q];
        v[q] = run;
        run += t;
    }
    // exclusive scan of the per-thread totals across the block
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    int warp_off = 0;
    for (int w = 0; w < warp; ++w) warp_off += warp_tot[w];
    const int excl = warp_off + inc - run;
#pragma unroll
    for (int q = 0; q < kScanItems; ++q)
        if (base + q < len) out[base + q] = v[q] + excl;
    if (threadIdx.x == 255) sums[blockIdx.x] = warp_off + inc;
}

// Exclusive scan of the n block totals in one CTA, in place: 4 consecutive
// totals a thread (16-byte coalesced loads), 4096 a pass, carried across passes.
// A target's start is then starts[t] + sums[t / kScanBlock] (seg_start).
__global__ void __launch_bounds__(1024) k_scan_totals(int *sums, int n) {
    __shared__ int warp_tot[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int carry = 0;
    for (int base = 0; base < n; base += 1024 * 4) {
        const int i0 = base + static_cast<int>(threadIdx.x) * 4;
        int v[4];
        int run = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int t = i0 + q < n ? sums[i0 + q] : 0;
            v[q] = run;
            run += t;
        }
        int inc = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
        }
        if (lane == 31) warp_tot[warp] = inc;
        __syncthreads();
        if (warp == 0) {
            int x = warp_tot[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            warp_tot[lane] = x;  // inclusive over the warps
        }
        __syncthreads();
        const int excl = carry + (warp > 0 ? warp_tot[warp - 1] : 0) + inc - run;
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (i0 + q < n) sums[i0 + q] = v[q] + excl;
        carry += warp_tot[31];
        __syncthreads();  // warp_tot is rewritten by the next pass
    }
}

// Start of target t's segment in perm (t = targets gives the end of the last);
// sums is null when starts already holds the final offsets.
__device__ __forceinline__ int seg_start(const int *starts, const int *sums, long long t) {
    return __ldg(starts + t) + (sums != nullptr ? __ldg(sums + t / kScanBlock) : 0);
}

// perm[starts[j] + rank[i]] = i for the update rows whose target j lies in
// [lo, hi): every update row in the slot the count pass gave it (no atomics;
// the order within a segment is fixed by the sort).  Run over slices of the
// targets, the randomly addressed parts of starts and perm stay in L2.
__global__ void __launch_bounds__(256) k_seg_fill(const RowArgs a, const int *rank, const int *starts,
                                                  const int *sums, int *perm, long long lo, long long hi) {
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.rows;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long j = __ldg(a.idx + a.idx_off + i * a.idx_rs);
        if (j < lo || j >= hi) continue;  // also every index outside the target
        perm[seg_start(starts, sums, j) + __ldcs(rank + i)] = static_cast<int>(i);
    }
}

// Sorts the segments of up to 32 rows in place, one thread per target; longer
// segments (up to kLongSegment) go to a list for k_seg_sort_long.
__global__ void __launch_bounds__(256) k_seg_sort(const int *starts, const int *sums, int *perm, long long targets,
                                                  int *long_list, int *long_count, int long_capacity) {
    for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; t < targets;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int s = seg_start(starts, sums, t), e = seg_start(starts, sums, t + 1);
        const int len = e - s;
        if (len < 2) continue;
        if (len > 32) {
            const int k = atomicAdd(long_count, 1);
            if (k < long_capacity) long_list[k] = static_cast<int>(t);
            continue;
        }
        int *p = perm + s;
        for (int q = 1; q < len; ++q) {
            const int key = p[q];
            int w = q - 1;
            while (w >= 0 && p[w] > key) {
                p[w + 1] = p[w];
                --w;
            }
            p[w + 1] = key;
        }
    }
}

// Bitonic sort of one long segment per CTA iteration in shared memory (padded
// with INT_MAX to a power of two); segments above kLongSegment stay in fill order.
__global__ void __launch_bounds__(256) k_seg_sort_long(const int *starts, const int *sums, int *perm,
                                                       const int *long_list, const int *long_count, int long_capacity) {
    __shared__ int keys[kLongSegment];
    const int count = min(*long_count, long_capacity);
    for (int e = blockIdx.x; e < count; e += gridDim.x) {
        const int t = long_list[e];
        const int s = seg_start(starts, sums, t), len = seg_start(starts, sums, t + 1) - s;
        if (len > kLongSegment) continue;
        int n2 = 64;
        while (n2 < len) n2 <<= 1;
        for (int q = threadIdx.x; q < n2; q += blockDim.x) keys[q] = q < len ? perm[s + q] : 0x7fffffff;
        __syncthreads();
        for (int k = 2; k <= n2; k <<= 1) {
            for (int jj = k >> 1; jj > 0; jj >>= 1) {
                for (int q = threadIdx.x; q < n2; q += blockDim.x) {
                    const int partner = q ^ jj;
                    if (partner > q) {
                        const bool up = (q & k) == 0;
                        const int x = keys[q], y = keys[partner];
                        if ((x > y) == up) {
                            keys[q] = y;
                            keys[partner] = x;
                        }
                    }
                }
                __syncthreads();
            }
        }
        for (int q = threadIdx.x; q < len; q += blockDim.x) perm[s + q] = keys[q];
        __syncthreads();
    }
}

__device__ __forceinline__ void add4(float4 &acc, const uint4 w) {
    acc.x = __fadd_rn(acc.x, __uint_as_float(w.x));
    acc.y = __fadd_rn(acc.y, __uint_as_float(w.y));
    acc.z = __fadd_rn(acc.z, __uint_as_float(w.z));
    acc.w = __fadd_rn(acc.w, __uint_as_float(w.w));
}

// ---- bucketed prelude (targets from 2^22 to 2^26 rows) -------------------
// The same starts and sorted perm, built without global atomics: a counting
// sort by target in two levels whose counters live in shared memory.  At 2^24
// rows of 64 floats: hist 53 us, scan 16, part 116, sort 160, against count
// 206, scan 48, fill 233, sort 113 for the atomic prelude (0.35 / 0.60 ms;
// the whole scatter-add 1.92 / 2.17 ms).
//   hist : per chunk of kChunk updates, how many fall in each bucket of
//          kBucketRows target rows, written bucket-major
//   scan : of that matrix (the scan kernels above) -> where each chunk's
//          updates of each bucket go
//   part : each chunk stages its updates by bucket in shared memory and writes
//          (update row, target row within the bucket) runs to their places
//   sort : a CTA per bucket counts its target rows in shared memory, scans,
//          writes starts, places the update rows into perm and sorts each
//          segment (the long ones go to k_seg_sort_long as before)
constexpr int kBucketShift = 13;
constexpr int kBucketRows = 1 << kBucketShift;     // target rows a bucket
constexpr int kChunk = 8192;                       // updates a partition CTA
constexpr int kMaxBuckets = 8192;                  // so targets <= 2^26
constexpr int kPartThreads = 1024;
constexpr int kPerThread = kChunk / kPartThreads;  // 8
constexpr int kStageCap = 16384;                   // a bucket's updates placed and sorted in shared memory
// partition smem: the stage, then 2 * nb counters and offsets, then 32 ints
constexpr size_t part_smem(int nb) { return kChunk * sizeof(int2) + (2 * static_cast<size_t>(nb) + 32) * sizeof(int); }
constexpr size_t kBktSortSmem = (kBucketRows + kStageCap + 32) * sizeof(int);

// Exclusive scan of v[0, len) in shared memory by a CTA of kPartThreads threads
// (len <= 16 * kPartThreads, v 16-byte aligned); returns the total.  Each
// thread owns a run of a multiple of 4 entries, read and written as int4 (a
// scalar run of 8 per thread made the bucket sort shared-memory-bound through
// 8-way bank conflicts).  wtot: 32 ints of shared scratch.
__device__ int block_exclusive_scan(int *v, int len, int *wtot) {
    const int per = ((len + kPartThreads - 1) / kPartThreads + 3) & ~3;
    const int b0 = static_cast<int>(threadIdx.x) * per;
    int run = 0;
    for (int q = 0; q < per; q += 4) {
        if (b0 + q + 3 < len) {
            const int4 x = *reinterpret_cast<const int4 *>(v + b0 + q);
            run += x.x + x.y + x.z + x.w;
        } else {
            for (int k = q; k < q + 4; ++k)
                if (b0 + k < len) run += v[b0 + k];
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) wtot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int x = wtot[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        wtot[lane] = x;
    }
    __syncthreads();
    int off = (warp > 0 ? wtot[warp - 1] : 0) + inc - run;
    for (int q = 0; q < per; q += 4) {
        if (b0 + q + 3 < len) {
            int4 x = *reinterpret_cast<const int4 *>(v + b0 + q);
            const int a0 = off, a1 = a0 + x.x, a2 = a1 + x.y, a3 = a2 + x.z;
            off = a3 + x.w;
            x = make_int4(a0, a1, a2, a3);
            *reinterpret_cast<int4 *>(v + b0 + q) = x;
        } else {
            for (int k = q; k < q + 4; ++k) {
                if (b0 + k < len) {
                    const int t = v[b0 + k];
                    v[b0 + k] = off;
                    off += t;
                }
            }
        }
    }
    const int total = wtot[31];
    __syncthreads();
    return total;
}

__global__ void __launch_bounds__(kPartThreads, 2) k_bkt_hist(const RowArgs a, int *hist, int nb, long long chunks) {
    __shared__ int h[kMaxBuckets];
    for (int b = threadIdx.x; b < nb; b += kPartThreads) h[b] = 0;
    __syncthreads();
    const long long base = static_cast<long long>(blockIdx.x) * kChunk;
    long long jv[kPerThread];  // all of a thread's index loads in flight before its first count
#pragma unroll
    for (int q = 0; q < kPerThread; ++q) {
        const long long i = base + threadIdx.x + q * kPartThreads;
        jv[q] = i < a.rows ? __ldg(a.idx + a.idx_off + i * a.idx_rs) : LLONG_MIN;
    }
#pragma unroll
    for (int q = 0; q < kPerThread; ++q) {
        if (jv[q] == LLONG_MIN) continue;
        if (jv[q] < 0 || jv[q] >= a.extent) record_device_error(MTC_ERR_OUT_OF_RANGE, jv[q]);
        else atomicAdd(&h[jv[q] >> kBucketShift], 1);
    }
    __syncthreads();
    for (int b = threadIdx.x; b < nb; b += kPartThreads) hist[static_cast<long long>(b) * chunks + blockIdx.x] = h[b];
}

// off / off_sums: the scanned histogram (offset of chunk c's bucket-b updates
// at b * chunks + c, plus its scan block's sum).
__global__ void __launch_bounds__(kPartThreads, 2) k_bkt_part(const RowArgs a, const int *off, const int *off_sums,
                                                           int2 *pairs, int nb, long long chunks) {
    extern __shared__ __align__(16) unsigned char bkt_smem[];
    int2 *stage = reinterpret_cast<int2 *>(bkt_smem);     // kChunk: the chunk's updates by bucket
    int *h = reinterpret_cast<int *>(stage + kChunk);      // nb counts, then chunk-local offsets
    int *goff = h + nb;                                    // nb: the chunk's place in each bucket
    int *wtot = goff + nb;
    const long long c = blockIdx.x;
    for (int b = threadIdx.x; b < nb; b += kPartThreads) {
        h[b] = 0;
        const long long x = static_cast<long long>(b) * chunks + c;
        goff[b] = off[x] + off_sums[x / kScanBlock];
    }
    __syncthreads();
    const long long base = c * kChunk;
    int jj[kPerThread], rr[kPerThread];
#pragma unroll
    for (int q = 0; q < kPerThread; ++q) {  // the loads first, all in flight
        const long long i = base + threadIdx.x + q * kPartThreads;
        const long long j = i < a.rows ? __ldg(a.idx + a.idx_off + i * a.idx_rs) : -1;
        jj[q] = j >= 0 && j < a.extent ? static_cast<int>(j) : -1;  // the histogram pass recorded the others
    }
#pragma unroll
    for (int q = 0; q < kPerThread; ++q) rr[q] = jj[q] >= 0 ? atomicAdd(&h[jj[q] >> kBucketShift], 1) : 0;
    __syncthreads();
    const int valid = block_exclusive_scan(h, nb, wtot);
#pragma unroll
    for (int q = 0; q < kPerThread; ++q)
        if (jj[q] >= 0)
            stage[h[jj[q] >> kBucketShift] + rr[q]] =
                make_int2(static_cast<int>(base + threadIdx.x + q * kPartThreads), jj[q]);
    __syncthreads();
    for (int p = threadIdx.x; p < valid; p += kPartThreads) {
        const int2 e = stage[p];
        const int b = e.y >> kBucketShift;
        pairs[goff[b] + (p - h[b])] = make_int2(e.x, e.y & (kBucketRows - 1));
    }
}

// Insertion sort of a short segment (at most 32 entries) in place.
template <class P>
__device__ __forceinline__ void sort_short(P pp, int len) {
    for (int q = 1; q < len; ++q) {
        const int key = pp[q];
        int w = q - 1;
        while (w >= 0 && pp[w] > key) {
            pp[w + 1] = pp[w];
            --w;
        }
        pp[w + 1] = key;
    }
}

// A CTA per bucket: counts its target rows in shared memory, scans them into
// starts, places the update rows (in shared memory when the bucket holds at
// most kStageCap updates, else straight into perm) and sorts each segment.
// Segments above 32 updates go to the long list, sorted in perm afterwards.
__global__ void __launch_bounds__(kPartThreads, 2) k_bkt_sort(const int2 *pairs, const int *off, const int *off_sums,
                                                           long long chunks, int nb, long long targets, int *starts,
                                                           int *perm, int *long_list, int *long_count,
                                                           int long_capacity) {
    extern __shared__ __align__(16) unsigned char bkt_smem[];
    int *cnt = reinterpret_cast<int *>(bkt_smem);  // kBucketRows
    int *stage = cnt + kBucketRows;                // kStageCap
    int *wtot = stage + kStageCap;
    const int b = blockIdx.x;
    const long long t0 = static_cast<long long>(b) << kBucketShift;
    const int wt = static_cast<int>(targets - t0 < kBucketRows ? targets - t0 : kBucketRows);
    const long long x0 = static_cast<long long>(b) * chunks, x1 = x0 + chunks;
    const int beg = off[x0] + off_sums[x0 / kScanBlock];
    const int end = off[x1] + off_sums[x1 / kScanBlock];
    const bool staged = end - beg <= kStageCap;  // uniform in the CTA
    for (int t = threadIdx.x; t < wt; t += kPartThreads) cnt[t] = 0;
    __syncthreads();
    constexpr int kIn = 8;  // pair loads in flight per thread
    for (int e0 = beg; e0 < end; e0 += kIn * kPartThreads) {
        int y[kIn];
#pragma unroll
        for (int u = 0; u < kIn; ++u) {
            const int e = e0 + static_cast<int>(threadIdx.x) + u * kPartThreads;
            y[u] = e < end ? pairs[e].y : -1;
        }
#pragma unroll
        for (int u = 0; u < kIn; ++u)
            if (y[u] >= 0) atomicAdd(&cnt[y[u]], 1);
    }
    __syncthreads();
    block_exclusive_scan(cnt, wt, wtot);
    for (int t = threadIdx.x; t < wt; t += kPartThreads) starts[t0 + t] = beg + cnt[t];
    if (b == nb - 1 && threadIdx.x == 0) starts[targets] = end;
    __syncthreads();  // every start is read before the placement moves cnt on
    for (int e0 = beg; e0 < end; e0 += kIn * kPartThreads) {
        int2 pe[kIn];
#pragma unroll
        for (int u = 0; u < kIn; ++u) {
            const int e = e0 + static_cast<int>(threadIdx.x) + u * kPartThreads;
            pe[u] = e < end ? pairs[e] : make_int2(0, -1);
        }
#pragma unroll
        for (int u = 0; u < kIn; ++u) {
            if (pe[u].y < 0) continue;
            const int p = atomicAdd(&cnt[pe[u].y], 1);
            if (staged) stage[p] = pe[u].x;
            else perm[beg + p] = pe[u].x;
        }
    }
    __syncthreads();
    // cnt[t] is now the end of segment t within the bucket; sort each segment
    for (int t = threadIdx.x; t < wt; t += kPartThreads) {
        const int s0 = t == 0 ? 0 : cnt[t - 1];
        const int len = cnt[t] - s0;
        if (len > 32) {
            const int k = atomicAdd(long_count, 1);
            if (k < long_capacity) long_list[k] = static_cast<int>(t0 + t);
        } else if (len > 1) {
            if (staged) sort_short(stage + s0, len);
            else sort_short(perm + beg + s0, len);
        }
    }
    if (staged) {
        __syncthreads();
        for (int e = threadIdx.x; e < end - beg; e += kPartThreads) perm[beg + e] = stage[e];
    }
}

// out[t] = +0 + upd[perm[s]] + upd[perm[s + 1]] + ... for every target row t,
// walking the sorted update list: a half-warp owns kWalkTargets consecutive
// target rows and consumes their update rows in list order, four rows in
// flight per lane at a time whatever the segment lengths; a row is stored as
// soon as its segment ends (zeros for rows no index names).  Measured at 2^24
// rows of 64 floats: 1.56 ms (5.6 TB/s), against 1.88 ms for a warp per 32
// target rows with each row's first three updates prefetched (two to four rows
// in flight per lane), and 1.67 ms when the walk also sorted each group of up
// to 16 updates in registers (a bitonic network over the half-warp) in place of
// the segment sort.  Four rows a batch at 64 registers (4 CTAs of 256 per SM)
// measured best: 2 rows at 40 registers 2.37 ms for the whole scatter-add, 4
// at 48 (spilling) 2.20, 4 at 72 2.45, 8 at 80 2.27, 8 at 94 2.62, against 2.16.
constexpr int kWalkTargets = 8;  // target rows per half-warp step (at most 15)

__global__ void __launch_bounds__(256, 4) k_seg_walk(const RowArgs a, const int *starts, const int *sums,
                                                     const int *perm) {
    constexpr int kBatch = 4;
    const int hl = threadIdx.x & 15;
    const unsigned hmask = 0xffffu << (threadIdx.x & 16);
    const long long half = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 4;
    const long long halves = (static_cast<long long>(gridDim.x) * blockDim.x) >> 4;
    const long long targets = a.extent;
    for (long long t0 = half * kWalkTargets; t0 < targets; t0 += halves * kWalkTargets) {
        const int g = static_cast<int>(targets - t0 < kWalkTargets ? targets - t0 : kWalkTargets);
        // lane l: the start of target t0 + l; lane g: the end of target t0 + g - 1
        // (loading the next group's bounds a group ahead measured no faster)
        const int sb = hl <= g ? seg_start(starts, sums, t0 + hl) : 0;
        const int e_beg = __shfl_sync(hmask, sb, 0, 16);
        const int e_end = __shfl_sync(hmask, sb, g, 16);
        for (int c0 = 0; c0 < a.row_vec; c0 += 16) {
            const int c = c0 + hl;
            const bool col = c < a.row_vec;
            int q = 0;                                        // current target of the group
            int seg_end = __shfl_sync(hmask, sb, 1, 16);      // end of target t0 + q
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int e = e_beg; e < e_end; e += kBatch) {
                const int nb = e_end - e < kBatch ? e_end - e : kBatch;  // uniform in the half-warp
                const int pl = hl < nb ? __ldg(perm + e + hl) : 0;
                int p[kBatch];
                uint4 v[kBatch];
#pragma unroll
                for (int u = 0; u < kBatch; ++u) p[u] = __shfl_sync(hmask, pl, u, 16);
#pragma unroll
                for (int u = 0; u < kBatch; ++u)
                    if (u < nb && col) v[u] = __ldg(row_in(a, p[u], c));
#pragma unroll
                for (int u = 0; u < kBatch; ++u) {
                    if (u >= nb) break;
                    while (e + u >= seg_end) {  // finish the targets that end before this entry
                        if (col) __stcs(reinterpret_cast<float4 *>(row_out(a, t0 + q, c)), acc);
                        acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                        ++q;
                        seg_end = __shfl_sync(hmask, sb, q + 1, 16);
                    }
                    if (col) add4(acc, v[u]);
                }
            }
            for (; q < g; ++q) {
                if (col) __stcs(reinterpret_cast<float4 *>(row_out(a, t0 + q, c)), acc);
                acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
    }
}

int grid_for(long long work, int per_block = 256) {
    const int sms = sm_count(current_device());
    long long b = (work + per_block - 1) / per_block;
    if (b > static_cast<long long>(sms) * 8) b = static_cast<long long>(sms) * 8;
    return b < 1 ? 1 : static_cast<int>(b);
}

void fill_divs(MoveArgs &a, const IterSpace &s) {
    a.numel = s.numel;
    a.rank = s.rank;
    for (int d = 0; d < s.rank; ++d) {
        a.shape[d] = static_cast<unsigned int>(s.shape[d]);
        a.div[d] = make_fastdiv(static_cast<uint32_t>(s.shape[d]));
        for (int k = 0; k < s.nops; ++k) a.str[k][d] = s.stride[k][d];
    }
    for (int k = 0; k < s.nops; ++k) a.off[k] = s.offset[k];
}

bool aligned16(const void *p, long long off_elems, int elem) {
    return (reinterpret_cast<uintptr_t>(static_cast<const char *>(p) + off_elems * elem) % 16) == 0;
}

// Rank-2 row operands along axis 0 with the index broadcast along the row
// (table / target, updates or output, and indices all [rows, W] views whose
// inner axis is contiguous, 16-byte aligned rows of whole vectors): the row
// gather and the segment-sum scatter-add.  `in` is the table (gather) or the
// updates (scatter); `indexed` is the operand the index selects rows of.
bool row_operands(const mtc_desc &out, const mtc_desc &in, const mtc_desc &idx, const mtc_desc &indexed, int64_t axis,
                  RowArgs &r) {
    if (axis != 0 || out.rank != 2 || in.rank != 2 || idx.rank != 2) return false;
    const int64_t w = idx.shape[1];
    if (w < 4 || w % 4 != 0 || out.shape[1] != w || in.shape[1] != w) return false;
    if (out.strides[1] != 1 || in.strides[1] != 1 || idx.strides[1] != 0) return false;
    if (!aligned16(out.data, out.offset, 4) || !aligned16(in.data, in.offset, 4)) return false;
    if (out.strides[0] % 4 != 0 || in.strides[0] % 4 != 0) return false;
    std::memset(&r, 0, sizeof(r));
    r.out = static_cast<char *>(out.data);
    r.in = static_cast<const char *>(in.data);
    r.idx = static_cast<const long long *>(idx.data);
    r.out_off = out.offset;
    r.out_rs = out.strides[0];
    r.in_off = in.offset;
    r.in_rs = in.strides[0];
    r.idx_off = idx.offset;
    r.idx_rs = idx.strides[0];
    r.rows = idx.shape[0];
    r.extent = indexed.shape[0];
    r.row_vec = static_cast<int>(w / 4);
    return w / 4 < (int64_t{1} << 30);
}

int row_gather(const RowArgs &r, cudaStream_t st) {
    if (r.rows == 0) return MTC_OK;
    k_gather_rows2<<<grid_for(r.rows * 4), 256, 0, st>>>(r);  // 16 lanes per kRowsPerHalf rows
    return check_launch("row gather");
}

// Segment-sum scatter-add (see k_seg_walk); MTC_ERR_UNSUPPORTED when the sizes
// exceed the int32 bookkeeping or the two-level scan (the caller then takes
// the atomic kernel).
// The bucketed prelude (k_bkt_*) and the walk, for 2^22 <= T <= 2^26 target rows.
int bucketed_scatter_add(const RowArgs &r, cudaStream_t st) {
    const long long T = r.extent, n = r.rows;
    const int nb = static_cast<int>((T + kBucketRows - 1) / kBucketRows);
    const long long chunks = (n + kChunk - 1) / kChunk;
    const long long hlen = static_cast<long long>(nb) * chunks + 1;  // + the total after the scan
    const long long hblk = (hlen + kScanBlock - 1) / kScanBlock;
    const long long cap = n / 33 + 1;
    // hist (scanned in place) | hist block sums | starts (T + 1) | perm (n) | long list | count | pairs (n int2)
    size_t words = static_cast<size_t>(hlen + hblk + (T + 1) + n + cap + 1);
    words = (words + 1) & ~size_t(1);  // 8-byte alignment of the pairs
    void *scratch = nullptr;
    MTC_TRY(scratch_alloc(words * sizeof(int) + static_cast<size_t>(n) * sizeof(int2), st, &scratch));
    int *hist = static_cast<int *>(scratch);
    int *hsums = hist + hlen;
    int *starts = hsums + hblk;
    int *perm = starts + (T + 1);
    int *long_list = perm + n;
    int *long_count = long_list + cap;
    int2 *pairs = reinterpret_cast<int2 *>(static_cast<int *>(scratch) + words);
    int rc = MTC_OK;
    auto launched = [&](const char *what) {
        if (rc == MTC_OK) rc = check_launch(what);
    };
    if (cudaMemsetAsync(hist + hlen - 1, 0, sizeof(int), st) != cudaSuccess ||
        cudaMemsetAsync(long_count, 0, sizeof(int), st) != cudaSuccess ||
        cudaFuncSetAttribute(k_bkt_part, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(part_smem(kMaxBuckets))) != cudaSuccess ||
        cudaFuncSetAttribute(k_bkt_sort, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kBktSortSmem)) != cudaSuccess) {
        rc = fail(MTC_ERR_RUNTIME, "bucketed scatter-add set-up failed: %s", cudaGetErrorString(cudaGetLastError()));
    }
    if (rc == MTC_OK) {
        k_bkt_hist<<<static_cast<unsigned>(chunks), kPartThreads, 0, st>>>(r, hist, nb, chunks);
        launched("bucketed scatter-add histogram");
    }
    if (rc == MTC_OK) {
        k_scan_blocks<<<static_cast<unsigned>(hblk), 256, 0, st>>>(hist, hist, hlen, hsums);
        launched("bucketed scatter-add scan");
    }
    if (rc == MTC_OK) {
        k_scan_totals<<<1, 1024, 0, st>>>(hsums, static_cast<int>(hblk));
        launched("bucketed scatter-add scan totals");
    }
    if (rc == MTC_OK) {
        k_bkt_part<<<static_cast<unsigned>(chunks), kPartThreads, part_smem(nb), st>>>(r, hist, hsums, pairs, nb,
                                                                                        chunks);
        launched("bucketed scatter-add partition");
    }
    if (rc == MTC_OK) {
        k_bkt_sort<<<static_cast<unsigned>(nb), kPartThreads, kBktSortSmem, st>>>(
            pairs, hist, hsums, chunks, nb, T, starts, perm, long_list, long_count, static_cast<int>(cap));
        launched("bucketed scatter-add bucket sort");
    }
    if (rc == MTC_OK) {
        k_seg_sort_long<<<sm_count(current_device()) * 2, 256, 0, st>>>(starts, nullptr, perm, long_list, long_count,
                                                                          static_cast<int>(cap));
        launched("bucketed scatter-add long sort");
    }
    if (rc == MTC_OK) {
        k_seg_walk<<<grid_for(T * 16 / kWalkTargets), 256, 0, st>>>(r, starts, nullptr, perm);
        launched("bucketed scatter-add sum");
    }
    scratch_free(scratch, st);
    return rc;
}

int segment_scatter_add(const RowArgs &r, cudaStream_t st) {
    const long long T = r.extent, n = r.rows;
    {
        const char *bv = std::getenv("MTC_SEG_BUCKETS");  // measurement switch: "0" keeps the atomic count
        const bool allow = bv == nullptr || bv[0] != '0';
        if (allow && T >= (1ll << 22) && T <= static_cast<long long>(kMaxBuckets) * kBucketRows && n > 0 &&
            n < (int64_t{1} << 31) - 1 && ((n + kChunk - 1) / kChunk) * ((T + kBucketRows - 1) / kBucketRows) <
                                              (int64_t{1} << 30) &&
            (n + kChunk - 1) / kChunk < 65536 * 32)
            return bucketed_scatter_add(r, st);
    }
    if (n >= (int64_t{1} << 31) - 1 || T + 1 > static_cast<long long>(kScanBlock) * 256 * 64)
        return fail(MTC_ERR_UNSUPPORTED, "scatter-add beyond the segment path's sizes");
    if (T == 0) {
        if (n > 0) {  // every index is out of range: record it like the other paths
            k_seg_count<<<grid_for(n), 256, 0, st>>>(r, nullptr, nullptr);
            return check_launch("segment scatter-add count");
        }
        return MTC_OK;
    }
    const long long nblk = (T + 1 + kScanBlock - 1) / kScanBlock;
    const long long cap = n / 33 + 1;
    const long long nn = n > 0 ? n : 1;
    // counts (scanned in place into starts) | rank | perm | block sums | long-segment list | count
    const size_t words = static_cast<size_t>((T + 1) + 2 * nn + nblk + cap + 1);
    void *scratch = nullptr;
    MTC_TRY(scratch_alloc(words * sizeof(int), st, &scratch));
    int *counts = static_cast<int *>(scratch);
    int *starts = counts;
    int *rank = counts + (T + 1);
    int *perm = rank + nn;
    int *sums = perm + nn;
    int *long_list = sums + nblk;
    int *long_count = long_list + cap;
    int rc = MTC_OK;
    auto launched = [&](const char *what) {
        if (rc == MTC_OK) rc = check_launch(what);
    };
    if (cudaMemsetAsync(counts, 0, static_cast<size_t>(T + 1) * sizeof(int), st) != cudaSuccess ||
        cudaMemsetAsync(long_count, 0, sizeof(int), st) != cudaSuccess) {
        rc = fail(MTC_ERR_RUNTIME, "segment scatter-add: clearing the counters failed: %s",
                  cudaGetErrorString(cudaGetLastError()));
    }
    if (rc == MTC_OK && n > 0) {
        k_seg_count<<<grid_for(n), 256, 0, st>>>(r, counts, rank);
        launched("segment scatter-add count");
    }
    if (rc == MTC_OK) {
        k_scan_blocks<<<static_cast<unsigned>(nblk), 256, 0, st>>>(counts, starts, T + 1, sums);  // in place
        launched("segment scatter-add scan");
    }
    if (rc == MTC_OK) {
        k_scan_totals<<<1, 1024, 0, st>>>(sums, static_cast<int>(nblk));
        launched("segment scatter-add scan totals");
    }
    if (rc == MTC_OK && n > 0) {
        // slices of the targets whose starts and perm regions (4 bytes per target
        // and per update) take at most 64 MB together, half of the 126 MB L2:
        // at 2^24 rows two slices took the fill from 0.50 to 0.23 ms (four: 0.25)
        const long long slice_bytes = 64ll << 20;
        const long long slices = ((T + n) * 4 + slice_bytes - 1) / slice_bytes;
        const long long per = (T + slices - 1) / slices;
        for (long long lo = 0; lo < T && rc == MTC_OK; lo += per) {
            k_seg_fill<<<grid_for(n), 256, 0, st>>>(r, rank, starts, sums, perm, lo, lo + per < T ? lo + per : T);
            launched("segment scatter-add fill");
        }
        if (rc == MTC_OK) {
            k_seg_sort<<<grid_for(T), 256, 0, st>>>(starts, sums, perm, T, long_list, long_count,
                                                   static_cast<int>(cap));
            launched("segment scatter-add sort");
        }
        if (rc == MTC_OK) {
            k_seg_sort_long<<<sm_count(current_device()) * 2, 256, 0, st>>>(starts, sums, perm, long_list,
                                                                              long_count, static_cast<int>(cap));
            launched("segment scatter-add long sort");
        }
    }
    if (rc == MTC_OK) {
        k_seg_walk<<<grid_for(T * 16 / kWalkTargets), 256, 0, st>>>(r, starts, sums, perm);  // 16 lanes a group
        launched("segment scatter-add sum");
    }
    scratch_free(scratch, st);
    return rc;
}

// Strided copy of src into dst (same shape, same dtype).
int copy_impl(const mtc_desc &src, const mtc_desc &dst, cudaStream_t stream) {
    IterSpace s;
    s.rank = src.rank;
    s.nops = 2;
    for (int d = 0; d < src.rank; ++d) {
        s.shape[d] = src.shape[d];
        s.stride[0][d] = dst.strides[d];
        s.stride[1][d] = src.strides[d];
    }
    s.offset[0] = dst.offset;
    s.offset[1] = src.offset;
    simplify(s);
    if (s.numel == 0) return MTC_OK;
    const int es = static_cast<int>(dtype_size(src.dtype));
    if (s.rank == 1 && s.stride[0][0] == 1 && s.stride[1][0] == 1) {
        MTC_CUDA_TRY(cudaMemcpyAsync(static_cast<char *>(dst.data) + s.offset[0] * es,
                                     static_cast<const char *>(src.data) + s.offset[1] * es,
                                     static_cast<size_t>(s.numel) * es, cudaMemcpyDeviceToDevice, stream));
        return MTC_OK;
    }
    if (s.numel >= (int64_t{1} << 32)) return fail(MTC_ERR_UNSUPPORTED, "strided copy of 2^32 or more elements");
    MoveArgs a;
    std::memset(&a, 0, sizeof(a));
    fill_divs(a, s);
    a.ptr[0] = static_cast<char *>(dst.data);
    a.ptr[1] = static_cast<char *>(const_cast<void *>(src.data));
    const int r = s.rank;
    // contiguous rows, 16-byte multiples: vector row copy
    if (r == 2 && s.stride[0][1] == 1 && s.stride[1][1] == 1 && (s.shape[1] * es) % 16 == 0 &&
        (s.stride[0][0] * es) % 16 == 0 && (s.stride[1][0] * es) % 16 == 0 && aligned16(dst.data, s.offset[0], es) &&
        aligned16(src.data, s.offset[1], es)) {
        const long long row_vec = s.shape[1] * es / 16;
        k_copy_rows16<<<grid_for(s.shape[0] * row_vec), 256, 0, stream>>>(a, row_vec);
        return check_launch("row copy");
    }
    if (r >= 2 && s.stride[0][r - 1] == 1 && s.stride[1][r - 2] == 1 && s.stride[1][r - 1] != 1) {
        int64_t batch = 1;
        for (int d = 0; d < r - 2; ++d) batch *= s.shape[d];
        const int64_t ty = (s.shape[r - 2] + 63) / 64;
        if (batch <= 65535 && ty <= 65535) {
            dim3 grid(static_cast<unsigned>((s.shape[r - 1] + 63) / 64), static_cast<unsigned>(ty),
                      static_cast<unsigned>(batch));
            if (es == 4) k_copy_tiled<uint32_t><<<grid, 256, 0, stream>>>(a);
            else k_copy_tiled<unsigned long long><<<grid, 256, 0, stream>>>(a);
            return check_launch("tiled copy");
        }
    }
    if (es == 4) k_copy_strided<uint32_t><<<grid_for(s.numel), 256, 0, stream>>>(a);
    else k_copy_strided<unsigned long long><<<grid_for(s.numel), 256, 0, stream>>>(a);
    return check_launch("strided copy");
}

int fill_impl(const mtc_desc &out, const void *value, cudaStream_t stream) {
    const int es = static_cast<int>(dtype_size(out.dtype));
    IterSpace s;
    s.rank = out.rank;
    s.nops = 1;
    for (int d = 0; d < out.rank; ++d) {
        s.shape[d] = out.shape[d];
        s.stride[0][d] = out.strides[d];
    }
    s.offset[0] = out.offset;
    simplify(s);
    if (s.numel == 0) return MTC_OK;
    uint64_t bits = 0;
    std::memcpy(&bits, value, es);
    char *base = static_cast<char *>(out.data);
    if (s.rank == 1 && (s.stride[0][0] == 1 || s.numel == 1)) {
        if (bits == 0) {
            MTC_CUDA_TRY(cudaMemsetAsync(base + s.offset[0] * es, 0, static_cast<size_t>(s.numel) * es, stream));
            return MTC_OK;
        }
        if (es == 4)
            k_fill_flat<uint32_t><<<grid_for(s.numel), 256, 0, stream>>>(
                reinterpret_cast<uint32_t *>(base) + s.offset[0], s.numel, static_cast<uint32_t>(bits));
        else
            k_fill_flat<unsigned long long><<<grid_for(s.numel), 256, 0, stream>>>(
                reinterpret_cast<unsigned long long *>(base) + s.offset[0], s.numel, static_cast<unsigned long long>(bits));
        return check_launch("fill");
    }
    if (s.numel >= (int64_t{1} << 32)) return fail(MTC_ERR_UNSUPPORTED, "strided fill of 2^32 or more elements");
    MoveArgs a;
    std::memset(&a, 0, sizeof(a));
    fill_divs(a, s);
    a.ptr[0] = base;
    if (es == 4) k_fill_strided<uint32_t><<<grid_for(s.numel), 256, 0, stream>>>(a, static_cast<uint32_t>(bits));
    else k_fill_strided<unsigned long long><<<grid_for(s.numel), 256, 0, stream>>>(a, static_cast<unsigned long long>(bits));
    return check_launch("strided fill");
}

bool same_shape(const mtc_desc &x, const mtc_desc &y) {
    if (x.rank != y.rank) return false;
    for (int d = 0; d < x.rank; ++d)
        if (x.shape[d] != y.shape[d]) return false;
    return true;
}

// Shared set-up of gather (role 0 = out, 1 = src, 2 = idx) and scatter-add
// (role 0 = target, 1 = updates, 2 = idx): the indexed tensor's axis stride is
// zeroed and supplied separately, the walk runs over idx.shape.
int index_space(const mtc_desc &indexed, const mtc_desc &walked, const mtc_desc &idx, int64_t axis, bool indexed_is_out,
                MoveArgs &a, IterSpace &s) {
    const int rank = idx.rank;
    s.rank = rank;
    s.nops = 3;
    for (int d = 0; d < rank; ++d) {
        s.shape[d] = idx.shape[d];
        const int64_t st = (d == axis) ? 0 : indexed.strides[d];
        s.stride[indexed_is_out ? 0 : 1][d] = st;
        s.stride[indexed_is_out ? 1 : 0][d] = walked.strides[d];
        s.stride[2][d] = idx.strides[d];
    }
    s.offset[indexed_is_out ? 0 : 1] = indexed.offset;
    s.offset[indexed_is_out ? 1 : 0] = walked.offset;
    s.offset[2] = idx.offset;
    // Keep the innermost axis separate from the coalescing so the row kernels can
    // recognise it: simplification still merges the outer axes.
    simplify(s);
    if (s.numel >= (int64_t{1} << 32)) return fail(MTC_ERR_UNSUPPORTED, "index space of 2^32 or more elements");
    std::memset(&a, 0, sizeof(a));
    fill_divs(a, s);
    a.axis_extent = indexed.shape[axis];
    a.axis_stride = indexed.strides[axis];
    return MTC_OK;
}

// out = 0 first when `clear`, then out[..idx..] += upd.
int scatter_add_impl(const mtc_desc *upd, const mtc_desc *idx, int64_t axis, const mtc_desc *out, bool clear,
                     cudaStream_t st) {
    MTC_TRY(validate(upd, "updates"));
    MTC_TRY(validate(idx, "indices"));
    MTC_TRY(validate(out, "output"));
    if (idx->dtype != MTC_INT64) return fail(MTC_ERR_INVALID_ARGUMENT, "scatter indices must be Int64");
    if (upd->dtype != MTC_FLOAT32 || out->dtype != MTC_FLOAT32)
        return fail(MTC_ERR_LOGIC, "scatter-add requires Float32");
    if (upd->rank != idx->rank || upd->rank != out->rank || !same_shape(*upd, *idx))
        return fail(MTC_ERR_INVALID_ARGUMENT, "scatter-add shapes are inconsistent");
    if (axis < 0 || axis >= out->rank) return fail(MTC_ERR_OUT_OF_RANGE, "scatter-add axis out of range");
    RowArgs ra;
    if (row_operands(*out, *upd, *idx, *out, axis, ra)) {
        if (!clear) {  // add into the values already there: 128-bit reductions into L2
            if (ra.rows == 0) return MTC_OK;
            k_scatter_rows2<<<grid_for(ra.rows * 4), 256, 0, st>>>(ra);
            return check_launch("row scatter-add into");
        }
        const int rc = segment_scatter_add(ra, st);
        if (rc != MTC_ERR_UNSUPPORTED) return rc;
        clear_error();
    }
    if (clear) {
        const float zero = 0.0f;
        MTC_TRY(fill_impl(*out, &zero, st));
    }
    MoveArgs a;
    IterSpace s;
    MTC_TRY(index_space(*out, *upd, *idx, axis, true, a, s));
    if (s.numel == 0) return MTC_OK;
    a.ptr[0] = static_cast<char *>(out->data);
    a.ptr[1] = static_cast<char *>(const_cast<void *>(upd->data));
    a.ptr[2] = static_cast<char *>(const_cast<void *>(idx->data));
    const int r = s.rank;
    if (r >= 2 && s.stride[0][r - 1] == 1 && s.stride[1][r - 1] == 1 && s.stride[2][r - 1] == 0 &&
        (s.shape[r - 1] * 4) % 16 == 0 && (a.axis_stride * 4) % 16 == 0) {
        bool ok = aligned16(out->data, 0, 4) && aligned16(upd->data, 0, 4);
        for (int d = 0; d < r - 1 && ok; ++d) ok = (s.stride[0][d] * 4) % 16 == 0 && (s.stride[1][d] * 4) % 16 == 0;
        ok = ok && (s.offset[0] * 4) % 16 == 0 && (s.offset[1] * 4) % 16 == 0;
        if (ok) {
            const long long rows = s.numel / s.shape[r - 1];
            const long long row_vec = s.shape[r - 1] / 4;
            k_scatter_add_rows16<<<grid_for(rows * row_vec), 256, 0, st>>>(a, rows, row_vec);
            return check_launch("row scatter-add");
        }
    }
    k_scatter_add<<<grid_for(s.numel), 256, 0, st>>>(a);
    return check_launch("scatter-add");
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" {

int mtc_copy(const mtc_desc *src, const mtc_desc *dst, void *stream) {
    clear_error();
    MTC_TRY(validate(src, "source"));
    MTC_TRY(validate(dst, "destination"));
    if (src->dtype != dst->dtype) return fail(MTC_ERR_INVALID_ARGUMENT, "copy between different dtypes");
    if (!same_shape(*src, *dst)) return fail(MTC_ERR_INVALID_ARGUMENT, "copy between different shapes");
    return copy_impl(*src, *dst, static_cast<cudaStream_t>(stream));
}

int mtc_concat(const mtc_desc *inputs, int32_t n_inputs, int64_t axis, const mtc_desc *out, void *stream) {
    clear_error();
    MTC_TRY(validate(out, "output"));
    if (n_inputs < 1 || inputs == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "concatenate needs inputs");
    if (axis < 0 || axis >= out->rank) return fail(MTC_ERR_OUT_OF_RANGE, "concatenate axis out of range");
    int64_t start = 0;
    for (int i = 0; i < n_inputs; ++i) {
        MTC_TRY(validate(&inputs[i], "input"));
        const mtc_desc &in = inputs[i];
        if (in.dtype != out->dtype || in.rank != out->rank)
            return fail(MTC_ERR_INVALID_ARGUMENT, "concatenate input %d does not match the output", i);
        for (int d = 0; d < out->rank; ++d)
            if (d != axis && in.shape[d] != out->shape[d])
                return fail(MTC_ERR_INVALID_ARGUMENT, "concatenate input %d has a mismatched extent", i);
        start += in.shape[axis];
    }
    if (start != out->shape[axis]) return fail(MTC_ERR_INVALID_ARGUMENT, "concatenate extents do not sum to the output");
    start = 0;
    for (int i = 0; i < n_inputs; ++i) {
        const mtc_desc &in = inputs[i];
        mtc_desc section = *out;
        for (int d = 0; d < out->rank; ++d) section.shape[d] = in.shape[d];
        section.offset = out->offset + start * out->strides[axis];
        start += in.shape[axis];
        int64_t n = 1;
        for (int d = 0; d < in.rank; ++d) n *= in.shape[d];
        if (n == 0) continue;
        MTC_TRY(copy_impl(in, section, static_cast<cudaStream_t>(stream)));
    }
    return MTC_OK;
}

int mtc_index_scatter(const mtc_desc *in, const mtc_desc *dst_view, const mtc_desc *out, void *stream) {
    clear_error();
    MTC_TRY(validate(in, "input"));
    MTC_TRY(validate(dst_view, "destination view"));
    MTC_TRY(validate(out, "output"));
    if (dst_view->data != out->data) return fail(MTC_ERR_INVALID_ARGUMENT, "scatter view must alias the output buffer");
    if (!same_shape(*in, *dst_view)) return fail(MTC_ERR_INVALID_ARGUMENT, "scatter view shape differs from input");
    if (in->dtype != out->dtype) return fail(MTC_ERR_INVALID_ARGUMENT, "scatter dtype mismatch");
    const uint64_t zero = 0;
    MTC_TRY(fill_impl(*out, &zero, static_cast<cudaStream_t>(stream)));
    return copy_impl(*in, *dst_view, static_cast<cudaStream_t>(stream));
}

int mtc_fill(const mtc_desc *out, const void *value, void *stream) {
    clear_error();
    MTC_TRY(validate(out, "output"));
    if (value == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null fill value");
    return fill_impl(*out, value, static_cast<cudaStream_t>(stream));
}

int mtc_gather(const mtc_desc *src, const mtc_desc *idx, int64_t axis, const mtc_desc *out, void *stream) {
    clear_error();
    MTC_TRY(validate(src, "source"));
    MTC_TRY(validate(idx, "indices"));
    MTC_TRY(validate(out, "output"));
    if (idx->dtype != MTC_INT64) return fail(MTC_ERR_INVALID_ARGUMENT, "gather indices must be Int64");
    if (src->dtype != out->dtype) return fail(MTC_ERR_INVALID_ARGUMENT, "gather dtype mismatch");
    if (src->rank != idx->rank || !same_shape(*idx, *out))
        return fail(MTC_ERR_INVALID_ARGUMENT, "gather shapes are inconsistent");
    if (axis < 0 || axis >= src->rank) return fail(MTC_ERR_OUT_OF_RANGE, "gather axis out of range");
    for (int d = 0; d < src->rank; ++d)
        if (d != axis && idx->shape[d] != src->shape[d])
            return fail(MTC_ERR_INVALID_ARGUMENT, "gather index extent differs from source off the axis");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    RowArgs rows;
    if (src->dtype == MTC_FLOAT32 && row_operands(*out, *src, *idx, *src, axis, rows)) return row_gather(rows, st);
    MoveArgs a;
    IterSpace s;
    MTC_TRY(index_space(*src, *out, *idx, axis, false, a, s));
    if (s.numel == 0) return MTC_OK;
    a.ptr[0] = static_cast<char *>(out->data);
    a.ptr[1] = static_cast<char *>(const_cast<void *>(src->data));
    a.ptr[2] = static_cast<char *>(const_cast<void *>(idx->data));
    const int r = s.rank;
    const int es = static_cast<int>(dtype_size(src->dtype));
    if (r >= 2 && es == 4 && s.stride[0][r - 1] == 1 && s.stride[1][r - 1] == 1 && s.stride[2][r - 1] == 0 &&
        (s.shape[r - 1] * 4) % 16 == 0 && (a.axis_stride * 4) % 16 == 0) {
        bool ok = aligned16(out->data, 0, 4) && aligned16(src->data, 0, 4);
        for (int d = 0; d < r - 1 && ok; ++d) ok = (s.stride[0][d] * 4) % 16 == 0 && (s.stride[1][d] * 4) % 16 == 0;
        ok = ok && (s.offset[0] * 4) % 16 == 0 && (s.offset[1] * 4) % 16 == 0;
        if (ok) {
            const long long rows = s.numel / s.shape[r - 1];
            const long long row_vec = s.shape[r - 1] / 4;
            k_gather_rows16<<<grid_for(rows * row_vec), 256, 0, st>>>(a, rows, row_vec);
            return check_launch("row gather");
        }
    }
    if (es == 4) k_gather<uint32_t><<<grid_for(s.numel), 256, 0, st>>>(a);
    else k_gather<unsigned long long><<<grid_for(s.numel), 256, 0, st>>>(a);
    return check_launch("gather");
}

int mtc_gather_scatter_add(const mtc_desc *upd, const mtc_desc *idx, int64_t axis, const mtc_desc *out, void *stream) {
    clear_error();
    return scatter_add_impl(upd, idx, axis, out, true, static_cast<cudaStream_t>(stream));
}

int mtc_gather_scatter_add_into(const mtc_desc *upd, const mtc_desc *idx, int64_t axis, const mtc_desc *out,
                                void *stream) {
    clear_error();
    return scatter_add_impl(upd, idx, axis, out, false, static_cast<cudaStream_t>(stream));
}

int mtc_check_device_errors(int device, void *stream, int64_t *detail) {
    clear_error();
    int prev = 0;
    MTC_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != device) MTC_CUDA_TRY(cudaSetDevice(device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned long long word[2] = {0, 0};
    int rc = MTC_OK;
    if (cudaMemcpyFromSymbolAsync(word, g_device_error, sizeof(word), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        rc = fail(MTC_ERR_RUNTIME, "reading the device error word failed: %s", cudaGetErrorString(cudaGetLastError()));
    } else {
        if (detail) *detail = static_cast<int64_t>(word[1]);
        if (word[0] != 0) {
            const unsigned long long zero[2] = {0, 0};
            cudaMemcpyToSymbolAsync(g_device_error, zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
            cudaStreamSynchronize(s);
            if (word[0] == MTC_ERR_OUT_OF_RANGE)
                rc = fail(MTC_ERR_OUT_OF_RANGE, "an index kernel met index %lld outside its axis",
                          static_cast<long long>(word[1]));
            else
                rc = fail(static_cast<int>(word[0]), "a device kernel gave up waiting (error %llu)", word[0]);
        }
    }
    if (prev != device) cudaSetDevice(prev);
    return rc;
}

// Asynchronous form: a snapshot of the error word is copied to pinned host
// memory on `stream` behind the work queued so far, and an event marks its
// arrival.  mtc_poll_device_errors reads the latest snapshot once its event has
// completed (or waits for it), so a caller can check for index errors without
// synchronising every evaluation.
namespace {
struct ErrorSnapshot {
    unsigned long long *host = nullptr;  // pinned [2]
    cudaEvent_t ready = nullptr;
    bool pending = false;
};
std::mutex g_snap_mutex;
ErrorSnapshot g_snaps[64];
}  // namespace

int mtc_watch_device_errors(int device, void *stream) {
    clear_error();
    if (device < 0 || device >= 64) return fail(MTC_ERR_INVALID_ARGUMENT, "device index %d out of range", device);
    int prev = 0;
    MTC_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != device) MTC_CUDA_TRY(cudaSetDevice(device));
    std::lock_guard<std::mutex> lock(g_snap_mutex);
    ErrorSnapshot &sn = g_snaps[device];
    int rc = MTC_OK;
    if (sn.host == nullptr) {
        if (cudaHostAlloc(reinterpret_cast<void **>(&sn.host), 2 * sizeof(unsigned long long), cudaHostAllocDefault) !=
                cudaSuccess ||
            cudaEventCreateWithFlags(&sn.ready, cudaEventDisableTiming) != cudaSuccess) {
            rc = fail(MTC_ERR_RUNTIME, "error-word snapshot set-up failed: %s", cudaGetErrorString(cudaGetLastError()));
        }
    }
    if (rc == MTC_OK) {
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (cudaMemcpyFromSymbolAsync(sn.host, g_device_error, 2 * sizeof(unsigned long long), 0,
                                      cudaMemcpyDeviceToHost, s) != cudaSuccess ||
            cudaEventRecord(sn.ready, s) != cudaSuccess) {
            rc = fail(MTC_ERR_RUNTIME, "error-word snapshot failed: %s", cudaGetErrorString(cudaGetLastError()));
        } else {
            sn.pending = true;
        }
    }
    if (prev != device) cudaSetDevice(prev);
    return rc;
}

int mtc_poll_device_errors(int device, int wait, int64_t *detail) {
    clear_error();
    if (device < 0 || device >= 64) return fail(MTC_ERR_INVALID_ARGUMENT, "device index %d out of range", device);
    unsigned long long word[2] = {0, 0};
    {
        std::lock_guard<std::mutex> lock(g_snap_mutex);
        ErrorSnapshot &sn = g_snaps[device];
        if (!sn.pending) return MTC_OK;
        const cudaError_t q = wait ? cudaEventSynchronize(sn.ready) : cudaEventQuery(sn.ready);
        if (q == cudaErrorNotReady) {
            cudaGetLastError();
            return MTC_OK;  // not known yet
        }
        if (q != cudaSuccess) return fail(MTC_ERR_RUNTIME, "error-word snapshot: %s", cudaGetErrorString(q));
        word[0] = sn.host[0];
        word[1] = sn.host[1];
        sn.pending = false;
    }
    if (word[0] == 0) return MTC_OK;
    // an error was recorded: clear the word (synchronously; this is the error path)
    int prev = 0;
    MTC_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != device) MTC_CUDA_TRY(cudaSetDevice(device));
    MTC_CUDA_TRY(cudaDeviceSynchronize());
    const unsigned long long zero[2] = {0, 0};
    MTC_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, zero, sizeof(zero)));
    if (prev != device) cudaSetDevice(prev);
    if (detail) *detail = static_cast<int64_t>(word[1]);
    if (word[0] == MTC_ERR_OUT_OF_RANGE)
        return fail(MTC_ERR_OUT_OF_RANGE, "an index kernel met index %lld outside its axis",
                    static_cast<long long>(word[1]));
    return fail(static_cast<int>(word[0]), "a device kernel gave up waiting (error %llu)", word[0]);
}

}  // extern "C"
