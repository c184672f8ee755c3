// Axis reductions: Sum (0x0301), LogSumExp (0x0302), Max, ArgMax, and the
// single-pass log-softmax.  Reference: reduce_values / reduce_logsumexp
// (src/tensor/backend/cpu/kernels/reduction/loops.hpp:21-136) over ReductionPlan
// (src/tensor/backend/cpu/iteration/reduction.cpp:14-121).
//
// Two kernel shapes:
//  - row kernel: the reduced elements of one output form one run (stride +-1
//    after folding), e.g. sum over the last axis; a warp (short rows) or a CTA
//    (long rows) reduces a row with 128-bit loads, shuffle and shared-memory trees.
//  - per-output kernel: one thread per output and reduction chunk; consecutive
//    threads own consecutive outputs, so reducing a strided axis (sum over axis
//    0 of a row-major matrix) reads full 128-byte lines.  Long reductions are cut
//    into chunks whose partial states are merged in order by a second kernel.
// The CPU accumulates sequentially in float; the GPU order is a fixed tree, so
// results agree to rounding (parity tolerance 1e-5 * sqrt(K) relative).
#include <cfloat>
#include <cmath>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"

namespace mtc {
namespace {

constexpr long long kEmpty = 0x7fffffffffffffffLL;

// Accumulator state shared by every reduction op.
struct State {
    float a;      // sum / running max
    float b;      // logsumexp: running sum of exp(x - a)
    long long i;  // argmax: index of the best element, kEmpty when none
    int flags;    // logsumexp: bit0 = NaN seen, bit1 = +inf seen
    int pad;
};

template <int OP>
struct Reducer;

template <>
struct Reducer<MTC_OP_SUM> {
    __device__ static State init() { return State{0.0f, 0.0f, kEmpty, 0, 0}; }
    __device__ static void add(State &s, float x, long long) { s.a += x; }
    __device__ static void merge(State &s, const State &o) { s.a += o.a; }
    __device__ static float result(const State &s) { return s.a; }
};

// Maximum that returns NaN when either operand is NaN (one instruction).
__device__ __forceinline__ float max_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

template <>
struct Reducer<MTC_OP_MAX> {
    // NaN propagates; an empty reduction gives -inf.
    __device__ static State init() { return State{-INFINITY, 0.0f, kEmpty, 0, 0}; }
    __device__ static void add(State &s, float x, long long) { s.a = max_nan(s.a, x); }
    __device__ static void merge(State &s, const State &o) { add(s, o.a, 0); }
    __device__ static float result(const State &s) { return s.a; }
};

template <>
struct Reducer<MTC_OP_ARGMAX> {
    // First index of the maximum; a NaN counts as the maximum (first NaN wins).
    __device__ static State init() { return State{-INFINITY, 0.0f, kEmpty, 0, 0}; }
    __device__ static void add(State &s, float x, long long idx) {
        if (s.i == kEmpty || (s.a == s.a && (x != x || x > s.a))) {
            s.a = x;
            s.i = idx;
        }
    }
    __device__ static void merge(State &s, const State &o) {
        if (o.i == kEmpty) return;
        if (s.i == kEmpty) {
            s = o;
            return;
        }
        const bool sn = s.a != s.a, on = o.a != o.a;
        bool take;
        if (sn || on) take = (sn && on) ? (o.i < s.i) : on;
        else take = (o.a > s.a) || (o.a == s.a && o.i < s.i);
        if (take) s = o;
    }
    __device__ static long long result(const State &s) { return s.i == kEmpty ? 0 : s.i; }
    // The update of a thread that walks its elements in increasing index order
    // from a state seeded with (-inf, first index): x replaces the best when it
    // is larger or NaN, unless the best is already NaN (the first NaN wins).
    __device__ static void add_seeded(State &s, float x, long long idx) {
        if (!(x <= s.a) && s.a == s.a) {
            s.a = x;
            s.i = idx;
        }
    }
};

template <>
struct Reducer<MTC_OP_LOGSUMEXP> {
    // Online (max, sum) form of the two-pass CPU loop; NaN -> NaN, a +inf element
    // or an all -inf / empty input returns the maximum (loops.hpp:59-136).
    __device__ static State init() { return State{-INFINITY, 0.0f, kEmpty, 0, 0}; }
    __device__ static void add(State &s, float x, long long) {
        if (x != x) {
            s.flags |= 1;
        } else if (x == INFINITY) {
            s.flags |= 2;
        } else if (x == -INFINITY) {
        } else if (x > s.a) {
            s.b = s.b * expf(s.a - x) + 1.0f;
            s.a = x;
        } else {
            s.b += expf(x - s.a);
        }
    }
    __device__ static void merge(State &s, const State &o) {
        s.flags |= o.flags;
        if (o.a == -INFINITY) return;
        if (s.a == -INFINITY) {
            s.a = o.a;
            s.b = o.b;
            return;
        }
        if (o.a > s.a) {
            s.b = s.b * expf(s.a - o.a) + o.b;
            s.a = o.a;
        } else {
            s.b += o.b * expf(o.a - s.a);
        }
    }
    __device__ static float result(const State &s) {
        if (s.flags & 1) return NAN;
        if (s.flags & 2) return INFINITY;
        if (s.a == -INFINITY) return -INFINITY;
        return s.a + logf(s.b);
    }
};

// Element update for a thread that visits its elements in increasing index
// order and has at least one: ARGMAX uses the seeded form (state seeded with
// the first index), every other op its ordinary add.
template <int OP>
__device__ __forceinline__ State seeded_init(long long first) {
    State s = Reducer<OP>::init();
    if constexpr (OP == MTC_OP_ARGMAX) s.i = first;
    return s;
}

template <int OP>
__device__ __forceinline__ void add_in_order(State &s, float x, long long idx) {
    if constexpr (OP == MTC_OP_ARGMAX) Reducer<OP>::add_seeded(s, x, idx);
    else Reducer<OP>::add(s, x, idx);
}

__device__ __forceinline__ State shfl_down(const State &s, int delta) {
    State o;
    o.a = __shfl_down_sync(0xffffffffu, s.a, delta);
    o.b = __shfl_down_sync(0xffffffffu, s.b, delta);
    o.i = __shfl_down_sync(0xffffffffu, s.i, delta);
    o.flags = __shfl_down_sync(0xffffffffu, s.flags, delta);
    o.pad = 0;
    return o;
}

template <int OP>
__device__ __forceinline__ State warp_reduce(State s) {
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) {
        const State o = shfl_down(s, d);
        Reducer<OP>::merge(s, o);
    }
    return s;
}

struct RedArgs {
    const float *in;
    long long in_off;
    void *out;
    long long out_off;
    long long nout;
    long long R;
    int krank;
    unsigned int kshape[MTC_MAX_RANK];
    FastDiv kdiv[MTC_MAX_RANK];
    long long kstr[MTC_MAX_RANK];
    int rrank;
    unsigned int rshape[MTC_MAX_RANK];
    long long rstr[MTC_MAX_RANK];
    long long rrun_stride;  // row kernel: stride of the single reduced run
    int vec4;               // row kernel: 128-bit loads allowed
    int chunks;             // per-output kernel: reduction chunks per output
    State *partial;         // chunks > 1: partial states [nout][chunks]
    float *out_f;           // log-softmax output
    long long out_row_stride;
};

__device__ __forceinline__ long long kept_offset(const RedArgs &a, unsigned int o) {
    long long off = a.in_off;
    unsigned int rem = o;
#pragma unroll
    for (int d = MTC_MAX_RANK - 1; d >= 1; --d) {
        if (d < a.krank) {
            const unsigned int q = fastdiv(rem, a.kdiv[d]);
            off += static_cast<long long>(rem - q * a.kshape[d]) * a.kstr[d];
            rem = q;
        }
    }
    if (a.krank > 0) off += static_cast<long long>(rem) * a.kstr[0];
    return off;
}

template <int OP>
__device__ __forceinline__ void store_result(const RedArgs &a, long long o, const State &s) {
    if constexpr (OP == MTC_OP_ARGMAX) {
        static_cast<long long *>(a.out)[a.out_off + o] = Reducer<OP>::result(s);
    } else {
        static_cast<float *>(a.out)[a.out_off + o] = Reducer<OP>::result(s);
    }
}

// Accumulates the run [base, base + R*stride) handled by `lane` of `lanes`.
template <int OP>
__device__ __forceinline__ State accumulate_row(const RedArgs &a, long long base, int lane, int lanes) {
    State s = Reducer<OP>::init();
    const long long R = a.R;
    if (a.vec4) {
        const float4 *p = reinterpret_cast<const float4 *>(a.in + base);
        const long long nv = R / 4;
        long long v = lane;
        if (v < nv) s = seeded_init<OP>(4 * v);
        // eight independent 128-bit loads in flight per thread, consumed in index order
        for (; v + 7LL * lanes < nv; v += 8LL * lanes) {
            float4 q[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) q[u] = __ldg(p + v + u * lanes);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const long long e = 4 * (v + u * lanes);
                add_in_order<OP>(s, q[u].x, e);
                add_in_order<OP>(s, q[u].y, e + 1);
                add_in_order<OP>(s, q[u].z, e + 2);
                add_in_order<OP>(s, q[u].w, e + 3);
            }
        }
        for (; v < nv; v += lanes) {
            const float4 q = __ldg(p + v);
            add_in_order<OP>(s, q.x, 4 * v);
            add_in_order<OP>(s, q.y, 4 * v + 1);
            add_in_order<OP>(s, q.z, 4 * v + 2);
            add_in_order<OP>(s, q.w, 4 * v + 3);
        }
    } else {
        const long long st = a.rrun_stride;
        for (long long j = lane; j < R; j += lanes) Reducer<OP>::add(s, __ldg(a.in + base + j * st), j);
    }
    return s;
}

template <int OP>
__device__ __forceinline__ State block_reduce(State s, State *shared) {
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    s = warp_reduce<OP>(s);
    if (lane == 0) shared[warp] = s;
    __syncthreads();
    if (warp == 0) {
        s = lane < static_cast<int>(blockDim.x / 32) ? shared[lane] : Reducer<OP>::init();
        s = warp_reduce<OP>(s);
        if (lane == 0) shared[0] = s;
    }
    __syncthreads();
    s = shared[0];
    __syncthreads();
    return s;
}

// One warp per row (short rows).
template <int OP>
__global__ void __launch_bounds__(256) k_row_warp(const RedArgs a) {
    const int lane = threadIdx.x % 32;
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x / 32);
    for (long long o = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32; o < a.nout; o += warps) {
        const long long base = kept_offset(a, static_cast<unsigned int>(o));
        State s = accumulate_row<OP>(a, base, lane, 32);
        s = warp_reduce<OP>(s);
        if (lane == 0) store_result<OP>(a, o, s);
    }
}

// One CTA per row (long rows).
template <int OP>
__global__ void __launch_bounds__(512) k_row_block(const RedArgs a) {
    __shared__ State shared[32];
    for (long long o = blockIdx.x; o < a.nout; o += gridDim.x) {
        const long long base = kept_offset(a, static_cast<unsigned int>(o));
        State s = accumulate_row<OP>(a, base, threadIdx.x, blockDim.x);
        s = block_reduce<OP>(s, shared);
        if (threadIdx.x == 0) store_result<OP>(a, o, s);
    }
}

// One thread per (output, chunk); reduced coordinates walked with an odometer.
template <int OP>
__global__ void __launch_bounds__(256) k_per_output(const RedArgs a) {
    const long long total = a.nout * a.chunks;
    for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long c = t / a.nout;  // chunk-major: neighbouring threads share a chunk
        const long long o = t - c * a.nout;
        const long long per = (a.R + a.chunks - 1) / a.chunks;
        const long long r0 = c * per;
        const long long r1 = r0 + per < a.R ? r0 + per : a.R;
        State s = Reducer<OP>::init();
        if (r0 < r1) {
            const long long base = kept_offset(a, static_cast<unsigned int>(o));
            unsigned int coord[MTC_MAX_RANK];
            long long off = base;
            long long rem = r0;
            for (int d = a.rrank - 1; d >= 0; --d) {
                coord[d] = static_cast<unsigned int>(rem % a.rshape[d]);
                rem /= a.rshape[d];
                off += static_cast<long long>(coord[d]) * a.rstr[d];
            }
            const int inner = a.rrank - 1;
            long long r = r0;
            if (a.rrank == 1) {
                // single reduced axis: eight independent loads in flight, consumed in order
                const long long st = a.rstr[0];
                const float *q = a.in + off;
                for (; r + 8 <= r1; r += 8, q += 8 * st) {
                    float v[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) v[u] = __ldg(q + u * st);
#pragma unroll
                    for (int u = 0; u < 8; ++u) Reducer<OP>::add(s, v[u], r + u);
                }
                off = q - a.in;
                coord[0] = static_cast<unsigned int>(r);
            }
            for (; r < r1; ++r) {
                Reducer<OP>::add(s, __ldg(a.in + off), r);
                // advance the odometer
                if (++coord[inner] < a.rshape[inner]) {
                    off += a.rstr[inner];
                } else {
                    off -= static_cast<long long>(a.rshape[inner] - 1) * a.rstr[inner];
                    coord[inner] = 0;
                    for (int d = inner - 1; d >= 0; --d) {
                        if (++coord[d] < a.rshape[d]) {
                            off += a.rstr[d];
                            break;
                        }
                        off -= static_cast<long long>(a.rshape[d] - 1) * a.rstr[d];
                        coord[d] = 0;
                    }
                }
            }
        }
        if (a.chunks == 1) store_result<OP>(a, o, s);
        else a.partial[o * a.chunks + c] = s;
    }
}

// Column reduction: the innermost kept axis is contiguous and one strided axis
// is reduced (sum over axis 0 of a row-major matrix, or over the middle axis of
// [B, R, C]).  A CTA owns 128 consecutive outputs - one float4 per lane, so a
// warp load is one 512-byte row segment - of one batch index (blockIdx.z) and a
// chunk of the reduced axis (blockIdx.y).  Its 8 warps take interleaved rows
// with ROWS vector loads in flight per thread, then merge in warp order through
// shared memory (a fixed order: results are deterministic).  The grid is one
// wave of resident CTAs: the row chunks are sized so that every SM holds its
// full complement for the whole kernel.
constexpr int kColWarps = 8;
#ifndef MTC_COL_ROWS_IN_FLIGHT
#define MTC_COL_ROWS_IN_FLIGHT 8
#endif
constexpr int kColRows = MTC_COL_ROWS_IN_FLIGHT;  // rows (vector loads) in flight per thread
#ifndef MTC_COL_ARGMAX_VEC
#define MTC_COL_ARGMAX_VEC 2
#endif

template <int OP, int VEC, int ROWS = kColRows>
__global__ void __launch_bounds__(256) k_col_tile(const RedArgs a, long long ncols, long long batch_stride,
                                                  unsigned int *arrivals) {
    constexpr int CW = 32 * VEC;  // outputs per CTA
    __shared__ State part[kColWarps][CW];
    const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    const long long col = static_cast<long long>(blockIdx.x) * CW + lane * VEC;
    const long long per = (a.R + a.chunks - 1) / a.chunks;
    const long long r0 = static_cast<long long>(blockIdx.y) * per;
    const long long r1 = r0 + per < a.R ? r0 + per : a.R;
    State s[VEC];
    const long long first = r0 + warp;
#pragma unroll
    for (int j = 0; j < VEC; ++j) s[j] = first < r1 ? seeded_init<OP>(first) : Reducer<OP>::init();
    auto load = [&](const float *p, float (&q)[VEC]) {
        if constexpr (VEC == 4) {
            const float4 t = __ldg(reinterpret_cast<const float4 *>(p));
            q[0] = t.x;
            q[1] = t.y;
            q[2] = t.z;
            q[3] = t.w;
        } else if constexpr (VEC == 2) {
            const float2 t = __ldg(reinterpret_cast<const float2 *>(p));
            q[0] = t.x;
            q[1] = t.y;
        } else {
            q[0] = __ldg(p);
        }
    };
    if (col < ncols) {
        const long long rs = a.rstr[0];
        const float *base = a.in + a.in_off + static_cast<long long>(blockIdx.z) * batch_stride + col;
        long long r = first;
        // ROWS rows (vector loads) in flight per thread
        for (; r + (ROWS - 1) * kColWarps < r1; r += ROWS * kColWarps) {
            float q[ROWS][VEC];
#pragma unroll
            for (int u = 0; u < ROWS; ++u) load(base + (r + u * kColWarps) * rs, q[u]);
#pragma unroll
            for (int u = 0; u < ROWS; ++u) {
                const long long e = r + u * kColWarps;
#pragma unroll
                for (int j = 0; j < VEC; ++j) add_in_order<OP>(s[j], q[u][j], e);
            }
        }
        for (; r < r1; r += kColWarps) {
            float q[VEC];
            load(base + r * rs, q);
#pragma unroll
            for (int j = 0; j < VEC; ++j) add_in_order<OP>(s[j], q[j], r);
        }
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) part[warp][lane * VEC + j] = s[j];
    __syncthreads();
    const long long c = static_cast<long long>(blockIdx.x) * CW + threadIdx.x;
    const long long o = static_cast<long long>(blockIdx.z) * ncols + c;
    if (threadIdx.x < CW) {
        State t = part[0][threadIdx.x];
#pragma unroll
        for (int w = 1; w < kColWarps; ++w) Reducer<OP>::merge(t, part[w][threadIdx.x]);
        if (c < ncols) {
            if (a.chunks == 1) store_result<OP>(a, o, t);
            else a.partial[static_cast<long long>(blockIdx.y) * a.nout + o] = t;  // chunk-major
        }
    }
    if (a.chunks == 1) return;
    // the last CTA of this column group to finish merges the chunk partials in
    // chunk order and re-arms the group's arrival counter for the next launch
    __shared__ unsigned int last;
    __threadfence();
    __syncthreads();
    const unsigned int group = blockIdx.z * gridDim.x + blockIdx.x;
    if (threadIdx.x == 0) last = atomicAdd(&arrivals[group], 1u) == static_cast<unsigned int>(a.chunks) - 1u;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (threadIdx.x < CW && c < ncols) {
        // one coalesced row of partials per chunk; four chunks' loads in flight
        auto load = [&](int k) {
            const State *q = a.partial + static_cast<long long>(k) * a.nout + o;
            State r;
            r.a = __ldcg(&q->a);
            r.b = __ldcg(&q->b);
            r.i = __ldcg(&q->i);
            r.flags = __ldcg(&q->flags);
            r.pad = 0;
            return r;
        };
        State t = load(0);
        int k = 1;
        for (; k + 3 < a.chunks; k += 4) {
            const State q0 = load(k), q1 = load(k + 1), q2 = load(k + 2), q3 = load(k + 3);
            Reducer<OP>::merge(t, q0);
            Reducer<OP>::merge(t, q1);
            Reducer<OP>::merge(t, q2);
            Reducer<OP>::merge(t, q3);
        }
        for (; k < a.chunks; ++k) Reducer<OP>::merge(t, load(k));
        store_result<OP>(a, o, t);
    }
    if (threadIdx.x == 0) arrivals[group] = 0u;
}

// Resident CTAs per SM of one column-kernel instance (queried once).
template <int OP, int VEC, int ROWS>
int col_tile_occupancy() {
    static const int occ = [] {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_col_tile<OP, VEC, ROWS>, 256, 0) != cudaSuccess || n < 1) {
            cudaGetLastError();
            n = 1;
        }
        return n;
    }();
    return occ;
}

// Arrival counters of the column kernel, one array per (device, stream): zeroed
// once on the stream that uses them, then re-armed by the kernel itself.
constexpr unsigned int kColGroups = 1u << 16;
std::mutex g_arrivals_mutex;
std::vector<std::pair<std::pair<int, cudaStream_t>, unsigned int *>> g_arrivals;

int col_arrivals(cudaStream_t stream, unsigned int **out) {
    int dev = 0;
    MTC_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(g_arrivals_mutex);
    for (auto &e : g_arrivals)
        if (e.first.first == dev && e.first.second == stream) {
            *out = e.second;
            return MTC_OK;
        }
    void *p = nullptr;
    MTC_CUDA_TRY(cudaMalloc(&p, kColGroups * sizeof(unsigned int)));
    MTC_CUDA_TRY(cudaMemsetAsync(p, 0, kColGroups * sizeof(unsigned int), stream));
    g_arrivals.push_back({{dev, stream}, static_cast<unsigned int *>(p)});
    *out = static_cast<unsigned int *>(p);
    return MTC_OK;
}

// Visits the reduced elements of one output in the reference's order (reduced
// axes row-major, ReductionPlan, iteration/reduction.cpp:14-121).
template <class F>
__device__ __forceinline__ void walk_reduced(const RedArgs &a, long long base, F &&f) {
    if (a.rrank == 1) {
        // one reduced axis: sixteen loads in flight, consumed strictly in order
        const long long st = a.rstr[0];
        const float *p = a.in + base;
        long long r = 0;
        for (; r + 16 <= a.R; r += 16, p += 16 * st) {
            float v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = __ldg(p + u * st);
#pragma unroll
            for (int u = 0; u < 16; ++u) f(v[u], r + u);
        }
        for (; r < a.R; ++r, p += st) f(__ldg(p), r);
        return;
    }
    unsigned int coord[MTC_MAX_RANK];
    for (int d = 0; d < a.rrank; ++d) coord[d] = 0;
    long long off = base;
    const int inner = a.rrank - 1;
    for (long long r = 0; r < a.R; ++r) {
        f(__ldg(a.in + off), r);
        if (++coord[inner] < a.rshape[inner]) {
            off += a.rstr[inner];
        } else {
            off -= static_cast<long long>(a.rshape[inner] - 1) * a.rstr[inner];
            coord[inner] = 0;
            for (int d = inner - 1; d >= 0; --d) {
                if (++coord[d] < a.rshape[d]) {
                    off += a.rstr[d];
                    break;
                }
                off -= static_cast<long long>(a.rshape[d] - 1) * a.rstr[d];
                coord[d] = 0;
            }
        }
    }
}

// Small reductions in the reference's exact arithmetic: one thread per output,
// sequential float accumulation for sum (reduction/loops.hpp:21-57) and the
// two-pass max / sum-of-exp form for logsumexp (loops.hpp:59-136).  Sums are
// bit-identical to the CPU; logsumexp differs only by the libm ulps of exp/log.
template <int OP>
__global__ void __launch_bounds__(128) k_exact_small(const RedArgs a) {
    for (long long o = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; o < a.nout;
         o += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long base = kept_offset(a, static_cast<unsigned int>(o));
        if constexpr (OP == MTC_OP_LOGSUMEXP) {
            float mx = -INFINITY;
            bool nan = false;
            walk_reduced(a, base, [&](float x, long long) {
                if (x != x) nan = true;
                else mx = (mx < x) ? x : mx;  // std::max(mx, x)
            });
            float result;
            if (nan) {
                result = NAN;
            } else if (isinf(mx)) {
                result = mx;
            } else {
                float s = 0.0f;
                walk_reduced(a, base, [&](float x, long long) { s = __fadd_rn(s, expf(__fsub_rn(x, mx))); });
                result = __fadd_rn(mx, logf(s));
            }
            static_cast<float *>(a.out)[a.out_off + o] = result;
        } else {
            State s = Reducer<OP>::init();
            walk_reduced(a, base, [&](float x, long long r) { Reducer<OP>::add(s, x, r); });
            store_result<OP>(a, o, s);
        }
    }
}

// Offset of the reduced element with walk index r from its output's base (the
// reduced axes row-major, the order walk_reduced visits them in).
__device__ __forceinline__ long long reduced_offset(const RedArgs &a, long long r) {
    long long off = 0;
    for (int d = a.rrank - 1; d >= 0; --d) {
        const long long c = r % a.rshape[d];
        r /= a.rshape[d];
        off += c * a.rstr[d];
    }
    return off;
}

constexpr int kStagedFloats = 12288;  // 48 KB of shared memory per CTA

// Small reductions whose outputs each read many elements (bias gradients,
// means): a CTA stages the inputs of up to G consecutive outputs in shared
// memory with all of its threads (asynchronous copies, coalesced along the
// kept axis when that is contiguous and along the reduced axis otherwise), so
// the loads are in flight together.  Then one thread per output combines its elements from shared
// memory in the reference's order, exactly as k_exact_small does from memory.
template <int OP>
__global__ void __launch_bounds__(256) k_exact_staged(const RedArgs a, int G) {
    extern __shared__ float tile[];  // tile[r * gp + g]: conflict-free for both phases
    const long long o0 = static_cast<long long>(blockIdx.x) * G;
    const int gn = static_cast<int>(a.nout - o0 < G ? a.nout - o0 : G);
    const int gp = G == 1 ? 1 : G + 1;
    const int R = static_cast<int>(a.R);  // <= 8192
    const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    const bool one_axis = a.rrank == 1;
    const long long rs = a.rstr[0];
    if (a.krank > 0 && a.kstr[a.krank - 1] == 1 && gn > 1) {
        // consecutive outputs are contiguous: lanes take outputs, warps take rows
        if (lane < gn) {
            const long long base = kept_offset(a, static_cast<unsigned int>(o0 + lane));
            for (int r = warp; r < R; r += 8) {
                const long long off = one_axis ? base + r * rs : base + reduced_offset(a, r);
                cp_async4(&tile[r * gp + lane], a.in + off);
            }
        }
    } else {
        // lanes walk the reduced elements of one output, warps take outputs
        for (int g = warp; g < gn; g += 8) {
            const long long base = kept_offset(a, static_cast<unsigned int>(o0 + g));
            for (int r = lane; r < R; r += 32) {
                const long long off = one_axis ? base + r * rs : base + reduced_offset(a, r);
                cp_async4(&tile[r * gp + g], a.in + off);
            }
        }
    }
    cp_async_wait_all();
    __syncthreads();
    const int t = threadIdx.x;
    if (t >= gn) return;
    const long long o = o0 + t;
    const float *col = tile + t;
    if constexpr (OP == MTC_OP_LOGSUMEXP) {
        float mx = -INFINITY;
        bool nan = false;
        for (int r = 0; r < R; ++r) {
            const float x = col[r * gp];
            if (x != x) nan = true;
            else mx = (mx < x) ? x : mx;  // std::max(mx, x)
        }
        float result;
        if (nan) {
            result = NAN;
        } else if (isinf(mx)) {
            result = mx;
        } else {
            float s = 0.0f;
            for (int r = 0; r < R; ++r) s = __fadd_rn(s, expf(__fsub_rn(col[r * gp], mx)));
            result = __fadd_rn(mx, logf(s));
        }
        static_cast<float *>(a.out)[a.out_off + o] = result;
    } else {
        State s = Reducer<OP>::init();
        int r = 0;
        // eight shared-memory reads ahead of the in-order updates
        for (; r + 8 <= R; r += 8) {
            float x[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) x[u] = col[(r + u) * gp];
#pragma unroll
            for (int u = 0; u < 8; ++u) Reducer<OP>::add(s, x[u], r + u);
        }
        for (; r < R; ++r) Reducer<OP>::add(s, col[r * gp], r);
        store_result<OP>(a, o, s);
    }
}

// Merges the chunk partials of every output in chunk order.
template <int OP>
__global__ void __launch_bounds__(256) k_finalize(const RedArgs a) {
    for (long long o = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; o < a.nout;
         o += static_cast<long long>(gridDim.x) * blockDim.x) {
        State s = a.partial[o * a.chunks];
        for (int c = 1; c < a.chunks; ++c) Reducer<OP>::merge(s, a.partial[o * a.chunks + c]);
        store_result<OP>(a, o, s);
    }
}

// log-softmax of contiguous rows: online (max, sum) pass, then x - lse written
// in a second pass that re-reads the row from L2.
__global__ void __launch_bounds__(512) k_log_softmax_rows(const RedArgs a) {
    __shared__ State shared[32];
    for (long long o = blockIdx.x; o < a.nout; o += gridDim.x) {
        const long long base = kept_offset(a, static_cast<unsigned int>(o));
        State s = accumulate_row<MTC_OP_LOGSUMEXP>(a, base, threadIdx.x, blockDim.x);
        s = block_reduce<MTC_OP_LOGSUMEXP>(s, shared);
        const float lse = Reducer<MTC_OP_LOGSUMEXP>::result(s);
        float *dst = a.out_f + a.out_off + o * a.out_row_stride;
        if (a.vec4) {
            const float4 *p = reinterpret_cast<const float4 *>(a.in + base);
            float4 *q = reinterpret_cast<float4 *>(dst);
            for (long long v = threadIdx.x; v < a.R / 4; v += blockDim.x) {
                float4 x = __ldg(p + v);
                x.x = __fsub_rn(x.x, lse);
                x.y = __fsub_rn(x.y, lse);
                x.z = __fsub_rn(x.z, lse);
                x.w = __fsub_rn(x.w, lse);
                q[v] = x;
            }
        } else {
            for (long long j = threadIdx.x; j < a.R; j += blockDim.x)
                dst[j] = __fsub_rn(__ldg(a.in + base + j * a.rrun_stride), lse);
        }
    }
}

// Row-resident logsumexp / log-softmax for contiguous rows of R <= 8192 floats
// (R % 4 == 0): 256 threads hold the row in registers (NV4 float4 each), take the
// NaN-ignoring maximum, then sum exp(x - max) exactly like the reference's two
// passes (reduction/loops.hpp:59-136) but reading HBM once.  With a.out_f set,
// x - lse is written from the registers (log-softmax: 8 bytes per element).
template <int NV4>
__global__ void __launch_bounds__(256) k_lse_resident(const RedArgs a) {
    __shared__ float red_f[8];
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const long long nv = a.R / 4;
    for (long long o = blockIdx.x; o < a.nout; o += gridDim.x) {
        const long long base = kept_offset(a, static_cast<unsigned int>(o));
        const float4 *p = reinterpret_cast<const float4 *>(a.in + base);
        float4 v[NV4];
#pragma unroll
        for (int i = 0; i < NV4; ++i) {
            const long long idx = threadIdx.x + 256LL * i;
            v[i] = idx < nv ? __ldg(p + idx) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        }
        // NaN-propagating maximum: NaN anywhere -> NaN, +inf -> +inf, all -inf -> -inf
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < NV4; ++i)
            mx = max_nan(max_nan(mx, v[i].x), max_nan(max_nan(v[i].y, v[i].z), v[i].w));
#pragma unroll
        for (int d = 16; d >= 1; d >>= 1) mx = max_nan(mx, __shfl_xor_sync(0xffffffffu, mx, d));
        if (lane == 0) red_f[warp] = mx;
        __syncthreads();
        mx = red_f[0];
#pragma unroll
        for (int w = 1; w < 8; ++w) mx = max_nan(mx, red_f[w]);
        __syncthreads();
        float lse;
        if (mx != mx || isinf(mx)) {
            lse = mx;  // NaN, +inf (a +inf element), or -inf (every element -inf)
        } else {
            // x - max <= 0: the hardware exponential's relative error (~2^-21) is far
            // inside the 1e-5*sqrt(K) reduction bound
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < NV4; ++i) {
                s += __expf(__fsub_rn(v[i].x, mx));
                s += __expf(__fsub_rn(v[i].y, mx));
                s += __expf(__fsub_rn(v[i].z, mx));
                s += __expf(__fsub_rn(v[i].w, mx));
            }
#pragma unroll
            for (int d = 16; d >= 1; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
            if (lane == 0) red_f[warp] = s;
            __syncthreads();
            s = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; ++w) s += red_f[w];
            __syncthreads();
            lse = __fadd_rn(mx, logf(s));
        }
        if (a.out_f != nullptr) {
            float4 *q = reinterpret_cast<float4 *>(a.out_f + a.out_off + o * a.out_row_stride);
#pragma unroll
            for (int i = 0; i < NV4; ++i) {
                const long long idx = threadIdx.x + 256LL * i;
                if (idx < nv)
                    q[idx] = make_float4(__fsub_rn(v[i].x, lse), __fsub_rn(v[i].y, lse), __fsub_rn(v[i].z, lse),
                                         __fsub_rn(v[i].w, lse));
            }
        } else if (threadIdx.x == 0) {
            static_cast<float *>(a.out)[a.out_off + o] = lse;
        }
    }
}

int launch_lse_resident(RedArgs &a, cudaStream_t stream, int sms) {
    const long long nv = a.R / 4;
    long long blocks = a.nout;
    if (blocks > static_cast<long long>(sms) * 8) blocks = static_cast<long long>(sms) * 8;
    const dim3 grid(static_cast<unsigned>(blocks < 1 ? 1 : blocks));
    if (nv <= 256) k_lse_resident<1><<<grid, 256, 0, stream>>>(a);
    else if (nv <= 512) k_lse_resident<2><<<grid, 256, 0, stream>>>(a);
    else if (nv <= 1024) k_lse_resident<4><<<grid, 256, 0, stream>>>(a);
    else k_lse_resident<8><<<grid, 256, 0, stream>>>(a);
    return check_launch("row-resident logsumexp");
}

struct RedPlan {
    RedArgs args;
    bool row = false;
    bool empty_out = false;
};

int plan_reduction(const mtc_desc *in, const int64_t *axes, int n_axes, RedPlan &plan) {
    RedArgs &a = plan.args;
    std::memset(&a, 0, sizeof(a));
    bool reduced[MTC_MAX_RANK] = {};
    for (int i = 0; i < n_axes; ++i) {
        if (axes[i] < 0 || axes[i] >= in->rank) return fail(MTC_ERR_OUT_OF_RANGE, "reduction axis out of range");
        if (reduced[axes[i]]) return fail(MTC_ERR_INVALID_ARGUMENT, "reduction axes contain a duplicate");
        reduced[axes[i]] = true;
    }
    // kept and reduced axes, extent-1 axes dropped, then folded where strides chain
    long long nout = 1, R = 1;
    int kr = 0, rr = 0;
    int64_t kshape[MTC_MAX_RANK], kstr[MTC_MAX_RANK], rshape[MTC_MAX_RANK], rstr[MTC_MAX_RANK];
    for (int d = 0; d < in->rank; ++d) {
        const int64_t e = in->shape[d];
        if (reduced[d]) R *= e; else nout *= e;
        if (e == 1) continue;
        if (reduced[d]) {
            if (rr > 0 && rstr[rr - 1] == in->strides[d] * e) {
                rshape[rr - 1] *= e;
                rstr[rr - 1] = in->strides[d];
            } else {
                rshape[rr] = e;
                rstr[rr] = in->strides[d];
                ++rr;
            }
        } else {
            if (kr > 0 && kstr[kr - 1] == in->strides[d] * e) {
                kshape[kr - 1] *= e;
                kstr[kr - 1] = in->strides[d];
            } else {
                kshape[kr] = e;
                kstr[kr] = in->strides[d];
                ++kr;
            }
        }
    }
    a.nout = nout;
    a.R = R;
    a.in = static_cast<const float *>(in->data);
    a.in_off = in->offset;
    plan.empty_out = (nout == 0);
    if (nout >= (1ll << 32)) return fail(MTC_ERR_UNSUPPORTED, "reduction with 2^32 or more outputs");
    a.krank = kr;
    for (int d = 0; d < kr; ++d) {
        a.kshape[d] = static_cast<unsigned int>(kshape[d]);
        a.kdiv[d] = make_fastdiv(static_cast<uint32_t>(kshape[d]));
        a.kstr[d] = kstr[d];
    }
    a.rrank = rr;
    for (int d = 0; d < rr; ++d) {
        if (rshape[d] >= (1ll << 32)) return fail(MTC_ERR_UNSUPPORTED, "reduced extent of 2^32 or more");
        a.rshape[d] = static_cast<unsigned int>(rshape[d]);
        a.rstr[d] = rstr[d];
    }
    plan.row = (rr == 1 && (rstr[0] == 1 || rstr[0] == -1) && R >= 32);
    if (a.rrank == 0) {
        // every reduced axis has extent 1 (or there is none): a one-element walk
        a.rrank = 1;
        a.rshape[0] = 1;
        a.rstr[0] = 0;
    }
    if (plan.row) {
        a.rrun_stride = rstr[0];
        bool vec = rstr[0] == 1 && R % 4 == 0 && (reinterpret_cast<uintptr_t>(a.in + a.in_off) % 16) == 0;
        for (int d = 0; d < kr && vec; ++d) vec = (kstr[d] % 4) == 0;
        a.vec4 = vec ? 1 : 0;
    }
    return MTC_OK;
}

template <int OP>
int run_reduction(RedPlan &p, cudaStream_t stream) {
    RedArgs &a = p.args;
    if (p.empty_out) return MTC_OK;
    const int sms = sm_count(current_device());
    if (a.R <= 8192 && a.nout * a.R <= (1LL << 21)) {
        // small: the reference's own order and rounding
        if (a.R >= 32) {
            // long walks: stage up to 32 outputs' elements per CTA in shared memory
            const int G = a.R * 2 <= kStagedFloats ? static_cast<int>(std::min<long long>(32, kStagedFloats / a.R - 1)) : 1;
            const int gp = G == 1 ? 1 : G + 1;
            const long long blocks = (a.nout + G - 1) / G;
            const size_t smem = static_cast<size_t>(a.R) * gp * sizeof(float);
            k_exact_staged<OP><<<static_cast<unsigned>(blocks), 256, smem, stream>>>(a, G);
            return check_launch("staged exact reduction");
        }
        long long blocks = (a.nout + 127) / 128;
        if (blocks > static_cast<long long>(sms) * 16) blocks = static_cast<long long>(sms) * 16;
        k_exact_small<OP><<<static_cast<unsigned>(blocks < 1 ? 1 : blocks), 128, 0, stream>>>(a);
        return check_launch("exact reduction");
    }
    if (p.row && OP == MTC_OP_LOGSUMEXP && a.vec4 && a.R <= 8192) {
        // whole row held in registers: max, then sum of exp(x - max), one read of HBM
        a.out_f = nullptr;
        return launch_lse_resident(a, stream, sms);
    }
    if (p.row) {
        if (a.R <= 2048 || a.nout >= 4LL * sms) {
            long long blocks = (a.nout + 7) / 8;
            if (blocks > static_cast<long long>(sms) * 8) blocks = static_cast<long long>(sms) * 8;
            k_row_warp<OP><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
        } else {
            long long blocks = a.nout;
            if (blocks > static_cast<long long>(sms) * 4) blocks = static_cast<long long>(sms) * 4;
            k_row_block<OP><<<static_cast<unsigned>(blocks), 512, 0, stream>>>(a);
        }
        return check_launch("row reduction");
    }
    // column kernel: contiguous innermost kept axis, one reduced axis, float4 aligned
    if (a.rrank == 1 && (a.krank == 1 || a.krank == 2) && a.kstr[a.krank - 1] == 1) {
        const long long ncols = a.kshape[a.krank - 1];
        const long long nbatch = a.krank == 2 ? a.kshape[0] : 1;
        const long long bstride = a.krank == 2 ? a.kstr[0] : 0;
        const bool v4 = ncols % 4 == 0 && a.rstr[0] % 4 == 0 && bstride % 4 == 0 &&
                        (reinterpret_cast<uintptr_t>(a.in + a.in_off) % 16) == 0;
        // argmax: 2 outputs per lane (fewer registers per thread, twice the CTAs);
        // sum: 16 rows in flight at no register cost (5.8 -> 5.9 TB/s)
        constexpr int vec = OP == MTC_OP_ARGMAX ? MTC_COL_ARGMAX_VEC : 4;
        constexpr int rows = OP == MTC_OP_SUM ? 16 : kColRows;
        if (v4 && nbatch <= 65535 && ((ncols + 32 * vec - 1) / (32 * vec)) * nbatch <= kColGroups) {
            const long long gx = (ncols + 32 * vec - 1) / (32 * vec);
            // exactly one wave of resident CTAs: a partial second wave of these
            // streaming CTAs leaves most of the machine idle (measured: 1.44
            // waves ran argmax at 4.7 TB/s, one wave at 5.7 TB/s)
            const long long want = static_cast<long long>(sms) * col_tile_occupancy<OP, vec, rows>();
            long long chunks = want / (gx * nbatch);
            const long long max_chunks = (a.R + 63) / 64;  // at least 64 rows per chunk
            if (chunks > max_chunks) chunks = max_chunks;
            if (chunks > 65535) chunks = 65535;
            if (chunks < 1) chunks = 1;
            a.chunks = static_cast<int>(chunks);
            void *scratch = nullptr;
            if (chunks > 1) {
                MTC_TRY(scratch_alloc(static_cast<size_t>(a.nout * chunks) * sizeof(State), stream, &scratch));
                a.partial = static_cast<State *>(scratch);
            }
            unsigned int *arrivals = nullptr;
            if (chunks > 1) MTC_TRY(col_arrivals(stream, &arrivals));
            const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(chunks), static_cast<unsigned>(nbatch));
            k_col_tile<OP, vec, rows><<<grid, 256, 0, stream>>>(a, ncols, bstride, arrivals);
            const int rc = check_launch("column reduction");
            scratch_free(scratch, stream);
            return rc;
        }
    }
    // per-output kernel: split the reduction so the grid fills the machine
    const long long target = static_cast<long long>(sms) * 2048;
    long long chunks = 1;
    if (a.nout < target && a.R > 64) {
        chunks = (target + a.nout - 1) / a.nout;
        const long long max_chunks = (a.R + 63) / 64;
        if (chunks > max_chunks) chunks = max_chunks;
        if (chunks > 4096) chunks = 4096;
    }
    a.chunks = static_cast<int>(chunks);
    void *scratch = nullptr;
    if (chunks > 1) {
        MTC_TRY(scratch_alloc(static_cast<size_t>(a.nout * chunks) * sizeof(State), stream, &scratch));
        a.partial = static_cast<State *>(scratch);
    }
    long long blocks = (a.nout * a.chunks + 255) / 256;
    if (blocks > static_cast<long long>(sms) * 8) blocks = static_cast<long long>(sms) * 8;
    if (blocks < 1) blocks = 1;
    k_per_output<OP><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
    int rc = check_launch("reduction");
    if (rc == MTC_OK && a.chunks > 1) {
        long long fb = (a.nout + 255) / 256;
        if (fb > static_cast<long long>(sms) * 8) fb = static_cast<long long>(sms) * 8;
        k_finalize<OP><<<static_cast<unsigned>(fb), 256, 0, stream>>>(a);
        rc = check_launch("reduction finalize");
    }
    scratch_free(scratch, stream);
    return rc;
}

bool contiguous(const mtc_desc &d) {
    int64_t expect = 1;
    for (int i = d.rank - 1; i >= 0; --i) {
        if (d.shape[i] != 1 && d.strides[i] != expect) return false;
        expect *= d.shape[i];
    }
    return true;
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" int mtc_reduce(int32_t op, const mtc_desc *in, const int64_t *axes, int32_t n_axes, const mtc_desc *out,
                          void *stream) {
    clear_error();
    MTC_TRY(validate(in, "input"));
    MTC_TRY(validate(out, "output"));
    if (in->dtype != MTC_FLOAT32) return fail(MTC_ERR_LOGIC, "reductions require a Float32 input");
    const int want = op == MTC_OP_ARGMAX ? MTC_INT64 : MTC_FLOAT32;
    if (out->dtype != want) return fail(MTC_ERR_INVALID_ARGUMENT, "reduction output has the wrong dtype");
    if (n_axes < 0 || n_axes > in->rank || (n_axes > 0 && axes == nullptr))
        return fail(MTC_ERR_INVALID_ARGUMENT, "bad reduction axes");
    if (!contiguous(*out)) return fail(MTC_ERR_INVALID_ARGUMENT, "reduction output must be contiguous");
    RedPlan p;
    MTC_TRY(plan_reduction(in, axes, n_axes, p));
    if (numel_of(*out) != p.args.nout) return fail(MTC_ERR_INVALID_ARGUMENT, "reduction output size mismatch");
    if (op == MTC_OP_ARGMAX && n_axes != 1) return fail(MTC_ERR_INVALID_ARGUMENT, "argmax reduces exactly one axis");
    if (op == MTC_OP_ARGMAX && p.args.R == 0 && p.args.nout > 0)
        return fail(MTC_ERR_INVALID_ARGUMENT, "argmax of an empty axis");
    p.args.out = out->data;
    p.args.out_off = out->offset;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (op) {
    case MTC_OP_SUM: return run_reduction<MTC_OP_SUM>(p, s);
    case MTC_OP_LOGSUMEXP: return run_reduction<MTC_OP_LOGSUMEXP>(p, s);
    case MTC_OP_MAX: return run_reduction<MTC_OP_MAX>(p, s);
    case MTC_OP_ARGMAX: return run_reduction<MTC_OP_ARGMAX>(p, s);
    default: return fail(MTC_ERR_INVALID_ARGUMENT, "unknown reduction op 0x%04x", op);
    }
}

extern "C" int mtc_log_softmax(const mtc_desc *in, int64_t axis, const mtc_desc *out, void *stream) {
    clear_error();
    MTC_TRY(validate(in, "input"));
    MTC_TRY(validate(out, "output"));
    if (in->dtype != MTC_FLOAT32 || out->dtype != MTC_FLOAT32) return fail(MTC_ERR_LOGIC, "log-softmax requires Float32");
    if (axis < 0 || axis >= in->rank) return fail(MTC_ERR_OUT_OF_RANGE, "log-softmax axis out of range");
    if (in->rank != out->rank) return fail(MTC_ERR_INVALID_ARGUMENT, "log-softmax shape mismatch");
    for (int d = 0; d < in->rank; ++d)
        if (in->shape[d] != out->shape[d]) return fail(MTC_ERR_INVALID_ARGUMENT, "log-softmax shape mismatch");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool last = (axis == in->rank - 1);
    if (last && contiguous(*out) && in->shape[axis] >= 32) {
        RedPlan p;
        MTC_TRY(plan_reduction(in, &axis, 1, p));
        if (p.empty_out) return MTC_OK;
        if (p.row) {
            RedArgs &a = p.args;
            a.out_f = static_cast<float *>(out->data);
            a.out_off = out->offset;
            a.out_row_stride = in->shape[axis];
            if (a.vec4) a.vec4 = ((reinterpret_cast<uintptr_t>(a.out_f + a.out_off) % 16) == 0) ? 1 : 0;
            const int sms = sm_count(current_device());
            if (a.vec4 && a.R <= 8192) return launch_lse_resident(a, s, sms);
            long long blocks = a.nout;
            if (blocks > static_cast<long long>(sms) * 4) blocks = static_cast<long long>(sms) * 4;
            k_log_softmax_rows<<<static_cast<unsigned>(blocks), 512, 0, s>>>(a);
            return check_launch("log-softmax");
        }
    }
    // general layout: logsumexp into scratch (kept dimension of extent 1), then subtract
    mtc_desc lse = *in;
    int64_t n = 1;
    for (int d = in->rank - 1; d >= 0; --d) {
        lse.shape[d] = (d == axis) ? 1 : in->shape[d];
        lse.strides[d] = n;
        n *= lse.shape[d];
    }
    lse.offset = 0;
    lse.capacity = n;
    void *buf = nullptr;
    MTC_TRY(scratch_alloc(static_cast<size_t>(n > 0 ? n : 1) * 4, s, &buf));
    lse.data = buf;
    int rc = mtc_reduce(MTC_OP_LOGSUMEXP, in, &axis, 1, &lse, stream);
    if (rc == MTC_OK) rc = mtc_binary(MTC_OP_SUBTRACT, in, &lse, out, stream);
    scratch_free(buf, s);
    return rc;
}
