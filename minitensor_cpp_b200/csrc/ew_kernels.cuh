// Elementwise kernel templates of libmtcuda.
//
// This header is compiled twice: by nvcc into the precompiled single-op kernels
// (elementwise.cu), and, embedded as text, by NVRTC into the kernels generated
// for fused elementwise programs (fused.cu).  It therefore uses only builtin
// types and CUDA device intrinsics (no host or standard-library headers).
//
// Op semantics follow the reference CPU kernels
// (src/tensor/backend/cpu/kernels/elementwise/kernels.cpp:58-167).  Every
// arithmetic step uses an explicitly rounded intrinsic (__fadd_rn, __fmul_rn,
// ...) so the compiler cannot contract a multiply and an add of two different
// graph nodes into one FMA: a fused chain then rounds exactly like the chain of
// materialised single ops the CPU evaluates.
#ifndef MTC_EW_KERNELS_CUH
#define MTC_EW_KERNELS_CUH

#define MTC_EW_MAX_RANK 8
#define MTC_EW_MAX_IN 12
#define MTC_EW_MAX_OUT 4
#define MTC_EW_TILE 64
#define MTC_EW_TILE_THREADS 256
#define MTC_EW_MAX_IMM 48

// ------------------------------------------------------------------- ops --

template <int OP>
__device__ __forceinline__ float mtc_unary(float x);

template <> __device__ __forceinline__ float mtc_unary<0x0101>(float x) { return fabsf(x); }
template <> __device__ __forceinline__ float mtc_unary<0x0102>(float x) {
    // sign keeps +-0 and NaN (kernels.cpp:96-107)
    return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : x);
}
template <> __device__ __forceinline__ float mtc_unary<0x0103>(float x) { return -x; }
template <> __device__ __forceinline__ float mtc_unary<0x0104>(float x) { return expf(x); }
template <> __device__ __forceinline__ float mtc_unary<0x0105>(float x) { return logf(x); }
template <> __device__ __forceinline__ float mtc_unary<0x0106>(float x) { return __fsqrt_rn(x); }
// tanh in double, rounded once: (nearly always) the correctly rounded float, so
// the result stays within the host libm's own error of the CPU reference (the
// float tanhf of either library alone can sit 3 ulp from the other's)
template <> __device__ __forceinline__ float mtc_unary<0x0107>(float x) {
    return __double2float_rn(tanh(static_cast<double>(x)));
}
template <> __device__ __forceinline__ float mtc_unary<0x0108>(float x) {
    // branch form of the CPU sigmoid (kernels.cpp:113-124)
    if (x >= 0.0f) {
        const float e = expf(-x);
        return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    }
    const float e = expf(x);
    return __fdiv_rn(e, __fadd_rn(1.0f, e));
}
template <> __device__ __forceinline__ float mtc_unary<0x0180>(float x) {
    // relu: max(x, 0) for every input; NaN propagates, -0 and -inf give +0
    return x > 0.0f ? x : (x != x ? x : 0.0f);
}

template <int OP>
__device__ __forceinline__ float mtc_binary(float a, float b);

template <> __device__ __forceinline__ float mtc_binary<0x0110>(float a, float b) { return __fadd_rn(a, b); }
template <> __device__ __forceinline__ float mtc_binary<0x0111>(float a, float b) { return __fsub_rn(a, b); }
template <> __device__ __forceinline__ float mtc_binary<0x0112>(float a, float b) { return __fmul_rn(a, b); }
template <> __device__ __forceinline__ float mtc_binary<0x0113>(float a, float b) { return __fdiv_rn(a, b); }
template <> __device__ __forceinline__ float mtc_binary<0x0114>(float a, float b) {
    // logaddexp with the CPU's NaN and infinity rules (kernels.cpp:150-167)
    if (a != a || b != b) return __fadd_rn(a, b);
    const float m = (a < b) ? b : a;  // std::max(a, b)
    if (isinf(m)) return m;
    return __fadd_rn(m, log1pf(expf(-fabsf(__fsub_rn(a, b)))));
}

template <int OP>
struct MtcUnaryOp {
    static constexpr int kIn = 1;
    static constexpr int kOut = 1;
    __device__ __forceinline__ void operator()(const float *x, float *y, const float *) const { y[0] = mtc_unary<OP>(x[0]); }
};

template <int OP>
struct MtcBinaryOp {
    static constexpr int kIn = 2;
    static constexpr int kOut = 1;
    __device__ __forceinline__ void operator()(const float *x, float *y, const float *) const { y[0] = mtc_binary<OP>(x[0], x[1]); }
};

// ------------------------------------------------------------ arguments --

struct MtcFastDiv {
    unsigned int d;
    unsigned int mul;
    unsigned int shift;
};

// Division by an invariant divisor (Granlund & Montgomery 1994, round-up variant).
__device__ __forceinline__ unsigned int mtc_fastdiv(unsigned int n, const MtcFastDiv &f) {
    if (f.d <= 1u) return n;
    const unsigned int t = __umulhi(n, f.mul);
    return (t + ((n - t) >> 1)) >> (f.shift - 1u);
}

// One launch's operands over a common (simplified) logical shape.
struct MtcEwArgs {
    long long numel;
    int rank;
    unsigned int shape[MTC_EW_MAX_RANK];
    MtcFastDiv div[MTC_EW_MAX_RANK];
    const float *in[MTC_EW_MAX_IN];
    long long in_off[MTC_EW_MAX_IN];
    long long in_str[MTC_EW_MAX_IN][MTC_EW_MAX_RANK];
    float *out[MTC_EW_MAX_OUT];
    long long out_off[MTC_EW_MAX_OUT];
    long long out_str[MTC_EW_MAX_OUT][MTC_EW_MAX_RANK];
    unsigned int transposed;  // tiled kernel: bit k set when input k is read through shared memory
    unsigned int batch_rank;  // tiled kernel: number of leading (batch) axes
    float imm[MTC_EW_MAX_IMM]; // fused programs: constants, passed by value so one compiled program serves all
};

// ------------------------------------------------------------ flat kernel --
// Every operand is contiguous (stride 1) or a broadcast scalar (stride 0) over
// a single axis.  VEC = 4 uses 128-bit loads/stores (all pointers 16-byte aligned).

template <class Op, int VEC>
__global__ void __launch_bounds__(256) mtc_ew_flat(const MtcEwArgs a) {
    constexpr int NIN = Op::kIn;
    constexpr int NOUT = Op::kOut;
    const Op op;
    const long long nvec = a.numel / VEC;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    auto load = [&](long long v, float (&x)[VEC][NIN > 0 ? NIN : 1]) {
#pragma unroll
        for (int k = 0; k < NIN; ++k) {
            if (a.in_str[k][0] == 0) {
                const float s = __ldg(a.in[k] + a.in_off[k]);
#pragma unroll
                for (int l = 0; l < VEC; ++l) x[l][k] = s;
            } else if (VEC == 4) {
                const float4 q = __ldg(reinterpret_cast<const float4 *>(a.in[k] + a.in_off[k]) + v);
                x[0][k] = q.x;
                x[1][k] = q.y;
                x[2][k] = q.z;
                x[3][k] = q.w;
            } else {
#pragma unroll
                for (int l = 0; l < VEC; ++l) x[l][k] = __ldg(a.in[k] + a.in_off[k] + v * VEC + l);
            }
        }
    };
    auto compute_store = [&](long long v, float (&x)[VEC][NIN > 0 ? NIN : 1]) {
        float y[VEC][NOUT];
#pragma unroll
        for (int l = 0; l < VEC; ++l) op(x[l], y[l], a.imm);
#pragma unroll
        for (int j = 0; j < NOUT; ++j) {
            if (VEC == 4) {
                float4 q;
                q.x = y[0][j];
                q.y = y[1][j];
                q.z = y[2][j];
                q.w = y[3][j];
                reinterpret_cast<float4 *>(a.out[j] + a.out_off[j])[v] = q;
            } else {
#pragma unroll
                for (int l = 0; l < VEC; ++l) a.out[j][a.out_off[j] + v * VEC + l] = y[l][j];
            }
        }
    };
    // two grid-stride units per iteration: both units' loads are in flight together
    for (long long v = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += 2 * stride) {
        float x0[VEC][NIN > 0 ? NIN : 1];
        float x1[VEC][NIN > 0 ? NIN : 1];
        const long long v1 = v + stride;
        load(v, x0);
        if (v1 < nvec) load(v1, x1);
        compute_store(v, x0);
        if (v1 < nvec) compute_store(v1, x1);
    }
    // scalar tail (numel not a multiple of VEC)
    const long long tail = nvec * VEC;
    const long long t = tail + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (VEC > 1 && t < a.numel) {
        float x[NIN > 0 ? NIN : 1];
        float y[NOUT];
#pragma unroll
        for (int k = 0; k < NIN; ++k) x[k] = __ldg(a.in[k] + a.in_off[k] + (a.in_str[k][0] == 0 ? 0 : t));
        op(x, y, a.imm);
#pragma unroll
        for (int j = 0; j < NOUT; ++j) a.out[j][a.out_off[j] + t] = y[j];
    }
}

// --------------------------------------------------------- strided kernel --
// Any strides (zero, negative, transposed); the linear index is decomposed into
// coordinates with precomputed divisors.  numel < 2^32.

template <class Op>
__global__ void __launch_bounds__(256) mtc_ew_strided(const MtcEwArgs a) {
    constexpr int NIN = Op::kIn;
    constexpr int NOUT = Op::kOut;
    const Op op;
    const unsigned int n = static_cast<unsigned int>(a.numel);
    const unsigned int stride = gridDim.x * blockDim.x;
    for (unsigned int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        long long io[NIN > 0 ? NIN : 1];
        long long oo[NOUT];
#pragma unroll
        for (int k = 0; k < NIN; ++k) io[k] = a.in_off[k];
#pragma unroll
        for (int j = 0; j < NOUT; ++j) oo[j] = a.out_off[j];
        unsigned int rem = i;
#pragma unroll
        for (int d = MTC_EW_MAX_RANK - 1; d >= 1; --d) {
            if (d < a.rank) {
                const unsigned int q = mtc_fastdiv(rem, a.div[d]);
                const long long c = static_cast<long long>(rem - q * a.shape[d]);
                rem = q;
#pragma unroll
                for (int k = 0; k < NIN; ++k) io[k] += c * a.in_str[k][d];
#pragma unroll
                for (int j = 0; j < NOUT; ++j) oo[j] += c * a.out_str[j][d];
            }
        }
#pragma unroll
        for (int k = 0; k < NIN; ++k) io[k] += static_cast<long long>(rem) * a.in_str[k][0];
#pragma unroll
        for (int j = 0; j < NOUT; ++j) oo[j] += static_cast<long long>(rem) * a.out_str[j][0];
        float x[NIN > 0 ? NIN : 1];
        float y[NOUT];
#pragma unroll
        for (int k = 0; k < NIN; ++k) x[k] = __ldg(a.in[k] + io[k]);
        op(x, y, a.imm);
#pragma unroll
        for (int j = 0; j < NOUT; ++j) a.out[j][oo[j]] = y[j];
    }
}

// ------------------------------------------------------------ rows kernel --
// Spaces whose innermost axis is contiguous for every output and, for every
// input, contiguous (stride 1) or broadcast (stride 0): a bias row, a column
// vector, a scalar.  Each task is a 4*blockDim-wide strip of one row; the row's
// outer offsets are decoded once per task (not per element) and VEC = 4 moves
// 128 bits per contiguous operand (row starts 16-byte aligned, cols % 4 == 0).

template <class Op, int VEC>
__global__ void __launch_bounds__(256) mtc_ew_rows(const MtcEwArgs a) {
    constexpr int NIN = Op::kIn;
    constexpr int NOUT = Op::kOut;
    const Op op;
    const int r = a.rank;
    const long long cols = a.shape[r - 1];
    const long long strip = static_cast<long long>(blockDim.x) * VEC;
    const long long strips = (cols + strip - 1) / strip;
    const long long rows = a.numel / cols;
    for (long long task = blockIdx.x; task < rows * strips; task += gridDim.x) {
        const long long row = task / strips;
        const long long c0 = (task - row * strips) * strip + static_cast<long long>(threadIdx.x) * VEC;
        long long ib[NIN > 0 ? NIN : 1];
        long long ob[NOUT];
#pragma unroll
        for (int k = 0; k < NIN; ++k) ib[k] = a.in_off[k];
#pragma unroll
        for (int j = 0; j < NOUT; ++j) ob[j] = a.out_off[j];
        unsigned int rem = static_cast<unsigned int>(row);
#pragma unroll
        for (int d = MTC_EW_MAX_RANK - 2; d >= 0; --d) {
            if (d < r - 1) {
                const unsigned int q = (d > 0) ? mtc_fastdiv(rem, a.div[d]) : 0u;
                const long long c = static_cast<long long>(d > 0 ? rem - q * a.shape[d] : rem);
                rem = q;
#pragma unroll
                for (int k = 0; k < NIN; ++k) ib[k] += c * a.in_str[k][d];
#pragma unroll
                for (int j = 0; j < NOUT; ++j) ob[j] += c * a.out_str[j][d];
            }
        }
        if (c0 >= cols) continue;
        float x[VEC][NIN > 0 ? NIN : 1];
        float y[VEC][NOUT];
        if (VEC == 4 && c0 + 4 <= cols) {
#pragma unroll
            for (int k = 0; k < NIN; ++k) {
                if (a.in_str[k][r - 1] == 0) {
                    const float s = __ldg(a.in[k] + ib[k]);
#pragma unroll
                    for (int l = 0; l < VEC; ++l) x[l][k] = s;
                } else {
                    const float4 q = __ldg(reinterpret_cast<const float4 *>(a.in[k] + ib[k] + c0));
                    x[0][k] = q.x;
                    x[1][k] = q.y;
                    x[2][k] = q.z;
                    x[3][k] = q.w;
                }
            }
#pragma unroll
            for (int l = 0; l < VEC; ++l) op(x[l], y[l], a.imm);
#pragma unroll
            for (int j = 0; j < NOUT; ++j)
                *reinterpret_cast<float4 *>(a.out[j] + ob[j] + c0) = make_float4(y[0][j], y[1][j], y[2][j], y[3][j]);
        } else {
            for (int l = 0; l < VEC && c0 + l < cols; ++l) {
#pragma unroll
                for (int k = 0; k < NIN; ++k)
                    x[0][k] = __ldg(a.in[k] + ib[k] + (c0 + l) * a.in_str[k][r - 1]);
                op(x[0], y[0], a.imm);
#pragma unroll
                for (int j = 0; j < NOUT; ++j) a.out[j][ob[j] + c0 + l] = y[0][j];
            }
        }
    }
}

// ----------------------------------------------------------- tiled kernel --
// For spaces whose innermost output axis is contiguous while some inputs are
// contiguous along the second-innermost axis instead (a transposed view, e.g.
// B^T in A * B^T).  A 64x64 output tile is produced per CTA; every transposed
// input is first staged through shared memory with loads coalesced along its own
// contiguous axis, so both the reads and the writes are full 128-byte lines.
// grid = (ceil(cols/64), ceil(rows/64), batch).

template <class Op, int NT>
__global__ void __launch_bounds__(MTC_EW_TILE_THREADS) mtc_ew_tiled(const MtcEwArgs a) {
    constexpr int NIN = Op::kIn;
    constexpr int NOUT = Op::kOut;
    constexpr int T = MTC_EW_TILE;
    __shared__ float stage[NT > 0 ? NT : 1][T][T + 1];
    const Op op;
    const int r = a.rank;
    const unsigned int rows = a.shape[r - 2];
    const unsigned int cols = a.shape[r - 1];
    const unsigned int r0 = blockIdx.y * T;
    const unsigned int c0 = blockIdx.x * T;

    long long ib[NIN > 0 ? NIN : 1];
    long long ob[NOUT];
#pragma unroll
    for (int k = 0; k < NIN; ++k) ib[k] = a.in_off[k];
#pragma unroll
    for (int j = 0; j < NOUT; ++j) ob[j] = a.out_off[j];
    unsigned int rem = blockIdx.z;
    for (int d = static_cast<int>(a.batch_rank) - 1; d >= 0; --d) {
        const unsigned int c = rem % a.shape[d];
        rem /= a.shape[d];
#pragma unroll
        for (int k = 0; k < NIN; ++k) ib[k] += static_cast<long long>(c) * a.in_str[k][d];
#pragma unroll
        for (int j = 0; j < NOUT; ++j) ob[j] += static_cast<long long>(c) * a.out_str[j][d];
    }

    const int tx = threadIdx.x % T;
    const int ty = threadIdx.x / T;  // 0..3
    constexpr int STEPS = T * T / MTC_EW_TILE_THREADS;

    if (NT > 0) {
        int slot = 0;
#pragma unroll
        for (int k = 0; k < NIN; ++k) {
            if (a.transposed & (1u << k)) {
#pragma unroll 4
                for (int s = 0; s < STEPS; ++s) {
                    const unsigned int lr = tx;                  // along the input's contiguous axis
                    const unsigned int lc = ty + s * (T / STEPS);
                    if (r0 + lr < rows && c0 + lc < cols) {
                        stage[slot][lc][lr] = __ldg(a.in[k] + ib[k] + static_cast<long long>(r0 + lr) * a.in_str[k][r - 2] +
                                                    static_cast<long long>(c0 + lc) * a.in_str[k][r - 1]);
                    }
                }
                ++slot;
            }
        }
        __syncthreads();
    }

#pragma unroll 4
    for (int s = 0; s < STEPS; ++s) {
        const unsigned int lc = tx;
        const unsigned int lr = ty + s * (T / STEPS);
        if (r0 + lr < rows && c0 + lc < cols) {
            float x[NIN > 0 ? NIN : 1];
            float y[NOUT];
            int slot = 0;
#pragma unroll
            for (int k = 0; k < NIN; ++k) {
                if (NT > 0 && (a.transposed & (1u << k))) {
                    x[k] = stage[slot][lc][lr];
                    ++slot;
                } else {
                    x[k] = __ldg(a.in[k] + ib[k] + static_cast<long long>(r0 + lr) * a.in_str[k][r - 2] +
                                 static_cast<long long>(c0 + lc) * a.in_str[k][r - 1]);
                }
            }
            op(x, y, a.imm);
#pragma unroll
            for (int j = 0; j < NOUT; ++j)
                a.out[j][ob[j] + static_cast<long long>(r0 + lr) * a.out_str[j][r - 2] +
                         static_cast<long long>(c0 + lc) * a.out_str[j][r - 1]] = y[j];
        }
    }
}

// Tiled, 128-bit: the same tile walk with float4 traffic.  Requirements (checked
// by the planner): column count a multiple of 4; outputs and row-contiguous
// inputs 16-byte aligned along their rows; column-broadcast inputs (stride 0
// along the row) read as one scalar per row; transposed inputs 16-byte aligned
// along their contiguous axis (the tile's rows) with a row count that is a
// multiple of 4.  A transposed input is staged in shared memory in the tile's
// row-major order with the 16-byte chunks of each row XOR-swizzled by
// (row / 4) % 8: the scalar stores of the staging pass and the float4 reads of
// the compute pass are then at most 2-way bank conflicted.
// grid = (ceil(cols/64), ceil(rows/64), batch); a thread owns 4 columns of 4 rows.

template <class Op, int NT>
__global__ void __launch_bounds__(MTC_EW_TILE_THREADS) mtc_ew_tiled4(const MtcEwArgs a) {
    constexpr int NIN = Op::kIn;
    constexpr int NOUT = Op::kOut;
    constexpr int T = MTC_EW_TILE;
    __shared__ __align__(16) float stage[NT > 0 ? NT : 1][T][T];
    const Op op;
    const int r = a.rank;
    const unsigned int rows = a.shape[r - 2];
    const unsigned int cols = a.shape[r - 1];
    const unsigned int r0 = blockIdx.y * T;
    const unsigned int c0 = blockIdx.x * T;

    long long ib[NIN > 0 ? NIN : 1];
    long long ob[NOUT];
#pragma unroll
    for (int k = 0; k < NIN; ++k) ib[k] = a.in_off[k];
#pragma unroll
    for (int j = 0; j < NOUT; ++j) ob[j] = a.out_off[j];
    unsigned int rem = blockIdx.z;
    for (int d = static_cast<int>(a.batch_rank) - 1; d >= 0; --d) {
        const unsigned int c = rem % a.shape[d];
        rem /= a.shape[d];
#pragma unroll
        for (int k = 0; k < NIN; ++k) ib[k] += static_cast<long long>(c) * a.in_str[k][d];
#pragma unroll
        for (int j = 0; j < NOUT; ++j) ob[j] += static_cast<long long>(c) * a.out_str[j][d];
    }

    const int q = threadIdx.x % 16;  // 16-byte chunk of a 64-wide tile row
    const int g = threadIdx.x / 16;  // 0..15

    if (NT > 0) {
        // staging: a thread loads rows 4q..4q+3 of tile columns g, g+16, g+32, g+48
        int slot = 0;
#pragma unroll
        for (int k = 0; k < NIN; ++k) {
            if (a.transposed & (1u << k)) {
                const long long cs = a.in_str[k][r - 1];
                const float *src = a.in[k] + ib[k] + (r0 + 4u * q);
                const bool row_in = r0 + 4u * q < rows;
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const unsigned int lc = g + 16 * p;
                    if (row_in && c0 + lc < cols) {
                        const float4 v = __ldg(reinterpret_cast<const float4 *>(src + static_cast<long long>(c0 + lc) * cs));
                        float *dst = &stage[slot][4 * q][(((lc >> 2) ^ (q & 7)) << 2) | (lc & 3)];
                        dst[0] = v.x;
                        dst[T] = v.y;
                        dst[2 * T] = v.z;
                        dst[3 * T] = v.w;
                    }
                }
                ++slot;
            }
        }
        __syncthreads();
    }

    const unsigned int cc = c0 + 4u * q;
    if (cc >= cols) return;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const unsigned int lr = g + 16 * p;
        if (r0 + lr >= rows) break;
        const long long row = r0 + lr;
        float x[NIN > 0 ? NIN : 1][4];
        int slot = 0;
#pragma unroll
        for (int k = 0; k < NIN; ++k) {
            if (NT > 0 && (a.transposed & (1u << k))) {
                const float4 v = *reinterpret_cast<const float4 *>(&stage[slot][lr][(q ^ ((lr >> 2) & 7)) << 2]);
                x[k][0] = v.x;
                x[k][1] = v.y;
                x[k][2] = v.z;
                x[k][3] = v.w;
                ++slot;
            } else if (a.in_str[k][r - 1] == 0) {
                const float v = __ldg(a.in[k] + ib[k] + row * a.in_str[k][r - 2]);
                x[k][0] = x[k][1] = x[k][2] = x[k][3] = v;
            } else {
                const float4 v = __ldg(reinterpret_cast<const float4 *>(a.in[k] + ib[k] + row * a.in_str[k][r - 2] + cc));
                x[k][0] = v.x;
                x[k][1] = v.y;
                x[k][2] = v.z;
                x[k][3] = v.w;
            }
        }
        float y[NOUT][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float xi[NIN > 0 ? NIN : 1];
            float yi[NOUT];
#pragma unroll
            for (int k = 0; k < NIN; ++k) xi[k] = x[k][i];
            op(xi, yi, a.imm);
#pragma unroll
            for (int j = 0; j < NOUT; ++j) y[j][i] = yi[j];
        }
#pragma unroll
        for (int j = 0; j < NOUT; ++j)
            *reinterpret_cast<float4 *>(a.out[j] + ob[j] + row * a.out_str[j][r - 2] + cc) =
                make_float4(y[j][0], y[j][1], y[j][2], y[j][3]);
    }
}

#endif  // MTC_EW_KERNELS_CUH
