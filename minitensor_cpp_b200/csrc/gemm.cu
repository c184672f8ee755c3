// mtc_matmul: reference matmul semantics and the exact float32 SIMT GEMM.
//
// Shape and stride rules follow matmul_dispatch / MatmulPlan
// (src/tensor/backend/cpu/kernels/linalg/loops.hpp:288-324,
//  src/tensor/backend/cpu/iteration/matmul.cpp:32-82): 1-D operands become a
// row (lhs) or column (rhs) of stride 0, batch axes are right-aligned and
// broadcast with stride 0.  The SIMT kernel computes each product in float32
// and accumulates with FFMA (one rounding per step instead of the CPU's two),
// so it matches the CPU to rounding, not bit for bit.
#include <cstring>

#include <atomic>

#include "gemm.cuh"

namespace mtc {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, PAD = 4;

struct SimtArgs {
    GemmProblem p;
    int a_kmajor;  // A is contiguous along k (row-major A)
    int b_nmajor;  // B is contiguous along n (row-major B)
};

template <bool EXACT>
__global__ void __launch_bounds__(256, 2) k_gemm_simt(const SimtArgs args) {
    const GemmProblem &p = args.p;
    __shared__ __align__(16) float As[2][BK][BM + PAD];
    __shared__ __align__(16) float Bs[2][BK][BN + PAD];

    // batch offsets
    long long ao = p.a_off, bo = p.b_off, co = p.c_off;
    {
        unsigned int rem = blockIdx.z;
        for (int d = p.batch_rank - 1; d >= 0; --d) {
            const unsigned int e = static_cast<unsigned int>(p.batch_shape[d]);
            const unsigned int c = rem % e;
            rem /= e;
            ao += static_cast<long long>(c) * p.a_bs[d];
            bo += static_cast<long long>(c) * p.b_bs[d];
            co += static_cast<long long>(c) * p.c_bs[d];
        }
    }
    const long long m0 = static_cast<long long>(blockIdx.y) * BM;
    const long long n0 = static_cast<long long>(blockIdx.x) * BN;
    const int t = threadIdx.x;

    // global -> register staging of one k-tile: 4 A values and 4 B values per thread
    float ra[4], rb[4];
    auto load_tile = [&](long long k0) {
        if (args.a_kmajor) {  // row m = t/2, k = (t%2)*4 + i
            const long long m = m0 + t / 2;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const long long k = k0 + (t % 2) * 4 + i;
                ra[i] = (m < p.M && k < p.K) ? __ldg(p.A + ao + m * p.a_rs + k * p.a_cs) : 0.0f;
            }
        } else {  // k = t/32, m = (t%32)*4 + i
            const long long k = k0 + t / 32;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const long long m = m0 + (t % 32) * 4 + i;
                ra[i] = (m < p.M && k < p.K) ? __ldg(p.A + ao + m * p.a_rs + k * p.a_cs) : 0.0f;
            }
        }
        if (args.b_nmajor) {  // k = t/32, n = (t%32)*4 + i
            const long long k = k0 + t / 32;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const long long n = n0 + (t % 32) * 4 + i;
                rb[i] = (n < p.N && k < p.K) ? __ldg(p.B + bo + k * p.b_rs + n * p.b_cs) : 0.0f;
            }
        } else {  // n = t/2, k = (t%2)*4 + i
            const long long n = n0 + t / 2;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const long long k = k0 + (t % 2) * 4 + i;
                rb[i] = (n < p.N && k < p.K) ? __ldg(p.B + bo + k * p.b_rs + n * p.b_cs) : 0.0f;
            }
        }
    };
    auto store_tile = [&](int buf) {
        if (args.a_kmajor) {
#pragma unroll
            for (int i = 0; i < 4; ++i) As[buf][(t % 2) * 4 + i][t / 2] = ra[i];
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) As[buf][t / 32][(t % 32) * 4 + i] = ra[i];
        }
        if (args.b_nmajor) {
#pragma unroll
            for (int i = 0; i < 4; ++i) Bs[buf][t / 32][(t % 32) * 4 + i] = rb[i];
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) Bs[buf][(t % 2) * 4 + i][t / 2] = rb[i];
        }
    };

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    const int tx = t % 16, ty = t / 16;
    const long long ktiles = (p.K + BK - 1) / BK;
    load_tile(0);
    store_tile(0);
    __syncthreads();
    for (long long kt = 0; kt < ktiles; ++kt) {
        const int buf = static_cast<int>(kt & 1);
        if (kt + 1 < ktiles) load_tile((kt + 1) * BK);
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][k][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][k][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][k][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][k][64 + tx * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    // EXACT: the reference's rounding, a float product then a float
                    // sum per k in ascending order (linalg/loops.hpp:231-245)
                    if (EXACT) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
                    else acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
                }
        }
        if (kt + 1 < ktiles) store_tile(buf ^ 1);
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const long long m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const long long n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (n < p.N) p.C[co + m * p.c_rs + n * p.c_cs] = acc[i][j];
        }
    }
}

}  // namespace

// Small problems in the CPU's exact order: one thread per output element, the
// k loop ascending with __fmul_rn then __fadd_rn as the reference's loop, and
// sixteen (A, B) pairs loaded ahead of the dependent adds.  Latency, not
// bandwidth, bounds these sizes, so spreading outputs over threads wins.
__global__ void __launch_bounds__(128) k_gemm_small_exact(const GemmProblem p) {
    const long long total = p.batch * p.M * p.N;
    for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long n = t % p.N;
        const long long rest = t / p.N;
        const long long m = rest % p.M;
        long long rem = rest / p.M;
        long long ao = p.a_off, bo = p.b_off, co = p.c_off;
        for (int d = p.batch_rank - 1; d >= 0; --d) {
            const long long c = rem % p.batch_shape[d];
            rem /= p.batch_shape[d];
            ao += c * p.a_bs[d];
            bo += c * p.b_bs[d];
            co += c * p.c_bs[d];
        }
        const float *a = p.A + ao + m * p.a_rs;
        const float *b = p.B + bo + n * p.b_cs;
        float acc = 0.0f;
        long long k = 0;
        for (; k + 16 <= p.K; k += 16) {
            float x[16], y[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                x[u] = __ldg(a + (k + u) * p.a_cs);
                y[u] = __ldg(b + (k + u) * p.b_rs);
            }
#pragma unroll
            for (int u = 0; u < 16; ++u) acc = __fadd_rn(acc, __fmul_rn(x[u], y[u]));
        }
        for (; k < p.K; ++k) acc = __fadd_rn(acc, __fmul_rn(__ldg(a + k * p.a_cs), __ldg(b + k * p.b_rs)));
        p.C[co + m * p.c_rs + n * p.c_cs] = acc;
    }
}

// Small problems with a long contraction: a 16x16 output tile per CTA, the A
// and B panels of the tile staged in shared memory by all 256 threads at once
// (asynchronous copies, coalesced along whichever axis has unit stride), then each thread runs its
// output's k loop in the reference's order from shared memory.  The loads of a
// panel are all in flight together, so the latency of memory is paid once per
// chunk of kSmallKc k values instead of once per sixteen.
constexpr int kSmallT = 16;     // output tile edge
constexpr int kSmallPad = 17;   // shared row pitch: conflict-free stores along k
constexpr int kSmallKc = 360;   // k values per staged chunk: 2 * 360 * 17 * 4 B = 48960 B

__global__ void __launch_bounds__(256) k_gemm_small_staged(const GemmProblem p) {
    __shared__ float As[kSmallKc * kSmallPad];  // As[k * pad + m]
    __shared__ float Bs[kSmallKc * kSmallPad];  // Bs[k * pad + n]
    const int t = threadIdx.x;
    const int tm = t / kSmallT, tn = t % kSmallT;  // this thread's output in the tile
    const long long m0 = static_cast<long long>(blockIdx.y) * kSmallT;
    const long long n0 = static_cast<long long>(blockIdx.x) * kSmallT;
    long long ao = p.a_off, bo = p.b_off, co = p.c_off;
    long long rem = blockIdx.z;
    for (int d = p.batch_rank - 1; d >= 0; --d) {
        const long long c = rem % p.batch_shape[d];
        rem /= p.batch_shape[d];
        ao += c * p.a_bs[d];
        bo += c * p.b_bs[d];
        co += c * p.c_bs[d];
    }
    const int mt = static_cast<int>(p.M - m0 < kSmallT ? p.M - m0 : kSmallT);
    const int nt = static_cast<int>(p.N - n0 < kSmallT ? p.N - n0 : kSmallT);
    const bool a_kfast = p.a_cs == 1 && p.a_rs != 1;  // A rows contiguous along k
    const bool b_kfast = p.b_rs == 1 && p.b_cs != 1;  // B columns contiguous along k
    float acc = 0.0f;
    for (long long k0 = 0; k0 < p.K; k0 += kSmallKc) {
        const int kn = static_cast<int>(p.K - k0 < kSmallKc ? p.K - k0 : kSmallKc);
        // coalesced along whichever axis has unit stride; no division per element
        const int lane = t % 32, warp = t / 32;
        if (a_kfast) {
            for (int m = warp; m < mt; m += 8)
                for (int k = lane; k < kn; k += 32)
                    cp_async4(&As[k * kSmallPad + m], p.A + ao + (m0 + m) * p.a_rs + (k0 + k) * p.a_cs);
        } else {
            const int m = t % kSmallT;
            for (int k = t / kSmallT; k < kn; k += 256 / kSmallT)
                if (m < mt) cp_async4(&As[k * kSmallPad + m], p.A + ao + (m0 + m) * p.a_rs + (k0 + k) * p.a_cs);
        }
        if (b_kfast) {
            for (int n = warp; n < nt; n += 8)
                for (int k = lane; k < kn; k += 32)
                    cp_async4(&Bs[k * kSmallPad + n], p.B + bo + (k0 + k) * p.b_rs + (n0 + n) * p.b_cs);
        } else {
            const int n = t % kSmallT;
            for (int k = t / kSmallT; k < kn; k += 256 / kSmallT)
                if (n < nt) cp_async4(&Bs[k * kSmallPad + n], p.B + bo + (k0 + k) * p.b_rs + (n0 + n) * p.b_cs);
        }
        cp_async_wait_all();
        __syncthreads();
        if (tm < mt && tn < nt) {
            // the reference's rounding and order: float product, float sum, k ascending
            int k = 0;
            for (; k + 4 <= kn; k += 4) {
                const float a0 = As[k * kSmallPad + tm], b0 = Bs[k * kSmallPad + tn];
                const float a1 = As[(k + 1) * kSmallPad + tm], b1 = Bs[(k + 1) * kSmallPad + tn];
                const float a2 = As[(k + 2) * kSmallPad + tm], b2 = Bs[(k + 2) * kSmallPad + tn];
                const float a3 = As[(k + 3) * kSmallPad + tm], b3 = Bs[(k + 3) * kSmallPad + tn];
                acc = __fadd_rn(acc, __fmul_rn(a0, b0));
                acc = __fadd_rn(acc, __fmul_rn(a1, b1));
                acc = __fadd_rn(acc, __fmul_rn(a2, b2));
                acc = __fadd_rn(acc, __fmul_rn(a3, b3));
            }
            for (; k < kn; ++k) acc = __fadd_rn(acc, __fmul_rn(As[k * kSmallPad + tm], Bs[k * kSmallPad + tn]));
        }
        __syncthreads();
    }
    if (tm < mt && tn < nt) p.C[co + (m0 + tm) * p.c_rs + (n0 + tn) * p.c_cs] = acc;
}

int gemm_simt(const GemmProblem &p, cudaStream_t stream, bool exact) {
    if (p.M == 0 || p.N == 0 || p.batch == 0) return MTC_OK;
    const double work = double(p.batch) * double(p.M) * double(p.N) * double(p.K);
    const long long tiles_m = (p.M + kSmallT - 1) / kSmallT, tiles_n = (p.N + kSmallT - 1) / kSmallT;
    // staged tiles pay off when a tile holds a warp's worth of outputs and k is long
    const bool staged_fits = (p.M < kSmallT ? p.M : kSmallT) * (p.N < kSmallT ? p.N : kSmallT) >= 32 &&
                             p.K >= 32 && tiles_m <= 65535 && p.batch <= 65535;
    if (exact && work <= double(1 << 22) && staged_fits) {
        const dim3 grid(static_cast<unsigned>(tiles_n), static_cast<unsigned>(tiles_m), static_cast<unsigned>(p.batch));
        k_gemm_small_staged<<<grid, 256, 0, stream>>>(p);
        return check_launch("small staged exact GEMM");
    }
    if (exact && work <= double(1 << 22)) {
        const long long total = p.batch * p.M * p.N;
        long long blocks = (total + 127) / 128;
        if (blocks > 148 * 16) blocks = 148 * 16;
        k_gemm_small_exact<<<static_cast<unsigned>(blocks), 128, 0, stream>>>(p);
        return check_launch("small exact GEMM");
    }
    SimtArgs args;
    args.p = p;
    args.a_kmajor = (p.a_cs == 1 || p.a_rs != 1) ? 1 : 0;
    args.b_nmajor = (p.b_cs == 1 || p.b_rs != 1) ? 1 : 0;
    const int64_t gx = (p.N + BN - 1) / BN, gy = (p.M + BM - 1) / BM;
    if (gy > 65535) return fail(MTC_ERR_UNSUPPORTED, "matmul with more than %d row tiles", 65535);
    if (p.batch > 65535) return fail(MTC_ERR_UNSUPPORTED, "matmul with more than 65535 batch entries");
    dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy), static_cast<unsigned>(p.batch));
    if (exact) k_gemm_simt<true><<<grid, 256, 0, stream>>>(args);
    else k_gemm_simt<false><<<grid, 256, 0, stream>>>(args);
    MTC_TRY(check_launch("SIMT GEMM"));
    return MTC_OK;
}

// Builds the GEMM problem from the three descriptors with the reference's
// matmul shape rules; fails with the reference's exception kinds.
static int build_problem(const mtc_desc &lhs, const mtc_desc &rhs, const mtc_desc &out, GemmProblem &p) {
    if (lhs.rank < 1 || rhs.rank < 1) return fail(MTC_ERR_INVALID_ARGUMENT, "matmul operands must have rank >= 1");
    const bool lv = lhs.rank == 1, rv = rhs.rank == 1;
    const int lb = lv ? 0 : lhs.rank - 2, rb = rv ? 0 : rhs.rank - 2;
    const int ob = lb > rb ? lb : rb;
    std::memset(&p, 0, sizeof(p));
    p.M = lv ? 1 : lhs.shape[lhs.rank - 2];
    p.K = lhs.shape[lhs.rank - 1];
    const int64_t rk = rv ? rhs.shape[0] : rhs.shape[rhs.rank - 2];
    if (rk != p.K) return fail(MTC_ERR_INVALID_ARGUMENT, "matmul contraction extents differ");
    p.N = rv ? 1 : rhs.shape[rhs.rank - 1];
    // expected output shape: batch..., [M], [N]
    const int out_rank = ob + (lv ? 0 : 1) + (rv ? 0 : 1);
    if (out.rank != out_rank) return fail(MTC_ERR_INVALID_ARGUMENT, "matmul output rank mismatch");
    p.batch = 1;
    p.batch_rank = ob;
    for (int d = 0; d < ob; ++d) {
        const int la = d - (ob - lb), ra = d - (ob - rb);
        const int64_t le = la >= 0 ? lhs.shape[la] : 1, re = ra >= 0 ? rhs.shape[ra] : 1;
        if (le != re && le != 1 && re != 1) return fail(MTC_ERR_INVALID_ARGUMENT, "matmul batch extents do not broadcast");
        const int64_t e = le == 1 ? re : le;
        if (out.shape[d] != e) return fail(MTC_ERR_INVALID_ARGUMENT, "matmul output batch extent mismatch");
        p.batch_shape[d] = e;
        p.batch *= e;
        p.a_bs[d] = (la >= 0 && lhs.shape[la] != 1) ? lhs.strides[la] : 0;
        p.b_bs[d] = (ra >= 0 && rhs.shape[ra] != 1) ? rhs.strides[ra] : 0;
        p.c_bs[d] = out.strides[d];
    }
    if (!lv && out.shape[ob] != p.M) return fail(MTC_ERR_INVALID_ARGUMENT, "matmul output row extent mismatch");
    if (!rv && out.shape[ob + (lv ? 0 : 1)] != p.N) return fail(MTC_ERR_INVALID_ARGUMENT, "matmul output column extent mismatch");
    p.A = static_cast<const float *>(lhs.data);
    p.B = static_cast<const float *>(rhs.data);
    p.C = static_cast<float *>(out.data);
    p.a_off = lhs.offset;
    p.a_rs = lv ? 0 : lhs.strides[lhs.rank - 2];
    p.a_cs = lhs.strides[lhs.rank - 1];
    p.b_off = rhs.offset;
    p.b_rs = rv ? rhs.strides[0] : rhs.strides[rhs.rank - 2];
    p.b_cs = rv ? 0 : rhs.strides[rhs.rank - 1];
    p.c_off = out.offset;
    p.c_rs = lv ? 0 : out.strides[ob];
    p.c_cs = rv ? 0 : out.strides[ob + (lv ? 0 : 1)];
    return MTC_OK;
}

}  // namespace mtc

using namespace mtc;

namespace {
// matmul calls served by each kernel family (mtc_gemm_path_counts)
std::atomic<uint64_t> g_tc_calls{0}, g_simt_calls{0};
}  // namespace

extern "C" int mtc_matmul(const mtc_desc *lhs, const mtc_desc *rhs, const mtc_desc *out, int32_t algo, void *stream) {
    clear_error();
    MTC_TRY(validate(lhs, "lhs"));
    MTC_TRY(validate(rhs, "rhs"));
    MTC_TRY(validate(out, "output"));
    if (lhs->dtype != MTC_FLOAT32 || rhs->dtype != MTC_FLOAT32 || out->dtype != MTC_FLOAT32)
        return fail(MTC_ERR_LOGIC, "matmul requires Float32");
    GemmProblem p;
    MTC_TRY(build_problem(*lhs, *rhs, *out, p));
    if (numel_of(*out) == 0) return MTC_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (p.K == 0) {
        // empty contraction: every output element is 0 (the CPU zero-fills, loops.hpp:224)
        const float zero = 0.0f;
        return mtc_fill(out, &zero, stream);
    }
    if (algo != MTC_GEMM_SIMT && algo != MTC_GEMM_3XTF32 && algo != MTC_GEMM_AUTO && algo != MTC_GEMM_SIMT_FFMA)
        return fail(MTC_ERR_INVALID_ARGUMENT, "unknown matmul algorithm %d", algo);
    void *mark = profiling() ? profile_begin(s) : nullptr;
    int rc;
    bool used_tensor_cores = false;
    // AUTO: tensor cores for problems large enough to amortise the split pack,
    // otherwise the exact-order SIMT kernel (bit-identical to the CPU reference)
    const double macs = double(p.M) * double(p.N) * double(p.K) * double(p.batch);
    const bool large = p.M >= 128 && p.N >= 128 && p.K >= 64 && macs >= double(1 << 28);
    if (algo == MTC_GEMM_SIMT || (algo == MTC_GEMM_AUTO && !large)) {
        rc = gemm_simt(p, s, true);
    } else if (algo == MTC_GEMM_SIMT_FFMA) {
        rc = gemm_simt(p, s, false);
    } else {
        rc = gemm_3xtf32(p, s);
        used_tensor_cores = rc == MTC_OK;
        if (rc == MTC_ERR_UNSUPPORTED && algo == MTC_GEMM_AUTO) {
            clear_error();
            rc = gemm_simt(p, s, true);
        }
    }
    if (mark != nullptr) profile_end(mark, s, 2.0 * double(p.M) * double(p.N) * double(p.K) * double(p.batch));
    if (rc == MTC_OK) (used_tensor_cores ? g_tc_calls : g_simt_calls).fetch_add(1, std::memory_order_relaxed);
    return rc;
}

extern "C" int mtc_gemm_path_counts(uint64_t *tensor_core, uint64_t *simt) {
    clear_error();
    if (tensor_core) *tensor_core = g_tc_calls.load(std::memory_order_relaxed);
    if (simt) *simt = g_simt_calls.load(std::memory_order_relaxed);
    return MTC_OK;
}

extern "C" int mtc_matmul_3xtf32_static(const mtc_desc *lhs, const mtc_desc *rhs, const mtc_desc *out, void *stream) {
    clear_error();
    MTC_TRY(validate(lhs, "lhs"));
    MTC_TRY(validate(rhs, "rhs"));
    MTC_TRY(validate(out, "output"));
    if (lhs->dtype != MTC_FLOAT32 || rhs->dtype != MTC_FLOAT32 || out->dtype != MTC_FLOAT32)
        return fail(MTC_ERR_LOGIC, "matmul requires Float32");
    GemmProblem p;
    MTC_TRY(build_problem(*lhs, *rhs, *out, p));
    if (numel_of(*out) == 0) return MTC_OK;
    if (p.K == 0) {
        const float zero = 0.0f;
        return mtc_fill(out, &zero, stream);
    }
    return gemm_3xtf32_static(p, static_cast<cudaStream_t>(stream));
}
