// Tensor-core GEMM for sm_100a with float32 accuracy: 3xTF32 on tcgen05.
//
// Every float32 operand x is split into hi = x with the low 13 mantissa bits
// cleared (exactly representable in TF32) and lo = x - hi (exact in float32).
// The product is accumulated in TMEM as Ahi*Bhi + Ahi*Blo + Alo*Bhi; the
// dropped Alo*Blo term and the TF32 rounding of lo are below 2^-20 relative.
// The accumulation in TMEM dominates the error: measured against an exact
// product it grows about as sqrt(K) (median 7e-7 of (|A||B|)_ij at K = 8192,
// 9e-7 at K = 16384), well inside the 1e-5*sqrt(K) parity bound of the float32
// reference; split-K (shorter chains summed in float32) shrinks it.  Rounding
// hi and lo to nearest TF32 instead of truncating was measured to change it by
// under 20 %, and made the raw-operand converters the bottleneck.
//
// Pipeline (one persistent CTA per SM, 192 threads):
//   pack kernel  : A -> Ahi/Alo [batch][M][Kp], B -> Bhi/Blo [batch][N][Kp],
//                  both K-major (transposing strided views through shared memory).
//   warp 0       : TMA producer, 128xBK (A) and 256xBK (B) fp32 boxes into a ring
//                  of shared-memory stages: BK=16 with the 64-byte swizzle in 4
//                  stages of 48 KB (default), or BK=32 with the 128-byte swizzle
//                  in 2 stages of 96 KB (MTC_TC_PIPELINE=32x2).
//   warp 1       : allocates 512 TMEM columns (two 128x256 fp32 accumulators);
//                  one thread issues tcgen05.mma.kind::tf32 (M=128, N=256, K=8),
//                  3 per k-step, and tcgen05.commit releases stages / accumulators.
//   warps 2..5   : epilogue, tcgen05.ld of the accumulator lane quadrant of the
//                  warp, stores to C (any strides), then frees the accumulator.
// Every mbarrier wait is bounded; on expiry the CTA records an error in the
// device error word and leaves its loops (no hang).
#include <cuda.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "gemm.cuh"

namespace mtc {

// Device error word (copy.cu) as a device address, for kernels in other files.
int device_error_word(unsigned long long **out);

namespace {

constexpr int TC_BM = 128;
constexpr int TC_BN = 256;
constexpr int TC_THREADS = 192;

// Pipeline shape: BK fp32 elements along K per stage (one swizzle row of BK*4
// bytes), STAGES stages in the ring.
template <int BK_, int STAGES_>
struct TcPipe {
    static constexpr int BK = BK_;
    static constexpr int STAGES = STAGES_;
    static constexpr int A_BYTES = TC_BM * BK * 4;
    static constexpr int B_BYTES = TC_BN * BK * 4;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 512;
    // smem descriptor layout code (tcgen05): 2 = 128-byte swizzle, 4 = 64-byte swizzle
    static constexpr uint64_t LAYOUT = BK == 32 ? 2ull : 4ull;
    // byte distance between 8-row core-matrix groups: 8 rows x one swizzle row
    static constexpr uint64_t SBO = 8ull * BK * 4;
    static_assert(BK == 16 || BK == 32, "BK is one 64- or 128-byte swizzle row");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};
using PipeDeep = TcPipe<16, 4>;     // 4 x 48 KB
using PipeWide = TcPipe<32, 2>;     // 2 x 96 KB
constexpr uint32_t TC_TMEM_COLS = 512;
constexpr long long kWaitLimit = 20000000;  // bounded spins per wait
constexpr int kErrTimeout = MTC_ERR_RUNTIME;

struct TcArgs {
    int64_t M, N, Kp;
    int64_t batch;
    int tiles_m, tiles_n;
    int64_t total_tiles;
    float *C;
    int64_t c_off, c_rs, c_cs;
    int batch_rank;
    int64_t batch_shape[kMaxBatchRank];
    int64_t c_bs[kMaxBatchRank];
    int vec_store;  // C rows contiguous and 16-byte aligned: float4 stores
    unsigned long long *err;
    // split-K: work unit u = tile u / splits, K blocks [(u % splits) * kb_per_split, +kb_per_split);
    // with splits > 1 each unit writes its partial tile to ws[split][batch][M][N]
    int splits;
    int64_t kb_per_split;
    float *ws;
    int group;  // row tiles per column sweep of the tile order (L2 reuse)
    // Work units are handed out at run time: each CTA (CTA pair) starts with the
    // unit of its own index, then takes the next from this counter (zeroed
    // before the launch), so a CTA that starts late -- its SM still busy with
    // another kernel, e.g. a collective on another stream -- takes fewer units
    // instead of holding up the whole GEMM.  Null: static round-robin.
    unsigned long long *counter;
};

constexpr int kUnitRing = 4;  // units published ahead of the slowest role

// Tile and K-block range of work unit u.
__device__ __forceinline__ void unit_range(const TcArgs &a, int64_t u, int64_t kblocks, int64_t &t, int &split,
                                           int64_t &kb0, int64_t &kb1) {
    t = u / a.splits;
    split = static_cast<int>(u - t * a.splits);
    kb0 = static_cast<int64_t>(split) * a.kb_per_split;
    kb1 = kb0 + a.kb_per_split < kblocks ? kb0 + a.kb_per_split : kblocks;
}

// ------------------------------------------------------------ PTX helpers --

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: false when the limit expired or another role aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    for (long long i = 0; i < kWaitLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 1023) == 1023 && *abort_flag) return false;
    }
    *abort_flag = 1;
    return false;
}

// The unit after `u` for a CTA (or CTA pair) among `workers`.
__device__ __forceinline__ int64_t next_unit(const TcArgs &a, int64_t u, int64_t workers) {
    return a.counter != nullptr ? workers + static_cast<int64_t>(atomicAdd(a.counter, 1ull)) : u + workers;
}

// Reads entry i of the unit ring once the producer has published it.  The
// caller arrives on unit_empty after every thread of its group has read it.
__device__ __forceinline__ bool unit_take(uint64_t *unit_full, const volatile int64_t *ring, int64_t i,
                                          volatile int *abort_flag, int64_t &u) {
    const int r = static_cast<int>(i % kUnitRing);
    if (!mbar_wait(&unit_full[r], static_cast<uint32_t>(i / kUnitRing) & 1u, abort_flag)) return false;
    u = ring[r];
    return true;
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// Shared-memory matrix descriptor: K-major, swizzled rows of BK*4 bytes, 8-row
// groups SBO bytes apart, descriptor version 1 (bit 46).
template <class P>
__device__ __forceinline__ uint64_t smem_desc(const void *tile) {
    const uint64_t addr = smem_u32(tile);
    return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | ((P::SBO >> 4) << 32) | (1ull << 46) | (P::LAYOUT << 61);
}

// Instruction descriptor: D=F32, A=B=TF32, both K-major, M=128, N=TC_BN.
constexpr uint32_t kInstrDesc = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(TC_BN >> 3) << 17) |
                                (uint32_t(TC_BM >> 4) << 24);

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(kInstrDesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// x = hi + lo with hi = x truncated to TF32 (low 13 mantissa bits cleared) and
// lo = x - hi exact in float32; non-finite values keep hi = x, lo = 0.
__device__ __forceinline__ void split_tf32(float x, float &hi, float &lo) {
    if (!isfinite(x)) {
        hi = x;
        lo = 0.0f;
        return;
    }
    hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
    lo = __fsub_rn(x, hi);
}

__device__ __forceinline__ void tile_coords(const TcArgs &a, int64_t t, int &tm, int &tn, int &tb) {
    const int64_t per_batch = static_cast<int64_t>(a.tiles_m) * a.tiles_n;
    tb = static_cast<int>(t / per_batch);
    const int64_t r = t - tb * per_batch;
    // grouped rasterisation: `group` row tiles share each column sweep for L2 reuse
    const int G = a.group;
    const int64_t group_span = static_cast<int64_t>(G) * a.tiles_n;
    const int group = static_cast<int>(r / group_span);
    const int first_m = group * G;
    const int gsize = (a.tiles_m - first_m) < G ? (a.tiles_m - first_m) : G;
    const int64_t in_group = r - group * group_span;
    tm = first_m + static_cast<int>(in_group % gsize);
    tn = static_cast<int>(in_group / gsize);
}

// DIRECT bit 0 / bit 1: operand A / B is loaded raw (fp32, K-major) from its own
// tensor into the "hi" slot, and four converter warps write lo = x - trunc(x)
// into the "lo" slot in shared memory.  The tensor core reads a TF32 operand
// from the upper 19 bits of each 32-bit word, so the raw value acts as hi.
template <class P, int DIRECT>
__global__ void __launch_bounds__(DIRECT ? TC_THREADS + 128 : TC_THREADS, 1)
    k_gemm_3xtf32(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
                  const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_blo,
                  const TcArgs args) {
    constexpr bool AD = (DIRECT & 1) != 0;
    constexpr bool BD = (DIRECT & 2) != 0;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int TC_STAGES = P::STAGES;
    constexpr int TC_BK = P::BK;
    constexpr int TC_A_BYTES = P::A_BYTES;
    constexpr int TC_B_BYTES = P::B_BYTES;
    constexpr int TC_STAGE_BYTES = P::STAGE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + TC_STAGES * TC_STAGE_BYTES);
    uint64_t *full = bars;                       // [TC_STAGES]
    uint64_t *empty = bars + TC_STAGES;          // [TC_STAGES]
    uint64_t *acc_full = bars + 2 * TC_STAGES;   // [2]
    uint64_t *acc_empty = acc_full + 2;          // [2]
    uint64_t *drain = acc_empty + 2;             // [1] completion of the MMA issuer's work
    uint64_t *conv = drain + 1;                  // [TC_STAGES] lo slots written (DIRECT)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(conv + TC_STAGES);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    // unit ring: the producer publishes every work unit it takes; the MMA issuer,
    // the epilogue warps and the converter warps read the same sequence
    uint64_t *unit_full = reinterpret_cast<uint64_t *>(tmem_slot + 2);  // [kUnitRing]
    uint64_t *unit_empty = unit_full + kUnitRing;                        // [kUnitRing]
    volatile int64_t *unit_ring = reinterpret_cast<volatile int64_t *>(unit_empty + kUnitRing);
    const int64_t units = args.total_tiles * args.splits;
    // bytes the TMA delivers per stage: raw operands fill one slot, packed ones two
    constexpr uint32_t kStageTx = (AD ? TC_A_BYTES : 2 * TC_A_BYTES) + (BD ? TC_B_BYTES : 2 * TC_B_BYTES);

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int64_t kblocks = (args.Kp + TC_BK - 1) / TC_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&conv[s], 128);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 128);
        }
        for (int r = 0; r < kUnitRing; ++r) {
            mbar_init(&unit_full[r], 1);
            mbar_init(&unit_empty[r], DIRECT ? 9 : 5);  // MMA issuer, 4 epilogue (+ 4 converter) warps
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TC_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int64_t it = 0;
            bool ok = true;
            int64_t u = blockIdx.x;
            for (int64_t i = 0; ok; ++i) {
                const int r = static_cast<int>(i % kUnitRing);
                if (!mbar_wait(&unit_empty[r], (static_cast<uint32_t>(i / kUnitRing) & 1u) ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                unit_ring[r] = u;
                mbar_arrive(&unit_full[r]);
                if (u >= units) break;
                const int64_t next = next_unit(args, u, gridDim.x);  // its latency overlaps this unit's loads
                int64_t t, kb0, kb1;
                int split;
                unit_range(args, u, kblocks, t, split, kb0, kb1);
                int tm, tn, tb;
                tile_coords(args, t, tm, tn, tb);
                for (int64_t kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = static_cast<int>(it % TC_STAGES);
                    const uint32_t round = static_cast<uint32_t>(it / TC_STAGES);
                    if (!mbar_wait(&empty[s], (round & 1u) ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    unsigned char *st = smem + s * TC_STAGE_BYTES;
                    mbar_expect_tx(&full[s], kStageTx);
                    const int kx = static_cast<int>(kb * TC_BK);
                    tma_load_3d(st, &tm_ahi, &full[s], kx, tm * TC_BM, tb);
                    if (!AD) tma_load_3d(st + TC_A_BYTES, &tm_alo, &full[s], kx, tm * TC_BM, tb);
                    tma_load_3d(st + 2 * TC_A_BYTES, &tm_bhi, &full[s], kx, tn * TC_BN, tb);
                    if (!BD) tma_load_3d(st + 2 * TC_A_BYTES + TC_B_BYTES, &tm_blo, &full[s], kx, tn * TC_BN, tb);
                }
                u = next;
            }
            if (!ok) atomicCAS(args.err, 0ull, static_cast<unsigned long long>(kErrTimeout));
            // drain: every issued stage must have landed before the CTA exits
            for (int64_t d = it > TC_STAGES ? it - TC_STAGES : 0; d < it; ++d) {
                const int s = static_cast<int>(d % TC_STAGES);
                const uint32_t round = static_cast<uint32_t>(d / TC_STAGES);
                for (long long i = 0; i < kWaitLimit && !mbar_try_wait(&full[s], round & 1u); ++i) {
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int64_t it = 0;
            bool ok = true;
            for (int64_t local = 0; ok; ++local) {
                int64_t u;
                if (!unit_take(unit_full, unit_ring, local, abort_flag, u)) {
                    ok = false;
                    break;
                }
                mbar_arrive(&unit_empty[local % kUnitRing]);
                if (u >= units) break;
                int64_t t, kb0, kb1;
                int split;
                unit_range(args, u, kblocks, t, split, kb0, kb1);
                const int b = static_cast<int>(local & 1);
                const uint32_t use = static_cast<uint32_t>(local >> 1);
                if (!mbar_wait(&acc_empty[b], (use & 1u) ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * TC_BN);
                for (int64_t kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = static_cast<int>(it % TC_STAGES);
                    const uint32_t round = static_cast<uint32_t>(it / TC_STAGES);
                    // with raw operands the converters' barrier completes after the TMA's
                    if (!mbar_wait(DIRECT ? &conv[s] : &full[s], round & 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    unsigned char *st = smem + s * TC_STAGE_BYTES;
                    const uint64_t a_hi = smem_desc<P>(st);
                    const uint64_t a_lo = smem_desc<P>(st + TC_A_BYTES);
                    const uint64_t b_hi = smem_desc<P>(st + 2 * TC_A_BYTES);
                    const uint64_t b_lo = smem_desc<P>(st + 2 * TC_A_BYTES + TC_B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 8; ++kk) {
                        const uint64_t adv = static_cast<uint64_t>(kk * 32) >> 4;  // 8 tf32 = 32 bytes along K
                        const uint32_t acc = (kb > kb0 || kk > 0) ? 1u : 0u;
                        umma_tf32(d_tmem, a_hi + adv, b_hi + adv, acc);
                        umma_tf32(d_tmem, a_hi + adv, b_lo + adv, 1u);
                        umma_tf32(d_tmem, a_lo + adv, b_hi + adv, 1u);
                    }
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                umma_commit(&acc_full[b]);
            }
            if (!ok) atomicCAS(args.err, 0ull, static_cast<unsigned long long>(kErrTimeout));
            // drain: all MMAs this thread issued complete before TMEM is released
            umma_commit(drain);
            for (long long i = 0; i < kWaitLimit && !mbar_try_wait(drain, 0u); ++i) {
            }
        }
    } else if (DIRECT && warp >= 6) {
        // converters: lo = x - trunc(x) of every raw operand tile, position for
        // position (the swizzled layout of the hi slot is reused as is)
        const int ct = threadIdx.x - TC_THREADS;  // 0..127
        int64_t it = 0;
        bool ok = true;
        for (int64_t i = 0; ok; ++i) {
            int64_t u;
            if (!unit_take(unit_full, unit_ring, i, abort_flag, u)) {
                ok = false;
                break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&unit_empty[i % kUnitRing]);
            if (u >= units) break;
            int64_t t, kb0, kb1;
            int split;
            unit_range(args, u, kblocks, t, split, kb0, kb1);
            for (int64_t kb = kb0; kb < kb1; ++kb, ++it) {
                const int s = static_cast<int>(it % TC_STAGES);
                const uint32_t round = static_cast<uint32_t>(it / TC_STAGES);
                if (!mbar_wait(&full[s], round & 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                unsigned char *st = smem + s * TC_STAGE_BYTES;
                auto convert = [&](const unsigned char *raw, unsigned char *lo, int bytes) {
                    const float4 *src = reinterpret_cast<const float4 *>(raw);
                    float4 *dst = reinterpret_cast<float4 *>(lo);
#pragma unroll 4
                    for (int i = ct; i < bytes / 16; i += 128) {
                        const float4 v = src[i];
                        float4 h, l;
                        split_tf32(v.x, h.x, l.x);
                        split_tf32(v.y, h.y, l.y);
                        split_tf32(v.z, h.z, l.z);
                        split_tf32(v.w, h.w, l.w);
                        dst[i] = l;
                    }
                };
                if (AD) convert(st, st + TC_A_BYTES, TC_A_BYTES);
                if (BD) convert(st + 2 * TC_A_BYTES, st + 2 * TC_A_BYTES + TC_B_BYTES, TC_B_BYTES);
                // make the generic-proxy stores visible to the tensor core before arriving
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(&conv[s]);
            }
        }
        if (!ok) atomicCAS(args.err, 0ull, static_cast<unsigned long long>(kErrTimeout));
    } else if (warp >= 2 && warp < 6) {
        // epilogue: warps 2..5 cover TMEM lane quadrants (warp % 4)
        const int quadrant = warp % 4;
        const int row_in_tile = quadrant * 32 + lane;
        for (int64_t local = 0;; ++local) {
            int64_t u;
            if (!unit_take(unit_full, unit_ring, local, abort_flag, u)) {
                atomicCAS(args.err, 0ull, static_cast<unsigned long long>(kErrTimeout));
                break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&unit_empty[local % kUnitRing]);
            if (u >= units) break;
            int64_t t, kb0, kb1;
            int split;
            unit_range(args, u, kblocks, t, split, kb0, kb1);
            const int b = static_cast<int>(local & 1);
            const uint32_t use = static_cast<uint32_t>(local >> 1);
            if (!mbar_wait(&acc_full[b], use & 1u, abort_flag)) {
                atomicCAS(args.err, 0ull, static_cast<unsigned long long>(kErrTimeout));
                break;
            }
            tc_fence_after();
            int tm, tn, tb;
            tile_coords(args, t, tm, tn, tb);
            // destination: C, or with split-K this split's partial tile in ws
            float *out = args.C;
            int64_t co = args.c_off, c_rs = args.c_rs, c_cs = args.c_cs;
            bool vec = args.vec_store != 0;
            if (args.splits > 1) {
                out = args.ws;
                co = (static_cast<int64_t>(split) * args.batch + tb) * args.M * args.N;
                c_rs = args.N;
                c_cs = 1;
                vec = (args.N % 4) == 0;
            } else {
                int64_t rem = tb;
                for (int d = args.batch_rank - 1; d >= 0; --d) {
                    const int64_t c = rem % args.batch_shape[d];
                    rem /= args.batch_shape[d];
                    co += c * args.c_bs[d];
                }
            }
            const int64_t m = static_cast<int64_t>(tm) * TC_BM + row_in_tile;
            const int64_t n0 = static_cast<int64_t>(tn) * TC_BN;
            const uint32_t taddr_row = tmem_base + (static_cast<uint32_t>(quadrant * 32) << 16) +
                                       static_cast<uint32_t>(b * TC_BN);
#pragma unroll 1
            for (int c = 0; c < TC_BN / 32; ++c) {
                float v[32];
                tmem_ld32(taddr_row + static_cast<uint32_t>(c * 32), v);
                if (m < args.M) {
                    const int64_t nb = n0 + c * 32;
                    float *dst = out + co + m * c_rs;
                    if (vec && nb + 32 <= args.N) {
                        float4 *d4 = reinterpret_cast<float4 *>(dst + nb);
#pragma unroll
                        for (int j = 0; j < 8; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (nb + j < args.N) dst[(nb + j) * c_cs] = v[j];
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[b]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TC_TMEM_COLS));
    }
}

// Split-K reduction: C = ws[0] + ws[1] + ... in split order (deterministic),
// written through C's strides; one thread per output element.
__global__ void __launch_bounds__(256) k_splitk_reduce(const TcArgs a) {
    const int64_t total = a.batch * a.M * a.N;
    const int64_t plane = a.batch * a.M * a.N;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float acc = a.ws[i];
        for (int s = 1; s < a.splits; ++s) acc = __fadd_rn(acc, a.ws[s * plane + i]);
        const int64_t n = i % a.N;
        const int64_t rest = i / a.N;
        const int64_t m = rest % a.M;
        int64_t rem = rest / a.M;
        int64_t co = a.c_off;
        for (int d = a.batch_rank - 1; d >= 0; --d) {
            const int64_t c = rem % a.batch_shape[d];
            rem /= a.batch_shape[d];
            co += c * a.c_bs[d];
        }
        a.C[co + m * a.c_rs + n * a.c_cs] = acc;
    }
}

// The same reduction four columns at a time (N a multiple of 4, C rows
// contiguous and 16-byte aligned): a CTA row per output row, 128-bit loads
// and stores, no per-element index division.
__global__ void __launch_bounds__(256) k_splitk_reduce4(const TcArgs a) {
    const int64_t rows = a.batch * a.M;
    const int64_t nv = a.N / 4;
    const int64_t plane4 = rows * nv;
    const float4 *ws4 = reinterpret_cast<const float4 *>(a.ws);
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
        const int64_t m = r % a.M;
        int64_t rem = r / a.M;
        int64_t co = a.c_off + m * a.c_rs;
        for (int d = a.batch_rank - 1; d >= 0; --d) {
            const int64_t c = rem % a.batch_shape[d];
            rem /= a.batch_shape[d];
            co += c * a.c_bs[d];
        }
        float4 *dst = reinterpret_cast<float4 *>(a.C + co);
        for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < nv;
             c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
            float4 acc = ws4[r * nv + c];
            for (int s = 1; s < a.splits; ++s) {
                const float4 v = ws4[s * plane4 + r * nv + c];
                acc.x = __fadd_rn(acc.x, v.x);
                acc.y = __fadd_rn(acc.y, v.y);
                acc.z = __fadd_rn(acc.z, v.z);
                acc.w = __fadd_rn(acc.w, v.w);
            }
            dst[c] = acc;
        }
    }
}

// ------------------------------------------------------- CTA-pair kernel --
// The same 3xTF32 product with tcgen05.mma.cta_group::2: a cluster of two CTAs
// on two SMs computes one 256x256 tile.  Each CTA stages its own 128 rows of A
// and its own 128 columns of B, so every SM moves half the B bytes of the
// single-CTA kernel per MMA; the leader CTA (rank 0) issues M=256, N=256 MMAs
// that read both CTAs' shared memory and write each CTA's 128 accumulator rows
// into that CTA's TMEM.
//   both CTAs, warp 0 : TMA producer into the own ring, completion counted on
//                       the leader's full barrier (.cta_group::2 loads)
//   leader, warp 1    : MMA issuer; tcgen05.commit arrives on the empty /
//                       accumulator-full barriers of both CTAs (CTA mask 0b11)
//   both, warp 1      : allocates / frees TMEM together (cta_group::2)
//   both, warps 2..5  : epilogue of the own 128 rows; one lane per warp
//                       arrives on the leader's accumulator-empty barrier

template <int BK_, int STAGES_>
struct PairPipe {
    static constexpr int BK = BK_;
    static constexpr int STAGES = STAGES_;
    static constexpr int A_BYTES = 128 * BK * 4;  // this CTA's 128 rows of A
    static constexpr int B_BYTES = 128 * BK * 4;  // this CTA's 128 columns of B
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 512;
    static constexpr uint64_t LAYOUT = BK == 32 ? 2ull : 4ull;
    static constexpr uint64_t SBO = 8ull * BK * 4;
    static_assert(BK == 16 || BK == 32, "BK is one 64- or 128-byte swizzle row");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};
using PairDeep = PairPipe<16, 6>;  // 6 x 32 KB
using PairWide = PairPipe<32, 3>;  // 3 x 64 KB

// D=F32, A=B=TF32, both K-major, M=256 (two CTAs), N=256.
constexpr uint32_t kPairInstrDesc = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(256 >> 3) << 17) |
                                    (uint32_t(256 >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t peer_addr(const void *p, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
    return out;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// Bounded wait with cluster-scope acquire: for barriers another CTA of the
// cluster arrives on after writing this CTA's shared memory.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    for (long long i = 0; i < kWaitLimit; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((i & 1023) == 1023 && *abort_flag) return false;
    }
    *abort_flag = 1;
    return false;
}

__device__ __forceinline__ void st_cluster_s64(uint32_t cluster_addr, int64_t v) {
    asm volatile("st.shared::cluster.s64 [%0], %1;" ::"r"(cluster_addr), "l"(v) : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void *dst, const CUtensorMap *map, uint32_t leader_bar, int x, int y,
                                                 int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void umma_tf32_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(kPairInstrDesc), "r"(accumulate)
        : "memory");
}

// Arrive once on the barrier at this offset in both CTAs of the pair when the
// issuing thread's prior MMAs complete.
__device__ __forceinline__ void umma_commit_both(uint64_t *bar) {
    const uint16_t mask = 0x3;
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(smem_u32(bar)), "h"(mask)
                 : "memory");
}

__device__ __forceinline__ void umma_commit_pair_local(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void pair_tile_coords(const TcArgs &a, int64_t t, int &tm, int &tn, int &tb) {
    tile_coords(a, t, tm, tn, tb);  // tiles_m / tiles_n count 256x256 pair tiles
}

template <class P>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TC_THREADS, 1)
    k_gemm_3xtf32_pair(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
                       const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_blo,
                       const TcArgs args) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // the same aligned offset in both CTAs (same dynamic size, same static layout)
    unsigned char *smem =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int S = P::STAGES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S * P::STAGE_BYTES);
    uint64_t *full = bars;               // [S]  leader's: both CTAs' TMA bytes
    uint64_t *empty = bars + S;          // [S]  each CTA's: stage consumed by the MMAs
    uint64_t *acc_full = bars + 2 * S;   // [2]  each CTA's: accumulator ready
    uint64_t *acc_empty = acc_full + 2;  // [2]  leader's: both epilogues done
    uint64_t *drain = acc_empty + 2;     // [1]  leader's: all MMAs complete
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    // unit ring in both CTAs, written by the leader's producer; unit_empty is the
    // leader's: its MMA issuer and epilogue warps, the peer's producer and
    // epilogue warps arrive once they have read an entry
    uint64_t *unit_full = reinterpret_cast<uint64_t *>(tmem_slot + 2);  // [kUnitRing]
    uint64_t *unit_empty = unit_full + kUnitRing;                        // [kUnitRing] (leader's)
    volatile int64_t *unit_ring = reinterpret_cast<volatile int64_t *>(unit_empty + kUnitRing);

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int64_t cluster = blockIdx.x / 2;
    const int64_t clusters = gridDim.x / 2;
    const int64_t kblocks = (args.Kp + P::BK - 1) / P::BK;
    // the entry's unit, and the release of its slot (the leader's barrier)
    auto take = [&](int64_t i, int64_t &u) -> bool {
        const int r = static_cast<int>(i % kUnitRing);
        const uint32_t par = static_cast<uint32_t>(i / kUnitRing) & 1u;
        if (!(leader ? mbar_wait(&unit_full[r], par, abort_flag) : mbar_wait_cluster(&unit_full[r], par, abort_flag)))
            return false;
        u = unit_ring[r];
        return true;
    };
    auto release = [&](int64_t i) {
        const int r = static_cast<int>(i % kUnitRing);
        if (leader) mbar_arrive(&unit_empty[r]);
        else mbar_arrive_remote(peer_addr(&unit_empty[r], 0));
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 8);  // 4 epilogue warps x 2 CTAs
        }
        for (int r = 0; r < kUnitRing; ++r) {
            mbar_init(&unit_full[r], 1);
            mbar_init(&unit_empty[r], 10);  // leader: MMA issuer + 4 epilogue warps; peer: producer + 4
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TC_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int64_t it = 0;
            bool ok = true;
            int64_t t = cluster;  // leader: the unit it publishes next
            for (int64_t i = 0; ok; ++i) {
                int64_t next = 0;
                if (leader) {
                    const int r = static_cast<int>(i % kUnitRing);
                    if (!mbar_wait_cluster(&unit_empty[r], (static_cast<uint32_t>(i / kUnitRing) & 1u) ^ 1u,
                                           abort_flag)) {
                        ok = false;
                        break;
                    }
                    unit_ring[r] = t;
                    st_cluster_s64(peer_addr(const_cast<int64_t *>(&unit_ring[r]), 1), t);
                    mbar_arrive(&unit_full[r]);
                    mbar_arrive_remote(peer_addr(&unit_full[r], 1));  // release: the remote store lands first
                    if (t >= args.total_tiles) break;
                    next = next_unit(args, t, clusters);
                } else {
                    if (!take(i, t)) {
                        ok = false;
                        break;
                    }
                    release(i);
                    if (t >= args.total_tiles) break;
                }
                int tm, tn, tb;
                pair_tile_coords(args, t, tm, tn, tb);
                const int a_row = tm * 256 + static_cast<int>(rank) * 128;
                const int b_row = tn * 256 + static_cast<int>(rank) * 128;
                for (int64_t kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = static_cast<int>(it % S);
                    const uint32_t round = static_cast<uint32_t>(it / S);
                    if (!mbar_wait(&empty[s], (round & 1u) ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    unsigned char *st = smem + s * P::STAGE_BYTES;
                    if (leader) mbar_expect_tx(&full[s], 2 * P::STAGE_BYTES);
                    const uint32_t fb = peer_addr(&full[s], 0);
                    const int kx = static_cast<int>(kb * P::BK);
                    tma_load_3d_pair(st, &tm_ahi, fb, kx, a_row, tb);
                    tma_load_3d_pair(st + P::A_BYTES, &tm_alo, fb, kx, a_row, tb);
                    tma_load_3d_pair(st + 2 * P::A_BYTES, &tm_bhi, fb, kx, b_row, tb);
                    tma_load_3d_pair(st + 2 * P::A_BYTES + P::B_BYTES, &tm_blo, fb, kx, b_row, tb);
                }
                if (leader) t = next;
            }
            if (!ok) atomicCAS(args.err, 0ull, static_cast<unsigned long long>(kErrTimeout));
            if (leader) {  // every stage issued by the pair has landed before the cluster exits
                for (int64_t d = it > S ? it - S : 0; d < it; ++d) {
                    const int s = static_cast<int>(d % S);
                    const uint32_t round = static_cast<uint32_t>(d / S);
                    for (long long i = 0; i < kWaitLimit && !mbar_try_wait(&full[s], round & 1u); ++i) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            int64_t it = 0;
            bool ok = true;
            for (int64_t local = 0; ok; ++local) {
                int64_t t;
                if (!take(local, t)) {
                    ok = false;
                    break;
                }
                release(local);
                if (t >= args.total_tiles) break;
                const int b = static_cast<int>(local & 1);
                const uint32_t use = static_cast<uint32_t>(local >> 1);
                if (!mbar_wait(&acc_empty[b], (use & 1u) ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * TC_BN);
                for (int64_t kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = static_cast<int>(it % S);
                    const uint32_t round = static_cast<uint32_t>(it / S);
                    if (!mbar_wait(&full[s], round & 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    unsigned char *st = smem + s * P::STAGE_BYTES;
                    const uint64_t a_hi = smem_desc<P>(st);
                    const uint64_t a_lo = smem_desc<P>(st + P::A_BYTES);
                    const uint64_t b_hi = smem_desc<P>(st + 2 * P::A_BYTES);
                    const uint64_t b_lo = smem_desc<P>(st + 2 * P::A_BYTES + P::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < P::BK / 8; ++kk) {
                        const uint64_t adv = static_cast<uint64_t>(kk * 32) >> 4;  // 8 tf32 = 32 bytes along K
                        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
                        umma_tf32_pair(d_tmem, a_hi + adv, b_hi + adv, acc);
                        umma_tf32_pair(d_tmem, a_hi + adv, b_lo + adv, 1u);
                        umma_tf32_pair(d_tmem, a_lo + adv, b_hi + adv, 1u);
                    }
                    umma_commit_both(&empty[s]);
                }
                if (!ok) break;
                umma_commit_both(&acc_full[b]);
            }
            if (!ok) atomicCAS(args.err, 0ull, static_cast<unsigned long long>(kErrTimeout));
            // drain: all MMAs of the pair complete before either CTA frees TMEM
            umma_commit_pair_local(drain);
            for (long long i = 0; i < kWaitLimit && !mbar_try_wait(drain, 0u); ++i) {
            }
        }
    } else {
        const int quadrant = warp % 4;
        const int row_in_tile = static_cast<int>(rank) * 128 + quadrant * 32 + lane;
        const uint32_t acc_empty_leader0 = peer_addr(&acc_empty[0], 0);
        const uint32_t acc_empty_leader1 = peer_addr(&acc_empty[1], 0);
        for (int64_t local = 0;; ++local) {
            int64_t t;
            if (!take(local, t)) {
                atomicCAS(args.err, 0ull, static_cast<unsigned long long>(kErrTimeout));
                break;
            }
            __syncwarp();
            if (lane == 0) release(local);
            if (t >= args.total_tiles) break;
            const int b = static_cast<int>(local & 1);
            const uint32_t use = static_cast<uint32_t>(local >> 1);
            if (!mbar_wait(&acc_full[b], use & 1u, abort_flag)) {
                atomicCAS(args.err, 0ull, static_cast<unsigned long long>(kErrTimeout));
                break;
            }
            tc_fence_after();
            int tm, tn, tb;
            pair_tile_coords(args, t, tm, tn, tb);
            int64_t co = args.c_off;
            {
                int64_t rem = tb;
                for (int d = args.batch_rank - 1; d >= 0; --d) {
                    const int64_t c = rem % args.batch_shape[d];
                    rem /= args.batch_shape[d];
                    co += c * args.c_bs[d];
                }
            }
            const int64_t m = static_cast<int64_t>(tm) * 256 + row_in_tile;
            const int64_t n0 = static_cast<int64_t>(tn) * 256;
            const uint32_t taddr_row = tmem_base + (static_cast<uint32_t>(quadrant * 32) << 16) +
                                       static_cast<uint32_t>(b * TC_BN);
#pragma unroll 1
            for (int c = 0; c < 256 / 32; ++c) {
                float v[32];
                tmem_ld32(taddr_row + static_cast<uint32_t>(c * 32), v);
                if (m < args.M) {
                    const int64_t nb = n0 + c * 32;
                    float *dst = args.C + co + m * args.c_rs;
                    if (args.vec_store && nb + 32 <= args.N) {
                        float4 *d4 = reinterpret_cast<float4 *>(dst + nb);
#pragma unroll
                        for (int j = 0; j < 8; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (nb + j < args.N) dst[(nb + j) * args.c_cs] = v[j];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(b == 0 ? acc_empty_leader0 : acc_empty_leader1);
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // the leader's MMAs into this CTA's TMEM have drained
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TC_TMEM_COLS));
    }
}

// Failure-path self-test: one thread waits on an mbarrier that nothing ever
// arrives at, with the same bounded try-wait loop as the GEMM's roles, then
// records the timeout in the device error word and returns.  It exercises the
// give-up path of a bounded wait without faulting or hanging the GPU.
__global__ void k_wait_selftest(long long spins, unsigned long long *err) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    bool done = false;
    for (long long i = 0; i < spins && !done; ++i) done = mbar_try_wait(&bar, 0u);
    if (!done) atomicCAS(err, 0ull, static_cast<unsigned long long>(kErrTimeout));
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(&bar)) : "memory");
}

// ------------------------------------------------------------- split pack --
// dst_hi/dst_lo: [batch][rows][Kp] row-major.  Source element (batch, r, k) at
// off + batch offsets + r*sr + k*sk.  A 32x32 tile goes through shared memory so
// both the strided read and the K-contiguous write are coalesced.

struct PackArgs {
    const float *src;
    int64_t off, sr, sk;
    int64_t rows, K, Kp;
    int batch_rank;
    int64_t batch_shape[kMaxBatchRank];
    int64_t bs[kMaxBatchRank];
    float *hi;
    float *lo;
    int k_contiguous;
};

__global__ void __launch_bounds__(256) k_split_pack(const PackArgs a) {
    __shared__ float tile[32][33];
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32;
    const int64_t b = blockIdx.z;
    int64_t base = a.off;
    {
        int64_t rem = b;
        for (int d = a.batch_rank - 1; d >= 0; --d) {
            const int64_t c = rem % a.batch_shape[d];
            rem /= a.batch_shape[d];
            base += c * a.bs[d];
        }
    }
    const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
    for (int i = ty; i < 32; i += 8) {
        // coalesced along whichever source axis is contiguous
        const int64_t r = a.k_contiguous ? r0 + i : r0 + tx;
        const int64_t k = a.k_contiguous ? k0 + tx : k0 + i;
        float v = 0.0f;
        if (r < a.rows && k < a.K) v = __ldg(a.src + base + r * a.sr + k * a.sk);
        if (a.k_contiguous) tile[i][tx] = v;
        else tile[tx][i] = v;
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int64_t r = r0 + i, k = k0 + tx;
        if (r < a.rows && k < a.Kp) {
            float hi, lo;
            split_tf32(tile[i][tx], hi, lo);
            const int64_t o = (b * a.rows + r) * a.Kp + k;
            a.hi[o] = hi;
            a.lo[o] = lo;
        }
    }
}

__device__ __forceinline__ long long pack_batch_offset(const PackArgs &a, long long b) {
    long long base = a.off;
    long long rem = b;
    for (int d = a.batch_rank - 1; d >= 0; --d) {
        const long long c = rem % a.batch_shape[d];
        rem /= a.batch_shape[d];
        base += c * a.bs[d];
    }
    return base;
}

__device__ __forceinline__ void split4(const float4 v, float4 &h, float4 &l) {
    split_tf32(v.x, h.x, l.x);
    split_tf32(v.y, h.y, l.y);
    split_tf32(v.z, h.z, l.z);
    split_tf32(v.w, h.w, l.w);
}

// K-contiguous source (k stride 1, K a multiple of 4, rows 16-byte aligned):
// one CTA per (batch, row), float4 along K, four loads in flight per thread.
__global__ void __launch_bounds__(256) k_split_rows4(const PackArgs a) {
    const long long row = blockIdx.x;  // b * rows + r
    const long long b = row / a.rows;
    const long long r = row - b * a.rows;
    const float4 *src = reinterpret_cast<const float4 *>(a.src + pack_batch_offset(a, b) + r * a.sr);
    float4 *hi = reinterpret_cast<float4 *>(a.hi + row * a.Kp);
    float4 *lo = reinterpret_cast<float4 *>(a.lo + row * a.Kp);
    const int n4 = static_cast<int>(a.K / 4);
    int c = threadIdx.x;
    for (; c + 768 < n4; c += 1024) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = __ldg(src + c + 256 * u);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            float4 h, l;
            split4(v[u], h, l);
            hi[c + 256 * u] = h;
            lo[c + 256 * u] = l;
        }
    }
    for (; c < n4; c += 256) {
        float4 h, l;
        split4(__ldg(src + c), h, l);
        hi[c] = h;
        lo[c] = l;
    }
}

// Row-contiguous source (the transpose of a K-major operand: row stride 1,
// rows a multiple of 4, 16-byte aligned columns): a 64 x 64 tile is read with
// float4 loads along the rows, staged in shared memory row-major with the
// 16-byte chunks of each row XOR-swizzled by (row / 4) % 8, and written with
// float4 stores along K.  Columns K..Kp-1 are written as zeros.
__global__ void __launch_bounds__(256) k_split_tile4(const PackArgs a) {
    __shared__ __align__(16) float stage[64][64];
    const long long r0 = static_cast<long long>(blockIdx.y) * 64;
    const long long k0 = static_cast<long long>(blockIdx.x) * 64;
    const long long b = blockIdx.z;
    const float *src = a.src + pack_batch_offset(a, b);
    const int q = threadIdx.x % 16, g = threadIdx.x / 16;
    const bool row_in = r0 + 4 * q < a.rows;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const int lc = g + 16 * p;
        const long long k = k0 + lc;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (row_in && k < a.K) v = __ldg(reinterpret_cast<const float4 *>(src + k * a.sk + r0 + 4 * q));
        float *dst = &stage[4 * q][(((lc >> 2) ^ (q & 7)) << 2) | (lc & 3)];
        dst[0] = v.x;
        dst[64] = v.y;
        dst[128] = v.z;
        dst[192] = v.w;
    }
    __syncthreads();
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const int lr = g + 16 * p;
        const long long r = r0 + lr;
        if (r >= a.rows || k0 + 4 * q >= a.Kp) continue;
        const float4 v = *reinterpret_cast<const float4 *>(&stage[lr][(q ^ ((lr >> 2) & 7)) << 2]);
        float4 h, l;
        split4(v, h, l);
        const long long o = (b * a.rows + r) * a.Kp + k0 + 4 * q;
        *reinterpret_cast<float4 *>(a.hi + o) = h;
        *reinterpret_cast<float4 *>(a.lo + o) = l;
    }
}

using PFN_EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                     const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                     CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_EncodeTiled encode_fn() {
    static PFN_EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess)
            fn = reinterpret_cast<PFN_EncodeTiled>(p);
    });
    return fn;
}

// One GEMM operand as its tensor maps see it: `rows` K-major rows of `kdim`
// elements, `pitch` elements apart, batches `bstride` elements apart.  Packed
// operands have split hi / lo arrays; a raw (direct) operand is the caller's own
// tensor, whose lo the kernel computes in shared memory.
struct TcOperand {
    const float *hi = nullptr;
    const float *lo = nullptr;
    int64_t kdim = 0;
    int64_t pitch = 0;
    int64_t bstride = 0;
    bool direct = false;
};

TcOperand packed_operand(const float *hi, const float *lo, int64_t Kp, int64_t rows) {
    TcOperand o;
    o.hi = hi;
    o.lo = lo;
    o.kdim = Kp;
    o.pitch = Kp;
    o.bstride = rows * Kp;
    return o;
}

// A strided operand can be read raw when K is its contiguous axis and its rows and
// batches start on 16-byte boundaries (TMA global-address and stride rules).
bool direct_operand(const float *base, int64_t off, int64_t row_stride, int64_t k_stride, int64_t rows,
                    const GemmProblem &p, const int64_t *bs, TcOperand &o) {
    // rows at least K apart and batches at least a whole matrix apart (no overlap)
    if (k_stride != 1 || row_stride < p.K || (row_stride * 4) % 16 != 0) return false;
    if ((reinterpret_cast<uintptr_t>(base + off) % 16) != 0) return false;
    int64_t bstride = rows * row_stride;
    if (p.batch_rank > 1) return false;
    if (p.batch_rank == 1) {
        if (bs[0] < rows * row_stride || (bs[0] * 4) % 16 != 0) return false;
        bstride = bs[0];
    }
    o.hi = base + off;
    o.lo = nullptr;
    o.kdim = p.K;
    o.pitch = row_stride;
    o.bstride = bstride;
    o.direct = true;
    return true;
}

template <class P>
int make_map(CUtensorMap &map, const float *base, int64_t kdim, int64_t rows, int64_t batch, int64_t pitch,
             int64_t bstride, uint32_t box_rows) {
    PFN_EncodeTiled enc = encode_fn();
    if (enc == nullptr) return fail(MTC_ERR_RUNTIME, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kdim), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(pitch) * 4, static_cast<cuuint64_t>(bstride) * 4};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(P::BK), box_rows, 1};
    const cuuint32_t elem[3] = {1, 1, 1};
    const CUtensorMapSwizzle swz = P::BK == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    const CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides, box,
                           elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MTC_ERR_RUNTIME, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return MTC_OK;
}

template <class P>
int operand_maps(const TcOperand &o, int64_t rows, int64_t batch, uint32_t box_rows, CUtensorMap &hi,
                 CUtensorMap &lo) {
    MTC_TRY(make_map<P>(hi, o.hi, o.kdim, rows, batch, o.pitch, o.bstride, box_rows));
    if (o.direct) {
        lo = hi;  // never loaded: the kernel writes lo itself
        return MTC_OK;
    }
    return make_map<P>(lo, o.lo, o.kdim, rows, batch, o.pitch, o.bstride, box_rows);
}

int pack(const float *src, int64_t off, int64_t sr, int64_t sk, int64_t rows, int64_t K, int64_t Kp,
         const GemmProblem &p, const int64_t *bs, float *hi, float *lo, cudaStream_t stream) {
    PackArgs a;
    std::memset(&a, 0, sizeof(a));
    a.src = src;
    a.off = off;
    a.sr = sr;
    a.sk = sk;
    a.rows = rows;
    a.K = K;
    a.Kp = Kp;
    a.batch_rank = p.batch_rank;
    for (int d = 0; d < p.batch_rank; ++d) {
        a.batch_shape[d] = p.batch_shape[d];
        a.bs[d] = bs[d];
    }
    a.hi = hi;
    a.lo = lo;
    a.k_contiguous = (sk == 1 || sr != 1) ? 1 : 0;
    bool aligned = (reinterpret_cast<uintptr_t>(src + off) % 16) == 0;
    for (int d = 0; d < p.batch_rank && aligned; ++d) aligned = bs[d] % 4 == 0;
    if (aligned && sk == 1 && K % 4 == 0 && sr % 4 == 0 && p.batch * rows < (int64_t{1} << 31)) {
        k_split_rows4<<<static_cast<unsigned>(p.batch * rows), 256, 0, stream>>>(a);
        return check_launch("3xTF32 split pack (rows)");
    }
    if (aligned && sr == 1 && rows % 4 == 0 && sk % 4 == 0 && (rows + 63) / 64 <= 65535) {
        const dim3 grid(static_cast<unsigned>((Kp + 63) / 64), static_cast<unsigned>((rows + 63) / 64),
                        static_cast<unsigned>(p.batch));
        k_split_tile4<<<grid, 256, 0, stream>>>(a);
        return check_launch("3xTF32 split pack (transpose)");
    }
    dim3 grid(static_cast<unsigned>((Kp + 31) / 32), static_cast<unsigned>((rows + 31) / 32),
              static_cast<unsigned>(p.batch));
    k_split_pack<<<grid, 256, 0, stream>>>(a);
    return check_launch("3xTF32 split pack");
}

// Tensor maps over the packed operands and the persistent GEMM launch with
// pipeline shape P (allocates nothing).
template <class P, int DIRECT>
int launch_tc_variant(const CUtensorMap &m_ahi, const CUtensorMap &m_alo, const CUtensorMap &m_bhi,
                      const CUtensorMap &m_blo, const TcArgs &a, cudaStream_t stream) {
    constexpr int threads = DIRECT ? TC_THREADS + 128 : TC_THREADS;
    MTC_CUDA_TRY(cudaFuncSetAttribute(k_gemm_3xtf32<P, DIRECT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      P::SMEM_BYTES));
    int dev = 0, sms = 0;
    MTC_CUDA_TRY(cudaGetDevice(&dev));
    MTC_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t units = a.total_tiles * a.splits;
    const int64_t grid = units < sms ? units : sms;
    k_gemm_3xtf32<P, DIRECT><<<static_cast<unsigned>(grid), threads, P::SMEM_BYTES, stream>>>(m_ahi, m_alo, m_bhi,
                                                                                             m_blo, a);
    return check_launch("3xTF32 GEMM");
}

// Tensor maps over the two operands and the persistent GEMM launch with
// pipeline shape P (allocates nothing).
// Row tiles per column sweep of the persistent tile order (environment
// override for measurements).
int tile_group(const char *env, int fallback) {
    const char *v = std::getenv(env);
    const int g = v != nullptr ? std::atoi(v) : fallback;
    return g >= 1 && g <= 256 ? g : fallback;
}

template <class P>
int launch_tc(const GemmProblem &p, int64_t Kp, const TcOperand &A, const TcOperand &B, cudaStream_t stream,
              int splits, float *split_ws, unsigned long long *counter) {
    CUtensorMap m_ahi, m_alo, m_bhi, m_blo;
    MTC_TRY(operand_maps<P>(A, p.M, p.batch, TC_BM, m_ahi, m_alo));
    MTC_TRY(operand_maps<P>(B, p.N, p.batch, TC_BN, m_bhi, m_blo));
    TcArgs a;
    std::memset(&a, 0, sizeof(a));
    a.M = p.M;
    a.N = p.N;
    a.Kp = Kp;
    a.batch = p.batch;
    a.tiles_m = static_cast<int>((p.M + TC_BM - 1) / TC_BM);
    a.tiles_n = static_cast<int>((p.N + TC_BN - 1) / TC_BN);
    a.total_tiles = static_cast<int64_t>(a.tiles_m) * a.tiles_n * p.batch;
    a.C = p.C;
    a.c_off = p.c_off;
    a.c_rs = p.c_rs;
    a.c_cs = p.c_cs;
    a.batch_rank = p.batch_rank;
    for (int d = 0; d < p.batch_rank; ++d) {
        a.batch_shape[d] = p.batch_shape[d];
        a.c_bs[d] = p.c_bs[d];
    }
    bool vec = p.c_cs == 1 && (p.c_rs % 4) == 0 && (p.c_off % 4) == 0 && (reinterpret_cast<uintptr_t>(p.C) % 16) == 0;
    for (int d = 0; d < p.batch_rank && vec; ++d) vec = (p.c_bs[d] % 4) == 0;
    a.vec_store = vec ? 1 : 0;
    MTC_TRY(device_error_word(&a.err));
    a.group = tile_group("MTC_TC_GROUP", 24);
    const int64_t kblocks = (Kp + P::BK - 1) / P::BK;
    a.splits = 1;
    a.kb_per_split = kblocks;
    if (splits > 1 && split_ws != nullptr) {
        a.kb_per_split = (kblocks + splits - 1) / splits;
        a.splits = static_cast<int>((kblocks + a.kb_per_split - 1) / a.kb_per_split);
        a.ws = split_ws;
    }
    a.counter = counter;
    int rc;
    switch ((A.direct ? 1 : 0) | (B.direct ? 2 : 0)) {
    case 0: rc = launch_tc_variant<P, 0>(m_ahi, m_alo, m_bhi, m_blo, a, stream); break;
    case 1: rc = launch_tc_variant<P, 1>(m_ahi, m_alo, m_bhi, m_blo, a, stream); break;
    case 2: rc = launch_tc_variant<P, 2>(m_ahi, m_alo, m_bhi, m_blo, a, stream); break;
    default: rc = launch_tc_variant<P, 3>(m_ahi, m_alo, m_bhi, m_blo, a, stream); break;
    }
    if (rc != MTC_OK || a.splits == 1) return rc;
    if (a.vec_store && a.N % 4 == 0) {
        const int64_t rows = a.batch * a.M;
        const int64_t bx = (a.N / 4 + 255) / 256;
        const dim3 grid(static_cast<unsigned>(bx < 64 ? bx : 64), static_cast<unsigned>(rows < 65535 ? rows : 65535));
        k_splitk_reduce4<<<grid, 256, 0, stream>>>(a);
        return check_launch("3xTF32 split-K reduction");
    }
    const int64_t total = a.batch * a.M * a.N;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    k_splitk_reduce<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
    return check_launch("3xTF32 split-K reduction");
}

// Clusters of the CTA-pair kernel that fit on the device at once (cached per device).
template <class P>
int pair_clusters(int *out) {
    static std::mutex mu;
    static int cached[64] = {};
    int dev = 0;
    MTC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(MTC_ERR_RUNTIME, "device index %d outside the supported range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == 0) {
        MTC_CUDA_TRY(cudaFuncSetAttribute(k_gemm_3xtf32_pair<P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          P::SMEM_BYTES));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2, 1, 1);
        cfg.blockDim = dim3(TC_THREADS, 1, 1);
        cfg.dynamicSmemBytes = P::SMEM_BYTES;
        int n = 0;
        MTC_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, k_gemm_3xtf32_pair<P>, &cfg));
        if (n <= 0) return fail(MTC_ERR_UNSUPPORTED, "no CTA pair of the tensor-core GEMM fits on this device");
        cached[dev] = n;
    }
    *out = cached[dev];
    return MTC_OK;
}

// The CTA-pair kernel: 256x256 tiles, each CTA stages 128 rows of A and 128 of B.
template <class P>
int launch_pair(const GemmProblem &p, int64_t Kp, float *ahi, float *alo, float *bhi, float *blo,
                cudaStream_t stream, unsigned long long *counter) {
    CUtensorMap m_ahi, m_alo, m_bhi, m_blo;
    MTC_TRY(operand_maps<P>(packed_operand(ahi, alo, Kp, p.M), p.M, p.batch, 128, m_ahi, m_alo));
    MTC_TRY(operand_maps<P>(packed_operand(bhi, blo, Kp, p.N), p.N, p.batch, 128, m_bhi, m_blo));
    TcArgs a;
    std::memset(&a, 0, sizeof(a));
    a.M = p.M;
    a.N = p.N;
    a.Kp = Kp;
    a.batch = p.batch;
    a.group = tile_group("MTC_TC_PAIR_GROUP", 16);
    a.tiles_m = static_cast<int>((p.M + 255) / 256);
    a.tiles_n = static_cast<int>((p.N + 255) / 256);
    a.total_tiles = static_cast<int64_t>(a.tiles_m) * a.tiles_n * p.batch;
    a.C = p.C;
    a.c_off = p.c_off;
    a.c_rs = p.c_rs;
    a.c_cs = p.c_cs;
    a.batch_rank = p.batch_rank;
    for (int d = 0; d < p.batch_rank; ++d) {
        a.batch_shape[d] = p.batch_shape[d];
        a.c_bs[d] = p.c_bs[d];
    }
    bool vec = p.c_cs == 1 && (p.c_rs % 4) == 0 && (p.c_off % 4) == 0 && (reinterpret_cast<uintptr_t>(p.C) % 16) == 0;
    for (int d = 0; d < p.batch_rank && vec; ++d) vec = (p.c_bs[d] % 4) == 0;
    a.vec_store = vec ? 1 : 0;
    MTC_TRY(device_error_word(&a.err));
    int max_clusters = 0;
    MTC_TRY(pair_clusters<P>(&max_clusters));
    a.counter = counter;
    const int64_t clusters = a.total_tiles < max_clusters ? a.total_tiles : max_clusters;
    k_gemm_3xtf32_pair<P><<<static_cast<unsigned>(2 * clusters), TC_THREADS, P::SMEM_BYTES, stream>>>(
        m_ahi, m_alo, m_bhi, m_blo, a);
    return check_launch("3xTF32 GEMM (CTA pair)");
}

// MTC_TC_PIPELINE picks the kernel and ring: "16x4" and "32x2" run the
// single-CTA kernel with 4 x 48 KB or 2 x 96 KB stages, "pair16x6" and
// "pair32x3" the CTA-pair kernel with 6 x 32 KB or 3 x 64 KB stages.  The
// single-CTA kernel reads a K-contiguous A raw (no split pack for it);
// MTC_TC_DIRECT selects the raw operands explicitly ("0", "a", "b", "ab").
//
// Unset: "16x4" when A can be read raw (the single-CTA kernel then streams A
// once instead of a split hi/lo copy), or when the CTA pair's 256 x 256 tiles
// would leave pairs of SMs idle (it also splits K for problems with few
// tiles); otherwise the CTA pair ("pair16x6").  Each CTA of a pair stages half
// of the B tile, so the pair reads half as much shared memory per MMA.
// Measured per GEMM of the wide-MLP training step (ncu, one pass):
//   weight gradients (both operands packed, K = 65536): pair 24 ms, single 31-34 ms;
//   forward / input gradients (raw A, K = 8192): single 28-30 ms and 57-62 GB of
//   DRAM traffic, pair (A packed) 30-33 ms and 105-121 GB.
enum class TcKernel { Deep, Wide, PairDeep, PairWide };

TcKernel selected_kernel(const GemmProblem &p, bool a_raw) {
    const char *sel = std::getenv("MTC_TC_PIPELINE");
    if (sel != nullptr) {
        if (std::strcmp(sel, "16x4") == 0) return TcKernel::Deep;
        if (std::strcmp(sel, "32x2") == 0) return TcKernel::Wide;
        if (std::strcmp(sel, "pair16x6") == 0) return TcKernel::PairDeep;
        if (std::strcmp(sel, "pair32x3") == 0) return TcKernel::PairWide;
    }
    if (a_raw) return TcKernel::Deep;
    const int64_t pair_tiles = ((p.M + 255) / 256) * ((p.N + 255) / 256) * p.batch;
    return 2 * pair_tiles >= sm_count(current_device()) ? TcKernel::PairDeep : TcKernel::Deep;
}

// Which operands may be read raw: MTC_TC_DIRECT = "0" (none), "a", "b", "ab";
// unset: the default policy of choose_direct.
int direct_mask(TcKernel k) {
    if (k == TcKernel::PairDeep || k == TcKernel::PairWide) return 0;
    const char *d = std::getenv("MTC_TC_DIRECT");
    if (d == nullptr) return -1;
    return (std::strchr(d, 'a') ? 1 : 0) | (std::strchr(d, 'b') ? 2 : 0);
}

// Packs the operands that cannot be read raw into `ws` (2 * batch * rows * Kp
// floats each), then launches the selected kernel.
// `counter`: 8 bytes of device memory for the run-time unit hand-out, zeroed
// here on the stream before the launch; null keeps the static round-robin.
int run_tc(const GemmProblem &p, int64_t Kp, TcKernel k, bool a_direct, bool b_direct, const TcOperand &a_raw,
           const TcOperand &b_raw, float *ws, cudaStream_t stream, int splits = 1, float *split_ws = nullptr,
           unsigned long long *counter = nullptr) {
    const size_t a_elems = a_direct ? 0 : static_cast<size_t>(p.batch * p.M * Kp);
    const size_t b_elems = b_direct ? 0 : static_cast<size_t>(p.batch * p.N * Kp);
    float *ahi = ws, *alo = ws + a_elems, *bhi = alo + a_elems, *blo = bhi + b_elems;
    {
        HostSpan span("3xTF32 operand packs");
        if (!a_direct) MTC_TRY(pack(p.A, p.a_off, p.a_rs, p.a_cs, p.M, p.K, Kp, p, p.a_bs, ahi, alo, stream));
        // B[k][n] packed as B'[n][k]: rows advance along n (b_cs), k along b_rs
        if (!b_direct) MTC_TRY(pack(p.B, p.b_off, p.b_cs, p.b_rs, p.N, p.K, Kp, p, p.b_bs, bhi, blo, stream));
    }
    HostSpan span("3xTF32 tensor maps and launch");
    const TcOperand A = a_direct ? a_raw : packed_operand(ahi, alo, Kp, p.M);
    const TcOperand B = b_direct ? b_raw : packed_operand(bhi, blo, Kp, p.N);
    if (counter != nullptr) MTC_CUDA_TRY(cudaMemsetAsync(counter, 0, sizeof(*counter), stream));
    switch (k) {
    case TcKernel::Wide: return launch_tc<PipeWide>(p, Kp, A, B, stream, splits, split_ws, counter);
    case TcKernel::PairDeep: return launch_pair<PairDeep>(p, Kp, ahi, alo, bhi, blo, stream, counter);
    case TcKernel::PairWide: return launch_pair<PairWide>(p, Kp, ahi, alo, bhi, blo, stream, counter);
    default: return launch_tc<PipeDeep>(p, Kp, A, B, stream, splits, split_ws, counter);
    }
}

// Decides which operands are read raw: A is K-contiguous when its column stride
// is 1; B (packed as B'[n][k]) when its row stride is 1.
void choose_direct(const GemmProblem &p, TcKernel k, bool &ad, bool &bd, TcOperand &a_raw, TcOperand &b_raw) {
    ad = bd = false;
    const int mask = direct_mask(k);
    if (mask == 0) return;
    // Default: A only.  Converting a raw 256-row B tile per stage costs the MMA
    // issuer more than its split pack saves (measured on B200: a raw B made the
    // 65536x8192x8192 GEMM 21 % slower, a raw A made it 1 % faster).
    ad = (mask < 0 || (mask & 1)) && direct_operand(p.A, p.a_off, p.a_rs, p.a_cs, p.M, p, p.a_bs, a_raw);
    bd = (mask > 0 && (mask & 2)) && direct_operand(p.B, p.b_off, p.b_cs, p.b_rs, p.N, p, p.b_bs, b_raw);
}

// Whether the single-CTA kernel would read A raw under the current policy.
bool a_readable_raw(const GemmProblem &p) {
    const int mask = direct_mask(TcKernel::Deep);
    if (mask == 0 || (mask > 0 && !(mask & 1))) return false;
    TcOperand unused;
    return direct_operand(p.A, p.a_off, p.a_rs, p.a_cs, p.M, p, p.a_bs, unused);
}

// Work units handed out at run time (TcArgs::counter) or round-robin.  Measured
// on one B200 with a kernel holding 16 SMs for 2 ms launched just before an
// 8192^3 GEMM: round-robin 4.0 -> 6.9 ms (the late CTAs' fixed shares finish
// last), run-time hand-out 4.0 -> 4.7 ms.  Alone, the hand-out was 0.5-1.5 %
// slower on the training step's large GEMMs (its waves spread a little wider),
// so it is used once a communicator exists in the process, i.e. when NCCL
// kernels may share the SMs.  MTC_TC_SCHEDULE=static / dynamic overrides.
std::atomic<bool> g_collectives{false};

bool run_time_units() {
    const char *v = std::getenv("MTC_TC_SCHEDULE");
    if (v != nullptr && std::strcmp(v, "static") == 0) return false;
    if (v != nullptr && std::strcmp(v, "dynamic") == 0) return true;
    return g_collectives.load(std::memory_order_relaxed);
}

}  // namespace

void gemm_note_collectives() { g_collectives.store(true, std::memory_order_relaxed); }

int gemm_3xtf32(const GemmProblem &p, cudaStream_t stream) {
    if (p.M < 64 || p.N < 64 || p.K < 16) return fail(MTC_ERR_UNSUPPORTED, "problem too small for the tensor-core path");
    if (p.batch > 65535 || (p.M + 31) / 32 > 65535 || (p.N + 31) / 32 > 65535)
        return fail(MTC_ERR_UNSUPPORTED, "problem too large for the tensor-core launch shape");
    const int64_t Kp = (p.K + 3) / 4 * 4;  // 16-byte row pitch for the tensor maps
    if (Kp >= (int64_t{1} << 31) || p.M >= (int64_t{1} << 31) || p.N >= (int64_t{1} << 31))
        return fail(MTC_ERR_UNSUPPORTED, "extent beyond the tensor-map range");
    const TcKernel k = selected_kernel(p, a_readable_raw(p));
    bool ad, bd;
    TcOperand a_raw, b_raw;
    choose_direct(p, k, ad, bd, a_raw, b_raw);
    const size_t a_elems = ad ? 0 : static_cast<size_t>(p.batch * p.M * Kp);
    const size_t b_elems = bd ? 0 : static_cast<size_t>(p.batch * p.N * Kp);
    // split-K when the output tiles fill less than half of the GPU and K is long:
    // each split of at least 8 K blocks writes a partial tile, summed in order
    int splits = 1;
    if (k == TcKernel::Deep || k == TcKernel::Wide) {
        int dev = 0, sms = 0;
        MTC_CUDA_TRY(cudaGetDevice(&dev));
        MTC_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        const int64_t tiles = ((p.M + TC_BM - 1) / TC_BM) * ((p.N + TC_BN - 1) / TC_BN) * p.batch;
        const int64_t kblocks = (Kp + (k == TcKernel::Deep ? PipeDeep::BK : PipeWide::BK) - 1) /
                                (k == TcKernel::Deep ? PipeDeep::BK : PipeWide::BK);
        if (2 * tiles <= sms && kblocks >= 16) {
            int64_t sp = sms / tiles;
            if (sp > kblocks / 8) sp = kblocks / 8;
            if (sp > 8) sp = 8;
            splits = sp > 1 ? static_cast<int>(sp) : 1;
        }
    }
    const size_t split_elems = splits > 1 ? static_cast<size_t>(splits) * p.batch * p.M * p.N : 0;
    // workspace: the unit counter (256 bytes, keeping the packs 256-byte aligned),
    // the split operands, the split-K partial tiles
    void *scratch = nullptr;
    {
        HostSpan span("3xTF32 workspace allocation");
        MTC_TRY(scratch_alloc(256 + (2 * a_elems + 2 * b_elems + split_elems) * sizeof(float) + 1024, stream,
                              &scratch));
    }
    unsigned long long *counter = run_time_units() ? static_cast<unsigned long long *>(scratch) : nullptr;
    float *ws = reinterpret_cast<float *>(static_cast<char *>(scratch) + 256);
    float *split_ws = splits > 1 ? ws + 2 * a_elems + 2 * b_elems : nullptr;
    const int rc = run_tc(p, Kp, k, ad, bd, a_raw, b_raw, ws, stream, splits, split_ws, counter);
    {
        HostSpan span("3xTF32 workspace release");
        scratch_free(scratch, stream);
    }
    return rc;
}

// ----------------------------------------------------- allocation-free variant --
// The same tensor-core GEMM for callers that must not allocate device memory
// (for example code running under another framework's memory manager, or a
// path that must not risk an allocation): the split operands live in this
// fixed array instead of a pool allocation.  Every GPU that loads the library
// holds it until the process exits.  All calls share it and each call
// overwrites the part it uses, so calls that overlap on the GPU (different
// streams, or different host threads) race; nothing in it needs to start zeroed
// because the pack kernels write every element the GEMM reads.

constexpr size_t kStaticWorkspaceFloats = size_t(8) << 20;  // 32 MiB
static __device__ __align__(256) float g_static_workspace[kStaticWorkspaceFloats];

namespace {
std::mutex g_static_mutex;
float *g_static_ptr[64] = {};

// Device address of g_static_workspace on the current device; looked up once per
// device (the host-side name is only a stand-in, never a device address).
int static_workspace(float **out) {
    int dev = 0;
    MTC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(MTC_ERR_RUNTIME, "device index %d outside the supported range", dev);
    std::lock_guard<std::mutex> lock(g_static_mutex);
    if (g_static_ptr[dev] == nullptr) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_workspace);
        if (e != cudaSuccess || p == nullptr)
            return fail(MTC_ERR_RUNTIME, "cudaGetSymbolAddress of the static workspace failed: %s",
                        cudaGetErrorString(e));
        g_static_ptr[dev] = static_cast<float *>(p);
    }
    *out = g_static_ptr[dev];
    return MTC_OK;
}
}  // namespace

int gemm_3xtf32_static(const GemmProblem &p, cudaStream_t stream) {
    if (p.M < 64 || p.N < 64 || p.K < 16) return fail(MTC_ERR_UNSUPPORTED, "problem too small for the tensor-core path");
    if (p.batch > 65535 || (p.M + 31) / 32 > 65535 || (p.N + 31) / 32 > 65535)
        return fail(MTC_ERR_UNSUPPORTED, "problem too large for the tensor-core launch shape");
    const int64_t Kp = (p.K + 3) / 4 * 4;
    const double need = 2.0 * double(p.batch) * (double(p.M) + double(p.N)) * double(Kp);
    if (need > double(kStaticWorkspaceFloats))
        return fail(MTC_ERR_INVALID_ARGUMENT,
                    "allocation-free GEMM needs 2*batch*(M+N)*round_up(K,4) = %.0f floats of workspace; the static "
                    "workspace holds %zu (32 MiB)",
                    need, kStaticWorkspaceFloats);
    float *ws = nullptr;
    MTC_TRY(static_workspace(&ws));
    const TcKernel k = selected_kernel(p, a_readable_raw(p));
    bool ad, bd;
    TcOperand a_raw, b_raw;
    choose_direct(p, k, ad, bd, a_raw, b_raw);
    return run_tc(p, Kp, k, ad, bd, a_raw, b_raw, ws, stream);
}

}  // namespace mtc

extern "C" int mtc_selftest_bounded_wait(int64_t spins, void *stream) {
    mtc::clear_error();
    if (spins < 1 || spins > (int64_t{1} << 24))
        return mtc::fail(MTC_ERR_INVALID_ARGUMENT, "spin limit %lld outside [1, 2^24]", static_cast<long long>(spins));
    unsigned long long *err = nullptr;
    MTC_TRY(mtc::device_error_word(&err));
    mtc::k_wait_selftest<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(spins, err);
    return mtc::check_launch("bounded-wait self-test");
}
