// Counter-based random creation kernels (Uniform 0x0002, Normal 0x0003).
//
// Philox-4x32-10 as the reference CPU backend runs it
// (src/tensor/backend/cpu/detail/random_engine.cpp:14-64): block b of four
// 32-bit words is keyed by RandomKey word 0 and uses counter
// {lo(b), hi(b), lo(word1), hi(word1)}.  Each thread produces one block, so
// output element 4b+l comes from word l of block b exactly as on the CPU
// (creation/loops.hpp:39-141), independent of the launch shape.
#include <cmath>

#include "common.cuh"

namespace mtc {
namespace {

struct Philox {
    uint32_t w[4];
};

__device__ __forceinline__ Philox philox_block(unsigned long long key0, unsigned long long key1,
                                               unsigned long long block) {
    const uint32_t m0 = 0xD2511F53u, m1 = 0xCD9E8D57u;
    const uint32_t weyl0 = 0x9E3779B9u, weyl1 = 0xBB67AE85u;
    uint32_t c0 = static_cast<uint32_t>(block), c1 = static_cast<uint32_t>(block >> 32);
    uint32_t c2 = static_cast<uint32_t>(key1), c3 = static_cast<uint32_t>(key1 >> 32);
    uint32_t k0 = static_cast<uint32_t>(key0), k1 = static_cast<uint32_t>(key0 >> 32);
#pragma unroll
    for (int round = 0; round < 10; ++round) {
        const uint32_t hi0 = __umulhi(m0, c0), lo0 = m0 * c0;
        const uint32_t hi1 = __umulhi(m1, c2), lo1 = m1 * c2;
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
        if (round != 9) {
            k0 += weyl0;
            k1 += weyl1;
        }
    }
    return Philox{{c0, c1, c2, c3}};
}

__global__ void __launch_bounds__(256) k_uniform(float *out, long long n, float low, float high,
                                                  unsigned long long key0, unsigned long long key1) {
    const double low_d = static_cast<double>(low);
    const double range = static_cast<double>(high) - low_d;
    const float largest_valid = nextafterf(high, low);
    const long long blocks = (n + 3) / 4;
    for (long long b = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; b < blocks;
         b += static_cast<long long>(gridDim.x) * blockDim.x) {
        const Philox p = philox_block(key0, key1, static_cast<unsigned long long>(b));
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const long long i = b * 4 + l;
            if (i < n) {
                // unit_uniform: 24 high bits scaled by 2^-24 in float, then the double affine map
                const float unit = static_cast<float>(p.w[l] >> 8) * 0x1.0p-24f;
                float v = static_cast<float>(__dadd_rn(low_d, __dmul_rn(range, static_cast<double>(unit))));
                if (v >= high) v = largest_valid;
                out[i] = v;
            }
        }
    }
}

__global__ void __launch_bounds__(256) k_normal(float *out, long long n, float mean, float std_dev,
                                                 unsigned long long key0, unsigned long long key1) {
    const double mean_d = static_cast<double>(mean);
    const double std_d = static_cast<double>(std_dev);
    const double two_pi = 6.283185307179586476925286766559;
    const long long blocks = (n + 3) / 4;
    for (long long b = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; b < blocks;
         b += static_cast<long long>(gridDim.x) * blockDim.x) {
        const Philox p = philox_block(key0, key1, static_cast<unsigned long long>(b));
        double z[4];
#pragma unroll
        for (int pair = 0; pair < 2; ++pair) {
            // open_unit_uniform: (bits + 0.5) * 2^-32, then Box-Muller in double
            const double u1 = (static_cast<double>(p.w[2 * pair]) + 0.5) * 0x1.0p-32;
            const double u2 = (static_cast<double>(p.w[2 * pair + 1]) + 0.5) * 0x1.0p-32;
            const double radius = sqrt(-2.0 * log(u1));
            const double angle = two_pi * u2;
            z[2 * pair] = radius * cos(angle);
            z[2 * pair + 1] = radius * sin(angle);
        }
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const long long i = b * 4 + l;
            if (i < n) out[i] = static_cast<float>(__dadd_rn(mean_d, __dmul_rn(std_d, z[l])));
        }
    }
}

int check_contiguous_f32(const mtc_desc *out) {
    MTC_TRY(validate(out, "output"));
    if (out->dtype != MTC_FLOAT32) return fail(MTC_ERR_LOGIC, "random creation requires Float32");
    int64_t expect = 1;
    for (int d = out->rank - 1; d >= 0; --d) {
        if (out->shape[d] > 1 && out->strides[d] != expect)
            return fail(MTC_ERR_INVALID_ARGUMENT, "random creation requires a contiguous output");
        expect *= out->shape[d] > 1 ? out->shape[d] : 1;
    }
    return MTC_OK;
}

int grid_blocks(long long work) {
    long long b = (work + 255) / 256;
    const long long cap = static_cast<long long>(sm_count(current_device())) * 8;
    if (b > cap) b = cap;
    return b < 1 ? 1 : static_cast<int>(b);
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" int mtc_uniform(const mtc_desc *out, float low, float high, uint64_t key0, uint64_t key1, void *stream) {
    clear_error();
    MTC_TRY(check_contiguous_f32(out));
    const long long n = numel_of(*out);
    if (n == 0) return MTC_OK;
    float *base = static_cast<float *>(out->data) + out->offset;
    if (low == high) return mtc_fill(out, &low, stream);
    k_uniform<<<grid_blocks((n + 3) / 4), 256, 0, static_cast<cudaStream_t>(stream)>>>(base, n, low, high, key0, key1);
    return check_launch("uniform");
}

extern "C" int mtc_normal(const mtc_desc *out, float mean, float std_dev, uint64_t key0, uint64_t key1, void *stream) {
    clear_error();
    MTC_TRY(check_contiguous_f32(out));
    const long long n = numel_of(*out);
    if (n == 0) return MTC_OK;
    float *base = static_cast<float *>(out->data) + out->offset;
    if (std_dev == 0.0f) return mtc_fill(out, &mean, stream);
    k_normal<<<grid_blocks((n + 3) / 4), 256, 0, static_cast<cudaStream_t>(stream)>>>(base, n, mean, std_dev, key0, key1);
    return check_launch("normal");
}
