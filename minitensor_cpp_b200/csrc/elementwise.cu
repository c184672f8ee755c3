// Precompiled single-op elementwise kernels: mtc_unary / mtc_binary.
// Replaces unary_elementwise / binary_elementwise
// (src/tensor/backend/cpu/kernels/elementwise/loops.hpp:19-153).
#include <cstring>

#include "elementwise.cuh"

namespace mtc {

int plan_elementwise(const mtc_desc *inputs, int n_in, const mtc_desc *outputs, int n_out, EwPlan &plan) {
    if (n_in < 0 || n_in > MTC_EW_MAX_IN) return fail(MTC_ERR_INVALID_ARGUMENT, "too many elementwise inputs (%d)", n_in);
    if (n_out < 1 || n_out > MTC_EW_MAX_OUT) return fail(MTC_ERR_INVALID_ARGUMENT, "bad elementwise output count (%d)", n_out);
    for (int j = 0; j < n_out; ++j) {
        MTC_TRY(validate(&outputs[j], "output"));
        if (outputs[j].dtype != MTC_FLOAT32) return fail(MTC_ERR_LOGIC, "elementwise kernels require Float32");
        if (outputs[j].rank != outputs[0].rank) return fail(MTC_ERR_INVALID_ARGUMENT, "fused outputs differ in rank");
        for (int d = 0; d < outputs[0].rank; ++d)
            if (outputs[j].shape[d] != outputs[0].shape[d])
                return fail(MTC_ERR_INVALID_ARGUMENT, "fused outputs differ in shape");
    }
    for (int k = 0; k < n_in; ++k) {
        MTC_TRY(validate(&inputs[k], "input"));
        if (inputs[k].dtype != MTC_FLOAT32) return fail(MTC_ERR_LOGIC, "elementwise kernels require Float32");
    }
    const mtc_desc &o0 = outputs[0];
    IterSpace s;
    s.rank = o0.rank;
    s.nops = n_out + n_in;
    for (int d = 0; d < o0.rank; ++d) s.shape[d] = o0.shape[d];
    for (int j = 0; j < n_out; ++j) {
        for (int d = 0; d < o0.rank; ++d) s.stride[j][d] = outputs[j].strides[d];
        s.offset[j] = outputs[j].offset;
    }
    for (int k = 0; k < n_in; ++k) {
        MTC_TRY(broadcast_strides(inputs[k], o0.shape, o0.rank, s.stride[n_out + k]));
        s.offset[n_out + k] = inputs[k].offset;
    }
    simplify(s);

    MtcEwArgs &a = plan.args;
    std::memset(&a, 0, sizeof(a));
    a.numel = s.numel;
    if (s.numel == 0) {
        plan.variant = EwVariant::Empty;
        return MTC_OK;
    }
    a.rank = s.rank;
    for (int j = 0; j < n_out; ++j) {
        a.out[j] = static_cast<float *>(outputs[j].data);
        a.out_off[j] = s.offset[j];
        for (int d = 0; d < s.rank; ++d) a.out_str[j][d] = s.stride[j][d];
    }
    for (int k = 0; k < n_in; ++k) {
        a.in[k] = static_cast<const float *>(inputs[k].data);
        a.in_off[k] = s.offset[n_out + k];
        for (int d = 0; d < s.rank; ++d) a.in_str[k][d] = s.stride[n_out + k][d];
    }
    const int sms = sm_count(current_device());
    plan.block = dim3(256);

    // Flat: one axis, every operand contiguous or a broadcast scalar.
    bool flat = (s.rank == 1);
    for (int k = 0; k < s.nops && flat; ++k) {
        const int64_t st = s.stride[k][0];
        const bool is_out = k < n_out;
        flat = (st == 1) || (st == 0 && (!is_out || s.numel == 1));
    }
    if (flat) {
        bool aligned = s.numel >= 4;
        for (int j = 0; j < n_out && aligned; ++j)
            aligned = (reinterpret_cast<uintptr_t>(a.out[j] + a.out_off[j]) % 16) == 0 && a.out_str[j][0] == 1;
        for (int k = 0; k < n_in && aligned; ++k)
            if (a.in_str[k][0] != 0) aligned = (reinterpret_cast<uintptr_t>(a.in[k] + a.in_off[k]) % 16) == 0;
        const int vec = aligned ? 4 : 1;
        plan.variant = aligned ? EwVariant::Flat4 : EwVariant::Flat1;
        const long long units = (s.numel + vec - 1) / vec;
        long long blocks = (units + 255) / 256;
        if (blocks > static_cast<long long>(sms) * 8) blocks = static_cast<long long>(sms) * 8;
        if (blocks < 1) blocks = 1;
        plan.grid = dim3(static_cast<unsigned>(blocks));
        return MTC_OK;
    }

    if (s.numel >= (int64_t{1} << 32)) {
        return fail(MTC_ERR_UNSUPPORTED, "strided elementwise space of %lld elements exceeds 2^32",
                    static_cast<long long>(s.numel));
    }
    for (int d = 0; d < s.rank; ++d) {
        a.shape[d] = static_cast<unsigned>(s.shape[d]);
        const FastDiv f = make_fastdiv(static_cast<uint32_t>(s.shape[d]));
        a.div[d] = MtcFastDiv{f.d, f.mul, f.shift};
    }

    // Rows: contiguous output rows; every input contiguous or broadcast along them.
    if (s.rank >= 2) {
        const int r = s.rank;
        bool rows_ok = true;
        for (int k = 0; k < s.nops && rows_ok; ++k) {
            const int64_t inner = s.stride[k][r - 1];
            rows_ok = k < n_out ? inner == 1 : (inner == 0 || inner == 1);
        }
        if (rows_ok) {
            const int64_t cols = s.shape[r - 1];
            bool vec = cols % 4 == 0;
            for (int k = 0; k < s.nops && vec; ++k) {
                const bool is_out = k < n_out;
                const float *p = is_out ? a.out[k] : a.in[k - n_out];
                const int64_t off = is_out ? a.out_off[k] : a.in_off[k - n_out];
                if (s.stride[k][r - 1] == 0) continue;
                vec = (reinterpret_cast<uintptr_t>(p + off) % 16) == 0;
                for (int d = 0; d < r - 1 && vec; ++d) vec = (s.stride[k][d] % 4) == 0;
            }
            plan.variant = vec ? EwVariant::Rows4 : EwVariant::Rows1;
            const int64_t strip = 256 * (vec ? 4 : 1);
            const int64_t tasks = (s.numel / cols) * ((cols + strip - 1) / strip);
            long long blocks = tasks;
            if (blocks > static_cast<long long>(sms) * 8) blocks = static_cast<long long>(sms) * 8;
            plan.grid = dim3(static_cast<unsigned>(blocks < 1 ? 1 : blocks));
            return MTC_OK;
        }
    }

    // Tiled: contiguous output rows, some input contiguous along the other axis.
    if (s.rank >= 2) {
        const int r = s.rank;
        bool out_rows = true;
        for (int j = 0; j < n_out; ++j) out_rows = out_rows && s.stride[j][r - 1] == 1;
        unsigned mask = 0;
        int nt = 0;
        for (int k = 0; k < n_in && nt < 2; ++k) {
            const int64_t inner = s.stride[n_out + k][r - 1];
            const int64_t outer = s.stride[n_out + k][r - 2];
            if (inner != 0 && inner != 1 && outer == 1) {
                mask |= 1u << k;
                ++nt;
            }
        }
        int64_t batch = 1;
        for (int d = 0; d < r - 2; ++d) batch *= s.shape[d];
        const int64_t tiles_y = (s.shape[r - 2] + MTC_EW_TILE - 1) / MTC_EW_TILE;
        const int64_t tiles_x = (s.shape[r - 1] + MTC_EW_TILE - 1) / MTC_EW_TILE;
        // a handful of tiles leaves the GPU idle while each CTA walks its tile:
        // below that the one-element-per-thread strided kernel has more in flight
        const bool enough_tiles = tiles_x * tiles_y * batch >= 32;
        if (out_rows && nt > 0 && enough_tiles && batch <= 65535 && tiles_y <= 65535) {
            a.transposed = mask;
            a.batch_rank = static_cast<unsigned>(r - 2);
            // 128-bit variant: every operand read or written as float4 along its contiguous axis
            auto aligned = [](const float *p, int64_t off) { return (reinterpret_cast<uintptr_t>(p + off) % 16) == 0; };
            bool v4 = s.shape[r - 1] % 4 == 0;
            for (int j = 0; j < n_out && v4; ++j) {
                v4 = aligned(a.out[j], a.out_off[j]);
                for (int d = 0; d < r - 1 && v4; ++d) v4 = s.stride[j][d] % 4 == 0;
            }
            for (int k = 0; k < n_in && v4; ++k) {
                const int64_t *st = s.stride[n_out + k];
                if (mask & (1u << k)) {
                    v4 = s.shape[r - 2] % 4 == 0 && aligned(a.in[k], a.in_off[k]) && st[r - 1] % 4 == 0;
                    for (int d = 0; d < r - 2 && v4; ++d) v4 = st[d] % 4 == 0;
                } else if (st[r - 1] == 1) {
                    v4 = aligned(a.in[k], a.in_off[k]);
                    for (int d = 0; d < r - 1 && v4; ++d) v4 = st[d] % 4 == 0;
                } else {
                    v4 = st[r - 1] == 0;
                }
            }
            if (v4) plan.variant = nt == 1 ? EwVariant::Tiled4x1 : EwVariant::Tiled4x2;
            else plan.variant = nt == 1 ? EwVariant::Tiled1 : EwVariant::Tiled2;
            plan.block = dim3(MTC_EW_TILE_THREADS);
            plan.grid = dim3(static_cast<unsigned>(tiles_x), static_cast<unsigned>(tiles_y), static_cast<unsigned>(batch));
            return MTC_OK;
        }
    }

    plan.variant = EwVariant::Strided;
    long long blocks = (s.numel + 255) / 256;
    if (blocks > static_cast<long long>(sms) * 8) blocks = static_cast<long long>(sms) * 8;
    plan.grid = dim3(static_cast<unsigned>(blocks));
    return MTC_OK;
}

namespace {

template <class Op>
int launch(const EwPlan &p, cudaStream_t stream) {
    switch (p.variant) {
    case EwVariant::Empty:
        return MTC_OK;
    case EwVariant::Flat4:
        mtc_ew_flat<Op, 4><<<p.grid, p.block, 0, stream>>>(p.args);
        break;
    case EwVariant::Flat1:
        mtc_ew_flat<Op, 1><<<p.grid, p.block, 0, stream>>>(p.args);
        break;
    case EwVariant::Strided:
        mtc_ew_strided<Op><<<p.grid, p.block, 0, stream>>>(p.args);
        break;
    case EwVariant::Rows4:
        mtc_ew_rows<Op, 4><<<p.grid, p.block, 0, stream>>>(p.args);
        break;
    case EwVariant::Rows1:
        mtc_ew_rows<Op, 1><<<p.grid, p.block, 0, stream>>>(p.args);
        break;
    case EwVariant::Tiled1:
        mtc_ew_tiled<Op, 1><<<p.grid, p.block, 0, stream>>>(p.args);
        break;
    case EwVariant::Tiled2:
        if constexpr (Op::kIn >= 2) {
            mtc_ew_tiled<Op, 2><<<p.grid, p.block, 0, stream>>>(p.args);
        } else {
            mtc_ew_tiled<Op, 1><<<p.grid, p.block, 0, stream>>>(p.args);
        }
        break;
    case EwVariant::Tiled4x1:
        mtc_ew_tiled4<Op, 1><<<p.grid, p.block, 0, stream>>>(p.args);
        break;
    case EwVariant::Tiled4x2:
        if constexpr (Op::kIn >= 2) {
            mtc_ew_tiled4<Op, 2><<<p.grid, p.block, 0, stream>>>(p.args);
        } else {
            mtc_ew_tiled4<Op, 1><<<p.grid, p.block, 0, stream>>>(p.args);
        }
        break;
    }
    return check_launch("elementwise kernel");
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" int mtc_unary(int32_t op, const mtc_desc *in, const mtc_desc *out, void *stream) {
    clear_error();
    if (in == nullptr || out == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null descriptor");
    if (in->rank != out->rank) return fail(MTC_ERR_INVALID_ARGUMENT, "unary input and output ranks differ");
    for (int d = 0; d < in->rank; ++d)
        if (in->shape[d] != out->shape[d]) return fail(MTC_ERR_INVALID_ARGUMENT, "unary input and output shapes differ");
    EwPlan p;
    MTC_TRY(plan_elementwise(in, 1, out, 1, p));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (op) {
    case MTC_OP_ABS: return launch<MtcUnaryOp<MTC_OP_ABS>>(p, s);
    case MTC_OP_SIGN: return launch<MtcUnaryOp<MTC_OP_SIGN>>(p, s);
    case MTC_OP_NEGATE: return launch<MtcUnaryOp<MTC_OP_NEGATE>>(p, s);
    case MTC_OP_EXP: return launch<MtcUnaryOp<MTC_OP_EXP>>(p, s);
    case MTC_OP_LOG: return launch<MtcUnaryOp<MTC_OP_LOG>>(p, s);
    case MTC_OP_SQRT: return launch<MtcUnaryOp<MTC_OP_SQRT>>(p, s);
    case MTC_OP_TANH: return launch<MtcUnaryOp<MTC_OP_TANH>>(p, s);
    case MTC_OP_SIGMOID: return launch<MtcUnaryOp<MTC_OP_SIGMOID>>(p, s);
    case MTC_OP_RELU: return launch<MtcUnaryOp<MTC_OP_RELU>>(p, s);
    default: return fail(MTC_ERR_INVALID_ARGUMENT, "unknown unary op 0x%04x", op);
    }
}

extern "C" int mtc_binary(int32_t op, const mtc_desc *lhs, const mtc_desc *rhs, const mtc_desc *out, void *stream) {
    clear_error();
    if (lhs == nullptr || rhs == nullptr || out == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null descriptor");
    mtc_desc ins[2] = {*lhs, *rhs};
    EwPlan p;
    MTC_TRY(plan_elementwise(ins, 2, out, 1, p));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (op) {
    case MTC_OP_ADD: return launch<MtcBinaryOp<MTC_OP_ADD>>(p, s);
    case MTC_OP_SUBTRACT: return launch<MtcBinaryOp<MTC_OP_SUBTRACT>>(p, s);
    case MTC_OP_MULTIPLY: return launch<MtcBinaryOp<MTC_OP_MULTIPLY>>(p, s);
    case MTC_OP_DIVIDE: return launch<MtcBinaryOp<MTC_OP_DIVIDE>>(p, s);
    case MTC_OP_LOGADDEXP: return launch<MtcBinaryOp<MTC_OP_LOGADDEXP>>(p, s);
    default: return fail(MTC_ERR_INVALID_ARGUMENT, "unknown binary op 0x%04x", op);
    }
}
