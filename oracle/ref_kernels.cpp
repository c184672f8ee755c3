// Oracle (test infrastructure only): the MiniTensor reference CPU kernels,
// exported through a C ABI that mirrors include/mtcuda.h but takes HOST
// pointers.  Every call builds reference TensorViews over copies of the host
// storage and invokes the kernel the reference registers for
// {PrimitiveId, DeviceType::Cpu} (src/tensor/backend/cpu/register_kernels.cpp),
// exactly like the reference's own CpuKernelHarness
// (tests/tensor/backend/cpu/support/kernel_harness.hpp:20-60).
//
// Built by oracle/Makefile into oracle/_ref/libmtref.so together with the
// unmodified reference sources.  Only tests/, __graft_entry__.smoke() and the
// CPU-baseline leg of bench.py load it.
#include <bit>
#include <cstring>
#include <exception>
#include <memory>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

#include <minitensor/host_scalar.hpp>
#include <minitensor/random.hpp>
#include <minitensor/types.hpp>

#include "mtcuda.h"
#include "tensor/backend/cpu/cpu_buffer.hpp"
#include "tensor/backend/cpu/cpu_runtime.hpp"
#include "tensor/backend/cpu/register_kernels.hpp"
#include "tensor/core/tensor_spec.hpp"
#include "tensor/dispatch/kernel_registry.hpp"
#include "tensor/dispatch/tensor_view.hpp"
#include "tensor/graph/primitive.hpp"
#include "tensor/primitives/creation/full.hpp"
#include "tensor/primitives/creation/normal.hpp"
#include "tensor/primitives/creation/uniform.hpp"
#include "tensor/primitives/elementwise/absolute_value.hpp"
#include "tensor/primitives/elementwise/add.hpp"
#include "tensor/primitives/elementwise/divide.hpp"
#include "tensor/primitives/elementwise/exponential.hpp"
#include "tensor/primitives/elementwise/hyperbolic_tangent.hpp"
#include "tensor/primitives/elementwise/logaddexp.hpp"
#include "tensor/primitives/elementwise/logarithm.hpp"
#include "tensor/primitives/elementwise/multiply.hpp"
#include "tensor/primitives/elementwise/negate.hpp"
#include "tensor/primitives/elementwise/sigmoid.hpp"
#include "tensor/primitives/elementwise/sign.hpp"
#include "tensor/primitives/elementwise/square_root.hpp"
#include "tensor/primitives/elementwise/subtract.hpp"
#include "tensor/primitives/linalg/matmul.hpp"
#include "tensor/primitives/manipulation/basic_index.hpp"
#include "tensor/primitives/manipulation/concatenate.hpp"
#include "tensor/primitives/manipulation/contiguous.hpp"
#include "tensor/primitives/manipulation/gather.hpp"
#include "tensor/primitives/reduction/logsumexp.hpp"
#include "tensor/primitives/reduction/sum.hpp"
#include "tensor/storage/layout.hpp"
#include "tensor/storage/materialization.hpp"

namespace md = minitensor::detail;
using minitensor::DType;
using minitensor::Shape;

namespace {

thread_local std::string t_error;

md::KernelRegistry &registry() {
    static md::KernelRegistry r = [] {
        md::KernelRegistry k;
        md::cpu::register_kernels(k);
        return k;
    }();
    return r;
}

md::cpu::CpuRuntime &runtime() {
    static md::cpu::CpuRuntime rt;
    return rt;
}

DType dtype_of(int32_t d) { return d == MTC_INT64 ? DType::Int64 : DType::Float32; }
size_t esize(int32_t d) { return d == MTC_INT64 ? 8 : 4; }

Shape shape_of(const mtc_desc &d) { return Shape(std::vector<std::int64_t>(d.shape, d.shape + d.rank)); }

// Host storage of a descriptor copied into a reference CpuBuffer.
struct Operand {
    md::TensorSpec spec;
    std::optional<md::Materialization> mat;
    md::BufferRef buffer;
    const mtc_desc *desc;

    explicit Operand(const mtc_desc &d) : desc(&d) {
        spec = md::TensorSpec{shape_of(d), dtype_of(d.dtype), minitensor::Device::cpu()};
        const size_t bytes = static_cast<size_t>(d.capacity) * esize(d.dtype);
        buffer = runtime().allocate(bytes);
        if (bytes) {
            auto *cpu = dynamic_cast<md::cpu::CpuBuffer *>(buffer.get());
            std::memcpy(cpu->data(), d.data, bytes);
        }
        mat.emplace(buffer, md::Layout(std::vector<std::int64_t>(d.strides, d.strides + d.rank), d.offset));
    }
    md::TensorView view() const { return md::TensorView(spec, *mat); }
    md::MutableTensorView mut() const { return md::MutableTensorView(spec, *mat); }
    void write_back() const {
        const size_t bytes = static_cast<size_t>(desc->capacity) * esize(desc->dtype);
        if (bytes) std::memcpy(desc->data, dynamic_cast<md::cpu::CpuBuffer *>(buffer.get())->data(), bytes);
    }
};

template <typename F>
int guarded(F &&f) {
    t_error.clear();
    try {
        f();
        return MTC_OK;
    } catch (const std::out_of_range &e) {
        t_error = e.what();
        return MTC_ERR_OUT_OF_RANGE;
    } catch (const std::invalid_argument &e) {
        t_error = e.what();
        return MTC_ERR_INVALID_ARGUMENT;
    } catch (const std::overflow_error &e) {
        t_error = e.what();
        return MTC_ERR_OVERFLOW;
    } catch (const std::logic_error &e) {
        t_error = e.what();
        return MTC_ERR_LOGIC;
    } catch (const std::exception &e) {
        t_error = e.what();
        return MTC_ERR_RUNTIME;
    }
}

void invoke(const md::Primitive &prim, const std::vector<const Operand *> &ins, const Operand &out) {
    std::vector<md::TensorView> views;
    for (const Operand *o : ins) views.push_back(o->view());
    const md::KernelFn &k = registry().get({prim.id(), minitensor::DeviceType::Cpu});
    k(runtime(), prim, views, out.mut());
    out.write_back();
}

std::unique_ptr<md::Primitive> elementwise_primitive(int op) {
    switch (op) {
    case MTC_OP_ABS: return std::make_unique<md::AbsoluteValuePrimitive>();
    case MTC_OP_SIGN: return std::make_unique<md::SignPrimitive>();
    case MTC_OP_NEGATE: return std::make_unique<md::NegatePrimitive>();
    case MTC_OP_EXP: return std::make_unique<md::ExponentialPrimitive>();
    case MTC_OP_LOG: return std::make_unique<md::LogarithmPrimitive>();
    case MTC_OP_SQRT: return std::make_unique<md::SquareRootPrimitive>();
    case MTC_OP_TANH: return std::make_unique<md::HyperbolicTangentPrimitive>();
    case MTC_OP_SIGMOID: return std::make_unique<md::SigmoidPrimitive>();
    case MTC_OP_ADD: return std::make_unique<md::AddPrimitive>();
    case MTC_OP_SUBTRACT: return std::make_unique<md::SubtractPrimitive>();
    case MTC_OP_MULTIPLY: return std::make_unique<md::MultiplyPrimitive>();
    case MTC_OP_DIVIDE: return std::make_unique<md::DividePrimitive>();
    case MTC_OP_LOGADDEXP: return std::make_unique<md::LogAddExpPrimitive>();
    default: throw std::invalid_argument{"the reference has no kernel for this op"};
    }
}

minitensor::RandomKey key_of(uint64_t w0, uint64_t w1) {
    // RandomKey is two 64-bit words (include/minitensor/random.hpp:45); its
    // two-word constructor is private, so the words are placed by value.
    return std::bit_cast<minitensor::RandomKey>(std::array<std::uint64_t, 2>{w0, w1});
}

}  // namespace

extern "C" {

const char *mtref_last_error(void) { return t_error.c_str(); }

int mtref_unary(int32_t op, const mtc_desc *in, const mtc_desc *out) {
    return guarded([&] {
        auto prim = elementwise_primitive(op);
        Operand i(*in), o(*out);
        invoke(*prim, {&i}, o);
    });
}

int mtref_binary(int32_t op, const mtc_desc *lhs, const mtc_desc *rhs, const mtc_desc *out) {
    return guarded([&] {
        auto prim = elementwise_primitive(op);
        Operand a(*lhs), b(*rhs), o(*out);
        invoke(*prim, {&a, &b}, o);
    });
}

int mtref_reduce(int32_t op, const mtc_desc *in, const int64_t *axes, int32_t n_axes, int32_t keep_dim,
                 const mtc_desc *out) {
    return guarded([&] {
        std::vector<std::int64_t> ax(axes, axes + n_axes);
        std::unique_ptr<md::Primitive> prim;
        if (op == MTC_OP_SUM) prim = std::make_unique<md::SumPrimitive>(ax, in->rank, keep_dim != 0);
        else if (op == MTC_OP_LOGSUMEXP) prim = std::make_unique<md::LogSumExpPrimitive>(ax, in->rank, keep_dim != 0);
        else throw std::invalid_argument{"the reference has no kernel for this reduction"};
        Operand i(*in), o(*out);
        invoke(*prim, {&i}, o);
    });
}

int mtref_matmul(const mtc_desc *lhs, const mtc_desc *rhs, const mtc_desc *out) {
    return guarded([&] {
        md::MatmulPrimitive prim;
        Operand a(*lhs), b(*rhs), o(*out);
        invoke(prim, {&a, &b}, o);
    });
}

int mtref_copy(const mtc_desc *src, const mtc_desc *dst) {
    return guarded([&] {
        md::ContiguousPrimitive prim;
        Operand i(*src), o(*dst);
        invoke(prim, {&i}, o);
    });
}

int mtref_concat(const mtc_desc *inputs, int32_t n_inputs, int64_t axis, const mtc_desc *out) {
    return guarded([&] {
        md::ConcatenatePrimitive prim(axis, out->rank);
        std::vector<std::unique_ptr<Operand>> ops;
        std::vector<const Operand *> ptrs;
        for (int i = 0; i < n_inputs; ++i) {
            ops.push_back(std::make_unique<Operand>(inputs[i]));
            ptrs.push_back(ops.back().get());
        }
        Operand o(*out);
        invoke(prim, ptrs, o);
    });
}

int mtref_gather(const mtc_desc *src, const mtc_desc *idx, int64_t axis, const mtc_desc *out) {
    return guarded([&] {
        md::GatherPrimitive prim(axis, src->rank);
        Operand s(*src), i(*idx), o(*out);
        invoke(prim, {&s, &i}, o);
    });
}

int mtref_gather_scatter_add(const mtc_desc *upd, const mtc_desc *idx, int64_t axis, const mtc_desc *out) {
    return guarded([&] {
        md::GatherScatterAddPrimitive prim(shape_of(*out), static_cast<Shape::size_type>(axis));
        Operand u(*upd), i(*idx), o(*out);
        invoke(prim, {&u, &i}, o);
    });
}

int mtref_fill(const mtc_desc *out, const void *value) {
    return guarded([&] {
        Operand o(*out);
        minitensor::HostScalar v = out->dtype == MTC_INT64 ? minitensor::HostScalar(*static_cast<const std::int64_t *>(value))
                                                           : minitensor::HostScalar(*static_cast<const float *>(value));
        md::FullPrimitive prim(o.spec, v);
        invoke(prim, {}, o);
    });
}

int mtref_uniform(const mtc_desc *out, float low, float high, uint64_t key0, uint64_t key1) {
    return guarded([&] {
        Operand o(*out);
        md::UniformPrimitive prim(o.spec, low, high, key_of(key0, key1));
        invoke(prim, {}, o);
    });
}

int mtref_normal(const mtc_desc *out, float mean, float std_dev, uint64_t key0, uint64_t key1) {
    return guarded([&] {
        Operand o(*out);
        md::NormalPrimitive prim(o.spec, mean, std_dev, key_of(key0, key1));
        invoke(prim, {}, o);
    });
}

namespace {
md::BasicIndexParameters index_parameters(int32_t select, int64_t axis, int32_t has_start, int64_t start,
                                          int32_t has_stop, int64_t stop, int64_t step_or_index, const Shape &shape) {
    if (select) return md::BasicIndexParameters::for_select(axis, step_or_index, shape);
    return md::BasicIndexParameters::for_slice(axis, has_start ? std::optional<std::int64_t>(start) : std::nullopt,
                                               has_stop ? std::optional<std::int64_t>(stop) : std::nullopt,
                                               step_or_index, shape);
}
}  // namespace

// BasicIndexScatter (copy/loops.hpp:129-153) for slice(axis, start, stop, step)
// or select(axis, index) of a tensor of out's shape.
int mtref_index_scatter(const mtc_desc *in, const mtc_desc *out, int32_t select, int64_t axis, int32_t has_start,
                        int64_t start, int32_t has_stop, int64_t stop, int64_t step_or_index) {
    return guarded([&] {
        const auto params = index_parameters(select, axis, has_start, start, has_stop, stop, step_or_index, shape_of(*out));
        md::BasicIndexScatterPrimitive prim(params);
        Operand i(*in), o(*out);
        invoke(prim, {&i}, o);
    });
}

// The view of `out`'s layout that the indexed slice/select occupies
// (BasicIndexParameters::derive_layout): strides and offset into view_out.
int mtref_index_layout(const mtc_desc *out, int32_t select, int64_t axis, int32_t has_start, int64_t start,
                       int32_t has_stop, int64_t stop, int64_t step_or_index, mtc_desc *view_out) {
    return guarded([&] {
        const auto params = index_parameters(select, axis, has_start, start, has_stop, stop, step_or_index, shape_of(*out));
        const md::Layout base(std::vector<std::int64_t>(out->strides, out->strides + out->rank), out->offset);
        const md::Layout view = params.derive_layout(base);
        *view_out = *out;
        const Shape &vs = params.output_shape();
        view_out->rank = static_cast<int32_t>(vs.rank());
        for (size_t d = 0; d < vs.rank(); ++d) {
            view_out->shape[d] = vs[d];
            view_out->strides[d] = view.stride(d);
        }
        view_out->offset = view.offset();
    });
}

// RandomKey derivations (src/tensor/random.cpp:13-32), for seeding tests.
void mtref_key_fold_in(uint64_t key0, uint64_t key1, uint64_t data, uint64_t *out2) {
    const auto k = minitensor::fold_in(key_of(key0, key1), data);
    const auto w = std::bit_cast<std::array<std::uint64_t, 2>>(k);
    out2[0] = w[0];
    out2[1] = w[1];
}

void mtref_key_split(uint64_t key0, uint64_t key1, uint64_t *out4) {
    const auto ks = minitensor::split(key_of(key0, key1));
    for (int i = 0; i < 2; ++i) {
        const auto w = std::bit_cast<std::array<std::uint64_t, 2>>(ks[i]);
        out4[2 * i] = w[0];
        out4[2 * i + 1] = w[1];
    }
}

}  // extern "C"
