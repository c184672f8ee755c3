// KernelFn adapters registered under DeviceType::Cuda: one per reference
// primitive that needs a kernel (the CPU registrations they mirror are in
// src/tensor/backend/cpu/kernels/*/kernels.cpp).  Each adapter downcasts the
// primitive exactly like its CPU twin, turns the views into mtc_desc operands
// and calls the C ABI on the device's stream.
#include <stdexcept>
#include <vector>

#include <minitensor/host_scalar.hpp>
#include <minitensor/random.hpp>

#include "cuda_backend.hpp"
#include "tensor/core/tensor_spec.hpp"
#include "tensor/dispatch/kernel_key.hpp"
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
#include "tensor/primitives/manipulation/reshape.hpp"
#include "tensor/primitives/reduction/logsumexp.hpp"
#include "tensor/primitives/reduction/sum.hpp"
#include "tensor/random_key_access.hpp"
#include "tensor/storage/layout.hpp"
#include "tensor/storage/materialization.hpp"

namespace minitensor::detail::cuda {

namespace {

template <typename View>
mtc_desc desc_of(const View &view) {
    mtc_desc d{};
    const auto *buffer = dynamic_cast<const CudaBuffer *>(&view.buffer());
    if (buffer == nullptr) throw std::invalid_argument{"CUDA kernel requires CUDA storage"};
    const std::size_t es = dtype_size(view.dtype());
    d.data = buffer->data();
    d.capacity = static_cast<int64_t>(buffer->size_bytes() / es);
    d.dtype = view.dtype() == DType::Int64 ? MTC_INT64 : MTC_FLOAT32;
    const Shape &shape = view.shape();
    if (shape.rank() > MTC_MAX_RANK) throw std::invalid_argument{"CUDA kernels support rank <= 8"};
    d.rank = static_cast<int32_t>(shape.rank());
    const Layout &layout = view.layout();
    d.offset = layout.offset();
    for (std::size_t i = 0; i < shape.rank(); ++i) {
        d.shape[i] = shape[i];
        d.strides[i] = layout.stride(i);
    }
    return d;
}

struct Launch {
    CudaRuntime &runtime;
    void *stream;
    explicit Launch(DeviceRuntime &rt) : runtime{dynamic_cast<CudaRuntime &>(rt)}, stream{nullptr} {
        runtime.activate();
        stream = runtime.stream();
    }
};

template <int OP, typename PrimitiveType>
void run_unary(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
               MutableTensorView output) {
    (void)dynamic_cast<const PrimitiveType &>(primitive);
    Launch l(rt);
    const mtc_desc in = desc_of(inputs[0]), out = desc_of(output);
    check(mtc_unary(OP, &in, &out, l.stream), "unary kernel");
}

template <int OP, typename PrimitiveType>
void run_binary(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
                MutableTensorView output) {
    (void)dynamic_cast<const PrimitiveType &>(primitive);
    Launch l(rt);
    const mtc_desc a = desc_of(inputs[0]), b = desc_of(inputs[1]), out = desc_of(output);
    check(mtc_binary(OP, &a, &b, &out, l.stream), "binary kernel");
}

void run_contiguous(DeviceRuntime &rt, const Primitive &, std::span<const TensorView> inputs,
                    MutableTensorView output) {
    // copy_to_contiguous (copy/loops.hpp:72-88): the output is written in the
    // input's logical order as a contiguous block at the output offset.
    Launch l(rt);
    const mtc_desc in = desc_of(inputs[0]);
    mtc_desc out = desc_of(output);
    const Layout dst = Layout::contiguous(inputs[0].shape(), output.layout().offset());
    out.rank = in.rank;
    for (int i = 0; i < in.rank; ++i) {
        out.shape[i] = in.shape[i];
        out.strides[i] = dst.stride(static_cast<std::size_t>(i));
    }
    check(mtc_copy(&in, &out, l.stream), "copy kernel");
}

void run_concatenate(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
                     MutableTensorView output) {
    const auto &concat = dynamic_cast<const ConcatenatePrimitive &>(primitive);
    Launch l(rt);
    std::vector<mtc_desc> ins;
    ins.reserve(inputs.size());
    for (const TensorView &v : inputs) ins.push_back(desc_of(v));
    const mtc_desc out = desc_of(output);
    check(mtc_concat(ins.data(), static_cast<int32_t>(ins.size()), static_cast<int64_t>(concat.axis()), &out, l.stream),
          "concatenate kernel");
}

void run_basic_index_scatter(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
                             MutableTensorView output) {
    const auto &scatter = dynamic_cast<const BasicIndexScatterPrimitive &>(primitive);
    const BasicIndexParameters &parameters = scatter.parameters();
    Launch l(rt);
    const mtc_desc in = desc_of(inputs[0]);
    const mtc_desc out = desc_of(output);
    const Layout view = parameters.derive_layout(output.layout());
    mtc_desc dst = out;
    const Shape &vs = parameters.output_shape();
    dst.rank = static_cast<int32_t>(vs.rank());
    for (std::size_t i = 0; i < vs.rank(); ++i) {
        dst.shape[i] = vs[i];
        dst.strides[i] = view.stride(i);
    }
    dst.offset = view.offset();
    check(mtc_index_scatter(&in, &dst, &out, l.stream), "basic index scatter kernel");
}

void run_gather(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
                MutableTensorView output) {
    const auto &gather = dynamic_cast<const GatherPrimitive &>(primitive);
    Launch l(rt);
    const mtc_desc src = desc_of(inputs[0]), idx = desc_of(inputs[1]), out = desc_of(output);
    check(mtc_gather(&src, &idx, static_cast<int64_t>(gather.axis()), &out, l.stream), "gather kernel");
}

void run_gather_scatter_add(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
                            MutableTensorView output) {
    const auto &scatter = dynamic_cast<const GatherScatterAddPrimitive &>(primitive);
    Launch l(rt);
    const mtc_desc upd = desc_of(inputs[0]), idx = desc_of(inputs[1]), out = desc_of(output);
    check(mtc_gather_scatter_add(&upd, &idx, static_cast<int64_t>(scatter.axis()), &out, l.stream),
          "gather scatter add kernel");
}

template <int OP, typename PrimitiveType>
void run_reduction(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
                   MutableTensorView output) {
    const auto &reduction = dynamic_cast<const PrimitiveType &>(primitive);
    Launch l(rt);
    std::vector<int64_t> axes(reduction.axes().begin(), reduction.axes().end());
    const mtc_desc in = desc_of(inputs[0]), out = desc_of(output);
    check(mtc_reduce(OP, &in, axes.data(), static_cast<int32_t>(axes.size()), &out, l.stream), "reduction kernel");
}

void run_matmul(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
                MutableTensorView output) {
    (void)dynamic_cast<const MatmulPrimitive &>(primitive);
    Launch l(rt);
    const mtc_desc a = desc_of(inputs[0]), b = desc_of(inputs[1]), out = desc_of(output);
    check(mtc_matmul(&a, &b, &out, MTC_GEMM_AUTO, l.stream), "matmul kernel");
}

void run_full(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView>, MutableTensorView output) {
    const auto &full = dynamic_cast<const FullPrimitive &>(primitive);
    Launch l(rt);
    const mtc_desc out = desc_of(output);
    if (output.dtype() == DType::Int64) {
        const std::int64_t v = full.fill_value().get<std::int64_t>();
        check(mtc_fill(&out, &v, l.stream), "fill kernel");
    } else {
        const float v = full.fill_value().get<float>();
        check(mtc_fill(&out, &v, l.stream), "fill kernel");
    }
}

void run_uniform(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView>, MutableTensorView output) {
    const auto &u = dynamic_cast<const UniformPrimitive &>(primitive);
    Launch l(rt);
    const mtc_desc out = desc_of(output);
    const auto &w = RandomKeyAccess::words(u.key());
    check(mtc_uniform(&out, u.low(), u.high(), w[0], w[1], l.stream), "uniform kernel");
}

void run_normal(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView>, MutableTensorView output) {
    const auto &n = dynamic_cast<const NormalPrimitive &>(primitive);
    Launch l(rt);
    const mtc_desc out = desc_of(output);
    const auto &w = RandomKeyAccess::words(n.key());
    check(mtc_normal(&out, n.mean(), n.std_dev(), w[0], w[1], l.stream), "normal kernel");
}

}  // namespace

mtc_desc make_desc(const TensorView &view) { return desc_of(view); }
mtc_desc make_desc(const MutableTensorView &view) { return desc_of(view); }

void register_cuda_kernels(KernelRegistry &registry) {
    const DeviceType C = DeviceType::Cuda;
    registry.register_kernel({NegatePrimitive::ID, C}, run_unary<MTC_OP_NEGATE, NegatePrimitive>);
    registry.register_kernel({ExponentialPrimitive::ID, C}, run_unary<MTC_OP_EXP, ExponentialPrimitive>);
    registry.register_kernel({LogarithmPrimitive::ID, C}, run_unary<MTC_OP_LOG, LogarithmPrimitive>);
    registry.register_kernel({SquareRootPrimitive::ID, C}, run_unary<MTC_OP_SQRT, SquareRootPrimitive>);
    registry.register_kernel({HyperbolicTangentPrimitive::ID, C}, run_unary<MTC_OP_TANH, HyperbolicTangentPrimitive>);
    registry.register_kernel({AbsoluteValuePrimitive::ID, C}, run_unary<MTC_OP_ABS, AbsoluteValuePrimitive>);
    registry.register_kernel({SignPrimitive::ID, C}, run_unary<MTC_OP_SIGN, SignPrimitive>);
    registry.register_kernel({SigmoidPrimitive::ID, C}, run_unary<MTC_OP_SIGMOID, SigmoidPrimitive>);
    registry.register_kernel({AddPrimitive::ID, C}, run_binary<MTC_OP_ADD, AddPrimitive>);
    registry.register_kernel({SubtractPrimitive::ID, C}, run_binary<MTC_OP_SUBTRACT, SubtractPrimitive>);
    registry.register_kernel({MultiplyPrimitive::ID, C}, run_binary<MTC_OP_MULTIPLY, MultiplyPrimitive>);
    registry.register_kernel({DividePrimitive::ID, C}, run_binary<MTC_OP_DIVIDE, DividePrimitive>);
    registry.register_kernel({LogAddExpPrimitive::ID, C}, run_binary<MTC_OP_LOGADDEXP, LogAddExpPrimitive>);
    registry.register_kernel({ContiguousPrimitive::ID, C}, run_contiguous);
    registry.register_kernel({ReshapePrimitive::ID, C}, run_contiguous);
    registry.register_kernel({ConcatenatePrimitive::ID, C}, run_concatenate);
    registry.register_kernel({BasicIndexScatterPrimitive::ID, C}, run_basic_index_scatter);
    registry.register_kernel({GatherPrimitive::ID, C}, run_gather);
    registry.register_kernel({GatherScatterAddPrimitive::ID, C}, run_gather_scatter_add);
    registry.register_kernel({SumPrimitive::ID, C}, run_reduction<MTC_OP_SUM, SumPrimitive>);
    registry.register_kernel({LogSumExpPrimitive::ID, C}, run_reduction<MTC_OP_LOGSUMEXP, LogSumExpPrimitive>);
    registry.register_kernel({MatmulPrimitive::ID, C}, run_matmul);
    registry.register_kernel({FullPrimitive::ID, C}, run_full);
    registry.register_kernel({UniformPrimitive::ID, C}, run_uniform);
    registry.register_kernel({NormalPrimitive::ID, C}, run_normal);
}

}  // namespace minitensor::detail::cuda
