// New primitives (relu, max, argmax, log-softmax), their CPU and CUDA kernels,
// and relu's VJP rule.  The CPU reduction kernels walk the reference's own
// ReductionPlan (src/tensor/backend/cpu/iteration/reduction.hpp:18-119) in its
// sequential order, and relu's CPU kernel runs the reference's unary loop
// (src/tensor/backend/cpu/kernels/elementwise/loops.hpp:19-67), so they are
// the CPU definition the CUDA kernels are checked against.
#include "ops_ext.hpp"

#include <algorithm>
#include <cmath>
#include <limits>
#include <memory>
#include <stdexcept>
#include <string_view>
#include <vector>

#include <minitensor/ops/elementwise.hpp>
#include <minitensor/ops/reduction.hpp>

#include "cuda_backend.hpp"
#include "tensor/apply_operation.hpp"
#include "tensor/autograd/vjp_registry.hpp"
#include "tensor/backend/cpu/kernels/elementwise/loops.hpp"
#include "tensor/backend/cpu/detail/buffer_access.hpp"
#include "tensor/backend/cpu/iteration/reduction.hpp"
#include "tensor/core/axis.hpp"
#include "tensor/core/reduction.hpp"
#include "tensor/core/tensor_spec.hpp"
#include "tensor/dispatch/kernel_key.hpp"
#include "tensor/graph/primitive.hpp"
#include "tensor/storage/layout.hpp"

namespace minitensor::detail::ext {

namespace {

std::vector<Shape::size_type> normalized_axes(std::span<const Axis> axes, Shape::size_type rank, const char *what) {
    if (axes.size() > rank) throw std::invalid_argument{std::string(what) + " cannot reduce more axes than the input rank"};
    std::vector<Shape::size_type> out;
    for (const Axis a : axes) out.push_back(normalize_axis(a, rank));
    std::ranges::sort(out);
    if (std::ranges::adjacent_find(out) != out.end())
        throw std::invalid_argument{std::string(what) + " axes cannot contain duplicates"};
    return out;
}

class ReluPrimitive final : public Primitive {
  public:
    static constexpr PrimitiveId ID{0x0180};
    [[nodiscard]] PrimitiveId id() const noexcept override { return ID; }
    [[nodiscard]] std::string_view name() const noexcept override { return "relu"; }
    [[nodiscard]] TensorSpec infer(std::span<const TensorSpec> inputs) const override {
        if (inputs.size() != 1) throw std::invalid_argument{"relu requires a single input"};
        if (!is_floating_point(inputs.front().dtype)) throw std::invalid_argument{"relu requires a floating-point input"};
        return inputs.front();
    }
};

class MaxPrimitive final : public Primitive {
  public:
    static constexpr PrimitiveId ID{0x0380};
    MaxPrimitive(std::span<const Axis> axes, Shape::size_type rank, bool keep_dim)
        : axes_{normalized_axes(axes, rank, "max")}, rank_{rank}, keep_dim_{keep_dim} {}
    [[nodiscard]] PrimitiveId id() const noexcept override { return ID; }
    [[nodiscard]] std::string_view name() const noexcept override { return "max"; }
    [[nodiscard]] TensorSpec infer(std::span<const TensorSpec> inputs) const override {
        if (inputs.size() != 1) throw std::invalid_argument{"max requires a single input"};
        const TensorSpec &in = inputs.front();
        if (in.shape.rank() != rank_) throw std::invalid_argument{"max primitive was normalized for a different rank"};
        if (!is_floating_point(in.dtype)) throw std::invalid_argument{"max requires a floating-point input"};
        return TensorSpec{reduction_shape(in.shape, axes_, keep_dim_), in.dtype, in.device};
    }
    [[nodiscard]] const std::vector<Shape::size_type> &axes() const noexcept { return axes_; }
    [[nodiscard]] bool keep_dim() const noexcept { return keep_dim_; }

  private:
    std::vector<Shape::size_type> axes_;
    Shape::size_type rank_;
    bool keep_dim_;
};

class ArgMaxPrimitive final : public Primitive {
  public:
    static constexpr PrimitiveId ID{0x0381};
    ArgMaxPrimitive(Axis axis, Shape::size_type rank, bool keep_dim)
        : axis_{normalize_axis(axis, rank)}, rank_{rank}, keep_dim_{keep_dim} {}
    [[nodiscard]] PrimitiveId id() const noexcept override { return ID; }
    [[nodiscard]] std::string_view name() const noexcept override { return "argmax"; }
    [[nodiscard]] TensorSpec infer(std::span<const TensorSpec> inputs) const override {
        if (inputs.size() != 1) throw std::invalid_argument{"argmax requires a single input"};
        const TensorSpec &in = inputs.front();
        if (in.shape.rank() != rank_) throw std::invalid_argument{"argmax primitive was normalized for a different rank"};
        if (!is_floating_point(in.dtype)) throw std::invalid_argument{"argmax requires a floating-point input"};
        if (in.shape[axis_] == 0) throw std::invalid_argument{"argmax of an empty axis"};
        const std::array<Shape::size_type, 1> ax{axis_};
        return TensorSpec{reduction_shape(in.shape, ax, keep_dim_), DType::Int64, in.device};
    }
    [[nodiscard]] Shape::size_type axis() const noexcept { return axis_; }
    [[nodiscard]] bool keep_dim() const noexcept { return keep_dim_; }

  private:
    Shape::size_type axis_;
    Shape::size_type rank_;
    bool keep_dim_;
};

class LogSoftmaxPrimitive final : public Primitive {
  public:
    static constexpr PrimitiveId ID{0x0382};
    LogSoftmaxPrimitive(Axis axis, Shape::size_type rank) : axis_{normalize_axis(axis, rank)}, rank_{rank} {}
    [[nodiscard]] PrimitiveId id() const noexcept override { return ID; }
    [[nodiscard]] std::string_view name() const noexcept override { return "log_softmax"; }
    [[nodiscard]] TensorSpec infer(std::span<const TensorSpec> inputs) const override {
        if (inputs.size() != 1) throw std::invalid_argument{"log_softmax requires a single input"};
        const TensorSpec &in = inputs.front();
        if (in.shape.rank() != rank_) throw std::invalid_argument{"log_softmax primitive was normalized for a different rank"};
        if (!is_floating_point(in.dtype)) throw std::invalid_argument{"log_softmax requires a floating-point input"};
        return in;
    }
    [[nodiscard]] Shape::size_type axis() const noexcept { return axis_; }

  private:
    Shape::size_type axis_;
    Shape::size_type rank_;
};

// ------------------------------------------------------------- CPU kernels --

// max(x, 0): x above 0 passes, NaN propagates, everything else (-0, -inf) is +0.
float relu_value(float x) { return x > 0.0F || std::isnan(x) ? x : 0.0F; }

void cpu_relu(DeviceRuntime &, const Primitive &primitive, std::span<const TensorView> inputs,
              MutableTensorView output) {
    (void)dynamic_cast<const ReluPrimitive &>(primitive);
    if (output.dtype() != DType::Float32) throw std::invalid_argument{"relu supports Float32"};
    cpu::unary_elementwise<float>(inputs.front(), output, relu_value);
}

void cpu_max(DeviceRuntime &, const Primitive &primitive, std::span<const TensorView> inputs, MutableTensorView output) {
    const auto &p = dynamic_cast<const MaxPrimitive &>(primitive);
    const TensorView &in = inputs.front();
    const cpu::ReductionPlan plan{in.shape(), in.layout(), p.axes()};
    if (plan.output_size() == 0) return;
    const float *x = cpu::data<float>(in);
    float *y = cpu::data<float>(output) + output.layout().offset();
    plan.for_each_output([&](Shape::size_type o, const cpu::ReductionPlan::ReductionRange &range) {
        float acc = -std::numeric_limits<float>::infinity();
        range.for_each_run([&](const cpu::ReductionPlan::Run &run) {
            Layout::offset_type off = run.offset;
            for (Shape::size_type i = 0; i < run.size; ++i, off += run.stride) {
                const float v = x[off];
                if (!std::isnan(acc) && (std::isnan(v) || v > acc)) acc = v;
            }
        });
        y[o] = acc;
    });
}

void cpu_argmax(DeviceRuntime &, const Primitive &primitive, std::span<const TensorView> inputs,
                MutableTensorView output) {
    const auto &p = dynamic_cast<const ArgMaxPrimitive &>(primitive);
    const TensorView &in = inputs.front();
    const std::array<Shape::size_type, 1> axes{p.axis()};
    const cpu::ReductionPlan plan{in.shape(), in.layout(), axes};
    if (plan.output_size() == 0) return;
    const float *x = cpu::data<float>(in);
    std::int64_t *y = cpu::data<std::int64_t>(output) + output.layout().offset();
    plan.for_each_output([&](Shape::size_type o, const cpu::ReductionPlan::ReductionRange &range) {
        float best = 0.0F;
        std::int64_t best_index = -1, index = 0;
        range.for_each_run([&](const cpu::ReductionPlan::Run &run) {
            Layout::offset_type off = run.offset;
            for (Shape::size_type i = 0; i < run.size; ++i, off += run.stride, ++index) {
                const float v = x[off];
                if (best_index < 0 || (!std::isnan(best) && (std::isnan(v) || v > best))) {
                    best = v;
                    best_index = index;
                }
            }
        });
        y[o] = best_index < 0 ? 0 : best_index;
    });
}

void cpu_log_softmax(DeviceRuntime &, const Primitive &primitive, std::span<const TensorView> inputs,
                     MutableTensorView output) {
    // the reference composite: logsumexp (reduction/loops.hpp:59-136), then x - lse
    const auto &p = dynamic_cast<const LogSoftmaxPrimitive &>(primitive);
    const TensorView &in = inputs.front();
    const Shape &shape = in.shape();
    const std::array<Shape::size_type, 1> axes{p.axis()};
    const cpu::ReductionPlan plan{shape, in.layout(), axes};
    if (shape.numel() == 0) return;
    const float *x = cpu::data<float>(in);
    float *y = cpu::data<float>(output);
    const Layout out_layout = output.layout();
    // output offset of the kept coordinates: contiguous output, axis extent folded in
    std::vector<std::size_t> kept;
    for (std::size_t d = 0; d < shape.rank(); ++d)
        if (d != p.axis()) kept.push_back(d);
    plan.for_each_output([&](Shape::size_type o, const cpu::ReductionPlan::ReductionRange &range) {
        float mx = -std::numeric_limits<float>::infinity();
        bool nan = false;
        range.for_each_run([&](const cpu::ReductionPlan::Run &run) {
            Layout::offset_type off = run.offset;
            for (Shape::size_type i = 0; i < run.size; ++i, off += run.stride) {
                if (std::isnan(x[off])) nan = true;
                else mx = std::max(mx, x[off]);
            }
        });
        float lse;
        if (nan) lse = std::numeric_limits<float>::quiet_NaN();
        else if (std::isinf(mx)) lse = mx;
        else {
            float s = 0.0F;
            range.for_each_run([&](const cpu::ReductionPlan::Run &run) {
                Layout::offset_type off = run.offset;
                for (Shape::size_type i = 0; i < run.size; ++i, off += run.stride) s += std::exp(x[off] - mx);
            });
            lse = mx + std::log(s);
        }
        // kept coordinates of output o
        std::size_t rem = o;
        Layout::offset_type base = out_layout.offset();
        for (std::size_t k = kept.size(); k > 0; --k) {
            const std::size_t d = kept[k - 1];
            const std::size_t e = static_cast<std::size_t>(shape[d]);
            base += static_cast<Layout::offset_type>(rem % e) * out_layout.stride(d);
            rem /= e;
        }
        Shape::size_type j = 0;
        range.for_each_run([&](const cpu::ReductionPlan::Run &run) {
            Layout::offset_type off = run.offset;
            for (Shape::size_type i = 0; i < run.size; ++i, off += run.stride, ++j)
                y[base + static_cast<Layout::offset_type>(j) * out_layout.stride(p.axis())] = x[off] - lse;
        });
    });
}

// ------------------------------------------------------------ CUDA kernels --

void cuda_relu(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
               MutableTensorView output) {
    (void)dynamic_cast<const ReluPrimitive &>(primitive);
    auto &cr = dynamic_cast<cuda::CudaRuntime &>(rt);
    cr.activate();
    const mtc_desc in = cuda::make_desc(inputs.front()), out = cuda::make_desc(output);
    cuda::check(mtc_unary(MTC_OP_RELU, &in, &out, cr.stream()), "relu kernel");
}

void cuda_max(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
              MutableTensorView output) {
    const auto &p = dynamic_cast<const MaxPrimitive &>(primitive);
    auto &cr = dynamic_cast<cuda::CudaRuntime &>(rt);
    cr.activate();
    std::vector<int64_t> axes(p.axes().begin(), p.axes().end());
    const mtc_desc in = cuda::make_desc(inputs.front()), out = cuda::make_desc(output);
    cuda::check(mtc_reduce(MTC_OP_MAX, &in, axes.data(), static_cast<int32_t>(axes.size()), &out, cr.stream()),
                "max kernel");
}

void cuda_argmax(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
                 MutableTensorView output) {
    const auto &p = dynamic_cast<const ArgMaxPrimitive &>(primitive);
    auto &cr = dynamic_cast<cuda::CudaRuntime &>(rt);
    cr.activate();
    const int64_t axis = static_cast<int64_t>(p.axis());
    const mtc_desc in = cuda::make_desc(inputs.front()), out = cuda::make_desc(output);
    cuda::check(mtc_reduce(MTC_OP_ARGMAX, &in, &axis, 1, &out, cr.stream()), "argmax kernel");
}

void cuda_log_softmax(DeviceRuntime &rt, const Primitive &primitive, std::span<const TensorView> inputs,
                      MutableTensorView output) {
    const auto &p = dynamic_cast<const LogSoftmaxPrimitive &>(primitive);
    auto &cr = dynamic_cast<cuda::CudaRuntime &>(rt);
    cr.activate();
    const mtc_desc in = cuda::make_desc(inputs.front()), out = cuda::make_desc(output);
    cuda::check(mtc_log_softmax(&in, static_cast<int64_t>(p.axis()), &out, cr.stream()), "log-softmax kernel");
}

}  // namespace

bool write_primitive_key(const Primitive &primitive, std::string &key) {
    auto put = [&key](std::int64_t v) { key.append(reinterpret_cast<const char *>(&v), sizeof(v)); };
    if (dynamic_cast<const ReluPrimitive *>(&primitive) != nullptr) return true;  // no parameters
    if (const auto *p = dynamic_cast<const MaxPrimitive *>(&primitive)) {
        put(static_cast<std::int64_t>(p->axes().size()));
        for (auto a : p->axes()) put(static_cast<std::int64_t>(a));
        put(p->keep_dim() ? 1 : 0);
        return true;
    }
    if (const auto *p = dynamic_cast<const ArgMaxPrimitive *>(&primitive)) {
        put(static_cast<std::int64_t>(p->axis()));
        put(p->keep_dim() ? 1 : 0);
        return true;
    }
    if (const auto *p = dynamic_cast<const LogSoftmaxPrimitive *>(&primitive)) {
        put(static_cast<std::int64_t>(p->axis()));
        return true;
    }
    return false;
}

void register_extension_kernels(KernelRegistry &registry) {
    registry.register_kernel({ReluPrimitive::ID, DeviceType::Cpu}, cpu_relu);
    registry.register_kernel({ReluPrimitive::ID, DeviceType::Cuda}, cuda_relu);
    registry.register_kernel({MaxPrimitive::ID, DeviceType::Cpu}, cpu_max);
    registry.register_kernel({ArgMaxPrimitive::ID, DeviceType::Cpu}, cpu_argmax);
    registry.register_kernel({LogSoftmaxPrimitive::ID, DeviceType::Cpu}, cpu_log_softmax);
    registry.register_kernel({MaxPrimitive::ID, DeviceType::Cuda}, cuda_max);
    registry.register_kernel({ArgMaxPrimitive::ID, DeviceType::Cuda}, cuda_argmax);
    registry.register_kernel({LogSoftmaxPrimitive::ID, DeviceType::Cuda}, cuda_log_softmax);
}

}  // namespace minitensor::detail::ext

namespace minitensor::detail {

// relu's VJP: the cotangent where the input is above 0, 0 where it is not
// (the derivative at 0 is taken as 0), NaN where the input is NaN.  The step
// (sign(x) + |sign(x)|) * 0.5 is built from reference ops, so the evaluator fuses
// it with the product into one kernel.  Called by the reference's VJP registry
// when it is built with this backend (the third edit of _build_host.py).
void register_backend_vjps(VjpRegistry &registry) {
    registry.register_rule<ext::ReluPrimitive>([](const ext::ReluPrimitive &, const VjpContext &context) {
        if (context.inputs.size() != 1) throw std::logic_error{"relu VJP expects 1 input"};
        const Tensor s = sign(context.inputs.front());
        return VjpContributions{context.output_cotangent * ((s + abs(s)) * 0.5F)};
    });
}

}  // namespace minitensor::detail

namespace minitensor::b200 {

Tensor relu(const Tensor &input) {
    return detail::apply_operation(std::make_unique<detail::ext::ReluPrimitive>(), input);
}

Tensor max(const Tensor &input, std::span<const Axis> axes, bool keep_dim) {
    return detail::apply_operation(std::make_unique<detail::ext::MaxPrimitive>(axes, input.rank(), keep_dim), input);
}

Tensor max(const Tensor &input, std::initializer_list<Axis> axes, bool keep_dim) {
    return max(input, std::span<const Axis>(axes.begin(), axes.size()), keep_dim);
}

Tensor argmax(const Tensor &input, Axis axis, bool keep_dim) {
    return detail::apply_operation(std::make_unique<detail::ext::ArgMaxPrimitive>(axis, input.rank(), keep_dim), input);
}

Tensor log_softmax(const Tensor &input, Axis axis) {
    return detail::apply_operation(std::make_unique<detail::ext::LogSoftmaxPrimitive>(axis, input.rank()), input);
}

}  // namespace minitensor::b200
