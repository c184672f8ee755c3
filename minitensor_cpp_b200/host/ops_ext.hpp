// Operations this backend adds to MiniTensor's public API.  The reference has
// no ReLU, max, argmax or log-softmax primitive (its activations are tanh and
// sigmoid, its reductions sum and logsumexp); the benchmark workloads need them.
//
//  relu(x)            new primitive 0x0180: max(x, 0) for every float32 input
//                     (x > 0 passes unchanged, -0 and -inf give +0, NaN
//                     propagates); VJP cotangent * [x > 0] (0 at 0, NaN for a
//                     NaN input).  Fused with its neighbours on the GPU.
//  max(x, axes)       new primitive 0x0380: NaN propagates, empty -> -inf.
//  argmax(x, axis)    new primitive 0x0381: Int64 index of the first maximum; a
//                     NaN counts as the maximum.
//  log_softmax(x, a)  new primitive 0x0382: x - logsumexp(x, {a}, keep_dim=true),
//                     one pass over memory on the GPU.
// max, argmax and log-softmax have no VJP rule (the workloads do not
// differentiate them); grad() through them raises the reference's missing-rule
// error.
#pragma once

#include <initializer_list>
#include <span>
#include <string>

#include <minitensor/tensor.hpp>
#include <minitensor/types.hpp>

namespace minitensor::detail {
class KernelRegistry;
class Primitive;
class VjpRegistry;
// relu's VJP rule; the reference's VJP registry calls this hook (weak there)
// after its own rules when it is built with this backend.
void register_backend_vjps(VjpRegistry &registry);
}

namespace minitensor::b200 {

[[nodiscard]] Tensor relu(const Tensor &input);
[[nodiscard]] Tensor max(const Tensor &input, std::span<const Axis> axes, bool keep_dim = false);
[[nodiscard]] Tensor max(const Tensor &input, std::initializer_list<Axis> axes, bool keep_dim = false);
[[nodiscard]] Tensor argmax(const Tensor &input, Axis axis, bool keep_dim = false);
[[nodiscard]] Tensor log_softmax(const Tensor &input, Axis axis);

}  // namespace minitensor::b200

namespace minitensor::detail::ext {
// CPU and CUDA kernels of the new primitives.
void register_extension_kernels(KernelRegistry &registry);
// Appends the parameters of a new primitive to a plan key (axes, keep_dim);
// false when `primitive` is none of them.
bool write_primitive_key(const Primitive &primitive, std::string &key);
}  // namespace minitensor::detail::ext
