// Operations this backend adds to MiniTensor's public API.  The reference has
// no ReLU, max, argmax or log-softmax primitive (its activations are tanh and
// sigmoid, its reductions sum and logsumexp); the benchmark workloads need them.
//
//  relu(x)            composite (x + |x|) * 0.5 of reference ops: exact ReLU in
//                     float32 for finite x (-0 -> +0), NaN propagates, and -inf
//                     gives NaN (-inf + inf); differentiable through the
//                     reference's own VJP rules (gradient 0.5 at 0), and one
//                     fused kernel on the GPU.
//  max(x, axes)       new primitive 0x0380: NaN propagates, empty -> -inf.
//  argmax(x, axis)    new primitive 0x0381: Int64 index of the first maximum; a
//                     NaN counts as the maximum.
//  log_softmax(x, a)  new primitive 0x0382: x - logsumexp(x, {a}, keep_dim=true),
//                     one pass over memory on the GPU.
// None of the three new primitives has a VJP rule (they are not differentiated
// by the workloads); grad() through them raises the reference's missing-rule error.
#pragma once

#include <initializer_list>
#include <span>
#include <string>

#include <minitensor/tensor.hpp>
#include <minitensor/types.hpp>

namespace minitensor::detail {
class KernelRegistry;
class Primitive;
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
