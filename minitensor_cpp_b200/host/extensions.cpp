// The two hooks the MiniTensor execution environment calls when it is built
// with this backend (src/tensor/execution/environment.cpp, ExecutionEnvironment's
// constructor and evaluate(); the build adds the calls, see _build_host.py):
//  - register_backend_extensions: one CudaRuntime per visible GPU
//    (Device::cuda(i)) and the CUDA kernels, next to the CPU runtime and kernels
//    the reference registers itself (environment.cpp:16-20);
//  - evaluate_with_backend_extensions: graphs that touch a CUDA device go to the
//    fusing evaluator; pure-CPU graphs stay with the reference Evaluator.
#include <memory>
#include <span>

#include "cuda_backend.hpp"
#include "ops_ext.hpp"

namespace minitensor::detail {

void register_backend_extensions(RuntimeRegistry &runtimes, KernelRegistry &kernels) {
    const int n = cuda::device_count();
    for (int i = 0; i < n; ++i) {
        runtimes.register_runtime(std::make_unique<cuda::CudaRuntime>(Device::cuda(static_cast<std::uint32_t>(i))));
    }
    cuda::register_cuda_kernels(kernels);
    ext::register_extension_kernels(kernels);
}

bool evaluate_with_backend_extensions(const RuntimeRegistry &runtimes, const KernelRegistry &kernels,
                                      std::span<const ValueRef> roots) {
    return cuda::evaluate_fused(runtimes, kernels, roots);
}

}  // namespace minitensor::detail
