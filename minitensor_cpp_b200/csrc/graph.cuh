// Recording state shared by the allocator (runtime.cu), the fused launcher
// (fused.cu) and the graph entry points (graph.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "ew_kernels.cuh"

namespace mtc {

// One mtc_fused launch inside a recording: what is needed to relaunch the same
// kernel node with other constants.  node == nullptr: the call launched nothing.
struct FusedNode {
    cudaGraphNode_t node = nullptr;
    CUfunction fn = nullptr;
    dim3 grid, block;
    MtcEwArgs args;
};

struct Capture {
    int device = -1;
    cudaStream_t stream = nullptr;
    uint64_t launches_at_begin = 0;
    std::vector<void *> retained;  // blocks released while recording: the graph keeps them
    std::vector<FusedNode> fused;
};

// The calling thread's recording, or nullptr.
Capture *active_capture();
void set_active_capture(Capture *c);
// Kernels launched by this library so far.
uint64_t launches_so_far();
// Adds `n` (negative: removes) to the launch counter.
void count_launches(int64_t n);
// Returns a block to the allocator as mtc_free would, even while recording.
int release_block(int device, void *ptr, cudaStream_t stream);

}  // namespace mtc
