// Graph replay of recorded launch sequences (mtc_capture_* / mtc_graph_*).
//
// The evaluator of a repeated plan records its launches once with stream
// capture and afterwards replays them as one CUDA graph: one launch call
// instead of one per kernel, and none of the host work that builds each
// kernel's arguments.  What a replay may touch is fixed at recording time:
//  - operand buffers: the caller guarantees that a replay sees the same input
//    buffers and has taken back (mtc_pool_take) the output blocks of the
//    recording;
//  - workspaces released while recording stay allocated and belong to the
//    graph (runtime.cu keeps them out of the pool);
//  - per-step constants of fused elementwise programs are patched into their
//    kernel nodes (mtc_graph_set_constants), so an optimizer step whose bias
//    corrections change every step replays the same graph.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "graph.cuh"

struct mtc_graph {
    int device = -1;
    cudaStream_t stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint64_t launches = 0;
    std::vector<void *> retained;
    std::vector<mtc::FusedNode> fused;
};

namespace mtc {
namespace {

using PFN_ExecKernelNodeSetParams = CUresult (*)(CUgraphExec, CUgraphNode, const CUDA_KERNEL_NODE_PARAMS *);

PFN_ExecKernelNodeSetParams set_params_fn() {
    static PFN_ExecKernelNodeSetParams fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuGraphExecKernelNodeSetParams", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<PFN_ExecKernelNodeSetParams>(nullptr);
        return reinterpret_cast<PFN_ExecKernelNodeSetParams>(p);
    }();
    return fn;
}

// Blocks a discarded or destroyed recording kept: back to the pool, in the
// order of `stream`.
void release_all(int device, cudaStream_t stream, std::vector<void *> &blocks) {
    for (void *p : blocks) (void)release_block(device, p, stream);
    blocks.clear();
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" {

int mtc_capture_begin(int device, void *stream) {
    clear_error();
    if (active_capture() != nullptr) return fail(MTC_ERR_LOGIC, "a recording is already active on this thread");
    if (stream == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "recording needs a non-default stream");
    if (profiling()) return fail(MTC_ERR_UNSUPPORTED, "GEMM profiling is on (its events cannot be recorded)");
    int cur = -1;
    MTC_CUDA_TRY(cudaGetDevice(&cur));
    if (cur != device) return fail(MTC_ERR_INVALID_ARGUMENT, "device %d is not current (%d is)", device, cur);
    auto c = std::make_unique<Capture>();
    c->device = device;
    c->stream = static_cast<cudaStream_t>(stream);
    c->launches_at_begin = launches_so_far();
    // relaxed: the allocator may still call cudaMalloc for a block it lacks
    MTC_CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
    set_active_capture(c.release());
    return MTC_OK;
}

int mtc_capture_fused_count(int32_t *count) {
    Capture *c = active_capture();
    if (c == nullptr) return fail(MTC_ERR_LOGIC, "no recording is active on this thread");
    *count = static_cast<int32_t>(c->fused.size());
    return MTC_OK;
}

int mtc_capture_end(int keep, mtc_graph **out) {
    clear_error();
    *out = nullptr;
    std::unique_ptr<Capture> c(active_capture());
    if (!c) return fail(MTC_ERR_LOGIC, "no recording is active on this thread");
    set_active_capture(nullptr);
    cudaGraph_t graph = nullptr;
    const cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
    const int64_t recorded = static_cast<int64_t>(launches_so_far() - c->launches_at_begin);
    // launches are counted when they run: at every mtc_graph_launch
    count_launches(-recorded);
    if (e != cudaSuccess || graph == nullptr || !keep) {
        cudaGetLastError();
        if (graph) cudaGraphDestroy(graph);
        release_all(c->device, c->stream, c->retained);
        if (!keep) return MTC_OK;
        return fail(MTC_ERR_RUNTIME, "stream capture failed: %s", cudaGetErrorString(e));
    }
    auto g = std::make_unique<mtc_graph>();
    g->device = c->device;
    g->stream = c->stream;
    g->graph = graph;
    g->launches = static_cast<uint64_t>(recorded);
    g->retained = std::move(c->retained);
    g->fused = std::move(c->fused);
    const cudaError_t ie = cudaGraphInstantiate(&g->exec, graph, 0);
    if (ie != cudaSuccess) {
        cudaGetLastError();
        cudaGraphDestroy(graph);
        release_all(g->device, g->stream, g->retained);
        return fail(MTC_ERR_RUNTIME, "graph instantiation failed: %s", cudaGetErrorString(ie));
    }
    *out = g.release();
    return MTC_OK;
}

int mtc_graph_launch(mtc_graph *g) {
    clear_error();
    if (g == nullptr || g->exec == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null graph");
    MTC_CUDA_TRY(cudaGraphLaunch(g->exec, g->stream));
    count_launches(static_cast<int64_t>(g->launches));
    return MTC_OK;
}

int mtc_graph_launches(const mtc_graph *g, uint64_t *count) {
    if (g == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null graph");
    *count = g->launches;
    return MTC_OK;
}

int mtc_graph_set_constants(mtc_graph *g, int32_t index, const float *imm, int32_t n_imm) {
    clear_error();
    if (g == nullptr || g->exec == nullptr) return fail(MTC_ERR_INVALID_ARGUMENT, "null graph");
    if (index < 0 || index >= static_cast<int32_t>(g->fused.size()))
        return fail(MTC_ERR_INVALID_ARGUMENT, "fused launch %d was not recorded", index);
    if (n_imm < 0 || n_imm > MTC_EW_MAX_IMM || (n_imm > 0 && imm == nullptr))
        return fail(MTC_ERR_INVALID_ARGUMENT, "%d constants outside [0, %d]", n_imm, MTC_EW_MAX_IMM);
    FusedNode &f = g->fused[index];
    if (f.node == nullptr) return MTC_OK;  // the call launched nothing (empty index space)
    std::memcpy(f.args.imm, imm, sizeof(float) * static_cast<size_t>(n_imm));
    PFN_ExecKernelNodeSetParams set = set_params_fn();
    if (set == nullptr) return fail(MTC_ERR_RUNTIME, "cuGraphExecKernelNodeSetParams is unavailable");
    void *params[] = {&f.args};
    CUDA_KERNEL_NODE_PARAMS p;
    std::memset(&p, 0, sizeof(p));
    p.func = f.fn;
    p.gridDimX = f.grid.x;
    p.gridDimY = f.grid.y;
    p.gridDimZ = f.grid.z;
    p.blockDimX = f.block.x;
    p.blockDimY = f.block.y;
    p.blockDimZ = f.block.z;
    p.kernelParams = params;
    const CUresult r = set(reinterpret_cast<CUgraphExec>(g->exec), reinterpret_cast<CUgraphNode>(f.node), &p);
    if (r != CUDA_SUCCESS) return fail(MTC_ERR_RUNTIME, "updating a fused kernel node failed (CUresult %d)", int(r));
    return MTC_OK;
}

int mtc_graph_destroy(mtc_graph *g) {
    if (g == nullptr) return MTC_OK;
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != g->device) cudaSetDevice(g->device);
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    release_all(g->device, g->stream, g->retained);
    if (cur >= 0 && cur != g->device) cudaSetDevice(cur);
    delete g;
    return MTC_OK;
}

}  // extern "C"
