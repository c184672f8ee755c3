// Fused elementwise programs (mtc_fused).
//
// A program is a short list of register instructions produced by the graph
// evaluator from a cluster of adjacent elementwise nodes.  For each distinct
// program a CUDA C functor is generated, compiled for sm_100a with NVRTC
// together with the same kernel templates the precompiled ops use
// (ew_kernels.cuh), loaded once per device and cached for the process.  The
// whole cluster then costs one pass over HBM instead of one pass per node.
#include <cuda.h>
#include <nvrtc.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "elementwise.cuh"

namespace mtc {
namespace {

const char *const kTemplateSource =
#include "ew_kernels_src.inc"
    ;

using PFN_ModuleLoadData = CUresult (*)(CUmodule *, const void *);
using PFN_ModuleGetFunction = CUresult (*)(CUfunction *, CUmodule, const char *);
using PFN_LaunchKernel = CUresult (*)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                                      CUstream, void **, void **);

struct Driver {
    PFN_ModuleLoadData load = nullptr;
    PFN_ModuleGetFunction get = nullptr;
    PFN_LaunchKernel launch = nullptr;
    bool ok = false;
};

Driver &driver() {
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuModuleLoadData", &p, cudaEnableDefault, &q) == cudaSuccess && p)
            d.load = reinterpret_cast<PFN_ModuleLoadData>(p);
        if (cudaGetDriverEntryPoint("cuModuleGetFunction", &p, cudaEnableDefault, &q) == cudaSuccess && p)
            d.get = reinterpret_cast<PFN_ModuleGetFunction>(p);
        if (cudaGetDriverEntryPoint("cuLaunchKernel", &p, cudaEnableDefault, &q) == cudaSuccess && p)
            d.launch = reinterpret_cast<PFN_LaunchKernel>(p);
        d.ok = d.load && d.get && d.launch;
    });
    return d;
}

constexpr int kVariants = 5;  // flat4, flat1, strided, tiled1, tiled2
const char *const kNameExpr[kVariants] = {"mtc_ew_flat<MtcFused, 4>", "mtc_ew_flat<MtcFused, 1>",
                                          "mtc_ew_strided<MtcFused>", "mtc_ew_tiled<MtcFused, 1>",
                                          "mtc_ew_tiled<MtcFused, 2>"};

struct CompiledProgram {
    CUmodule module = nullptr;
    CUfunction fn[kVariants] = {};
};

std::mutex g_cache_mutex;
std::unordered_map<std::string, std::unique_ptr<CompiledProgram>> g_cache;  // key: device + source

bool is_unary(int op) {
    return (op >= MTC_OP_ABS && op <= MTC_OP_SIGMOID) || op == MTC_OP_RELU;
}
bool is_binary(int op) { return op >= MTC_OP_ADD && op <= MTC_OP_LOGADDEXP; }

int generate(const mtc_instr *program, int n_instr, int n_in, const int32_t *out_regs, int n_out, std::string &src) {
    int n_reg = n_in;
    for (int i = 0; i < n_instr; ++i) {
        const mtc_instr &ins = program[i];
        if (ins.dst < 0 || ins.a < 0 || ins.b < 0 || ins.dst >= 256 || ins.a >= 256 || ins.b >= 256)
            return fail(MTC_ERR_INVALID_ARGUMENT, "fused instruction %d: register out of range", i);
        n_reg = std::max<int>(n_reg, ins.dst + 1);
        if (!(ins.op == MTC_OP_CONST || is_unary(ins.op) || is_binary(ins.op)))
            return fail(MTC_ERR_INVALID_ARGUMENT, "fused instruction %d: unknown op 0x%04x", i, ins.op);
    }
    std::vector<bool> written(n_reg, false);
    for (int k = 0; k < n_in; ++k) written[k] = true;
    std::string body;
    char line[160];
    if (n_reg > 0) {
        body += "        float ";
        for (int r = 0; r < n_reg; ++r) {
            snprintf(line, sizeof(line), "%sr%d", r ? ", " : "", r);
            body += line;
        }
        body += ";\n";
    }
    for (int k = 0; k < n_in; ++k) {
        snprintf(line, sizeof(line), "        r%d = x[%d];\n", k, k);
        body += line;
    }
    for (int i = 0; i < n_instr; ++i) {
        const mtc_instr &ins = program[i];
        if (ins.op == MTC_OP_CONST) {
            uint32_t bits;
            std::memcpy(&bits, &ins.imm, 4);
            snprintf(line, sizeof(line), "        r%d = __int_as_float(0x%08xu);\n", ins.dst, bits);
        } else if (is_unary(ins.op)) {
            if (ins.a >= n_reg || !written[ins.a])
                return fail(MTC_ERR_INVALID_ARGUMENT, "fused instruction %d reads an unwritten register", i);
            snprintf(line, sizeof(line), "        r%d = mtc_unary<0x%04x>(r%d);\n", ins.dst, ins.op, ins.a);
        } else {
            if (ins.a >= n_reg || ins.b >= n_reg || !written[ins.a] || !written[ins.b])
                return fail(MTC_ERR_INVALID_ARGUMENT, "fused instruction %d reads an unwritten register", i);
            snprintf(line, sizeof(line), "        r%d = mtc_binary<0x%04x>(r%d, r%d);\n", ins.dst, ins.op, ins.a, ins.b);
        }
        written[ins.dst] = true;
        body += line;
    }
    for (int j = 0; j < n_out; ++j) {
        if (out_regs[j] < 0 || out_regs[j] >= n_reg || !written[out_regs[j]])
            return fail(MTC_ERR_INVALID_ARGUMENT, "fused output %d reads an unwritten register", j);
        snprintf(line, sizeof(line), "        y[%d] = r%d;\n", j, out_regs[j]);
        body += line;
    }
    src = kTemplateSource;
    snprintf(line, sizeof(line),
             "\nstruct MtcFused {\n    static constexpr int kIn = %d;\n    static constexpr int kOut = %d;\n", n_in,
             n_out);
    src += line;
    src += "    __device__ __forceinline__ void operator()(const float *x, float *y) const {\n";
    src += body;
    src += "    }\n};\n";
    return MTC_OK;
}

int compile(const std::string &src, int n_in, CompiledProgram &out) {
    nvrtcProgram prog;
    if (nvrtcCreateProgram(&prog, src.c_str(), "mtc_fused.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
        return fail(MTC_ERR_RUNTIME, "nvrtcCreateProgram failed");
    const int variants = n_in >= 2 ? kVariants : kVariants - 1;
    for (int v = 0; v < variants; ++v) nvrtcAddNameExpression(prog, kNameExpr[v]);
    const char *opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", "-default-device"};
    nvrtcResult rc = nvrtcCompileProgram(prog, 3, opts);
    if (rc != NVRTC_SUCCESS) {
        size_t n = 0;
        nvrtcGetProgramLogSize(prog, &n);
        std::string log(n, '\0');
        nvrtcGetProgramLog(prog, log.data());
        nvrtcDestroyProgram(&prog);
        return fail(MTC_ERR_UNSUPPORTED, "NVRTC could not compile the fused program: %s", log.c_str());
    }
    size_t cubin_size = 0;
    nvrtcGetCUBINSize(prog, &cubin_size);
    std::vector<char> cubin(cubin_size);
    nvrtcGetCUBIN(prog, cubin.data());
    std::vector<std::string> lowered(variants);
    for (int v = 0; v < variants; ++v) {
        const char *name = nullptr;
        nvrtcGetLoweredName(prog, kNameExpr[v], &name);
        lowered[v] = name ? name : "";
    }
    nvrtcDestroyProgram(&prog);

    Driver &d = driver();
    if (!d.ok) return fail(MTC_ERR_RUNTIME, "CUDA driver entry points for module loading are unavailable");
    MTC_CUDA_TRY(cudaFree(nullptr));  // make the primary context current
    if (d.load(&out.module, cubin.data()) != CUDA_SUCCESS)
        return fail(MTC_ERR_RUNTIME, "cuModuleLoadData failed for a fused program");
    for (int v = 0; v < variants; ++v) {
        if (d.get(&out.fn[v], out.module, lowered[v].c_str()) != CUDA_SUCCESS)
            return fail(MTC_ERR_RUNTIME, "fused kernel %s not found in module", kNameExpr[v]);
    }
    return MTC_OK;
}

}  // namespace
}  // namespace mtc

using namespace mtc;

extern "C" int mtc_fused(const mtc_instr *program, int32_t n_instr, const mtc_desc *inputs, int32_t n_inputs,
                         const int32_t *out_regs, const mtc_desc *outputs, int32_t n_outputs, void *stream) {
    clear_error();
    if (n_instr < 0 || n_instr > MTC_MAX_FUSED_INSTRUCTIONS)
        return fail(MTC_ERR_INVALID_ARGUMENT, "fused program length %d outside [0, %d]", n_instr,
                    MTC_MAX_FUSED_INSTRUCTIONS);
    if (n_inputs < 0 || n_inputs > MTC_MAX_FUSED_OPERANDS || n_outputs < 1 || n_outputs > MTC_MAX_FUSED_OUTPUTS)
        return fail(MTC_ERR_INVALID_ARGUMENT, "fused operand counts %d/%d out of range", n_inputs, n_outputs);
    if ((n_instr > 0 && program == nullptr) || out_regs == nullptr)
        return fail(MTC_ERR_INVALID_ARGUMENT, "null fused program");
    EwPlan plan;
    MTC_TRY(plan_elementwise(inputs, n_inputs, outputs, n_outputs, plan));
    if (plan.variant == EwVariant::Empty) return MTC_OK;

    std::string src;
    MTC_TRY(generate(program, n_instr, n_inputs, out_regs, n_outputs, src));
    const int device = current_device();
    std::string key = std::to_string(device) + "\n" + src.substr(std::strlen(kTemplateSource));
    CompiledProgram *cp = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_cache_mutex);
        auto it = g_cache.find(key);
        if (it == g_cache.end()) {
            auto fresh = std::make_unique<CompiledProgram>();
            MTC_TRY(compile(src, n_inputs, *fresh));
            it = g_cache.emplace(key, std::move(fresh)).first;
        }
        cp = it->second.get();
    }
    int v = 0;
    switch (plan.variant) {
    case EwVariant::Flat4: v = 0; break;
    case EwVariant::Flat1: v = 1; break;
    case EwVariant::Strided: v = 2; break;
    case EwVariant::Tiled1: v = 3; break;
    case EwVariant::Tiled2: v = 4; break;
    default: return MTC_OK;
    }
    if (cp->fn[v] == nullptr) return fail(MTC_ERR_LOGIC, "fused variant %d was not compiled", v);
    void *params[] = {&plan.args};
    CUresult r = driver().launch(cp->fn[v], plan.grid.x, plan.grid.y, plan.grid.z, plan.block.x, plan.block.y,
                                 plan.block.z, 0, static_cast<CUstream>(stream), params, nullptr);
    if (r != CUDA_SUCCESS) return fail(MTC_ERR_RUNTIME, "launch of fused kernel failed (CUresult %d)", static_cast<int>(r));
    return MTC_OK;
}
