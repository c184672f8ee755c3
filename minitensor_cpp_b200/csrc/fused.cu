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

#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "elementwise.cuh"
#include "graph.cuh"

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

constexpr int kVariants = 9;  // flat4, flat1, strided, tiled1, tiled2, rows4, rows1, tiled4x1, tiled4x2
const char *const kNameExpr[kVariants] = {"mtc_ew_flat<MtcFused, 4>", "mtc_ew_flat<MtcFused, 1>",
                                          "mtc_ew_strided<MtcFused>", "mtc_ew_tiled<MtcFused, 1>",
                                          "mtc_ew_tiled<MtcFused, 2>", "mtc_ew_rows<MtcFused, 4>",
                                          "mtc_ew_rows<MtcFused, 1>", "mtc_ew_tiled4<MtcFused, 1>",
                                          "mtc_ew_tiled4<MtcFused, 2>"};

struct CompiledProgram {
    CUmodule module = nullptr;
    CUfunction fn = nullptr;
};

std::mutex g_cache_mutex;
std::unordered_map<std::string, std::unique_ptr<CompiledProgram>> g_cache;  // key: device + source
std::unordered_map<std::string, CompiledProgram *> g_bin_cache;               // key: program structure bytes

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
    int n_imm = 0;
    for (int i = 0; i < n_instr; ++i) {
        const mtc_instr &ins = program[i];
        if (ins.op == MTC_OP_CONST) {
            // constants are launch arguments, so programs that differ only in their
            // constants (an optimizer's per-step coefficients) share one kernel
            if (n_imm >= MTC_EW_MAX_IMM) return fail(MTC_ERR_UNSUPPORTED, "fused program has too many constants");
            snprintf(line, sizeof(line), "        r%d = imm[%d];\n", ins.dst, n_imm++);
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
    src.clear();  // the program-specific part only: kTemplateSource precedes it when compiled
    snprintf(line, sizeof(line),
             "\nstruct MtcFused {\n    static constexpr int kIn = %d;\n    static constexpr int kOut = %d;\n", n_in,
             n_out);
    src += line;
    src += "    __device__ __forceinline__ void operator()(const float *x, float *y, const float *imm) const {\n";
    src += body;
    src += "    }\n};\n";
    return MTC_OK;
}

uint64_t fnv1a(const std::string &text) {
    uint64_t h = 1469598103934665603ull;
    for (unsigned char c : text) {
        h ^= c;
        h *= 1099511628211ull;
    }
    return h;
}

// On-disk cache of compiled programs: <dir>/<hash>.cubin next to <hash>.src,
// whose text must equal the program's source (no trust in the hash alone).
std::string cache_dir() {
    const char *env = std::getenv("MTB_KERNEL_CACHE");
    if (env != nullptr) return env;
    return "/tmp/mtb_kernel_cache";
}

bool read_file(const std::string &path, std::string &out) {
    FILE *f = std::fopen(path.c_str(), "rb");
    if (!f) return false;
    std::fseek(f, 0, SEEK_END);
    const long n = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    out.resize(n > 0 ? static_cast<size_t>(n) : 0);
    const bool ok = n <= 0 || std::fread(out.data(), 1, out.size(), f) == out.size();
    std::fclose(f);
    return ok;
}

void write_file(const std::string &path, const std::string &data) {
    const std::string tmp = path + ".tmp" + std::to_string(static_cast<long long>(::getpid()));
    FILE *f = std::fopen(tmp.c_str(), "wb");
    if (!f) return;
    const bool ok = std::fwrite(data.data(), 1, data.size(), f) == data.size();
    std::fclose(f);
    if (ok) std::rename(tmp.c_str(), path.c_str());
    else std::remove(tmp.c_str());
}

// Compiles one kernel variant of a program (NVRTC, sm_100a) or loads it from the
// disk cache.  `program` is the generated MtcFused definition; the kernel
// templates precede it in the compiled source.
int compile(const std::string &program, int variant, CompiledProgram &out) {
    const std::string src = std::string(kTemplateSource) + program;
    const std::string full = src + "\n// variant " + kNameExpr[variant] + "\n";
    const std::string dir = cache_dir();
    char name[32];
    snprintf(name, sizeof(name), "%016llx", static_cast<unsigned long long>(fnv1a(full)));
    const std::string base = dir + "/" + name;
    std::string cubin, lowered, cached_src;
    if (!(read_file(base + ".src", cached_src) && cached_src == full && read_file(base + ".cubin", cubin) &&
          read_file(base + ".sym", lowered) && !cubin.empty() && !lowered.empty())) {
        nvrtcProgram prog;
        if (nvrtcCreateProgram(&prog, src.c_str(), "mtc_fused.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
            return fail(MTC_ERR_RUNTIME, "nvrtcCreateProgram failed");
        nvrtcAddNameExpression(prog, kNameExpr[variant]);
        const char *opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", "-default-device"};
        const nvrtcResult rc = nvrtcCompileProgram(prog, 3, opts);
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
        cubin.assign(cubin_size, '\0');
        nvrtcGetCUBIN(prog, cubin.data());
        const char *lname = nullptr;
        nvrtcGetLoweredName(prog, kNameExpr[variant], &lname);
        lowered = lname ? lname : "";
        nvrtcDestroyProgram(&prog);
        ::mkdir(dir.c_str(), 0777);
        write_file(base + ".cubin", cubin);
        write_file(base + ".sym", lowered);
        write_file(base + ".src", full);
    }
    Driver &d = driver();
    if (!d.ok) return fail(MTC_ERR_RUNTIME, "CUDA driver entry points for module loading are unavailable");
    MTC_CUDA_TRY(cudaFree(nullptr));  // make the primary context current
    if (d.load(&out.module, cubin.data()) != CUDA_SUCCESS)
        return fail(MTC_ERR_RUNTIME, "cuModuleLoadData failed for a fused program");
    if (d.get(&out.fn, out.module, lowered.c_str()) != CUDA_SUCCESS)
        return fail(MTC_ERR_RUNTIME, "fused kernel %s not found in module", kNameExpr[variant]);
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
    Capture *capture = active_capture();
    if (capture != nullptr && static_cast<cudaStream_t>(stream) != capture->stream)
        return fail(MTC_ERR_INVALID_ARGUMENT, "fused launch on a stream other than the recorded one");
    EwPlan plan;
    MTC_TRY(plan_elementwise(inputs, n_inputs, outputs, n_outputs, plan));
    if (plan.variant == EwVariant::Empty) {
        if (capture != nullptr) capture->fused.emplace_back();  // launches nothing
        return MTC_OK;
    }

    int n_imm = 0;
    for (int i = 0; i < n_instr && n_imm < MTC_EW_MAX_IMM; ++i)
        if (program[i].op == MTC_OP_CONST) plan.args.imm[n_imm++] = program[i].imm;
    const int device = current_device();
    int v = 0;
    switch (plan.variant) {
    case EwVariant::Flat4: v = 0; break;
    case EwVariant::Flat1: v = 1; break;
    case EwVariant::Strided: v = 2; break;
    case EwVariant::Tiled1: v = 3; break;
    case EwVariant::Tiled2: v = 4; break;
    case EwVariant::Rows4: v = 5; break;
    case EwVariant::Rows1: v = 6; break;
    case EwVariant::Tiled4x1: v = 7; break;
    case EwVariant::Tiled4x2: v = 8; break;
    default:
        if (capture != nullptr) capture->fused.emplace_back();
        return MTC_OK;
    }
    // First level: the program's structure as bytes (device, variant, operand
    // counts, output registers, and op / registers of every instruction; the
    // constants are launch arguments).  A hit skips source generation entirely.
    std::string bin;
    {
        const int32_t head[4] = {device, v, n_inputs, n_outputs};
        bin.append(reinterpret_cast<const char *>(head), sizeof(head));
        bin.append(reinterpret_cast<const char *>(out_regs), sizeof(int32_t) * static_cast<size_t>(n_outputs));
        for (int i = 0; i < n_instr; ++i) {
            const int32_t w[2] = {program[i].op, (int32_t(uint16_t(program[i].dst)) << 16) | uint16_t(program[i].a)};
            const int16_t b = program[i].b;
            bin.append(reinterpret_cast<const char *>(w), sizeof(w));
            bin.append(reinterpret_cast<const char *>(&b), sizeof(b));
        }
    }
    CompiledProgram *cp = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_cache_mutex);
        auto hit = g_bin_cache.find(bin);
        if (hit != g_bin_cache.end()) cp = hit->second;
    }
    if (cp == nullptr) {
        // Second level: the generated source text (validates the program), then
        // NVRTC or the disk cache on a miss.
        std::string src;
        MTC_TRY(generate(program, n_instr, n_inputs, out_regs, n_outputs, src));
        std::string key = std::to_string(device) + ":" + std::to_string(v) + "\n" + src;
        std::lock_guard<std::mutex> lock(g_cache_mutex);
        auto it = g_cache.find(key);
        if (it == g_cache.end()) {
            auto fresh = std::make_unique<CompiledProgram>();
            const auto t0 = std::chrono::steady_clock::now();
            MTC_TRY(compile(src, v, *fresh));
            if (std::getenv("MTB_TRACE") != nullptr)
                std::fprintf(stderr, "mtc fused program: variant %d compiled or loaded in %.1f ms\n", v,
                             std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
            it = g_cache.emplace(key, std::move(fresh)).first;
        }
        cp = it->second.get();
        g_bin_cache.emplace(std::move(bin), cp);
    }
    if (cp->fn == nullptr) return fail(MTC_ERR_LOGIC, "fused variant %d was not compiled", v);
    void *params[] = {&plan.args};
    CUresult r = driver().launch(cp->fn, plan.grid.x, plan.grid.y, plan.grid.z, plan.block.x, plan.block.y,
                                 plan.block.z, 0, static_cast<CUstream>(stream), params, nullptr);
    if (r != CUDA_SUCCESS) return fail(MTC_ERR_RUNTIME, "launch of fused kernel failed (CUresult %d)", static_cast<int>(r));
    count_launch();
    if (capture != nullptr) {
        // remember the kernel node, so replays can receive other constants
        cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
        const cudaGraphNode_t *deps = nullptr;
        size_t n_deps = 0;
        if (cudaStreamGetCaptureInfo(capture->stream, &status, nullptr, nullptr, &deps, &n_deps) != cudaSuccess ||
            status != cudaStreamCaptureStatusActive || n_deps != 1)
            return fail(MTC_ERR_RUNTIME, "the recorded fused kernel node cannot be identified");
        FusedNode f;
        f.node = deps[0];
        f.fn = cp->fn;
        f.grid = plan.grid;
        f.block = plan.block;
        f.args = plan.args;
        capture->fused.push_back(f);
    }
    return MTC_OK;
}
