// Graph evaluator for graphs with CUDA work.
//
// It keeps every observable rule of the reference Evaluator
// (src/tensor/execution/evaluator.cpp:49-206): depth-first topological plan,
// cached (materialised) values are not recomputed, shared sub-graphs run once,
// storage-sharing views need no kernel, a missing runtime or kernel throws
// before anything executes, and a failing kernel installs no storage.  On top of
// that, adjacent elementwise nodes on a CUDA device are fused:
//
//  - a cluster is a set of Float32 unary/binary elementwise nodes of one output
//    shape; a node joins the cluster of its consumers when all of its planned
//    consumers belong to that one cluster;
//  - a Float32 `Full` node whose consumers are all fused becomes an immediate
//    constant of those clusters (the rank-0 scalars of `tensor op scalar`);
//  - a member is written to memory only if something outside the cluster can
//    still see it: it is an evaluation root, a node outside the cluster consumes
//    it, or a handle outside this graph holds it (reference count above the
//    graph's own references);
//  - the cluster runs as one mtc_fused launch at the position of its last node.
// Values internal to a cluster stay unmaterialised and are recomputed from
// their producers if a later evaluation asks for them.
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <optional>
#include <stdexcept>
#include <unordered_map>
#include <utility>
#include <vector>

#include <minitensor/host_scalar.hpp>

#include "cuda_backend.hpp"
#include "tensor/core/tensor_spec.hpp"
#include "tensor/dispatch/kernel_key.hpp"
#include "tensor/graph/node.hpp"
#include "tensor/graph/primitive.hpp"
#include "tensor/graph/value.hpp"
#include "tensor/primitives/creation/full.hpp"
#include "tensor/storage/dense_size.hpp"
#include "tensor/storage/layout.hpp"
#include "tensor/storage/materialization.hpp"

namespace minitensor::detail::cuda {

EvaluatorOptions &evaluator_options() {
    static EvaluatorOptions options = [] {
        EvaluatorOptions o;
        if (const char *v = std::getenv("MTB_FUSION")) o.fusion = std::strcmp(v, "0") != 0;
        if (const char *v = std::getenv("MTB_INDEX_CHECKS")) o.check_index_errors = std::strcmp(v, "0") != 0;
        return o;
    }();
    return options;
}

EvaluatorStats &evaluator_stats() {
    static EvaluatorStats stats;
    return stats;
}

namespace {

constexpr std::uint32_t kFullId = 0x0001;
constexpr std::uint32_t kGatherId = 0x0208;
constexpr std::uint32_t kScatterAddId = 0x0209;

bool is_unary_id(std::uint32_t id) { return id >= 0x0101 && id <= 0x0108; }
bool is_binary_id(std::uint32_t id) { return id >= 0x0110 && id <= 0x0114; }

struct Step {
    ValueRef output;
    const Node *node = nullptr;
    DeviceRuntime *runtime = nullptr;  // null for view-only primitives
    const KernelFn *kernel = nullptr;
    bool on_cuda = false;
    bool fusible = false;  // Float32 elementwise node on a CUDA device
    bool constant = false; // Float32 Full node on a CUDA device
    bool folded = false;   // constant folded into the clusters of its consumers
    bool materialize = false;
    int cluster = -1;
    std::vector<int> consumers;
    int internal_refs = 0;
};

struct Cluster {
    std::vector<int> members;  // step indices, added in reverse plan order
    int root = -1;             // last member in plan order: the launch point
    Shape shape;
};

class Planner {
  public:
    Planner(const RuntimeRegistry &runtimes, const KernelRegistry &kernels) : runtimes_{runtimes}, kernels_{kernels} {}

    std::vector<Step> build(std::span<const ValueRef> roots, bool &has_cuda) {
        for (const ValueRef &v : roots) visit(v);
        has_cuda = has_cuda_;
        return std::move(plan_);
    }

    const std::unordered_map<const Value *, int> &index() const { return index_; }

  private:
    void visit(const ValueRef &value) {
        if (!value) throw std::invalid_argument{"cannot evaluate an empty value"};
        if (value->materialization() != nullptr) return;
        auto it = state_.find(value.get());
        if (it != state_.end()) {
            if (it->second == 0) throw std::logic_error{"cycle in computation graph"};
            return;
        }
        state_.emplace(value.get(), 0);
        const NodeRef &node = value->producer_ref();
        if (!node) throw std::runtime_error{"cannot evaluate unmaterialized leaf"};
        for (const ValueRef &input : node->inputs()) visit(input);
        Step step;
        step.output = value;
        step.node = node.get();
        const Primitive &primitive = node->primitive();
        const TensorSpec &spec = value->spec();
        step.on_cuda = spec.device.type() == DeviceType::Cuda;
        if (primitive.requires_kernel_support()) {
            step.runtime = &runtimes_.get(spec.device);
            step.kernel = &kernels_.get(KernelKey{primitive.id(), spec.device.type()});
        }
        if (step.on_cuda) {
            has_cuda_ = true;
            const std::uint32_t id = primitive.id().value();
            const bool f32 = spec.dtype == DType::Float32;
            step.fusible = f32 && (is_unary_id(id) || is_binary_id(id));
            step.constant = f32 && id == kFullId;
        }
        index_.emplace(value.get(), static_cast<int>(plan_.size()));
        plan_.push_back(std::move(step));
        state_[value.get()] = 1;
    }

    const RuntimeRegistry &runtimes_;
    const KernelRegistry &kernels_;
    std::unordered_map<const Value *, int> state_;
    std::unordered_map<const Value *, int> index_;
    std::vector<Step> plan_;
    bool has_cuda_ = false;
};

void execute_kernel_step(const Step &step) {
    Value &output = *step.output;
    const Node &node = *step.node;
    const Primitive &primitive = node.primitive();
    const auto inputs = node.inputs();
    std::vector<TensorView> views;
    views.reserve(inputs.size());
    for (const ValueRef &input : inputs) {
        const Materialization *m = input->materialization();
        if (m == nullptr) throw std::logic_error{"planned operation has unmaterialized input"};
        if (inputs.size() == 1) {
            auto shared = primitive.try_derive_shared_layout(input->spec(), m->layout(), output.spec());
            if (shared) {
                output.materialize(Materialization(m->buffer_ref(), std::move(*shared)));
                ++evaluator_stats().view_steps;
                return;
            }
        }
        views.emplace_back(input->spec(), *m);
    }
    if (step.kernel == nullptr) throw std::logic_error{"primitive must either share storage or plan a kernel"};
    const TensorSpec &spec = output.spec();
    BufferRef buffer = step.runtime->allocate(dense_size_bytes(spec));
    Materialization m(std::move(buffer), Layout::contiguous(spec.shape));
    {
        MutableTensorView out(spec, m);
        (*step.kernel)(*step.runtime, primitive, views, out);
    }
    output.materialize(std::move(m));
    if (step.on_cuda) ++evaluator_stats().kernel_steps;
}

class FusedEvaluator {
  public:
    FusedEvaluator(const RuntimeRegistry &runtimes, const KernelRegistry &kernels)
        : runtimes_{runtimes}, kernels_{kernels} {}

    bool run(std::span<const ValueRef> roots) {
        using clock = std::chrono::steady_clock;
        const auto t0 = clock::now();
        Planner planner(runtimes_, kernels_);
        bool has_cuda = false;
        plan_ = planner.build(roots, has_cuda);
        if (!has_cuda) return false;
        // an index error of an earlier evaluation whose snapshot has arrived
        for (const Step &s : plan_) {
            if (!s.on_cuda) continue;
            raise_device_errors(static_cast<int>(s.output->spec().device.index()), false);
            break;
        }
        index_cache_ = planner.index();
        ++evaluator_stats().evaluations;
        const auto &index = index_cache_;
        // consumers, graph-internal references and roots
        for (int i = 0; i < static_cast<int>(plan_.size()); ++i) {
            for (const ValueRef &in : plan_[i].node->inputs()) {
                auto it = index.find(in.get());
                if (it == index.end()) continue;
                plan_[it->second].consumers.push_back(i);
                ++plan_[it->second].internal_refs;
            }
        }
        for (const ValueRef &r : roots) {
            auto it = index.find(r.get());
            if (it != index.end()) plan_[it->second].materialize = true;
        }
        for (Step &s : plan_) {
            // the step itself holds one reference; anything beyond the graph's own
            // input slots means a handle outside this evaluation can see the value
            const long external = s.output.use_count() - 1 - s.internal_refs;
            if (external > 0) s.materialize = true;
        }
        if (evaluator_options().fusion) form_clusters();
        const auto t1 = clock::now();
        execute();
        const auto t2 = clock::now();
        auto &st = evaluator_stats();
        st.plan_ns += static_cast<std::uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count());
        st.execute_ns += static_cast<std::uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(t2 - t1).count());
        return true;
    }

  private:
    bool consumers_in_one_cluster(const Step &s, int &target) const {
        target = -1;
        if (s.consumers.empty()) return false;
        for (int c : s.consumers) {
            const Step &cs = plan_[c];
            if (!cs.fusible || cs.cluster < 0) return false;
            if (target == -1) target = cs.cluster;
            else if (target != cs.cluster) return false;
        }
        return true;
    }

    void form_clusters() {
        for (int i = static_cast<int>(plan_.size()) - 1; i >= 0; --i) {
            Step &s = plan_[i];
            if (s.constant && !s.materialize) {
                bool all_fused = !s.consumers.empty();
                for (int c : s.consumers) all_fused = all_fused && plan_[c].fusible && plan_[c].cluster >= 0;
                s.folded = all_fused;
                continue;
            }
            if (!s.fusible) continue;
            int target = -1;
            const Shape &shape = s.output->spec().shape;
            if (consumers_in_one_cluster(s, target) && clusters_[target].shape == shape && can_grow(target, i)) {
                clusters_[target].members.push_back(i);
                s.cluster = target;
            } else {
                Cluster c;
                c.root = i;
                c.shape = shape;
                c.members.push_back(i);
                clusters_.push_back(std::move(c));
                s.cluster = static_cast<int>(clusters_.size()) - 1;
                s.materialize = true;  // the cluster's result is always written
            }
            // a member consumed outside its cluster must be written
            for (int c : s.consumers)
                if (plan_[c].cluster != s.cluster) s.materialize = true;
        }
    }

    // Conservative operand budget: every input of every member counts as external.
    bool can_grow(int cluster, int candidate) const {
        const Cluster &c = clusters_[cluster];
        if (c.members.size() + 1 > 48) return false;
        int outputs = 0, inputs = 0;
        for (int m : c.members) {
            if (plan_[m].materialize) ++outputs;
            inputs += static_cast<int>(plan_[m].node->inputs().size());
        }
        inputs += static_cast<int>(plan_[candidate].node->inputs().size());
        if (plan_[candidate].materialize) ++outputs;
        return outputs <= MTC_MAX_FUSED_OUTPUTS && inputs - static_cast<int>(c.members.size()) <= MTC_MAX_FUSED_OPERANDS;
    }

    void execute() {
        bool index_kernels = false;
        DeviceRuntime *index_runtime = nullptr;
        static const bool trace = std::getenv("MTB_TRACE") != nullptr;
        for (int i = 0; i < static_cast<int>(plan_.size()); ++i) {
            Step &s = plan_[i];
            if (s.folded) {
                ++evaluator_stats().folded_constants;
                continue;
            }
            const auto t0 = std::chrono::steady_clock::now();
            if (s.cluster >= 0) {
                if (clusters_[s.cluster].root == i) launch_cluster(clusters_[s.cluster]);
                if (trace) report_slow(t0, "fused cluster", s);
                continue;
            }
            execute_kernel_step(s);
            if (trace) report_slow(t0, "kernel", s);
            const std::uint32_t id = s.node->primitive().id().value();
            if (s.on_cuda && (id == kGatherId || id == kScatterAddId)) {
                index_kernels = true;
                index_runtime = s.runtime;
            }
        }
        if (index_kernels && evaluator_options().check_index_errors && index_runtime != nullptr) {
            // queue a snapshot of the device error word; it is examined at the next
            // evaluation on this device or the next device-to-host read, so the
            // host does not wait for the GPU here
            auto &rt = dynamic_cast<CudaRuntime &>(*index_runtime);
            const auto c0 = std::chrono::steady_clock::now();
            check(mtc_watch_device_errors(rt.index(), rt.stream()), "device error check");
            evaluator_stats().check_ns += static_cast<std::uint64_t>(
                std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - c0).count());
        }
    }

    // MTB_TRACE: host calls of 20 ms or more (allocation, compilation or a
    // blocked launch) are reported with the primitive that made them.
    static void report_slow(std::chrono::steady_clock::time_point t0, const char *what, const Step &s) {
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if (ms >= 20.0)
            std::fprintf(stderr, "mtb slow host call: %s, primitive 0x%04x, %.1f ms\n", what,
                         static_cast<unsigned>(s.node->primitive().id().value()), ms);
    }

    // Members in plan order; registers: external inputs first, then one per
    // member and one per distinct folded constant.
    void launch_cluster(Cluster &c) {
        std::vector<int> members(c.members.rbegin(), c.members.rend());
        std::unordered_map<const Value *, int> reg;  // value -> register
        std::vector<mtc_desc> inputs;
        std::vector<mtc_instr> program;
        std::vector<int> out_steps;
        // external inputs
        for (int m : members) {
            for (const ValueRef &in : plan_[m].node->inputs()) {
                const Value *v = in.get();
                if (reg.count(v)) continue;
                auto it = plan_index(v);
                if (it >= 0 && plan_[it].cluster == plan_[m].cluster) continue;
                if (it >= 0 && plan_[it].folded) continue;
                const Materialization *mat = in->materialization();
                if (mat == nullptr) throw std::logic_error{"fused cluster has an unmaterialized input"};
                reg.emplace(v, static_cast<int>(inputs.size()));
                inputs.push_back(make_desc(TensorView(in->spec(), *mat)));
            }
        }
        int next = static_cast<int>(inputs.size());
        CudaRuntime *runtime = nullptr;
        for (int m : members) {
            const Step &s = plan_[m];
            runtime = &dynamic_cast<CudaRuntime &>(*s.runtime);
            int operand[2] = {0, 0};
            const auto ins = s.node->inputs();
            for (std::size_t k = 0; k < ins.size(); ++k) {
                const Value *v = ins[k].get();
                auto found = reg.find(v);
                if (found == reg.end()) {
                    // a folded constant: emit it once
                    const int pi = plan_index(v);
                    if (pi < 0 || !plan_[pi].folded) throw std::logic_error{"fused operand has no register"};
                    const auto &full = dynamic_cast<const FullPrimitive &>(plan_[pi].node->primitive());
                    mtc_instr ci{};
                    ci.op = MTC_OP_CONST;
                    ci.dst = static_cast<int16_t>(next);
                    ci.imm = full.fill_value().get<float>();
                    program.push_back(ci);
                    found = reg.emplace(v, next++).first;
                }
                operand[k] = found->second;
            }
            mtc_instr ins_op{};
            ins_op.op = static_cast<int32_t>(s.node->primitive().id().value());
            ins_op.dst = static_cast<int16_t>(next);
            ins_op.a = static_cast<int16_t>(operand[0]);
            ins_op.b = static_cast<int16_t>(ins.size() > 1 ? operand[1] : 0);
            program.push_back(ins_op);
            reg.emplace(s.output.get(), next++);
            if (s.materialize) out_steps.push_back(m);
        }
        if (program.size() > MTC_MAX_FUSED_INSTRUCTIONS || inputs.size() > MTC_MAX_FUSED_OPERANDS ||
            out_steps.size() > MTC_MAX_FUSED_OUTPUTS) {
            run_unfused(members);
            return;
        }
        std::vector<Materialization> mats;
        std::vector<mtc_desc> outputs;
        std::vector<int32_t> out_regs;
        for (int m : out_steps) {
            const TensorSpec &spec = plan_[m].output->spec();
            BufferRef buffer = plan_[m].runtime->allocate(dense_size_bytes(spec));
            mats.emplace_back(std::move(buffer), Layout::contiguous(spec.shape));
            out_regs.push_back(reg.at(plan_[m].output.get()));
        }
        for (std::size_t j = 0; j < out_steps.size(); ++j)
            outputs.push_back(make_desc(MutableTensorView(plan_[out_steps[j]].output->spec(), mats[j])));
        runtime->activate();
        const int rc = mtc_fused(program.data(), static_cast<int32_t>(program.size()), inputs.data(),
                                 static_cast<int32_t>(inputs.size()), out_regs.data(), outputs.data(),
                                 static_cast<int32_t>(outputs.size()), runtime->stream());
        if (rc == MTC_ERR_UNSUPPORTED) {
            // no runtime compiler available: run the members one kernel at a time
            run_unfused(members);
            return;
        }
        check(rc, "fused elementwise kernel");
        for (std::size_t j = 0; j < out_steps.size(); ++j) plan_[out_steps[j]].output->materialize(std::move(mats[j]));
        ++evaluator_stats().fused_launches;
        evaluator_stats().fused_nodes += members.size();
    }

    void run_unfused(const std::vector<int> &members) {
        for (int m : members) {
            for (const ValueRef &in : plan_[m].node->inputs()) {
                const int pi = plan_index(in.get());
                if (pi >= 0 && plan_[pi].folded && in->materialization() == nullptr) execute_kernel_step(plan_[pi]);
            }
            execute_kernel_step(plan_[m]);
        }
    }

    int plan_index(const Value *v) const {
        const auto it = index_cache_.find(v);
        return it == index_cache_.end() ? -1 : it->second;
    }

    const RuntimeRegistry &runtimes_;
    const KernelRegistry &kernels_;
    std::vector<Step> plan_;
    std::vector<Cluster> clusters_;
    std::unordered_map<const Value *, int> index_cache_;
};

}  // namespace

bool evaluate_fused(const RuntimeRegistry &runtimes, const KernelRegistry &kernels, std::span<const ValueRef> roots) {
    FusedEvaluator evaluator(runtimes, kernels);
    return evaluator.run(roots);
}

}  // namespace minitensor::detail::cuda
