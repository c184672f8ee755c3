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
#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <optional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include <minitensor/host_scalar.hpp>

#include "cuda_backend.hpp"
#include "ops_ext.hpp"
#include "tensor/core/tensor_spec.hpp"
#include "tensor/dispatch/kernel_key.hpp"
#include "tensor/graph/node.hpp"
#include "tensor/graph/primitive.hpp"
#include "tensor/graph/value.hpp"
#include "tensor/primitives/creation/full.hpp"
#include "tensor/primitives/creation/normal.hpp"
#include "tensor/primitives/creation/uniform.hpp"
#include "tensor/primitives/manipulation/basic_index.hpp"
#include "tensor/primitives/manipulation/concatenate.hpp"
#include "tensor/primitives/manipulation/gather.hpp"
#include "tensor/primitives/manipulation/permute.hpp"
#include "tensor/primitives/reduction/logsumexp.hpp"
#include "tensor/primitives/reduction/sum.hpp"
#include "tensor/random_key_access.hpp"
#include "tensor/storage/dense_size.hpp"
#include "tensor/storage/layout.hpp"
#include "tensor/storage/materialization.hpp"

namespace minitensor::detail::cuda {

EvaluatorOptions &evaluator_options() {
    static EvaluatorOptions options = [] {
        EvaluatorOptions o;
        if (const char *v = std::getenv("MTB_FUSION")) o.fusion = std::strcmp(v, "0") != 0;
        if (const char *v = std::getenv("MTB_INDEX_CHECKS")) {
            o.check_index_errors = std::strcmp(v, "0") != 0;
            o.sync_index_checks = std::strcmp(v, "sync") == 0;
        }
        if (const char *v = std::getenv("MTB_GRAPHS")) o.graphs = std::strcmp(v, "0") != 0;
        if (const char *v = std::getenv("MTB_GRAPH_MAX_BYTES")) o.graph_max_bytes = std::strtoull(v, nullptr, 10);
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
constexpr std::uint32_t kAddId = 0x0110;

// reference unary ops 0x0101-0x0108 and this backend's relu 0x0180 (MTC_OP_RELU)
bool is_unary_id(std::uint32_t id) { return (id >= 0x0101 && id <= 0x0108) || id == 0x0180; }
bool is_binary_id(std::uint32_t id) { return id >= 0x0110 && id <= 0x0114; }

// Open-addressing map from graph values to plan positions.  A plan visits a
// few hundred values per evaluation; std::unordered_map's node allocations and
// the copy of the planner's map cost a third of the host time of planning.
class ValueIndex {
  public:
    // Position of `v`, or nullptr when absent.
    int *find(const Value *v) {
        if (keys_.empty()) return nullptr;
        for (std::size_t i = slot(v);; i = (i + 1) & mask_) {
            if (keys_[i] == v) return &vals_[i];
            if (keys_[i] == nullptr) return nullptr;
        }
    }
    const int *find(const Value *v) const { return const_cast<ValueIndex *>(this)->find(v); }
    // Inserts (v, value) when absent; returns the stored value and whether it was inserted.
    std::pair<int *, bool> emplace(const Value *v, int value) {
        if (2 * (size_ + 1) > keys_.size()) grow();
        for (std::size_t i = slot(v);; i = (i + 1) & mask_) {
            if (keys_[i] == v) return {&vals_[i], false};
            if (keys_[i] == nullptr) {
                keys_[i] = v;
                vals_[i] = value;
                ++size_;
                return {&vals_[i], true};
            }
        }
    }

  private:
    std::size_t slot(const Value *v) const {
        auto x = static_cast<std::uint64_t>(reinterpret_cast<std::uintptr_t>(v));
        x ^= x >> 33;
        x *= 0xff51afd7ed558ccdULL;
        x ^= x >> 33;
        return static_cast<std::size_t>(x) & mask_;
    }
    void grow() {
        std::vector<const Value *> keys = std::move(keys_);
        std::vector<int> vals = std::move(vals_);
        const std::size_t cap = keys.empty() ? 256 : 2 * keys.size();
        keys_.assign(cap, nullptr);
        vals_.assign(cap, 0);
        mask_ = cap - 1;
        size_ = 0;
        for (std::size_t i = 0; i < keys.size(); ++i)
            if (keys[i] != nullptr) emplace(keys[i], vals[i]);
    }
    std::vector<const Value *> keys_;
    std::vector<int> vals_;
    std::size_t size_ = 0;
    std::size_t mask_ = 0;
};

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
    // a scatter-add deferred into the cluster rooted at this step: the cluster
    // reads 0 in its place and the updates are then added into its output
    int into = -1;
    int internal_refs = 0;  // input slots of planned nodes that read this value
};

struct Cluster {
    std::vector<int> members;  // step indices, added in reverse plan order
    int root = -1;             // last member in plan order: the launch point
    Shape shape;
    int outputs = 0;                     // members written
    std::vector<const Value *> external;  // distinct values read from outside the members
    std::vector<const Value *> constants; // distinct Full inputs (folded into the program)
};

class Planner {
  public:
    Planner(const RuntimeRegistry &runtimes, const KernelRegistry &kernels) : runtimes_{runtimes}, kernels_{kernels} {}

    std::vector<Step> build(std::span<const ValueRef> roots, bool &has_cuda) {
        for (const ValueRef &v : roots) visit(v);
        has_cuda = has_cuda_;
        return std::move(plan_);
    }

    // Plan position of every planned value (moved out: call once, after build).
    ValueIndex take_index() { return std::move(index_); }

  private:
    void visit(const ValueRef &value) {
        if (!value) throw std::invalid_argument{"cannot evaluate an empty value"};
        if (value->materialization() != nullptr) return;
        // -1 while the value's inputs are being visited, then its plan position
        auto [pos, fresh] = index_.emplace(value.get(), -1);
        if (!fresh) {
            if (*pos < 0) throw std::logic_error{"cycle in computation graph"};
            return;
        }
        const NodeRef &node = value->producer_ref();
        if (!node) throw std::runtime_error{"cannot evaluate unmaterialized leaf"};
        for (const ValueRef &input : node->inputs()) visit(input);
        Step step;
        step.output = value;
        step.node = node.get();
        const Primitive &primitive = node->primitive();
        const TensorSpec &spec = value->spec();
        step.on_cuda = spec.device.type() == DeviceType::Cuda;
        if (primitive.requires_kernel_support()) lookup(primitive, spec.device, step);
        if (step.on_cuda) {
            has_cuda_ = true;
            const std::uint32_t id = primitive.id().value();
            const bool f32 = spec.dtype == DType::Float32;
            step.fusible = f32 && (is_unary_id(id) || is_binary_id(id));
            step.constant = f32 && id == kFullId;
        }
        *index_.find(value.get()) = static_cast<int>(plan_.size());
        plan_.push_back(std::move(step));
    }

    // The registries' runtime and kernel for (primitive, device), remembered
    // for this plan: a plan has a few hundred nodes but a few dozen kinds.
    void lookup(const Primitive &primitive, const Device &device, Step &step) {
        const std::uint32_t id = primitive.id().value();
        for (const Known &k : known_)
            if (k.id == id && k.device == device) {
                step.runtime = k.runtime;
                step.kernel = k.kernel;
                return;
            }
        step.runtime = &runtimes_.get(device);
        step.kernel = &kernels_.get(KernelKey{primitive.id(), device.type()});
        known_.push_back(Known{id, device, step.runtime, step.kernel});
    }

    struct Known {
        std::uint32_t id;
        Device device;
        DeviceRuntime *runtime;
        const KernelFn *kernel;
    };

    const RuntimeRegistry &runtimes_;
    const KernelRegistry &kernels_;
    ValueIndex index_;
    std::vector<Known> known_;
    std::vector<Step> plan_;
    bool has_cuda_ = false;
};

// ------------------------------------------------------------- plan replay --
//
// A plan that repeats (a training step builds the same graph every step) is
// recorded once with stream capture and then replayed as one CUDA graph.  The
// key of a plan is its structure (every step's primitive, parameters, output
// spec, fusion decisions and input references) together with the data
// pointers and layouts of its leaf inputs.  A replay is sound because:
//  - an equal key means the same launches on the same operands, except for the
//    outputs and the constants folded into fused programs;
//  - the outputs are the very blocks the recording wrote, taken back from the
//    allocator (mtc_pool_take) before the replay; when one is still in use the
//    evaluation runs eagerly instead;
//  - folded constants (an optimizer's per-step coefficients) are compared with
//    the recorded ones and patched into their kernel nodes before the replay.
// When a plan is recorded while an earlier recording of the same structure
// exists, and that recording's outputs are this plan's leaves (the parameters
// of step t+1 are outputs of step t), the new outputs are placed in the blocks
// the earlier recording read.  The two recordings then alternate: every later
// step finds its leaves where one of them expects them.

// Appends plain values to a byte key.  Writes go through a cursor into a
// buffer grown by doubling: a plan key takes a few thousand small writes.
struct KeyWriter {
    std::string bytes;
    std::size_t used = 0;
    template <typename T>
    void pod(const T &v) {
        if (bytes.size() - used < sizeof(T)) bytes.resize(bytes.empty() ? 4096 : 2 * bytes.size());
        std::memcpy(bytes.data() + used, &v, sizeof(T));
        used += sizeof(T);
    }
    void raw(const void *p, std::size_t n) {
        while (bytes.size() - used < n) bytes.resize(bytes.empty() ? 4096 : 2 * bytes.size());
        std::memcpy(bytes.data() + used, p, n);
        used += n;
    }
    // The key: the bytes written so far.
    void finish() { bytes.resize(used); }
    void shape(const Shape &s) {
        pod(static_cast<std::uint32_t>(s.rank()));
        for (Extent e : s.dimensions()) pod(static_cast<std::int64_t>(e));
    }
    void layout(const Layout &l) {
        pod(static_cast<std::int64_t>(l.offset()));
        pod(static_cast<std::uint32_t>(l.rank()));
        for (auto st : l.strides()) pod(static_cast<std::int64_t>(st));
    }
    template <typename Seq>
    void seq(const Seq &v) {
        pod(static_cast<std::uint32_t>(v.size()));
        for (const auto &x : v) pod(static_cast<std::int64_t>(x));
    }
};

// Writes the parameters of `primitive` that shape its launches.  False for a
// primitive this evaluator does not know: such plans are never recorded.
bool write_parameters(const Primitive &primitive, std::uint32_t id, bool folded, KeyWriter &w) {
    switch (id) {
    case 0x0001: {  // Full; a folded value is a fused constant, patched at replay
        if (folded) return true;
        const HostScalar &v = dynamic_cast<const FullPrimitive &>(primitive).fill_value();
        w.pod(static_cast<std::uint8_t>(v.dtype()));
        if (v.dtype() == DType::Float32) w.pod(v.get<float>());
        else w.pod(v.get<std::int64_t>());
        return true;
    }
    case 0x0002: {
        const auto &u = dynamic_cast<const UniformPrimitive &>(primitive);
        const auto &k = RandomKeyAccess::words(u.key());
        w.pod(u.low());
        w.pod(u.high());
        w.pod(k[0]);
        w.pod(k[1]);
        return true;
    }
    case 0x0003: {
        const auto &n = dynamic_cast<const NormalPrimitive &>(primitive);
        const auto &k = RandomKeyAccess::words(n.key());
        w.pod(n.mean());
        w.pod(n.std_dev());
        w.pod(k[0]);
        w.pod(k[1]);
        return true;
    }
    case 0x0203: w.seq(dynamic_cast<const PermutePrimitive &>(primitive).permutation()); return true;
    case 0x0205: w.pod(static_cast<std::uint64_t>(dynamic_cast<const ConcatenatePrimitive &>(primitive).axis())); return true;
    case 0x0206: {  // the slice as a layout over a contiguous input
        const auto &p = dynamic_cast<const BasicIndexPrimitive &>(primitive).parameters();
        w.layout(p.derive_layout(Layout::contiguous(p.input_shape())));
        return true;
    }
    case 0x0207: {
        const auto &p = dynamic_cast<const BasicIndexScatterPrimitive &>(primitive).parameters();
        w.layout(p.derive_layout(Layout::contiguous(p.input_shape())));
        return true;
    }
    case 0x0208: w.pod(static_cast<std::uint64_t>(dynamic_cast<const GatherPrimitive &>(primitive).axis())); return true;
    case 0x0209:
        w.pod(static_cast<std::uint64_t>(dynamic_cast<const GatherScatterAddPrimitive &>(primitive).axis()));
        return true;
    case 0x0301: {
        const auto &r = dynamic_cast<const SumPrimitive &>(primitive);
        w.seq(r.axes());
        w.pod(static_cast<std::uint8_t>(r.keep_dim()));
        return true;
    }
    case 0x0302: {
        const auto &r = dynamic_cast<const LogSumExpPrimitive &>(primitive);
        w.seq(r.axes());
        w.pod(static_cast<std::uint8_t>(r.keep_dim()));
        return true;
    }
    case 0x0201:  // Contiguous, Reshape, BroadcastTo, Matmul: the specs say it all
    case 0x0202:
    case 0x0204:
    case 0x0401: return true;
    default: {
        if (is_unary_id(id) || is_binary_id(id)) return true;
        std::string ext_key;
        if (!ext::write_primitive_key(primitive, ext_key)) return false;
        w.raw(ext_key.data(), ext_key.size());
        return true;
    }
    }
}

// One materialisation a recorded plan installs, in execution order.
struct Install {
    int step = -1;
    bool view = false;
    void *ptr = nullptr;  // buffer: the block the recording wrote
    std::size_t bytes = 0;
    std::optional<Layout> layout;  // view: the layout over its input's buffer
};

// The folded constants of one recorded fused launch.
struct FusedConstants {
    std::int32_t index = 0;     // position among the recording's mtc_fused calls
    std::vector<int> steps;     // plan steps of the Full nodes, in program order
    std::vector<float> values;  // what the kernel node holds now
};

// Bytes of blocks protected for recordings, over all of them (bounded by
// kMaxProtectedBytes; guarded by the cache mutex).
std::size_t g_protected_bytes = 0;
constexpr std::size_t kMaxProtectedBytes = std::size_t(1) << 30;

struct Recording {
    int device = -1;
    std::vector<const void *> leaves;
    mtc_graph *graph = nullptr;
    std::vector<Install> installs;
    std::vector<FusedConstants> constants;
    bool index_kernels = false;
    EvaluatorStats work;  // evaluator counters of one evaluation of the plan
    // Blocks this recording reads (leaves) or writes (outputs).  They are
    // protected in the allocator: once released they wait for this recording's
    // replays (and the next recording of the plan) instead of serving other
    // requests, so the outputs are free whenever the plan comes back.
    std::vector<void *> protected_blocks;
    std::size_t protected_bytes = 0;
    // the output blocks a replay takes back, in one allocator call
    std::vector<void *> take_ptrs;
    std::vector<std::size_t> take_bytes;
    Recording() = default;
    Recording(const Recording &) = delete;
    Recording &operator=(const Recording &) = delete;
    ~Recording() {
        for (void *p : protected_blocks) (void)mtc_pool_protect(device, p, -1);
        g_protected_bytes -= protected_bytes;
        if (graph != nullptr) (void)mtc_graph_destroy(graph);
    }
    void protect(void *p, std::size_t bytes) {
        if (p == nullptr || mtc_pool_protect(device, p, 1) != MTC_OK) return;
        protected_blocks.push_back(p);
        protected_bytes += bytes;
        g_protected_bytes += bytes;
    }
};

struct PlanHistory {
    int seen = 0;
    std::uint64_t captures = 0;
    std::uint64_t replays = 0;
    std::uint64_t fallbacks = 0;
    bool disabled = false;
    std::vector<std::unique_ptr<Recording>> recordings;
};

constexpr std::size_t kMaxRecordings = 4;  // per plan structure
constexpr std::size_t kMaxPlans = 256;

struct GraphCache {
    std::mutex mu;
    std::unordered_map<std::string, PlanHistory> plans;
};

GraphCache &graph_cache() {
    // never destroyed: graphs must not be freed after the CUDA runtime at exit
    static GraphCache *cache = new GraphCache;
    return *cache;
}

void add_work(EvaluatorStats &to, const EvaluatorStats &w) {
    to.kernel_steps += w.kernel_steps;
    to.fused_launches += w.fused_launches;
    to.fused_nodes += w.fused_nodes;
    to.folded_constants += w.folded_constants;
    to.view_steps += w.view_steps;
}

// MTB_TRACE: why a plan is not recorded or a recording failed.
void trace_graph(const char *what, const char *detail) {
    static const bool on = std::getenv("MTB_TRACE") != nullptr;
    if (on) std::fprintf(stderr, "mtb plan replay: %s%s%s\n", what, detail[0] ? ": " : "", detail);
}

EvaluatorStats work_between(const EvaluatorStats &before, const EvaluatorStats &after) {
    EvaluatorStats w;
    w.kernel_steps = after.kernel_steps - before.kernel_steps;
    w.fused_launches = after.fused_launches - before.fused_launches;
    w.fused_nodes = after.fused_nodes - before.fused_nodes;
    w.folded_constants = after.folded_constants - before.folded_constants;
    w.view_steps = after.view_steps - before.view_steps;
    return w;
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
        index_cache_ = planner.take_index();
        ++evaluator_stats().evaluations;
        // consumers (one flat array, ascending per producer), graph-internal
        // references and roots
        const int n = static_cast<int>(plan_.size());
        cons_off_.assign(static_cast<std::size_t>(n) + 1, 0);
        for (int i = 0; i < n; ++i)
            for (const ValueRef &in : plan_[i].node->inputs()) {
                const int pi = plan_index(in.get());
                if (pi >= 0) ++cons_off_[static_cast<std::size_t>(pi) + 1];
            }
        for (int i = 0; i < n; ++i) cons_off_[i + 1] += cons_off_[i];
        cons_.assign(static_cast<std::size_t>(cons_off_[n]), 0);
        std::vector<int> fill(cons_off_.begin(), cons_off_.end() - 1);
        for (int i = 0; i < n; ++i)
            for (const ValueRef &in : plan_[i].node->inputs()) {
                const int pi = plan_index(in.get());
                if (pi < 0) continue;
                cons_[fill[pi]++] = i;
                ++plan_[pi].internal_refs;
            }
        for (const ValueRef &r : roots) {
            const int pi = plan_index(r.get());
            if (pi >= 0) plan_[pi].materialize = true;
        }
        for (Step &s : plan_) {
            // the step itself holds one reference; anything beyond the graph's own
            // input slots means a handle outside this evaluation can see the value
            const long external = s.output.use_count() - 1 - s.internal_refs;
            if (external > 0) s.materialize = true;
        }
        if (evaluator_options().fusion) form_clusters();
        const auto t1 = clock::now();
        if (!(evaluator_options().graphs && run_recorded())) execute();
        const auto t2 = clock::now();
        auto &st = evaluator_stats();
        st.plan_ns += static_cast<std::uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count());
        st.execute_ns += static_cast<std::uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(t2 - t1).count());
        return true;
    }

  private:
    // The planned consumers of step i, in plan order.
    std::span<const int> consumers(int i) const {
        return {cons_.data() + cons_off_[i], static_cast<std::size_t>(cons_off_[i + 1] - cons_off_[i])};
    }

    bool consumers_in_one_cluster(int i, int &target) const {
        target = -1;
        const auto cs_of = consumers(i);
        if (cs_of.empty()) return false;
        for (int c : cs_of) {
            const Step &cs = plan_[c];
            if (!cs.fusible || cs.cluster < 0) return false;
            if (target == -1) target = cs.cluster;
            else if (target != cs.cluster) return false;
        }
        return true;
    }

    // The gather VJP (rules/manipulation.cpp:81-91) with one index per position
    // along its axis, whose output only an elementwise Add at a cluster's root
    // reads -- in cross entropy, dLoss/dlogits = g * exp(x - lse) + scatter(-g):
    // instead of zero-filling [B, C], scattering into it and reading it back,
    // the cluster reads the constant 0 in its place and the updates are added
    // into the cluster's output afterwards (mtc_gather_scatter_add_into).  Bit
    // for bit the same: every target element receives at most one update, and
    // (y + 0) + (0 + u) equals y + (0 + u) in float32, signed zeros included.
    void defer_scatter(int i) {
        Step &s = plan_[i];
        if (!s.on_cuda || s.materialize || s.node->primitive().id().value() != kScatterAddId) return;
        const auto cons = consumers(i);
        if (cons.size() != 1) return;
        const int c = cons.front();
        const Step &cs = plan_[c];
        if (cs.cluster < 0 || clusters_[cs.cluster].root != c || cs.node->primitive().id().value() != kAddId) return;
        int uses = 0;
        for (const ValueRef &in : cs.node->inputs()) uses += in.get() == s.output.get() ? 1 : 0;
        if (uses != 1 || s.output->spec().shape != cs.output->spec().shape) return;
        const auto &scatter = dynamic_cast<const GatherScatterAddPrimitive &>(s.node->primitive());
        const auto ins = s.node->inputs();
        if (ins.size() != 2 || ins[1]->spec().shape[scatter.axis()] != 1) return;
        s.into = c;
    }

    void form_clusters() {
        for (int i = static_cast<int>(plan_.size()) - 1; i >= 0; --i) {
            Step &s = plan_[i];
            if (s.constant && !s.materialize) {
                bool all_fused = !consumers(i).empty();
                for (int c : consumers(i)) all_fused = all_fused && plan_[c].fusible && plan_[c].cluster >= 0;
                s.folded = all_fused;
                continue;
            }
            if (!s.fusible) {
                defer_scatter(i);
                continue;
            }
            int target = -1;
            const Shape &shape = s.output->spec().shape;
            Budget b;
            if (consumers_in_one_cluster(i, target) && clusters_[target].shape == shape && can_grow(target, i, b)) {
                Cluster &c = clusters_[target];
                c.members.push_back(i);
                c.external = std::move(b.external);
                c.constants = std::move(b.constants);
                if (s.materialize) ++c.outputs;
                s.cluster = target;
            } else {
                s.materialize = true;  // the cluster's result is always written
                b = with_member(-1, i);
                Cluster c;
                c.root = i;
                c.shape = shape;
                c.members.push_back(i);
                c.outputs = 1;
                c.external = std::move(b.external);
                c.constants = std::move(b.constants);
                clusters_.push_back(std::move(c));
                s.cluster = static_cast<int>(clusters_.size()) - 1;
            }
            // a member consumed outside its cluster must be written
            for (int c : consumers(i))
                if (plan_[c].cluster != s.cluster) s.materialize = true;
        }
    }

    // Operand budget: the distinct values the cluster would read from outside
    // itself once the candidate joins (constants fold into the program), its
    // outputs and its program length.  The earlier count, every input of every
    // member less one per member, split AdamW's update (four external tensors,
    // about sixteen operations) into four kernels moving about 51 bytes a
    // parameter instead of one moving 28.  A cluster that still ends up over
    // budget at launch (a constant that was not folded) runs unfused.  The
    // lists are kept per cluster and updated as members join, since planning
    // runs for every evaluation, replayed ones included.
    struct Budget {
        std::vector<const Value *> external, constants;
    };

    // The budget of `c` (cluster index, or -1 for a new cluster) with step i added.
    Budget with_member(int c, int i) const {
        Budget b;
        if (c >= 0) {
            b.external = clusters_[c].external;
            b.constants = clusters_[c].constants;
            const Value *own = plan_[i].output.get();  // now produced inside
            b.external.erase(std::remove(b.external.begin(), b.external.end(), own), b.external.end());
        }
        for (const ValueRef &in : plan_[i].node->inputs()) {
            const Value *v = in.get();
            const int pi = plan_index(v);
            if (pi >= 0 && c >= 0 && plan_[pi].cluster == c) continue;
            auto &set = pi >= 0 && plan_[pi].constant ? b.constants : b.external;
            if (std::find(set.begin(), set.end(), v) == set.end()) set.push_back(v);
        }
        return b;
    }

    bool can_grow(int cluster, int candidate, Budget &b) const {
        const Cluster &c = clusters_[cluster];
        if (c.members.size() + 1 > 48) return false;
        if (c.outputs + (plan_[candidate].materialize ? 1 : 0) > MTC_MAX_FUSED_OUTPUTS) return false;
        b = with_member(cluster, candidate);
        // the program: one instruction per member and per folded constant
        const std::size_t instructions = c.members.size() + 1 + b.constants.size();
        return static_cast<int>(b.external.size()) <= MTC_MAX_FUSED_OPERANDS &&
               instructions <= static_cast<std::size_t>(MTC_MAX_FUSED_INSTRUCTIONS);
    }

    // --------------------------------------------------------- eager steps --

    // The materialisation of `v` as this evaluation sees it: while recording,
    // outputs are held back until the recorded graph has run.
    const Materialization *mat_of(const Value *v) const {
        if (capturing_) {
            const int pi = plan_index(v);
            if (pi >= 0 && pending_[pi]) return &*pending_[pi];
        }
        return v->materialization();
    }

    void install(int pi, Materialization m, bool view) {
        if (!capturing_) {
            plan_[pi].output->materialize(std::move(m));
            return;
        }
        m.validate(plan_[pi].output->spec());
        Install rec;
        rec.step = pi;
        rec.view = view;
        if (view) {
            rec.layout = m.layout();
        } else {
            const auto *b = dynamic_cast<const CudaBuffer *>(m.buffer_ref().get());
            if (b == nullptr) throw std::logic_error{"a recorded output is not a device buffer"};
            rec.ptr = b->data();
            rec.bytes = b->size_bytes();
        }
        installs_.push_back(std::move(rec));
        pending_[pi].emplace(std::move(m));
    }

    BufferRef allocate_output(int pi, std::size_t bytes) {
        if (capturing_ && !reserved_.empty()) {
            auto r = reserved_.find(pi);
            if (r != reserved_.end() && r->second->size_bytes() == bytes) {
                BufferRef b = std::move(r->second);
                reserved_.erase(r);
                return b;
            }
        }
        return plan_[pi].runtime->allocate(bytes);
    }

    void execute_step(int pi) {
        Step &step = plan_[pi];
        Value &output = *step.output;
        const Node &node = *step.node;
        const Primitive &primitive = node.primitive();
        const auto inputs = node.inputs();
        std::vector<TensorView> views;
        views.reserve(inputs.size());
        for (const ValueRef &input : inputs) {
            const Materialization *m = mat_of(input.get());
            if (m == nullptr) throw std::logic_error{"planned operation has unmaterialized input"};
            if (inputs.size() == 1) {
                auto shared = primitive.try_derive_shared_layout(input->spec(), m->layout(), output.spec());
                if (shared) {
                    install(pi, Materialization(m->buffer_ref(), std::move(*shared)), true);
                    ++evaluator_stats().view_steps;
                    return;
                }
            }
            views.emplace_back(input->spec(), *m);
        }
        if (step.kernel == nullptr) throw std::logic_error{"primitive must either share storage or plan a kernel"};
        const TensorSpec &spec = output.spec();
        Materialization m(allocate_output(pi, dense_size_bytes(spec)), Layout::contiguous(spec.shape));
        {
            MutableTensorView out(spec, m);
            (*step.kernel)(*step.runtime, primitive, views, out);
        }
        if (step.on_cuda && evaluator_options().sync_index_checks) {
            const std::uint32_t id = primitive.id().value();
            if (id == kGatherId || id == kScatterAddId) check_index_now(*step.runtime, id);
        }
        install(pi, std::move(m), false);
        if (step.on_cuda) ++evaluator_stats().kernel_steps;
    }

    void execute() {
        index_kernels_ = false;
        index_runtime_ = nullptr;
        static const bool trace = std::getenv("MTB_TRACE") != nullptr;
        for (int i = 0; i < static_cast<int>(plan_.size()); ++i) {
            Step &s = plan_[i];
            if (s.folded) {
                ++evaluator_stats().folded_constants;
                continue;
            }
            if (s.into >= 0) continue;  // added by its consumer's cluster launch
            const auto t0 = std::chrono::steady_clock::now();
            if (s.cluster >= 0) {
                if (clusters_[s.cluster].root == i) launch_cluster(clusters_[s.cluster]);
                if (trace) report_slow(t0, "fused cluster", s);
                continue;
            }
            execute_step(i);
            if (trace) report_slow(t0, "kernel", s);
            const std::uint32_t id = s.node->primitive().id().value();
            if (s.on_cuda && (id == kGatherId || id == kScatterAddId)) {
                index_kernels_ = true;
                index_runtime_ = s.runtime;
            }
        }
        if (!capturing_) watch_index_errors();
    }

    // Synchronous index check (MTB_INDEX_CHECKS=sync): waits for the kernel just
    // queued and throws std::out_of_range before its output is installed.
    static void check_index_now(DeviceRuntime &runtime, std::uint32_t id) {
        auto &rt = dynamic_cast<CudaRuntime &>(runtime);
        const auto c0 = std::chrono::steady_clock::now();
        std::int64_t detail = 0;
        const int rc = mtc_check_device_errors(rt.index(), rt.stream(), &detail);
        evaluator_stats().check_ns += static_cast<std::uint64_t>(
            std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - c0).count());
        // the reference kernels' messages (copy/loops.hpp:208, :288)
        if (rc == MTC_ERR_OUT_OF_RANGE)
            throw std::out_of_range{id == kGatherId ? "gather index is out of range"
                                                    : "gather scatter add index is out of range"};
        check(rc, "device error check");
    }

    // Queues a snapshot of the device error word after an evaluation that ran
    // an index kernel; it is examined at the next evaluation on this device or
    // the next device-to-host read, so the host does not wait for the GPU here.
    void watch_index_errors() {
        if (!index_kernels_ || !evaluator_options().check_index_errors || index_runtime_ == nullptr) return;
        auto &rt = dynamic_cast<CudaRuntime &>(*index_runtime_);
        const auto c0 = std::chrono::steady_clock::now();
        check(mtc_watch_device_errors(rt.index(), rt.stream()), "device error check");
        evaluator_stats().check_ns += static_cast<std::uint64_t>(
            std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - c0).count());
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
        std::vector<int> const_steps;
        std::vector<float> const_values;
        int deferred = -1;  // a scatter-add added into the root's output afterwards
        // external inputs
        for (int m : members) {
            for (const ValueRef &in : plan_[m].node->inputs()) {
                const Value *v = in.get();
                if (reg.count(v)) continue;
                auto it = plan_index(v);
                if (it >= 0 && plan_[it].cluster == plan_[m].cluster) continue;
                if (it >= 0 && (plan_[it].folded || plan_[it].into >= 0)) continue;
                const Materialization *mat = mat_of(v);
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
                if (found == reg.end() && plan_index(v) >= 0 && plan_[plan_index(v)].into >= 0) {
                    // a deferred scatter-add: 0 here, its updates added afterwards
                    mtc_instr zi{};
                    zi.op = MTC_OP_CONST;
                    zi.dst = static_cast<int16_t>(next);
                    zi.imm = 0.0f;
                    program.push_back(zi);
                    deferred = plan_index(v);
                    found = reg.emplace(v, next++).first;
                }
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
                    const_steps.push_back(pi);
                    const_values.push_back(ci.imm);
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
        const Materialization *scatter_upd = nullptr, *scatter_idx = nullptr;
        if (deferred >= 0) {
            const auto sin = plan_[deferred].node->inputs();
            scatter_upd = mat_of(sin[0].get());
            scatter_idx = mat_of(sin[1].get());
            if (scatter_upd == nullptr || scatter_idx == nullptr)
                throw std::logic_error{"deferred scatter-add has an unmaterialized input"};
        }
        std::vector<Materialization> mats;
        std::vector<mtc_desc> outputs;
        std::vector<int32_t> out_regs;
        for (int m : out_steps) {
            const TensorSpec &spec = plan_[m].output->spec();
            mats.emplace_back(allocate_output(m, dense_size_bytes(spec)), Layout::contiguous(spec.shape));
            out_regs.push_back(reg.at(plan_[m].output.get()));
        }
        for (std::size_t j = 0; j < out_steps.size(); ++j)
            outputs.push_back(make_desc(MutableTensorView(plan_[out_steps[j]].output->spec(), mats[j])));
        runtime->activate();
        int32_t recorded_before = 0;
        if (capturing_) check(mtc_capture_fused_count(&recorded_before), "recording");
        const int rc = mtc_fused(program.data(), static_cast<int32_t>(program.size()), inputs.data(),
                                 static_cast<int32_t>(inputs.size()), out_regs.data(), outputs.data(),
                                 static_cast<int32_t>(outputs.size()), runtime->stream());
        if (rc == MTC_ERR_UNSUPPORTED) {
            // no runtime compiler available: run the members one kernel at a time
            run_unfused(members);
            return;
        }
        check(rc, "fused elementwise kernel");
        if (deferred >= 0) {
            const Step &sc = plan_[deferred];
            const auto sin = sc.node->inputs();
            const mtc_desc upd = make_desc(TensorView(sin[0]->spec(), *scatter_upd));
            const mtc_desc idx = make_desc(TensorView(sin[1]->spec(), *scatter_idx));
            std::size_t j = 0;
            while (out_steps[j] != c.root) ++j;
            const mtc_desc out = outputs[j];
            const auto axis = static_cast<int64_t>(
                dynamic_cast<const GatherScatterAddPrimitive &>(sc.node->primitive()).axis());
            check(mtc_gather_scatter_add_into(&upd, &idx, axis, &out, runtime->stream()), "scatter-add into");
            if (evaluator_options().sync_index_checks) check_index_now(*runtime, kScatterAddId);
            index_kernels_ = true;
            index_runtime_ = runtime;
            ++evaluator_stats().kernel_steps;
            ++evaluator_stats().scatters_deferred;
        }
        if (capturing_) {
            int32_t recorded_after = 0;
            check(mtc_capture_fused_count(&recorded_after), "recording");
            if (recorded_after != recorded_before + 1) capture_unsafe_ = true;
            else if (!const_steps.empty())
                constants_.push_back(FusedConstants{recorded_before, std::move(const_steps), std::move(const_values)});
        }
        for (std::size_t j = 0; j < out_steps.size(); ++j) install(out_steps[j], std::move(mats[j]), false);
        ++evaluator_stats().fused_launches;
        evaluator_stats().fused_nodes += members.size();
    }

    void run_unfused(const std::vector<int> &members) {
        // the folded constants become kernels with their values built in: a
        // recording of them could not follow later values
        if (capturing_) capture_unsafe_ = true;
        for (int m : members) {
            for (const ValueRef &in : plan_[m].node->inputs()) {
                const int pi = plan_index(in.get());
                if (pi >= 0 && (plan_[pi].folded || plan_[pi].into >= 0) && mat_of(in.get()) == nullptr) {
                    execute_step(pi);
                    if (plan_[pi].into >= 0) {
                        index_kernels_ = true;
                        index_runtime_ = plan_[pi].runtime;
                    }
                }
            }
            execute_step(m);
        }
    }

    int plan_index(const Value *v) const {
        const int *p = index_cache_.find(v);
        return p == nullptr ? -1 : *p;
    }

    // ---------------------------------------------------------- recording --

    // The plan's key (structure bytes) and its leaves' data pointers; false
    // when the plan is not recorded (host steps, several devices, an unknown
    // primitive, outputs above MTB_GRAPH_MAX_BYTES).
    bool plan_key(KeyWriter &w, std::vector<const void *> &leaves, CudaRuntime *&rt) {
        leaf_values_.clear();
        int device = -1;
        std::size_t out_bytes = 0;
        ValueIndex leaf_slot;
        w.bytes.resize(plan_.size() * 64);
        for (int i = 0; i < static_cast<int>(plan_.size()); ++i) {
            const Step &s = plan_[i];
            if (!s.on_cuda) return trace_graph("not recorded", "a step runs on the host"), false;
            const TensorSpec &spec = s.output->spec();
            const int dev = static_cast<int>(spec.device.index());
            if (device < 0) device = dev;
            else if (dev != device) return trace_graph("not recorded", "steps on several devices"), false;
            if (rt == nullptr && s.runtime != nullptr) rt = dynamic_cast<CudaRuntime *>(s.runtime);
            const Primitive &primitive = s.node->primitive();
            const std::uint32_t id = primitive.id().value();
            if ((id == kGatherId || id == kScatterAddId) && evaluator_options().sync_index_checks)
                return trace_graph("not recorded", "synchronous index checks"), false;
            w.pod(id);
            w.pod(static_cast<std::uint8_t>(spec.dtype));
            w.shape(spec.shape);
            w.pod(static_cast<std::uint8_t>((s.materialize ? 1 : 0) | (s.folded ? 2 : 0) | (s.into >= 0 ? 4 : 0)));
            w.pod(static_cast<std::int32_t>(s.cluster));
            if (!write_parameters(primitive, id, s.folded, w)) {
                trace_graph("not recorded, unknown primitive", std::string(primitive.name()).c_str());
                return false;
            }
            const auto ins = s.node->inputs();
            w.pod(static_cast<std::uint32_t>(ins.size()));
            for (const ValueRef &in : ins) {
                const int pi = plan_index(in.get());
                if (pi >= 0) {
                    w.pod(static_cast<std::int32_t>(pi));
                    continue;
                }
                auto [slot, fresh] = leaf_slot.emplace(in.get(), static_cast<int>(leaves.size()));
                if (fresh) {
                    leaf_values_.push_back(in.get());
                    const Materialization *m = in->materialization();
                    const auto *b = m != nullptr ? dynamic_cast<const CudaBuffer *>(m->buffer_ref().get()) : nullptr;
                    if (b == nullptr || static_cast<int>(b->device().index()) != device)
                        return trace_graph("not recorded", "a leaf is not a buffer of the plan's device"), false;
                    leaves.push_back(b->data());
                    w.pod(std::int32_t{-1});  // a new leaf: its spec and layout
                    w.pod(static_cast<std::uint8_t>(in->spec().dtype));
                    w.shape(in->spec().shape);
                    w.layout(m->layout());
                }
                w.pod(static_cast<std::int32_t>(-2 - *slot));
            }
            if (s.materialize && s.kernel != nullptr) out_bytes += dense_size_bytes(spec);
        }
        if (rt == nullptr || device < 0) return trace_graph("not recorded", "no device runtime"), false;
        if (out_bytes > evaluator_options().graph_max_bytes) return false;  // launch overhead does not matter
        w.pod(device);
        w.finish();
        return true;
    }

    bool run_recorded() {
        KeyWriter key;
        std::vector<const void *> leaves;
        CudaRuntime *rt = nullptr;
        if (!plan_key(key, leaves, rt)) return false;
        GraphCache &cache = graph_cache();
        std::lock_guard<std::mutex> lock(cache.mu);
        if (cache.plans.size() >= kMaxPlans && cache.plans.count(key.bytes) == 0) cache.plans.clear();
        PlanHistory &h = cache.plans[key.bytes];
        if (h.disabled) return false;
        static const bool trace = std::getenv("MTB_TRACE") != nullptr;
        char note[96];
        for (auto &r : h.recordings) {
            if (r->leaves != leaves) continue;
            if (replay(*r, *rt)) {
                ++h.replays;
                ++evaluator_stats().graph_replays;
                return true;
            }
            // an output block is still in use: this evaluation runs eagerly
            ++h.fallbacks;
            ++evaluator_stats().graph_fallbacks;
            if (trace) {
                std::snprintf(note, sizeof(note), "plan of %zu steps, %s", plan_.size(), mtc_last_error());
                trace_graph("recorded outputs in use", note);
            }
            if (h.fallbacks > 16 && h.fallbacks > h.replays) h.disabled = true;
            return false;
        }
        if (trace) {
            std::snprintf(note, sizeof(note), "plan of %zu steps, %zu leaves, seen %d, %zu recordings", plan_.size(),
                          leaves.size(), h.seen + 1, h.recordings.size());
            trace_graph("no recording matches", note);
        }
        if (++h.seen < 2) return false;  // a plan seen once is not recorded
        if (h.captures >= 4 * kMaxRecordings && h.replays < h.captures) {
            h.disabled = true;  // the leaves never come back to recorded blocks
            return false;
        }
        if (g_protected_bytes > kMaxProtectedBytes) {
            trace_graph("not recorded", "recordings already protect the allowed memory");
            return false;
        }
        return record(h, leaves, *rt);
    }

    bool record(PlanHistory &h, const std::vector<const void *> &leaves, CudaRuntime &rt) {
        reserved_.clear();
        if (!h.recordings.empty()) {
            // outputs of the previous recording that are leaves here: the outputs
            // of the same steps go to the blocks that recording read in their
            // place.  They are taken now, before any intermediate of this
            // evaluation can be given one of them.
            const Recording &prev = *h.recordings.back();
            std::unordered_map<const void *, const Install *> out_of;
            for (const Install &in : prev.installs)
                if (!in.view && in.ptr != nullptr) out_of.emplace(in.ptr, &in);
            for (std::size_t i = 0; i < leaves.size() && i < prev.leaves.size(); ++i) {
                auto f = out_of.find(leaves[i]);
                if (f == out_of.end() || reserved_.count(f->second->step)) continue;
                void *block = const_cast<void *>(prev.leaves[i]);
                if (mtc_pool_take(rt.index(), block, f->second->bytes, rt.stream()) == MTC_OK)
                    reserved_.emplace(f->second->step, rt.adopt(block, f->second->bytes));
            }
        }
        const EvaluatorStats before = evaluator_stats();
        auto restore = [&] {
            EvaluatorStats &st = evaluator_stats();
            st.kernel_steps = before.kernel_steps;
            st.fused_launches = before.fused_launches;
            st.fused_nodes = before.fused_nodes;
            st.folded_constants = before.folded_constants;
            st.view_steps = before.view_steps;
        };
        rt.activate();
        if (mtc_capture_begin(rt.index(), rt.stream()) != MTC_OK) {
            trace_graph("recording could not start", mtc_last_error());
            h.disabled = true;
            return false;
        }
        capturing_ = true;
        capture_unsafe_ = false;
        pending_.assign(plan_.size(), std::nullopt);
        installs_.clear();
        constants_.clear();
        bool ok = true;
        try {
            execute();
        } catch (const std::exception &e) {
            trace_graph("recording failed", e.what());
            ok = false;
        }
        capturing_ = false;
        if (capture_unsafe_) trace_graph("not recorded", "constants run as kernels (no runtime compiler)");
        ok = ok && !capture_unsafe_;
        mtc_graph *graph = nullptr;
        const int rc = mtc_capture_end(ok ? 1 : 0, &graph);
        reserved_.clear();  // blocks reserved for outputs this plan did not write
        auto rec = std::make_unique<Recording>();
        rec->graph = graph;
        if (ok && (rc != MTC_OK || graph == nullptr)) trace_graph("recording failed", mtc_last_error());
        if (!ok || rc != MTC_OK || graph == nullptr || mtc_graph_launch(graph) != MTC_OK) {
            // nothing ran: drop the held-back outputs; the caller evaluates eagerly
            pending_.clear();
            installs_.clear();
            restore();
            h.disabled = true;
            return false;
        }
        for (const Install &in : installs_) plan_[in.step].output->materialize(std::move(*pending_[in.step]));
        pending_.clear();
        rec->device = rt.index();
        for (const Install &in : installs_)
            if (!in.view) rec->protect(in.ptr, in.bytes);
        for (std::size_t i = 0; i < leaves.size(); ++i) {
            // the leaf's whole buffer (a view may start at an offset)
            const Value *v = leaf_values_[i];
            const auto *b = dynamic_cast<const CudaBuffer *>(v->materialization()->buffer_ref().get());
            rec->protect(const_cast<void *>(leaves[i]), b != nullptr ? b->size_bytes() : 0);
        }
        rec->leaves = leaves;
        for (const Install &in : installs_) {
            if (in.view || in.bytes == 0) continue;
            rec->take_ptrs.push_back(in.ptr);
            rec->take_bytes.push_back(in.bytes);
        }
        rec->installs = std::move(installs_);
        rec->constants = std::move(constants_);
        rec->index_kernels = index_kernels_;
        rec->work = work_between(before, evaluator_stats());
        watch_index_errors();
        ++h.captures;
        ++evaluator_stats().graph_captures;
        if (h.recordings.size() >= kMaxRecordings) h.recordings.erase(h.recordings.begin());
        h.recordings.push_back(std::move(rec));
        return true;
    }

    bool replay(Recording &r, CudaRuntime &rt) {
        const int device = rt.index();
        void *stream = rt.stream();
        // every output block at once, or none (some value still holds one)
        int32_t failed = -1;
        if (!r.take_ptrs.empty() &&
            mtc_pool_take_many(device, r.take_ptrs.data(), r.take_bytes.data(), static_cast<int32_t>(r.take_ptrs.size()),
                               stream, &failed) != MTC_OK)
            return false;
        std::vector<BufferRef> taken(r.installs.size());
        for (std::size_t k = 0; k < r.installs.size(); ++k) {
            const Install &in = r.installs[k];
            if (!in.view) taken[k] = rt.adopt(in.bytes != 0 ? in.ptr : nullptr, in.bytes);
        }
        for (FusedConstants &fc : r.constants) {
            bool changed = false;
            for (std::size_t j = 0; j < fc.steps.size(); ++j) {
                const float v =
                    dynamic_cast<const FullPrimitive &>(plan_[fc.steps[j]].node->primitive()).fill_value().get<float>();
                if (std::memcmp(&v, &fc.values[j], sizeof(float)) != 0) {
                    fc.values[j] = v;
                    changed = true;
                }
            }
            if (changed)
                check(mtc_graph_set_constants(r.graph, fc.index, fc.values.data(), static_cast<int32_t>(fc.values.size())),
                      "recorded fused constants");
        }
        rt.activate();
        check(mtc_graph_launch(r.graph), "recorded plan");
        for (std::size_t k = 0; k < r.installs.size(); ++k) {
            const Install &in = r.installs[k];
            const Value &out = *plan_[in.step].output;
            if (in.view) {
                const Materialization *src = plan_[in.step].node->inputs()[0]->materialization();
                if (src == nullptr) throw std::logic_error{"recorded view has an unmaterialized input"};
                out.materialize(Materialization(src->buffer_ref(), *in.layout));
            } else {
                out.materialize(Materialization(std::move(taken[k]), Layout::contiguous(out.spec().shape)));
            }
        }
        index_kernels_ = r.index_kernels;
        index_runtime_ = &rt;
        watch_index_errors();
        add_work(evaluator_stats(), r.work);
        return true;
    }

    const RuntimeRegistry &runtimes_;
    const KernelRegistry &kernels_;
    std::vector<Step> plan_;
    std::vector<Cluster> clusters_;
    ValueIndex index_cache_;
    std::vector<int> cons_off_;  // consumers of step i: cons_[cons_off_[i] .. cons_off_[i + 1])
    std::vector<int> cons_;
    bool index_kernels_ = false;
    DeviceRuntime *index_runtime_ = nullptr;
    // recording state
    bool capturing_ = false;
    bool capture_unsafe_ = false;
    std::vector<std::optional<Materialization>> pending_;
    std::vector<Install> installs_;
    std::vector<FusedConstants> constants_;
    std::unordered_map<int, BufferRef> reserved_;  // plan step -> block its output goes to
    std::vector<const Value *> leaf_values_;       // the plan's leaves, in key order
};

}  // namespace

bool evaluate_fused(const RuntimeRegistry &runtimes, const KernelRegistry &kernels, std::span<const ValueRef> roots) {
    FusedEvaluator evaluator(runtimes, kernels);
    return evaluator.run(roots);
}

void clear_graph_cache() {
    GraphCache &cache = graph_cache();
    std::lock_guard<std::mutex> lock(cache.mu);
    cache.plans.clear();
}

}  // namespace minitensor::detail::cuda
