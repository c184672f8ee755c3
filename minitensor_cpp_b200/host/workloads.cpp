// Benchmark and parity workloads over MiniTensor's public API (see workloads.hpp).
#include "workloads.hpp"

#include <array>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <unordered_map>
#include <cstring>
#include <limits>
#include <memory>
#include <optional>
#include <span>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

#include <minitensor/data.hpp>
#include <minitensor/evaluation.hpp>
#include <minitensor/autograd.hpp>
#include <minitensor/nn/gradients.hpp>
#include <minitensor/nn/leafification.hpp>
#include <minitensor/nn/loss.hpp>
#include <minitensor/nn/module.hpp>
#include <minitensor/nn/modules/linear.hpp>
#include <minitensor/nn/optimizers/adamw.hpp>
#include <minitensor/nn/optimizers/sgd.hpp>
#include <minitensor/nn/parameters.hpp>
#include <minitensor/nn/parameters/parameter_tree.hpp>
#include <minitensor/ops.hpp>
#include <minitensor/random.hpp>
#include <minitensor/tensor.hpp>

#include "mtcuda.h"

#ifndef MTB_CPU_ONLY
#include "cuda_backend.hpp"
#include "ops_ext.hpp"
#include "tensor/backend/cpu/cpu_buffer.hpp"
#include "tensor/execution/environment.hpp"
#include "tensor/graph/leaf.hpp"
#include "tensor/graph/value.hpp"
#include "tensor/storage/dense_size.hpp"
#include "tensor/storage/materialization.hpp"
#include "tensor/tensor_access.hpp"
#endif

namespace mt = minitensor;

#ifndef MTB_CPU_ONLY
namespace minitensor::nn {
// Step count and moments of AdamW::State, which keeps them private; the state
// befriends this struct in the backend build (the fourth edit of the reference).
struct AdamWStateAccess {
    static std::uint64_t step(const AdamW::State &s) { return s.step_; }
    static void set_step(AdamW::State &s, std::uint64_t step) { s.step_ = step; }
    static const Tensor &first(const AdamW::State &s, const ParameterId &id) { return s.moments_.at(id).first; }
    static const Tensor &second(const AdamW::State &s, const ParameterId &id) { return s.moments_.at(id).second; }
    static void set_moments(AdamW::State &s, const ParameterId &id, Tensor first, Tensor second) {
        auto &m = s.moments_.at(id);
        m.first = std::move(first);
        m.second = std::move(second);
    }
};
}  // namespace minitensor::nn
#endif

namespace {

thread_local std::string t_error;

template <typename F>
int guarded(F &&f) {
    t_error.clear();
    try {
        f();
        return MTC_OK;
    } catch (const std::out_of_range &e) {
        t_error = e.what();
        return MTC_ERR_OUT_OF_RANGE;
    } catch (const std::invalid_argument &e) {
        t_error = e.what();
        return MTC_ERR_INVALID_ARGUMENT;
    } catch (const std::overflow_error &e) {
        t_error = e.what();
        return MTC_ERR_OVERFLOW;
    } catch (const std::logic_error &e) {
        t_error = e.what();
        return MTC_ERR_LOGIC;
    } catch (const std::exception &e) {
        t_error = e.what();
        return MTC_ERR_RUNTIME;
    }
}

mt::Device device_of(int device) {
    if (device < 0) return mt::Device::cpu();
#ifdef MTB_CPU_ONLY
    throw std::invalid_argument{"this build has no CUDA device"};
#else
    return mt::Device::cuda(static_cast<std::uint32_t>(device));
#endif
}

// ReLU as the exact composite of reference ops (gradient 0.5 at 0); the CUDA
// evaluator fuses it into one kernel with its neighbours.
mt::Tensor relu(const mt::Tensor &x) { return (x + mt::abs(x)) * 0.5F; }

// Dense MLP: Linear layers with ReLU between them (none after the last).
class DenseMlp final {
  public:
    class ParameterTree final {
      public:
        [[nodiscard]] const std::vector<mt::nn::Linear::ParameterTree> &layers() const noexcept { return layers_; }

      private:
        explicit ParameterTree(std::vector<mt::nn::Linear::ParameterTree> layers) : layers_{std::move(layers)} {}

        template <typename Self, typename Visitor>
        static void visit_members(Self &self, Visitor &visitor) {
            static constexpr std::string_view names[] = {"layer0", "layer1", "layer2", "layer3",
                                                         "layer4", "layer5", "layer6", "layer7"};
            for (std::size_t i = 0; i < self.layers_.size(); ++i) visitor.child(names[i], self.layers_[i]);
        }

        std::vector<mt::nn::Linear::ParameterTree> layers_;
        friend class DenseMlp;
        friend class minitensor::nn::ParameterTreeAccess;
    };

    explicit DenseMlp(std::vector<mt::Extent> widths) {
        if (widths.size() < 2 || widths.size() > 9) throw std::invalid_argument{"MLP needs 1 to 8 layers"};
        for (std::size_t i = 0; i + 1 < widths.size(); ++i) layers_.emplace_back(widths[i], widths[i + 1]);
    }

    [[nodiscard]] ParameterTree initialize(mt::nn::ParameterBuilder &builder, mt::RandomKey key,
                                           mt::TensorOptions options = {}) const {
        // one key per layer: split off the first, keep splitting the rest
        std::vector<mt::nn::Linear::ParameterTree> trees;
        mt::RandomKey rest = key;
        for (std::size_t i = 0; i < layers_.size(); ++i) {
            auto [layer_key, next] = mt::split(rest);
            trees.push_back(layers_[i].initialize(builder, layer_key, options));
            rest = next;
        }
        return ParameterTree{std::move(trees)};
    }

    [[nodiscard]] mt::Tensor operator()(const mt::nn::ParameterMap &parameters, const ParameterTree &tree,
                                        const mt::Tensor &input) const {
        mt::Tensor h = input;
        for (std::size_t i = 0; i < layers_.size(); ++i) {
            h = layers_[i](parameters, tree.layers()[i], h);
            if (i + 1 < layers_.size()) h = relu(h);
        }
        return h;
    }

    [[nodiscard]] std::size_t depth() const noexcept { return layers_.size(); }

  private:
    std::vector<mt::nn::Linear> layers_;
};

// One parameter vector: the tree of the optimizer workload.
class VectorTree final {
  public:
    explicit VectorTree(mt::nn::ParameterId id) : id_{std::move(id)} {}
    [[nodiscard]] const mt::nn::ParameterId &id() const noexcept { return id_; }

  private:
    template <typename Self, typename Visitor>
    static void visit_members(Self &self, Visitor &visitor) {
        visitor.parameter("value", self.id_);
    }

    mt::nn::ParameterId id_;
    friend class minitensor::nn::ParameterTreeAccess;
};

using Snapshot = mt::nn::ParameterSnapshot<DenseMlp::ParameterTree>;

}  // namespace

extern "C" {

const char *mtb_last_error(void) { return t_error.c_str(); }

int mtb_has_cuda(void) {
#ifdef MTB_CPU_ONLY
    return 0;
#else
    return 1;
#endif
}

int mtb_spiral_train(int device, int steps, int points, int hidden, uint64_t seed, float lr, int loss_every,
                     float *losses, double *seconds) {
    return guarded([&] {
        if (points < 2 || steps < 0 || hidden < 1) throw std::invalid_argument{"bad spiral configuration"};
        const mt::Device dev = device_of(device);
        // keys as in demo.cpp:163-164
        auto [dataset_key, model_key] = mt::split(mt::RandomKey{seed});
        auto [train_key, test_key] = mt::split(dataset_key);
        (void)test_key;
        constexpr int classes = 3;
        const int n = classes * points;
        const std::vector<float> noise = mt::to_vector(mt::normal(mt::Shape{n}, 0.0F, 0.2F, train_key));
        std::vector<float> xs(static_cast<std::size_t>(n) * 2);
        std::vector<std::int64_t> ys(static_cast<std::size_t>(n));
        for (int k = 0; k < classes; ++k) {
            for (int i = 0; i < points; ++i) {
                const int s = k * points + i;
                const float r = static_cast<float>(i) / static_cast<float>(points - 1);  // linspace(0, 1)
                const float theta = 4.0F * static_cast<float>(k) + 4.0F * r + noise[static_cast<std::size_t>(s)];
                xs[2 * s] = r * std::sin(theta);
                xs[2 * s + 1] = r * std::cos(theta);
                ys[s] = k;
            }
        }
        const mt::Tensor x = mt::from_data(xs, mt::Shape{n, 2}, dev);
        const mt::Tensor y = mt::from_data(ys, mt::Shape{n}, dev);
        const DenseMlp model({2, hidden, hidden, classes});
        auto params = mt::nn::initialize(model, model_key, mt::TensorOptions{mt::DType::Float32, dev});
        const mt::nn::AdamW optimizer(lr, 0.0F);
        auto state = optimizer.initialize(params);
        const auto t0 = std::chrono::steady_clock::now();
        for (int step = 0; step < steps; ++step) {
            const mt::Tensor logits = mt::nn::forward(model, params, x);
            const mt::Tensor loss = mt::nn::categorical_cross_entropy_with_logits(logits, y);
            if (losses) {
                losses[step] = (loss_every > 0 && step % loss_every == 0) ? mt::item<float>(loss)
                                                                          : std::numeric_limits<float>::quiet_NaN();
            }
            auto grads = mt::nn::parameter_gradients(loss, params);
            auto [next_params, next_state] = optimizer.step(std::move(params), std::move(state), grads);
            params = mt::nn::leafify_parameter_values(std::move(next_params));
            state = mt::nn::leafify_optimizer_state(std::move(next_state));
        }
        // the final parameters are the step's result: wait for them
        for (const auto &[id, p] : params.parameters()) {
            (void)id;
            (void)mt::to_vector(mt::reshape(p.value, mt::Shape{static_cast<mt::Extent>(p.value.numel())}));
            break;
        }
        if (seconds) seconds[0] = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    });
}

}  // extern "C"

namespace {

// MTB_TRACE=1: one line per training step on stderr with the host time of each
// phase (graph construction, gradient exchange, evaluations), for telling a
// host-bound step from a device-bound one.
struct StepTrace {
    using clock = std::chrono::steady_clock;
    bool on = std::getenv("MTB_TRACE") != nullptr;
    clock::time_point last = clock::now();
    std::string line;
    void mark(const char *phase) {
        if (!on) return;
        const auto now = clock::now();
        char buf[96];
        std::snprintf(buf, sizeof(buf), "%s%s %.1f ms", line.empty() ? "" : ", ", phase,
                      std::chrono::duration<double, std::milli>(now - last).count());
        line += buf;
        last = now;
    }
    ~StepTrace() {
        if (on) std::fprintf(stderr, "mtb step: %s\n", line.c_str());
    }
};

struct MlpTrainer {
    mt::Device device;
    DenseMlp model;
    Snapshot params;
    mt::nn::AdamW optimizer;
    mt::nn::AdamW::State state;
    std::vector<mt::nn::ParameterId> order;  // layer order: weight, bias, ...
    std::vector<std::vector<mt::nn::ParameterId>> layers;  // the same ids grouped per layer
    void *comm = nullptr;
    int (*host_allreduce)(void *, std::size_t) = nullptr;
    int world = 1;
    std::optional<mt::Tensor> x_resident;
    std::optional<mt::Tensor> y_resident;
    // further resident batches (mtb_mlp_load_batch_slot); mtb_mlp_use_slot makes
    // one of them the resident batch without a copy
    std::vector<std::pair<mt::Tensor, mt::Tensor>> batch_slots;
    std::optional<mt::nn::SGD> sgd;  // set: SGD replaces Adam
#ifndef MTB_CPU_ONLY
    // Input pipeline of step_host on a CUDA device: two device slots for a
    // batch (x and labels) filled on a copy stream, so the next batch's copy
    // runs while the device stream still computes the previous step.
    struct InputSlot {
        std::optional<mt::Tensor> x, y;
        void *copied = nullptr;  // event: the slot holds its batch (copy stream)
        void *free = nullptr;    // event: the step that read the slot has run (device stream)
    };
    InputSlot slots[2];
    int next_slot = 0;
    std::int64_t slot_batch = -1;
    void *copy_stream = nullptr;
    void *loss_ready = nullptr;  // event: the step's loss is computed
    bool mark_loss = false;      // record loss_ready once the loss is queued
    // Phase profile (mtb_mlp_profile): timed events on the device stream at the
    // step's start, before the wait for the gradient exchange, after it, and
    // after the optimizer; read and released by mtb_mlp_profile_read.
    bool profile = false;
    std::vector<std::array<void *, 4>> phase_events;
    void *phase_mark(int which) {
        if (!profile || device.type() != mt::DeviceType::Cuda) return nullptr;
        if (which == 0) phase_events.push_back({nullptr, nullptr, nullptr, nullptr});
        void *&e = phase_events.back()[static_cast<std::size_t>(which)];
        const int dev = static_cast<int>(device.index());
        mt::detail::cuda::check(mtc_event_create_timed(dev, &e), "profile event");
        mt::detail::cuda::check(mtc_event_record(e, cuda_runtime().stream()), "profile event");
        return e;
    }
#endif

    MlpTrainer(mt::Device dev, std::vector<mt::Extent> widths, uint64_t seed, float lr)
        : device{dev}, model{std::move(widths)},
          params{mt::nn::initialize(model, mt::RandomKey{seed}, mt::TensorOptions{mt::DType::Float32, dev})},
          optimizer{lr, 0.0F}, state{optimizer.initialize(params)} {
        for (const auto &layer : params.tree().layers()) {
            layers.emplace_back();
            order.push_back(layer.weight());
            layers.back().push_back(layer.weight());
            if (layer.bias()) {
                order.push_back(*layer.bias());
                layers.back().push_back(*layer.bias());
            }
        }
    }

    ~MlpTrainer() {
#ifndef MTB_CPU_ONLY
        const int dev = static_cast<int>(device.index());
        for (auto &ev : phase_events)
            for (void *e : ev) (void)mtc_event_destroy(dev, e);
        if (copy_stream == nullptr) return;
        (void)mtc_stream_synchronize(copy_stream);
        for (InputSlot &sl : slots) {
            (void)mtc_event_destroy(dev, sl.copied);
            (void)mtc_event_destroy(dev, sl.free);
        }
        (void)mtc_event_destroy(dev, loss_ready);
        (void)mtc_stream_destroy(dev, copy_stream);
#endif
    }

#ifndef MTB_CPU_ONLY
    // Device milliseconds of the profiled steps so far, summed: [0] the whole
    // steps, [1] forward + backward up to the wait for the gradient exchange,
    // [2] the exchange's exposed part (the device stream waiting for NCCL),
    // [3] the optimizer after it.  With one rank only [0] is measured.  The
    // events are released.
    void profile_read(double *ms4) {
        for (int k = 0; k < 4; ++k) ms4[k] = 0.0;
        const int dev = static_cast<int>(device.index());
        for (auto &ev : phase_events) {
            float t = 0.0F;
            if (ev[0] && ev[3]) {
                mt::detail::cuda::check(mtc_event_elapsed(ev[0], ev[3], &t), "profile read");
                ms4[0] += t;
            }
            for (int k = 0; k < 3; ++k) {
                if (ev[static_cast<std::size_t>(k)] && ev[static_cast<std::size_t>(k) + 1]) {
                    mt::detail::cuda::check(mtc_event_elapsed(ev[static_cast<std::size_t>(k)],
                                                              ev[static_cast<std::size_t>(k) + 1], &t),
                                            "profile read");
                    ms4[k + 1] += t;
                }
            }
            for (void *e : ev) (void)mtc_event_destroy(dev, e);
        }
        phase_events.clear();
    }
#endif

    // early_loss: read the loss as soon as it is computed (a CUDA device): the
    // forward pass is evaluated first and marked, and the read waits for that
    // mark only, so the host returns while the device runs the backward pass
    // and the optimizer.  Otherwise the loss is read after the whole step.
    float step(const mt::Tensor &x, const mt::Tensor &y, bool read_loss, bool early_loss = false) {
        StepTrace trace;
#ifndef MTB_CPU_ONLY
        phase_mark(0);
#endif
        const mt::Tensor logits = mt::nn::forward(model, params, x);
        const mt::Tensor loss = mt::nn::categorical_cross_entropy_with_logits(logits, y);
#ifndef MTB_CPU_ONLY
        early_loss = early_loss && read_loss && device.type() == mt::DeviceType::Cuda && copy_stream != nullptr;
        if (early_loss && world == 1) {
            mt::eval(loss);  // materialises the loss; the graph stays for the gradients
            mark_loss_ready();
        }
        mark_loss = early_loss && world > 1;  // the first layer of the exchange materialises it
#else
        early_loss = false;
#endif
        auto grads = mt::nn::parameter_gradients(loss, params);
        trace.mark("graph");
        if (world > 1) allreduce(grads, loss);
        trace.mark("allreduce");
        if (sgd) {
            auto [next_params, sgd_state] = sgd->step(std::move(params), mt::nn::SGD::State{}, grads);
            (void)sgd_state;
            grads.clear();
            trace.mark("optimizer graph");
            params = mt::nn::leafify_parameter_values(std::move(next_params));
            trace.mark("evaluate parameters");
        } else {
            auto [next_params, next_state] = optimizer.step(std::move(params), std::move(state), grads);
            grads.clear();
            trace.mark("optimizer graph");
            params = mt::nn::leafify_parameter_values(std::move(next_params));
            trace.mark("evaluate parameters");
            state = mt::nn::leafify_optimizer_state(std::move(next_state));
            trace.mark("evaluate state");
        }
#ifndef MTB_CPU_ONLY
        phase_mark(3);
#endif
        float value = 0.0F;
#ifndef MTB_CPU_ONLY
        if (early_loss) value = read_marked_loss(loss);
        else
#endif
            if (read_loss) value = mt::item<float>(loss);
        trace.mark("loss");
        return value;
    }

    // Replaces every parameter's value with host values in the order of
    // mtb_mlp_parameters (weight [out, in] then bias [out], layer by layer).
    void set_parameters(const float *values, std::int64_t count) {
        std::int64_t pos = 0;
        std::vector<std::pair<mt::nn::ParameterId, std::int64_t>> offsets;
        for (const auto &id : order) {
            offsets.emplace_back(id, pos);
            pos += static_cast<std::int64_t>(params.parameters().get(id).value.numel());
        }
        if (pos != count) throw std::invalid_argument{"parameter count differs from the model's"};
        params = std::move(params).transform([&](mt::nn::ParameterId id, const mt::nn::ParameterState &state) {
            for (const auto &[pid, off] : offsets) {
                if (pid == id) {
                    const auto n = static_cast<std::size_t>(state.value.numel());
                    return mt::nn::ParameterState{
                        mt::from_data(std::span<const float>(values + off, n), state.value.shape(), device),
                        state.metadata};
                }
            }
            return state;
        });
        params = mt::nn::leafify_parameter_values(std::move(params));
    }

    // Checkpoint of the parameters under their tree paths (layer0.weight, ...).
    // Format, little-endian: "MTBCKPT1", u32 parameter count, then per parameter
    // u32 path length, the path, u32 rank, i64 extents, float32 values.
    void save(const char *file) const {
        std::FILE *f = std::fopen(file, "wb");
        if (f == nullptr) throw std::runtime_error{std::string("cannot open ") + file + " for writing"};
        std::vector<std::pair<std::string, mt::nn::ParameterId>> named;
        mt::nn::for_each_named_parameter(params.tree(), [&](std::string_view name, const mt::nn::ParameterId id) {
            named.emplace_back(std::string(name), id);
        });
#ifndef MTB_CPU_ONLY
        const bool with_state = !sgd;  // Adam's step count and moments follow the parameters
#else
        const bool with_state = false;
#endif
        bool ok = std::fwrite(with_state ? "MTBCKPT2" : "MTBCKPT1", 1, 8, f) == 8;
        const auto count = static_cast<std::uint32_t>(named.size());
        ok = ok && std::fwrite(&count, sizeof(count), 1, f) == 1;
        for (const auto &[name, id] : named) {
            const mt::Tensor &v = params.value(id);
            const std::vector<float> host = mt::to_vector(v);
            const auto len = static_cast<std::uint32_t>(name.size());
            const auto rank = static_cast<std::uint32_t>(v.rank());
            ok = ok && std::fwrite(&len, sizeof(len), 1, f) == 1 && std::fwrite(name.data(), 1, len, f) == len &&
                 std::fwrite(&rank, sizeof(rank), 1, f) == 1;
            for (std::size_t d = 0; d < v.rank(); ++d) {
                const auto extent = static_cast<std::int64_t>(v.shape()[d]);
                ok = ok && std::fwrite(&extent, sizeof(extent), 1, f) == 1;
            }
            ok = ok && std::fwrite(host.data(), sizeof(float), host.size(), f) == host.size();
        }
#ifndef MTB_CPU_ONLY
        if (with_state) {
            const std::uint64_t step = mt::nn::AdamWStateAccess::step(state);
            ok = ok && std::fwrite(&step, sizeof(step), 1, f) == 1;
            for (const auto &[name, id] : named) {
                for (const mt::Tensor *m : {&mt::nn::AdamWStateAccess::first(state, id),
                                            &mt::nn::AdamWStateAccess::second(state, id)}) {
                    const std::vector<float> host = mt::to_vector(*m);
                    ok = ok && std::fwrite(host.data(), sizeof(float), host.size(), f) == host.size();
                }
            }
        }
#endif
        ok = std::fclose(f) == 0 && ok;
        if (!ok) throw std::runtime_error{std::string("writing ") + file + " failed"};
    }

    // Replaces every parameter with the one saved under its path; the file must
    // hold each of the model's parameters with the same shape.
    void load(const char *file) {
        std::FILE *f = std::fopen(file, "rb");
        if (f == nullptr) throw std::runtime_error{std::string("cannot open ") + file};
        struct Record {
            std::vector<mt::Extent> shape;
            std::vector<float> values;
        };
        std::unordered_map<std::string, Record> records;
        char magic[8] = {};
        std::uint32_t count = 0;
        bool ok = std::fread(magic, 1, 8, f) == 8 &&
                  (std::memcmp(magic, "MTBCKPT1", 8) == 0 || std::memcmp(magic, "MTBCKPT2", 8) == 0) &&
                  std::fread(&count, sizeof(count), 1, f) == 1;
        const bool with_state = ok && magic[7] == '2';
        std::vector<std::string> order_in_file;
        for (std::uint32_t k = 0; ok && k < count; ++k) {
            std::uint32_t len = 0, rank = 0;
            ok = std::fread(&len, sizeof(len), 1, f) == 1 && len < 4096;
            std::string name(ok ? len : 0, '\0');
            ok = ok && std::fread(name.data(), 1, len, f) == len && std::fread(&rank, sizeof(rank), 1, f) == 1 &&
                 rank <= 8;
            Record r;
            std::size_t n = 1;
            for (std::uint32_t d = 0; ok && d < rank; ++d) {
                std::int64_t extent = 0;
                ok = std::fread(&extent, sizeof(extent), 1, f) == 1 && extent >= 0 && extent < (std::int64_t{1} << 40);
                r.shape.push_back(extent);
                n *= static_cast<std::size_t>(extent);
            }
            if (!ok) break;
            r.values.resize(n);
            ok = std::fread(r.values.data(), sizeof(float), n, f) == n;
            order_in_file.push_back(name);
            records.emplace(std::move(name), std::move(r));
        }
        // optimizer state (version 2): the step count, then each parameter's
        // first and second moments in the order of the parameters above
        std::uint64_t adam_step = 0;
        std::unordered_map<std::string, std::pair<std::vector<float>, std::vector<float>>> moments;
        if (ok && with_state) {
            ok = std::fread(&adam_step, sizeof(adam_step), 1, f) == 1;
            for (const std::string &name : order_in_file) {
                if (!ok) break;
                const std::size_t n = records.at(name).values.size();
                std::vector<float> m1(n), m2(n);
                ok = std::fread(m1.data(), sizeof(float), n, f) == n && std::fread(m2.data(), sizeof(float), n, f) == n;
                moments.emplace(name, std::make_pair(std::move(m1), std::move(m2)));
            }
        }
        std::fclose(f);
        if (!ok) throw std::runtime_error{std::string(file) + " is not a complete checkpoint"};
        std::unordered_map<mt::nn::ParameterId, const Record *> by_id;
        mt::nn::for_each_named_parameter(params.tree(), [&](std::string_view name, const mt::nn::ParameterId id) {
            const auto it = records.find(std::string(name));
            if (it == records.end()) throw std::invalid_argument{"checkpoint has no parameter " + std::string(name)};
            const mt::Tensor &v = params.value(id);
            if (it->second.shape.size() != v.rank()) throw std::invalid_argument{"checkpoint shape differs: " + std::string(name)};
            for (std::size_t d = 0; d < v.rank(); ++d)
                if (it->second.shape[d] != v.shape()[d])
                    throw std::invalid_argument{"checkpoint shape differs: " + std::string(name)};
            by_id.emplace(id, &it->second);
        });
        params = std::move(params).transform([&](mt::nn::ParameterId id, const mt::nn::ParameterState &state) {
            const auto it = by_id.find(id);
            if (it == by_id.end()) return state;
            return mt::nn::ParameterState{mt::from_data(std::span<const float>(it->second->values), state.value.shape(),
                                                        device),
                                          state.metadata};
        });
        params = mt::nn::leafify_parameter_values(std::move(params));
#ifndef MTB_CPU_ONLY
        if (with_state && !sgd) {
            mt::nn::for_each_named_parameter(params.tree(), [&](std::string_view name, const mt::nn::ParameterId id) {
                const auto &mv = moments.at(std::string(name));
                const mt::Shape shape = params.value(id).shape();
                mt::nn::AdamWStateAccess::set_moments(state, id,
                                                      mt::from_data(std::span<const float>(mv.first), shape, device),
                                                      mt::from_data(std::span<const float>(mv.second), shape, device));
            });
            mt::nn::AdamWStateAccess::set_step(state, adam_step);
            state = mt::nn::leafify_optimizer_state(std::move(state));
        }
#endif
    }

    // Loss and parameter gradients on the resident batch at the current
    // parameters (no update), evaluated together in one evaluation.
    float gradients(float *out, std::int64_t capacity) {
        if (!x_resident) throw std::logic_error{"no resident batch loaded"};
        const mt::Tensor logits = mt::nn::forward(model, params, *x_resident);
        const mt::Tensor loss = mt::nn::categorical_cross_entropy_with_logits(logits, *y_resident);
        const auto grads = mt::nn::parameter_gradients(loss, params);
        std::vector<mt::Tensor> roots{loss};
        for (const auto &id : order) roots.push_back(grads.at(id));
        const std::vector<mt::Tensor> leaves = mt::leafify(roots);
        std::int64_t pos = 0;
        for (std::size_t i = 0; i < order.size(); ++i) {
            const std::vector<float> host = mt::to_vector(leaves[i + 1]);
            if (pos + static_cast<std::int64_t>(host.size()) > capacity)
                throw std::out_of_range{"gradient buffer too small"};
            std::copy(host.begin(), host.end(), out + pos);
            pos += static_cast<std::int64_t>(host.size());
        }
        return mt::item<float>(leaves[0]);
    }

#ifndef MTB_CPU_ONLY
    mt::detail::cuda::CudaRuntime &cuda_runtime() const {
        return dynamic_cast<mt::detail::cuda::CudaRuntime &>(mt::detail::environment().runtime_for(device));
    }

    void mark_loss_ready() {
        mt::detail::cuda::check(mtc_event_record(loss_ready, cuda_runtime().stream()), "loss mark");
    }

    // The loss, read on the copy stream once the device stream passed the mark.
    float read_marked_loss(const mt::Tensor &loss) {
        mt::Tensor l = loss;
        const void *src = dense_region(l);
        float value = 0.0F;
        const int dev = static_cast<int>(device.index());
        mt::detail::cuda::check(mtc_stream_wait_event(copy_stream, loss_ready), "loss wait");
        mt::detail::cuda::check(mtc_copy_to_host(dev, &value, src, sizeof(float), copy_stream), "loss read");
        // an index error of this or an earlier step whose snapshot has arrived
        mt::detail::cuda::raise_device_errors(dev, false);
        return value;
    }

    // One step from host inputs through the input pipeline: the batch is copied
    // into the next slot on the copy stream (after the step that last read that
    // slot), the device stream waits for the copy, and the loss is read early.
    float step_pipelined(const float *x, const std::int64_t *labels, std::int64_t batch) {
        const int dev = static_cast<int>(device.index());
        const mt::Extent in = params.parameters().get(order.front()).value.shape()[1];
        auto &rt = cuda_runtime();
        if (copy_stream == nullptr) {
            mt::detail::cuda::check(mtc_stream_create(dev, &copy_stream), "copy stream");
            mt::detail::cuda::check(mtc_event_create(dev, &loss_ready), "event");
            for (InputSlot &sl : slots) {
                mt::detail::cuda::check(mtc_event_create(dev, &sl.copied), "event");
                mt::detail::cuda::check(mtc_event_create(dev, &sl.free), "event");
            }
        }
        if (batch != slot_batch) {
            // (re)allocate the slots for this batch size, after all earlier use
            mt::detail::cuda::check(mtc_stream_synchronize(rt.stream()), "stream");
            for (InputSlot &sl : slots) {
                sl.x = device_leaf(mt::detail::TensorSpec{mt::Shape{batch, in}, mt::DType::Float32, device}, rt);
                sl.y = device_leaf(mt::detail::TensorSpec{mt::Shape{batch}, mt::DType::Int64, device}, rt);
            }
            slot_batch = batch;
        }
        InputSlot &sl = slots[next_slot];
        next_slot ^= 1;
        const std::size_t xb = static_cast<std::size_t>(batch * in) * sizeof(float);
        const std::size_t yb = static_cast<std::size_t>(batch) * sizeof(std::int64_t);
        mt::detail::cuda::check(mtc_stream_wait_event(copy_stream, sl.free), "slot wait");
        mt::Tensor xs = *sl.x, ys = *sl.y;
        mt::detail::cuda::check(mtc_copy_from_host(dev, dense_region(xs), x, xb, copy_stream), "input copy");
        mt::detail::cuda::check(mtc_copy_from_host(dev, dense_region_i64(ys), labels, yb, copy_stream), "label copy");
        mt::detail::cuda::check(mtc_event_record(sl.copied, copy_stream), "copy mark");
        mt::detail::cuda::check(mtc_stream_wait_event(rt.stream(), sl.copied), "copy wait");
        const float l = step(xs, ys, true, true);
        mt::detail::cuda::check(mtc_event_record(sl.free, rt.stream()), "slot mark");
        return l;
    }

    // A materialised leaf over a fresh device buffer of the spec's dense size.
    static mt::Tensor device_leaf(mt::detail::TensorSpec spec, mt::detail::cuda::CudaRuntime &rt) {
        mt::detail::BufferRef buffer = rt.allocate(mt::detail::dense_size_bytes(spec));
        mt::detail::Materialization m(std::move(buffer), mt::detail::Layout::contiguous(spec.shape));
        return mt::detail::TensorAccess::make(mt::detail::make_materialized_leaf(std::move(spec), std::move(m)));
    }

    static void *dense_region_i64(mt::Tensor &t) {
        const auto *m = mt::detail::TensorAccess::value(t)->materialization();
        auto *cb = dynamic_cast<mt::detail::cuda::CudaBuffer *>(m->buffer_ref().get());
        if (cb == nullptr) throw std::logic_error{"label storage is not a device buffer"};
        return static_cast<std::int64_t *>(cb->data()) + m->layout().offset();
    }
#endif

    // Data-parallel gradient exchange.  Each gradient's dense storage region is
    // summed over the ranks in place and scaled by 1/world, then the unchanged
    // AdamW step runs.
    //  - CUDA device: layers are evaluated last to first, one evaluation per
    //    layer (the first also materialises the loss).  As soon as a layer's
    //    gradients are queued, their NCCL all-reduce is queued on the
    //    communicator's own stream behind them, so it runs while the next
    //    layer's backward GEMMs run on the device stream; the device stream
    //    waits for every reduction before the optimizer.
    //  - CPU device: one evaluation, then the host callback per gradient (used to
    //    run the same path with CPU process groups).
    void allreduce(mt::nn::ParameterGradients &grads, const mt::Tensor &loss) {
#ifdef MTB_CPU_ONLY
        (void)grads;
        (void)loss;
        throw std::invalid_argument{"data parallelism needs the backend build"};
#else
        if (device.type() == mt::DeviceType::Cuda) {
            if (comm == nullptr) throw std::logic_error{"no NCCL communicator attached"};
            auto &rt = dynamic_cast<mt::detail::cuda::CudaRuntime &>(mt::detail::environment().runtime_for(device));
            for (std::size_t l = layers.size(); l-- > 0;) {
                std::vector<mt::Tensor> roots;
                if (l + 1 == layers.size()) roots.push_back(loss);
                for (const auto &id : layers[l]) roots.push_back(grads.at(id));
                std::vector<mt::Tensor> leaves = mt::leafify(roots);
                const std::size_t skip = l + 1 == layers.size() ? 1 : 0;
                if (skip == 1 && mark_loss) mark_loss_ready();
                std::vector<void *> buffers;
                std::vector<std::size_t> counts;
                for (std::size_t i = 0; i < layers[l].size(); ++i) {
                    mt::Tensor g = leaves[i + skip];
                    buffers.push_back(dense_region(g));
                    counts.push_back(g.numel());
                    grads.at(layers[l][i]) = g;
                }
                mt::detail::cuda::check(mtc_comm_allreduce_f32_async(comm, buffers.data(), counts.data(),
                                                                     static_cast<int32_t>(buffers.size()),
                                                                     1.0F / world, rt.stream()),
                                        "gradient all-reduce");
            }
            phase_mark(1);
            mt::detail::cuda::check(mtc_comm_wait(comm, rt.stream()), "gradient all-reduce wait");
            phase_mark(2);
            return;
        }
        std::vector<mt::Tensor> roots{loss};
        for (const auto &id : order) roots.push_back(grads.at(id));
        std::vector<mt::Tensor> leaves = mt::leafify(roots);
        if (host_allreduce == nullptr) throw std::logic_error{"no host all-reduce attached"};
        const float scale = 1.0F / static_cast<float>(world);
        for (std::size_t i = 0; i < order.size(); ++i) {
            mt::Tensor g = leaves[i + 1];
            float *p = static_cast<float *>(dense_region(g));
            grads.at(order[i]) = g;
            if (host_allreduce(p, g.numel()) != 0) throw std::runtime_error{"host all-reduce failed"};
            for (std::size_t j = 0; j < g.numel(); ++j) p[j] *= scale;
        }
#endif
    }

#ifndef MTB_CPU_ONLY
    // Start of the dense storage region of a materialised gradient; a gradient
    // whose layout does not cover exactly numel elements is made contiguous first
    // (the region of a permuted dense layout is [lowest offset, + numel)).
    static void *dense_region(mt::Tensor &g) {
        {
            const auto &layout = mt::detail::TensorAccess::value(g)->materialization()->layout();
            std::int64_t span = 1;
            for (std::size_t d = 0; d < g.rank(); ++d) span += (g.shape()[d] - 1) * std::abs(layout.stride(d));
            if (span != static_cast<std::int64_t>(g.numel())) g = mt::leafify(mt::contiguous(g));
        }
        const auto *m = mt::detail::TensorAccess::value(g)->materialization();
        std::int64_t lo = m->layout().offset();
        for (std::size_t d = 0; d < g.rank(); ++d)
            if (m->layout().stride(d) < 0) lo += (g.shape()[d] - 1) * m->layout().stride(d);
        std::byte *base = nullptr;
        if (auto *cb = dynamic_cast<mt::detail::cuda::CudaBuffer *>(m->buffer_ref().get())) {
            base = static_cast<std::byte *>(cb->data());
        } else if (auto *hb = dynamic_cast<mt::detail::cpu::CpuBuffer *>(m->buffer_ref().get())) {
            base = hb->data();
        } else {
            throw std::logic_error{"gradient storage of an unknown buffer type"};
        }
        return reinterpret_cast<float *>(base) + lo;
    }
#endif
};

}  // namespace

extern "C" {

int mtb_mlp_create(int device, int64_t in_features, int64_t hidden, int32_t hidden_layers, int64_t classes,
                   uint64_t seed, float lr, void **handle) {
    return guarded([&] {
        std::vector<mt::Extent> widths{in_features};
        for (int i = 0; i < hidden_layers; ++i) widths.push_back(hidden);
        widths.push_back(classes);
        *handle = new MlpTrainer(device_of(device), std::move(widths), seed, lr);
    });
}

void mtb_mlp_destroy(void *handle) { delete static_cast<MlpTrainer *>(handle); }

int mtb_mlp_set_comm(void *handle, void *comm, int32_t world) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
        t->comm = comm;
        t->world = world;
    });
}

int mtb_mlp_set_host_allreduce(void *handle, int (*sum_in_place)(void *, size_t), int32_t world) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
        t->host_allreduce = sum_in_place;
        t->world = world;
    });
}

int mtb_mlp_load_batch(void *handle, const float *x, const int64_t *labels, int64_t batch) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
        const mt::Extent in = t->params.parameters().get(t->order.front()).value.shape()[1];
        t->x_resident = mt::from_data(std::span<const float>(x, static_cast<std::size_t>(batch * in)),
                                      mt::Shape{batch, in}, t->device);
        t->y_resident = mt::from_data(std::span<const std::int64_t>(labels, static_cast<std::size_t>(batch)),
                                      mt::Shape{batch}, t->device);
    });
}

int mtb_mlp_load_batch_slot(void *handle, int32_t slot, const float *x, const int64_t *labels, int64_t batch) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
        if (slot < 0 || slot > 64) throw std::out_of_range{"batch slot outside 0..64"};
        const mt::Extent in = t->params.parameters().get(t->order.front()).value.shape()[1];
        mt::Tensor xt = mt::from_data(std::span<const float>(x, static_cast<std::size_t>(batch * in)),
                                      mt::Shape{batch, in}, t->device);
        mt::Tensor yt = mt::from_data(std::span<const std::int64_t>(labels, static_cast<std::size_t>(batch)),
                                      mt::Shape{batch}, t->device);
        mt::eval({xt, yt});
        while (static_cast<int32_t>(t->batch_slots.size()) <= slot) t->batch_slots.emplace_back(xt, yt);
        t->batch_slots[static_cast<std::size_t>(slot)] = {std::move(xt), std::move(yt)};
    });
}

int mtb_mlp_use_slot(void *handle, int32_t slot) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
        if (slot < 0 || slot >= static_cast<int32_t>(t->batch_slots.size())) throw std::out_of_range{"no such batch slot"};
        t->x_resident = t->batch_slots[static_cast<std::size_t>(slot)].first;
        t->y_resident = t->batch_slots[static_cast<std::size_t>(slot)].second;
    });
}

int mtb_mlp_step_resident(void *handle, int32_t read_loss, float *loss) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
        if (!t->x_resident) throw std::logic_error{"no resident batch loaded"};
        const float l = t->step(*t->x_resident, *t->y_resident, read_loss != 0);
        if (loss) *loss = l;
    });
}

int mtb_mlp_step_host(void *handle, const float *x, const int64_t *labels, int64_t batch, float *loss) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
#ifndef MTB_CPU_ONLY
        if (t->device.type() == mt::DeviceType::Cuda) {
            const float l = t->step_pipelined(x, labels, batch);
            if (loss) *loss = l;
            return;
        }
#endif
        const mt::Extent in = t->params.parameters().get(t->order.front()).value.shape()[1];
        const mt::Tensor xt = mt::from_data(std::span<const float>(x, static_cast<std::size_t>(batch * in)),
                                            mt::Shape{batch, in}, t->device);
        const mt::Tensor yt = mt::from_data(std::span<const std::int64_t>(labels, static_cast<std::size_t>(batch)),
                                            mt::Shape{batch}, t->device);
        const float l = t->step(xt, yt, true);
        if (loss) *loss = l;
    });
}

int64_t mtb_mlp_parameter_count(void *handle) {
    auto *t = static_cast<MlpTrainer *>(handle);
    int64_t n = 0;
    for (const auto &id : t->order) n += static_cast<int64_t>(t->params.parameters().get(id).value.numel());
    return n;
}

int mtb_mlp_parameters(void *handle, float *out, int64_t capacity) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
        int64_t pos = 0;
        for (const auto &id : t->order) {
            const mt::Tensor &v = t->params.parameters().get(id).value;
            const std::vector<float> host = mt::to_vector(v);
            if (pos + static_cast<int64_t>(host.size()) > capacity) throw std::out_of_range{"parameter buffer too small"};
            std::copy(host.begin(), host.end(), out + pos);
            pos += static_cast<int64_t>(host.size());
        }
    });
}

int mtb_mlp_gradients(void *handle, float *loss, float *out, int64_t capacity) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
        const float l = t->gradients(out, capacity);
        if (loss) *loss = l;
    });
}

int mtb_mlp_profile(void *handle, int32_t on, double *ms4) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
#ifndef MTB_CPU_ONLY
        if (ms4) t->profile_read(ms4);
        t->profile = on != 0;
#else
        (void)t;
        (void)on;
        if (ms4)
            for (int k = 0; k < 4; ++k) ms4[k] = 0.0;
#endif
    });
}

int mtb_mlp_save(void *handle, const char *path) {
    return guarded([&] { static_cast<MlpTrainer *>(handle)->save(path); });
}

int mtb_mlp_load(void *handle, const char *path) {
    return guarded([&] { static_cast<MlpTrainer *>(handle)->load(path); });
}

int mtb_mlp_set_parameters(void *handle, const float *values, int64_t count) {
    return guarded([&] { static_cast<MlpTrainer *>(handle)->set_parameters(values, count); });
}

int mtb_mlp_use_sgd(void *handle, float lr) {
    return guarded([&] { static_cast<MlpTrainer *>(handle)->sgd.emplace(lr); });
}

int mtb_mlp_materialize(void *handle) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
        t->params = mt::nn::leafify_parameter_values(std::move(t->params));
        t->state = mt::nn::leafify_optimizer_state(std::move(t->state));
    });
}

int mtb_mlp_synchronize(void *handle) {
    return guarded([&] {
        auto *t = static_cast<MlpTrainer *>(handle);
#ifndef MTB_CPU_ONLY
        if (t->device.type() == mt::DeviceType::Cuda) {
            auto &rt = dynamic_cast<mt::detail::cuda::CudaRuntime &>(mt::detail::environment().runtime_for(t->device));
            mt::detail::cuda::check(mtc_stream_synchronize(rt.stream()), "synchronize");
        }
#else
        (void)t;
#endif
    });
}

void *mtb_mlp_stream(void *handle) {
#ifndef MTB_CPU_ONLY
    auto *t = static_cast<MlpTrainer *>(handle);
    if (t->device.type() != mt::DeviceType::Cuda) return nullptr;
    auto &rt = dynamic_cast<mt::detail::cuda::CudaRuntime &>(mt::detail::environment().runtime_for(t->device));
    return rt.stream();
#else
    (void)handle;
    return nullptr;
#endif
}

int mtb_chain(int device, int64_t n, int64_t m, const float *a, const float *b_storage, const float *row,
              const float *col, float *out, float *reductions) {
    return guarded([&] {
        const mt::Device dev = device_of(device);
        const auto N = static_cast<std::size_t>(n), M = static_cast<std::size_t>(m);
        const mt::Tensor A = mt::from_data(std::span<const float>(a, N * M), mt::Shape{n, m}, dev);
        const mt::Tensor Bs = mt::from_data(std::span<const float>(b_storage, N * M), mt::Shape{m, n}, dev);
        const mt::Tensor B = mt::transpose(Bs);  // [n, m] view with strides {1, n}
        const mt::Tensor r = mt::from_data(std::span<const float>(row, M), mt::Shape{1, m}, dev);
        const mt::Tensor c = mt::from_data(std::span<const float>(col, N), mt::Shape{n, 1}, dev);
        const mt::Tensor Y = relu(A * B + r) * mt::exp(-c);
        const std::vector<float> y = mt::to_vector(Y);
        std::copy(y.begin(), y.end(), out);
        if (reductions) {
            const std::vector<float> s0 = mt::to_vector(mt::sum(Y, {0}));
            const std::vector<float> s1 = mt::to_vector(mt::sum(Y, {1}));
            const std::vector<float> l1 = mt::to_vector(mt::logsumexp(Y, {1}));
            std::copy(s0.begin(), s0.end(), reductions);
            std::copy(s1.begin(), s1.end(), reductions + M);
            std::copy(l1.begin(), l1.end(), reductions + M + N);
        }
    });
}

int mtb_gather_rows(int device, int64_t rows, int64_t cols, const float *table, int64_t n, const int64_t *index,
                    float *out) {
    return guarded([&] {
        const mt::Device dev = device_of(device);
        const mt::Tensor t = mt::from_data(std::span<const float>(table, static_cast<std::size_t>(rows * cols)),
                                           mt::Shape{rows, cols}, dev);
        const mt::Tensor i = mt::from_data(std::span<const std::int64_t>(index, static_cast<std::size_t>(n)),
                                           mt::Shape{n, 1}, dev);
        const mt::Tensor g = mt::gather(t, 0, mt::broadcast_to(i, mt::Shape{n, cols}));
        const std::vector<float> v = mt::to_vector(g);
        std::copy(v.begin(), v.end(), out);
    });
}

int mtb_cross_entropy(int device, int64_t rows, int64_t cols, const float *logits, int32_t class_axis,
                      const int64_t *targets, float *loss, float *grad) {
    return guarded([&] {
        if (class_axis != 0 && class_axis != 1) throw std::invalid_argument{"class axis must be 0 or 1"};
        const mt::Device dev = device_of(device);
        const mt::Tensor X = mt::from_data(std::span<const float>(logits, static_cast<std::size_t>(rows * cols)),
                                           mt::Shape{rows, cols}, dev);
        const int64_t n = class_axis == 0 ? cols : rows;
        const mt::Tensor T = mt::from_data(std::span<const std::int64_t>(targets, static_cast<std::size_t>(n)),
                                           mt::Shape{n}, dev);
        const mt::Tensor L = mt::nn::categorical_cross_entropy_with_logits(X, T, class_axis);
        if (grad) {
            const std::vector<float> g = mt::to_vector(mt::grad(L, X).front());
            std::copy(g.begin(), g.end(), grad);
        }
        if (loss) *loss = mt::item<float>(L);
    });
}

int mtb_optimizer_steps(int device, int32_t kind, int64_t n, const float *params, int32_t steps, const float *grads,
                        float lr, float weight_decay, float beta1, float beta2, float eps, float *out) {
    return guarded([&] {
        if (kind != 0 && kind != 1) throw std::invalid_argument{"optimizer kind must be 0 (AdamW) or 1 (SGD)"};
        if (n < 0 || steps < 0) throw std::invalid_argument{"negative size"};
        const mt::Device dev = device_of(device);
        const auto count = static_cast<std::size_t>(n);
        mt::nn::ParameterBuilder builder;
        const mt::nn::ParameterId id =
            builder.add(mt::nn::ParameterState{mt::from_data(std::span<const float>(params, count), mt::Shape{n}, dev)});
        auto snapshot = std::move(builder).finish(VectorTree{id});
        auto gradient_of = [&](int32_t step) {
            mt::nn::ParameterGradients g;
            g.emplace(id, mt::from_data(std::span<const float>(grads + static_cast<std::size_t>(step) * count, count),
                                        mt::Shape{n}, dev));
            return g;
        };
        if (kind == 0) {
            const mt::nn::AdamW optimizer(lr, weight_decay, beta1, beta2, eps);
            auto state = optimizer.initialize(snapshot);
            for (int32_t s = 0; s < steps; ++s) {
                auto [next, next_state] = optimizer.step(std::move(snapshot), std::move(state), gradient_of(s));
                snapshot = mt::nn::leafify_parameter_values(std::move(next));
                state = mt::nn::leafify_optimizer_state(std::move(next_state));
            }
        } else {
            const mt::nn::SGD optimizer(lr);
            for (int32_t s = 0; s < steps; ++s) {
                auto [next, next_state] = optimizer.step(std::move(snapshot), optimizer.initialize(snapshot),
                                                         gradient_of(s));
                (void)next_state;
                snapshot = mt::nn::leafify_parameter_values(std::move(next));
            }
        }
        const std::vector<float> v = mt::to_vector(snapshot.value(id));
        std::copy(v.begin(), v.end(), out);
    });
}

#ifndef MTB_CPU_ONLY
int mtb_gather_eval_probe(int device, int64_t rows, int64_t cols, const float *table, int64_t n, const int64_t *index,
                          int32_t *threw, int32_t *materialized) {
    return guarded([&] {
        const mt::Device dev = device_of(device);
        const mt::Tensor t = mt::from_data(std::span<const float>(table, static_cast<std::size_t>(rows * cols)),
                                           mt::Shape{rows, cols}, dev);
        const mt::Tensor i = mt::from_data(std::span<const std::int64_t>(index, static_cast<std::size_t>(n)),
                                           mt::Shape{n, 1}, dev);
        const mt::Tensor g = mt::gather(t, 0, mt::broadcast_to(i, mt::Shape{n, cols}));
        *threw = 0;
        try {
            mt::eval(g);
        } catch (const std::out_of_range &) {
            *threw = 1;
        }
        *materialized = mt::detail::TensorAccess::value(g)->materialization() != nullptr ? 1 : 0;
        if (*threw == 0) (void)mt::to_vector(g);  // a deferred index error surfaces at this read
    });
}

int mtb_set_index_checks(int mode) {
    auto &o = mt::detail::cuda::evaluator_options();
    const int previous = !o.check_index_errors ? 0 : (o.sync_index_checks ? 2 : 1);
    o.check_index_errors = mode != 0;
    o.sync_index_checks = mode == 2;
    return previous;
}
#endif

#ifndef MTB_CPU_ONLY
// The operations this backend adds (ops_ext.hpp) on a [rows, cols] matrix,
// through MiniTensor's API: relu(x), and max, argmax and log-softmax along
// `axis` (0 or 1), and (relu_grad_out, may be NULL) the gradient of
// sum(relu(x)).  max_out and argmax_out hold the reduced extent, the others
// rows * cols values.
int mtb_added_ops(int device, int64_t rows, int64_t cols, const float *x, int32_t axis, float *relu_out,
                  float *max_out, int64_t *argmax_out, float *log_softmax_out, float *relu_grad_out) {
    return guarded([&] {
        if (axis != 0 && axis != 1) throw std::invalid_argument{"axis must be 0 or 1"};
        const mt::Device dev = device_of(device);
        const mt::Tensor X = mt::from_data(std::span<const float>(x, static_cast<std::size_t>(rows * cols)),
                                           mt::Shape{rows, cols}, dev);
        if (relu_grad_out) {
            // d sum(relu(X)) / dX through the autograd engine and relu's VJP rule
            const std::vector<float> g = mt::to_vector(mt::grad(mt::sum(mt::b200::relu(X)), X).front());
            std::copy(g.begin(), g.end(), relu_grad_out);
        }
        const std::vector<float> r = mt::to_vector(mt::b200::relu(X));
        const std::vector<float> m = mt::to_vector(mt::b200::max(X, {axis}));
        const std::vector<std::int64_t> a = mt::to_vector<std::int64_t>(mt::b200::argmax(X, axis));
        const std::vector<float> l = mt::to_vector(mt::b200::log_softmax(X, axis));
        std::copy(r.begin(), r.end(), relu_out);
        std::copy(m.begin(), m.end(), max_out);
        std::copy(a.begin(), a.end(), argmax_out);
        std::copy(l.begin(), l.end(), log_softmax_out);
    });
}
#endif

void mtb_evaluator_stats(uint64_t *out13) {
#ifndef MTB_CPU_ONLY
    const auto &s = mt::detail::cuda::evaluator_stats();
    out13[0] = s.kernel_steps;
    out13[1] = s.fused_launches;
    out13[2] = s.fused_nodes;
    out13[3] = s.folded_constants;
    out13[4] = s.view_steps;
    out13[5] = s.evaluations;
    out13[6] = s.plan_ns;
    out13[7] = s.execute_ns;
    out13[8] = s.check_ns;
    out13[9] = s.graph_captures;
    out13[10] = s.graph_replays;
    out13[11] = s.graph_fallbacks;
    out13[12] = s.scatters_deferred;
#else
    for (int i = 0; i < 13; ++i) out13[i] = 0;
#endif
}

void mtb_graph_cache_clear(void) {
#ifndef MTB_CPU_ONLY
    mt::detail::cuda::clear_graph_cache();
#endif
}

int mtb_set_fusion(int on) {
#ifndef MTB_CPU_ONLY
    const bool previous = mt::detail::cuda::evaluator_options().fusion;
    mt::detail::cuda::evaluator_options().fusion = on != 0;
    return previous ? 1 : 0;
#else
    (void)on;
    return 0;
#endif
}

int mtb_set_graphs(int on) {
#ifndef MTB_CPU_ONLY
    const bool previous = mt::detail::cuda::evaluator_options().graphs;
    mt::detail::cuda::evaluator_options().graphs = on != 0;
    return previous ? 1 : 0;
#else
    (void)on;
    return 0;
#endif
}

void mtb_evaluator_reset_stats(void) {
#ifndef MTB_CPU_ONLY
    mt::detail::cuda::evaluator_stats() = {};
#endif
}

}  // extern "C"
