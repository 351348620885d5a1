// extern "C" entry points of include/cpde_b200.h over cpde::Engine.
#include <cstring>
#include <string>

#include "../../include/cpde_b200.h"
#include "engine.hpp"

struct cpde_engine {
    cpde::Engine* engine = nullptr;
    std::string error;
};

namespace {

template <class F>
int guard(cpde_engine* h, F&& f) {
    if (!h) return CPDE_REJECTED;
    if (!h->engine) {
        h->error = "the engine was not created";
        return CPDE_REJECTED;
    }
    try {
        if (h->engine) CPDE_CUDA(cudaSetDevice(h->engine->device));
        f();
        return CPDE_OK;
    } catch (const cpde::DeviceError& e) {
        h->error = e.what();
        return CPDE_DEVICE_ERROR;
    } catch (const std::exception& e) {
        h->error = e.what();
        return CPDE_REJECTED;
    }
}

cpde::Engine& E(cpde_engine* h) { return *h->engine; }

}  // namespace

extern "C" {

int cpde_engine_create(int32_t device, cpde_engine** out) {
    if (!out) return CPDE_REJECTED;
    *out = nullptr;
    auto* h = new cpde_engine;
    try {
        h->engine = new cpde::Engine(device);
    } catch (const cpde::DeviceError& e) {
        h->error = e.what();
        *out = h;
        return CPDE_DEVICE_ERROR;
    } catch (const std::exception& e) {
        h->error = e.what();
        *out = h;
        return CPDE_REJECTED;
    }
    *out = h;
    return CPDE_OK;
}

int cpde_engine_create_sharded(int32_t device, int32_t rank, int32_t world, const void* unique_id,
                               cpde_engine** out) {
    if (!out) return CPDE_REJECTED;
    *out = nullptr;
    auto* h = new cpde_engine;
    *out = h;
    try {
        cpde::require(world >= 1 && rank >= 0 && rank < world && unique_id, "invalid shard rank or group size");
        h->engine = new cpde::Engine(device);
        h->engine->join(rank, world, unique_id);
    } catch (const cpde::DeviceError& e) {
        h->error = e.what();
        delete h->engine;
        h->engine = nullptr;
        return CPDE_DEVICE_ERROR;
    } catch (const std::exception& e) {
        h->error = e.what();
        delete h->engine;
        h->engine = nullptr;
        return CPDE_REJECTED;
    }
    return CPDE_OK;
}

int cpde_sharding_id(void* unique_id, size_t capacity) {
    if (!unique_id || capacity < sizeof(ncclUniqueId)) return CPDE_REJECTED;
    auto& nccl = cpde::Nccl::get();
    if (!nccl.available()) return CPDE_REJECTED;
    ncclUniqueId id;
    if (nccl.get_unique_id(&id) != ncclSuccess) return CPDE_DEVICE_ERROR;
    std::memcpy(unique_id, &id, sizeof(id));
    return CPDE_OK;
}

int cpde_shard_range(int64_t total, int32_t rank, int32_t world, int64_t* lo, int64_t* count) {
    if (total < 0 || world < 1 || rank < 0 || rank >= world || !lo || !count) return CPDE_REJECTED;
    const cpde::Shard s = cpde::shard_range(total, rank, world);
    *lo = s.lo;
    *count = s.count;
    return CPDE_OK;
}

void cpde_engine_destroy(cpde_engine* h) {
    if (!h) return;
    delete h->engine;
    delete h;
}

const char* cpde_last_error(const cpde_engine* h) { return h ? h->error.c_str() : "no engine"; }

int cpde_hello(cpde_engine* h, cpde_sink reply, void* ctx) {
    return guard(h, [&] {
        cpde::Payload out;
        out.put_string("CPDE/3");
        out.put<int32_t>(6);
        // 1 diagnostics, 2 graphs, 4 expressions, 8 RPROP restore, 16 wrapper
        // initialisation (cuda/cpde_server.cu:444), 128 tanh layers (new).
        out.put<uint32_t>(31u | 128u);
        reply(ctx, out.bytes.data(), out.bytes.size());
    });
}

int cpde_data_create(cpde_engine* h, int32_t d, int32_t c, int32_t s, int32_t v, const int32_t* table,
                     size_t table_count, const float* values, size_t count, uint64_t* id) {
    return guard(h, [&] { *id = E(h).create_data(d, c, s, v, table, table_count, values, count); });
}

int cpde_data_shape(cpde_engine* h, uint64_t id, int32_t* d, int32_t* c, int32_t* s) {
    return guard(h, [&] {
        auto& r = E(h).dat(id);
        *d = r.d;
        *c = r.h;
        *s = r.total;
    });
}

int cpde_data_download(cpde_engine* h, uint64_t id, float* values, size_t count) {
    return guard(h, [&] {
        auto& r = E(h).dat(id);
        cpde::require(count == size_t(r.d) * r.h * r.total, "download size mismatch");
        E(h).gather(r, values);
    });
}

int cpde_data_replace(cpde_engine* h, uint64_t id, const float* values, size_t count) {
    return guard(h, [&] { E(h).replace_data(id, values, count); });
}

int cpde_net_create(cpde_engine* h, const int32_t* neurons, const int32_t* linear, int32_t layers,
                    const float* const* initial, const size_t* counts, uint64_t* id) {
    return guard(h, [&] {
        cpde::require(layers >= 0 && layers <= 4096, "invalid architecture");
        std::vector<int> ns(neurons, neurons + layers), ls(linear, linear + layers);
        std::vector<std::vector<float>> init;
        if (initial && counts)
            for (int i = 0; i + 1 < layers; ++i) init.emplace_back(initial[i], initial[i] + counts[i]);
        *id = E(h).create_net(ns, ls, init);
    });
}

int cpde_net_evaluate(cpde_engine* h, uint64_t net, uint64_t data, int32_t chunk, uint64_t* output) {
    return guard(h, [&] { *output = E(h).evaluate(net, data, chunk); });
}

int cpde_net_snapshot(cpde_engine* h, uint64_t net, cpde_sink blob, void* ctx) {
    return guard(h, [&] {
        auto b = E(h).snapshot(E(h).net(net));
        blob(ctx, b.bytes.data(), b.bytes.size());
    });
}

int cpde_net_restore(cpde_engine* h, uint64_t net, const void* blob, size_t length) {
    return guard(h, [&] {
        cpde::Payload b(blob, length);
        E(h).restore(E(h).net(net), b);
    });
}

int cpde_cost_matching(cpde_engine* h, uint64_t net, uint64_t in, uint64_t tgt, int32_t chunk, const int32_t* rows,
                       size_t row_count, const int32_t* target_rows, size_t target_count, int32_t weight_samples,
                       const float* weights, size_t weight_count, uint64_t* id) {
    return guard(h, [&] {
        *id = E(h).cost_matching(net, in, tgt, chunk, std::vector<int>(rows, rows + row_count),
                                 std::vector<int>(target_rows, target_rows + target_count), weight_samples,
                                 std::vector<float>(weights, weights + weight_count));
    });
}

int cpde_cost_polynomial(cpde_engine* h, uint64_t net, uint64_t in, int32_t chunk, const int32_t* rows,
                         size_t row_count, int32_t equations, const int32_t* terms, size_t term_words,
                         const float* co, size_t co_count, const float* rhs, size_t rhs_count, const float* w,
                         size_t w_count, uint64_t* id) {
    return guard(h, [&] {
        *id = E(h).cost_polynomial(net, in, chunk, std::vector<int>(rows, rows + row_count), equations,
                                   std::vector<int>(terms, terms + term_words), std::vector<float>(co, co + co_count),
                                   std::vector<float>(rhs, rhs + rhs_count), std::vector<float>(w, w + w_count));
    });
}

int cpde_cost_integral(cpde_engine* h, uint64_t net, uint64_t in, int32_t chunk, int32_t samples,
                       const int32_t* nodes, size_t node_words, const double* constants, size_t constant_count,
                       int32_t fields, const double* field_values, size_t field_count, const double* weights,
                       size_t weight_count, uint64_t* id) {
    return guard(h, [&] {
        *id = E(h).cost_integral(net, in, chunk, samples, std::vector<int>(nodes, nodes + node_words),
                                 std::vector<double>(constants, constants + constant_count), fields,
                                 std::vector<double>(field_values, field_values + field_count),
                                 std::vector<double>(weights, weights + weight_count));
    });
}

int cpde_cost_source(cpde_engine* h, uint64_t id, int32_t compile, cpde_sink code, cpde_sink log, void* ctx) {
    return guard(h, [&] {
        auto& c = E(h).cost(id);
        cpde::require(bool(c.program), "not a compiled expression cost");
        if (compile) c.program->compile();
        code(ctx, c.program->code.data(), c.program->code.size());
        log(ctx, c.program->log.data(), c.program->log.size());
    });
}

int cpde_release(cpde_engine* h, int32_t kind, uint64_t id) {
    return guard(h, [&] { E(h).release(kind, id); });
}

int cpde_train(cpde_engine* h, int32_t graph_mode, const void* request, size_t length, cpde_event_sink events,
               void* ctx, const volatile int32_t* stop) {
    return guard(h, [&] {
        cpde::Payload b(request, length);
        E(h).train(b, graph_mode != 0, [&](uint32_t kind, const cpde::Payload& p) {
            events(ctx, kind, p.bytes.data(), p.bytes.size());
        }, stop);
    });
}

int cpde_graph_evaluate(cpde_engine* h, const void* request, size_t length, cpde_sink reply, void* ctx) {
    return guard(h, [&] {
        cpde::Payload b(request, length);
        auto out = E(h).graph_evaluate(b);
        reply(ctx, out.bytes.data(), out.bytes.size());
    });
}

int cpde_benchmark(cpde_engine* h, uint64_t net, uint64_t cost, int32_t warm, int32_t iterations, int32_t batches,
                   cpde_sink reply, void* ctx) {
    return guard(h, [&] {
        auto out = E(h).benchmark(net, cost, warm, iterations, batches);
        reply(ctx, out.bytes.data(), out.bytes.size());
    });
}

int cpde_epoch(cpde_engine* h, uint64_t net, const uint64_t* costs, size_t count) {
    return guard(h, [&] {
        std::vector<uint64_t> ids(costs, costs + count);
        auto& n = E(h).net(net);
        (void)n;
        E(h).epoch(net, ids);
    });
}

int cpde_epoch_result(cpde_engine* h, uint64_t net, double* objective, float* gradient, size_t count) {
    return guard(h, [&] {
        auto& e = E(h);
        auto& n = e.net(net);
        cpde::require(gradient == nullptr || count == size_t(n.params), "gradient size mismatch");
        e.check_device_errors();
        if (objective) {
            cpde::CostStats s;
            CPDE_CUDA(cudaMemcpy(&s, n.cost_totals.ptr, sizeof(s), cudaMemcpyDeviceToHost));
            *objective = s.value;
        }
        if (gradient)
            for (int l = 0; l < n.layers; ++l)
                CPDE_CUDA(cudaMemcpy(gradient + n.offset[l], n.gradient(l), n.count[l] * sizeof(float),
                                     cudaMemcpyDeviceToHost));
    });
}

int cpde_engine_stream(cpde_engine* h, void** stream) {
    return guard(h, [&] { *stream = (void*)E(h).stream; });
}

int cpde_kernel_timing(cpde_engine* h, int32_t enable) {
    return guard(h, [&] { E(h).timing(enable != 0); });
}

int cpde_kernel_timing_report(cpde_engine* h, cpde_sink report, void* ctx) {
    return guard(h, [&] {
        auto s = E(h).timing_report();
        report(ctx, s.data(), s.size());
    });
}

int cpde_set_tier(cpde_engine* h, int32_t tier) {
    return guard(h, [&] {
        cpde::require(tier >= 0 && tier <= 4,
                      "tier must be 0 (automatic), 1 (generic), 2 (tensor cores), 3 (point-tile epochs) or 4 "
                      "(exact-FP32 fast tier)");
        E(h).tier = tier;
    });
}

int cpde_jet_plan(const int32_t* counts, int32_t rows, int32_t variables, int32_t* packed, size_t capacity,
                  size_t* length) {
    try {
        if (rows <= 0 || variables <= 0 || !counts) return CPDE_REJECTED;
        std::vector<std::vector<int>> c(rows);
        for (int r = 0; r < rows; ++r) c[r].assign(counts + size_t(r) * variables, counts + size_t(r + 1) * variables);
        auto plan = cpde::JetPlan::build(c).pack();
        if (length) *length = plan.size();
        if (packed && capacity >= plan.size()) std::memcpy(packed, plan.data(), plan.size() * sizeof(int32_t));
        return CPDE_OK;
    } catch (...) {
        return CPDE_REJECTED;
    }
}

}  // extern "C"
