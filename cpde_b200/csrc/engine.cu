// Engine implementation: object commands, chunked passes, epochs, cost graphs.
//
// Command semantics (validation order and messages, pass ordering, reporting)
// follow the reference server cuda/cpde_server.cu; each function cites the
// lines it mirrors. Storage, kernels and reductions are this engine's own.
#include <algorithm>
#include <cfloat>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <numeric>

#include "engine_internal.hpp"

namespace cpde {

void Engine::timing(bool enable) {
    if (enable && !timer) timer.reset(new KernelTimer);
    if (!enable) timer.reset();
}

std::string Engine::timing_report() {
    std::string out;
    if (!timer) return out;
    timer->collect();
    for (auto& kv : timer->totals)
        out += kv.first + " " + std::to_string(kv.second.launches) + " " + std::to_string(kv.second.ms) + "\n";
    timer->totals.clear();
    return out;
}


// ---------------------------------------------------------------------------
// construction and lookup

Engine::Engine(int dev) : device(dev) {
    int count = 0;
    CPDE_CUDA(cudaGetDeviceCount(&count));
    require(dev >= 0 && dev < count, "invalid CUDA device");
    CPDE_CUDA(cudaSetDevice(device));
    CPDE_CUDA(cudaFree(nullptr));  // create the primary context
    CPDE_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    tc_error.resize(1);
    CPDE_CUDA(cudaMemsetAsync(tc_error.ptr, 0, sizeof(int), stream));
    CPDE_CUDA(cudaStreamSynchronize(stream));
}

// Cost totals <-> the buffers of the group reduction (sample indices made global).
__global__ void k_pack_costs(const CostStats* totals, const int* offsets, int count, double* values,
                             long long* keys) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += blockDim.x * gridDim.x) {
        const CostStats s = totals[i];
        values[i] = s.value;
        keys[i] = bad_entry_key(s.bad_sample == INT_MAX ? INT_MAX : s.bad_sample + offsets[i], s.bad_component);
    }
}
__global__ void k_unpack_costs(CostStats* totals, int count, const double* values, const long long* keys) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += blockDim.x * gridDim.x) {
        CostStats s;
        s.value = values[i];
        bad_entry_unkey(keys[i], s.bad_sample, s.bad_component);
        totals[i] = s;
    }
}

void Engine::check_device_errors() {
    int code = 0;
    CPDE_CUDA(cudaMemcpyAsync(&code, tc_error.ptr, sizeof(int), cudaMemcpyDeviceToHost, stream));
    CPDE_CUDA(cudaStreamSynchronize(stream));
    if (code) {
        CPDE_CUDA(cudaMemsetAsync(tc_error.ptr, 0, sizeof(int), stream));
        throw DeviceError(std::string("tensor-core kernel gave up waiting for ") +
                          (code == tcg::kErrTma ? "a TMA tile" : "an MMA") + "; results of this pass are invalid");
    }
}

// Joins a sharded group: one NCCL communicator per engine, on its device.
void Engine::join(int r, int n, const void* unique_id) {
    require(n >= 1 && r >= 0 && r < n && unique_id, "invalid shard rank or group size");
    auto& nccl = Nccl::get();
    if (!nccl.available()) throw DeviceError(nccl.load_error());
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    CPDE_CUDA(cudaSetDevice(device));
    nccl.check(nccl.comm_init_rank(&comm, n, id, r), "ncclCommInitRank");
    rank = r;
    world = n;
}

Engine::~Engine() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    if (comm_stream) cudaStreamSynchronize(comm_stream);
    if (comm) Nccl::get().comm_destroy(comm);
    for (auto e : layer_events) cudaEventDestroy(e);
    if (comm_done) cudaEventDestroy(comm_done);
    if (comm_stream) cudaStreamDestroy(comm_stream);
    costs.clear();
    nets.clear();
    data.clear();
    programs.clear();
    contexts.clear();
    timer.reset();
    if (stream) cudaStreamDestroy(stream);
}

template <class M>
static typename M::mapped_type::element_type& lookup(M& m, uint64_t id) {
    auto p = m.find(id);
    require(p != m.end(), "unknown or released object handle");
    return *p->second;
}
DataRecord& Engine::dat(uint64_t id) { return lookup(data, id); }
NetRecord& Engine::net(uint64_t id) { return lookup(nets, id); }
CostRecord& Engine::cost(uint64_t id) { return lookup(costs, id); }

// ---------------------------------------------------------------------------
// data (cuda/cpde_server.cu:449-454, 475-476)

uint64_t Engine::create_data(int d, int h, int w, int v, const int* table, size_t table_count, const float* values,
                             size_t count) {
    checked_size(d, h, w);
    require(v > 0 && v <= 26, "invalid variable count");
    require(table_count == size_t(d) * (v + 1) && count == size_t(d) * h * w, "data shape mismatch");
    auto rec = std::unique_ptr<DataRecord>(new DataRecord);
    const Shard part = shard(w);
    rec->d = d;
    rec->h = h;
    rec->w = int(part.count);
    rec->total = w;
    rec->lo = int(part.lo);
    rec->v = v;
    rec->table.assign(table, table + table_count);
    rec->values.resize(size_t(d) * h * part.count);
    upload_shard(*rec, values);
    CPDE_CUDA(cudaStreamSynchronize(stream));
    uint64_t id = next_id++;
    data[id] = std::move(rec);
    return id;
}

void Engine::replace_data(uint64_t id, const float* values, size_t count) {
    auto& d = dat(id);
    require(count == size_t(d.d) * d.h * d.total, "replacement data shape mismatch");
    upload_shard(d, values);
    CPDE_CUDA(cudaStreamSynchronize(stream));
    ++d.version;
}

// Copies this rank's samples of a host (row, sample, channel) array: one
// strided copy, a row of the shard per source row.
void Engine::upload_shard(DataRecord& d, const float* values) {
    if (d.w == 0) return;
    const size_t row = size_t(d.w) * d.h * sizeof(float);
    if (world == 1) {
        CPDE_CUDA(cudaMemcpyAsync(d.values.ptr, values, row * d.d, cudaMemcpyHostToDevice, stream));
        return;
    }
    CPDE_CUDA(cudaMemcpy2DAsync(d.values.ptr, row, values + size_t(d.lo) * d.h, size_t(d.total) * d.h * sizeof(float),
                                row, d.d, cudaMemcpyHostToDevice, stream));
}

// Download of a sharded array: every rank pads its shard to the largest one
// (rank 0's), one all-gather, then each rank's rows land at their samples.
void Engine::gather(DataRecord& d, float* host) {
    CPDE_CUDA(cudaStreamSynchronize(stream));
    if (world == 1) {
        CPDE_CUDA(cudaMemcpy(host, d.values.ptr, d.values.count * sizeof(float), cudaMemcpyDeviceToHost));
        return;
    }
    auto& nccl = Nccl::get();
    const long widest = shard_range(d.total, 0, world).count;
    const size_t slot = size_t(d.d) * widest * d.h;
    gather_send.reserve(std::max<size_t>(slot, 1));
    gather_recv.reserve(std::max<size_t>(slot * world, 1));
    if (d.w)
        CPDE_CUDA(cudaMemcpy2DAsync(gather_send.ptr, size_t(widest) * d.h * sizeof(float), d.values.ptr,
                                    size_t(d.w) * d.h * sizeof(float), size_t(d.w) * d.h * sizeof(float), d.d,
                                    cudaMemcpyDeviceToDevice, stream));
    nccl.check(nccl.all_gather(gather_send.ptr, gather_recv.ptr, slot, ncclFloat, comm, stream), "ncclAllGather");
    for (int q = 0; q < world; ++q) {
        const Shard s = shard_range(d.total, q, world);
        if (s.count)
            CPDE_CUDA(cudaMemcpy2DAsync(host + size_t(s.lo) * d.h, size_t(d.total) * d.h * sizeof(float),
                                        gather_recv.ptr + slot * q, size_t(widest) * d.h * sizeof(float),
                                        size_t(s.count) * d.h * sizeof(float), d.d, cudaMemcpyDeviceToHost, stream));
    }
    CPDE_CUDA(cudaStreamSynchronize(stream));
}

// Sums the cost totals over the group: values in double, and the first bad
// (global sample, component) by an integer minimum of its key.
void Engine::reduce_costs(NetRecord& n, const std::vector<uint64_t>& ids) {
    if (world == 1 || ids.empty()) return;
    auto& nccl = Nccl::get();
    const int count = int(ids.size());
    std::vector<int> offsets(count);
    for (int i = 0; i < count; ++i) {
        auto& c = cost(ids[i]);
        offsets[i] = c.input_id ? dat(c.input_id).lo : 0;
    }
    // a copy from pageable memory may wait for the stream to drain, which at
    // every epoch left the GPU idle while the host enqueued the next one; the
    // offsets change only with the cost set
    if (offsets != shard_offsets_host) {
        shard_offsets.upload(offsets, stream);
        shard_offsets_host = offsets;
    }
    shard_values.reserve(count);
    shard_keys.reserve(count);
    CPDE_RUN(*this, "pack_costs", k_pack_costs<<<grid_for(count), 256, 0, stream>>>(
                                      n.cost_totals.ptr, shard_offsets.ptr, count, shard_values.ptr, shard_keys.ptr));
    nccl.check(nccl.group_start(), "ncclGroupStart");
    nccl.check(nccl.all_reduce(shard_values.ptr, shard_values.ptr, count, ncclDouble, ncclSum, comm, stream),
               "ncclAllReduce");
    nccl.check(nccl.all_reduce(shard_keys.ptr, shard_keys.ptr, count, ncclInt64, ncclMin, comm, stream),
               "ncclAllReduce");
    nccl.check(nccl.group_end(), "ncclGroupEnd");
    CPDE_RUN(*this, "unpack_costs", k_unpack_costs<<<grid_for(count), 256, 0, stream>>>(
                                        n.cost_totals.ptr, count, shard_values.ptr, shard_keys.ptr));
}

// Marks layer `layer`'s gradient as complete so far in this epoch (the
// backward calls it after the last write of each chunk into that layer); the
// latest mark before reduce_gradient is the one its reduction waits for.
static void ensure_events(std::vector<cudaEvent_t>& events, std::vector<char>& marked, size_t count) {
    const size_t old = events.size();
    if (count <= old) return;
    events.resize(count);
    marked.resize(count, 0);
    for (size_t i = old; i < count; ++i) CPDE_CUDA(cudaEventCreateWithFlags(&events[i], cudaEventDisableTiming));
}

void Engine::layer_done(int layer) {
    if (world == 1) return;
    ensure_events(layer_events, layer_marked, size_t(layer) + 2);  // the last slot is the "now" event
    CPDE_CUDA(cudaEventRecord(layer_events[layer], stream));
    layer_marked[layer] = 1;
}

// Sums the weight gradients over the group: one all-reduce per layer, from
// the output layer down, on the communication stream, and the compute stream
// waits for all of them. Two schedules:
//  * tail (default): the reductions wait for the whole backward and go out
//    as one NCCL group (one launch);
//  * overlapped (CPDE_OVERLAP_ALLREDUCE=1): a layer's reduction waits only for
//    its completion mark of this epoch (or, unmarked, for everything enqueued
//    so far), so it runs beside the backward of the layers below.
// The tensor-core layers are persistent kernels with one CTA per SM that
// takes nearly all of its shared memory, so an NCCL kernel that starts in the
// middle of one holds SMs the next layer's CTAs wait for: measured on two
// B200s (config 2, order 6, 65,536 points per GPU) the overlapped schedule
// added 0.21 ms per epoch over one GPU's.
static bool overlap_allreduce() {
    static const bool on = [] {
        const char* v = std::getenv("CPDE_OVERLAP_ALLREDUCE");
        return v && v[0] == '1';
    }();
    return on;
}

void Engine::reduce_gradient(NetRecord& n, float* target) {
    if (world == 1) return;
    auto& nccl = Nccl::get();
    if (!comm_stream) {
        CPDE_CUDA(cudaStreamCreateWithFlags(&comm_stream, cudaStreamNonBlocking));
        CPDE_CUDA(cudaEventCreateWithFlags(&comm_done, cudaEventDisableTiming));
    }
    ensure_events(layer_events, layer_marked, size_t(n.layers) + 1);
    cudaEvent_t now = nullptr;
    KernelTimer* t = timer.get();
    cudaEvent_t t0 = nullptr, t1 = nullptr;
    const bool overlap = overlap_allreduce();
    if (!overlap) nccl.check(nccl.group_start(), "ncclGroupStart");
    for (int l = n.layers - 1; l >= 0; --l) {
        cudaEvent_t ready = overlap && layer_marked[l] ? layer_events[l] : nullptr;
        if (!ready) {
            if (!now) {
                now = layer_events.back();  // one past every layer index that marks use
                CPDE_CUDA(cudaEventRecord(now, stream));
            }
            ready = now;
        }
        CPDE_CUDA(cudaStreamWaitEvent(comm_stream, ready, 0));
        if (t && !t0) {
            t0 = t->get();
            CPDE_CUDA(cudaEventRecord(t0, comm_stream));
        }
        float* g = n.gradient_base(l, target);
        nccl.check(nccl.all_reduce(g, g, size_t(n.count[l]), ncclFloat, ncclSum, comm, comm_stream), "ncclAllReduce");
    }
    if (!overlap) nccl.check(nccl.group_end(), "ncclGroupEnd");
    std::fill(layer_marked.begin(), layer_marked.end(), 0);
    if (t) {
        t1 = t->get();
        CPDE_CUDA(cudaEventRecord(t1, comm_stream));
        t->marks.push_back({"allreduce_gradient", t0, t1});
    }
    CPDE_CUDA(cudaEventRecord(comm_done, comm_stream));
    CPDE_CUDA(cudaStreamWaitEvent(stream, comm_done, 0));
}

// ---------------------------------------------------------------------------
// schema contexts (cuda/cpde_server.cu:109-127)

std::vector<int> Engine::all_rows(DataRecord& d) {
    std::vector<int> rows(d.d);
    std::iota(rows.begin(), rows.end(), 0);
    std::stable_sort(rows.begin(), rows.end(), [&](int a, int b) { return d.order(a) < d.order(b); });
    return rows;
}

std::shared_ptr<Context> Engine::make_context(DataRecord& d, const std::vector<int>& rows, bool need_plan) {
    require(!rows.empty(), "empty derivative closure");
    int previous = -1;
    std::string key = std::to_string(d.v) + ":";
    for (int src : rows) {
        require(src >= 0 && src < d.d, "invalid derivative row");
        int order = d.order(src);
        require(order >= previous && order <= 6, "derivative closure must be sorted, orders 0..6");
        previous = order;
        for (int x : d.counts(src)) key.push_back(char('0' + x));
        key.push_back(',');
    }
    require(d.order(rows[0]) == 0, "value derivative must come first");
    std::string full = key + "|" + std::to_string(need_plan);
    // The context caches the copy-in row map too, so it is keyed by the data
    // rows themselves, not only by their multi-indices.
    for (int src : rows) full += std::to_string(src) + ";";
    auto it = contexts.find(full);
    if (it != contexts.end()) return it->second;
    auto ctx = std::make_shared<Context>();
    ctx->rows = rows;
    ctx->rows_dev.upload(rows, stream);
    if (need_plan) {
        std::vector<std::vector<int>> counts;
        for (int src : rows) counts.push_back(d.counts(src));
        ctx->plan = JetPlan::build(counts);
        ctx->tables.upload(ctx->plan.pack(), stream);
        ctx->planned = true;
        for (int sid = 0; sid < kStaticSchemas; ++sid) {
            const auto& info = kStaticSchemaInfo[sid];
            if (info.variables != d.v || info.rows != int(rows.size())) continue;
            bool same = true;
            for (int r = 0; r < info.rows && same; ++r)
                for (int v = 0; v < d.v; ++v)
                    same = same && kStaticSchemaCounts[info.offset + r * d.v + v] == counts[r][v];
            if (same) ctx->static_id = sid;
        }
    }
    CPDE_CUDA(cudaStreamSynchronize(stream));
    contexts[full] = ctx;
    return ctx;
}

// ---------------------------------------------------------------------------
// networks (cuda/cpde_server.cu:455-473; storage of cuda/cpde_engine.cuh:562-659)

uint64_t Engine::create_net(const std::vector<int>& ns, const std::vector<int>& ls,
                            const std::vector<std::vector<float>>& initial) {
    require(ns.size() >= 2 && ns.size() <= 256 && ns.size() == ls.size(), "invalid architecture");
    for (size_t i = 0; i < ns.size(); ++i) require(ns[i] > 0 && ls[i] >= 0 && ls[i] <= 2, "invalid layer");
    require(ls.front() == 1 && ls.back() == 1, "input and output layers must be linear");
    require(!initial.empty(), "initial weights required; update the Python wrapper");
    require(initial.size() == ns.size() - 1, "initial weight shape mismatch");
    for (size_t i = 1; i < ns.size(); ++i) {
        checked_size(ns[i], ns[i - 1] + 1);
        require(initial[i - 1].size() == size_t(ns[i]) * (size_t(ns[i - 1]) + 1), "initial weight shape mismatch");
        for (float x : initial[i - 1]) require(std::isfinite(x), "nonfinite initial weight");
    }
    auto r = std::unique_ptr<NetRecord>(new NetRecord);
    NetRecord& n = *r;
    n.neurons = ns;
    n.linear = ls;
    n.layers = int(ns.size()) - 1;
    long off = 0;
    for (int l = 0; l < n.layers; ++l) {
        n.offset.push_back(off);
        n.count.push_back(ns[l + 1] * (ns[l] + 1));
        off += n.count.back();
    }
    n.params = off;
    for (auto& b : n.bank) b.resize(n.params);
    std::vector<float> flat;
    flat.reserve(n.params);
    for (auto& a : initial) flat.insert(flat.end(), a.begin(), a.end());
    CPDE_CUDA(cudaMemcpyAsync(n.bank[0].ptr, flat.data(), flat.size() * 4, cudaMemcpyHostToDevice, stream));
    CPDE_CUDA(cudaMemsetAsync(n.bank[1].ptr, 0, n.params * 4, stream));
    CPDE_CUDA(cudaMemsetAsync(n.bank[2].ptr, 0, n.params * 4, stream));
    CPDE_RUN(*this, "fill", k_fill<<<grid_for(n.params), 256, 0, stream>>>(n.bank[3].ptr, n.params, .002f));
    n.active.assign(n.layers, 1);
    n.act.resize(n.layers + 1);
    n.pre.resize(n.layers + 1);
    std::vector<OptLayer> opt;
    for (int l = 0; l < n.layers; ++l) opt.push_back({n.offset[l], n.count[l], 1});
    n.opt_layers.upload(opt, stream);
    n.grad_counts.upload(n.count, stream);
    n.grad_ptrs.resize(n.layers);
    CPDE_CUDA(cudaStreamSynchronize(stream));
    uint64_t id = next_id++;
    nets[id] = std::move(r);
    return id;
}

static bool nonlinear_net(const NetRecord& n) {
    for (int x : n.linear)
        if (x != 1) return true;
    return false;
}

void Engine::ensure_arena(NetRecord& n, long columns, bool backward) {
    const int widest = *std::max_element(n.neurons.begin(), n.neurons.end());
    // an evaluation that grows the arena in the middle of training (the
    // outputs a training run prints) must leave the backward storage in place
    backward = backward || n.dz[0].ptr;
    if (columns > n.capacity) {
        CPDE_CUDA(cudaStreamSynchronize(stream));
        for (int l = 0; l <= n.layers; ++l) {
            n.act[l].resize(size_t(n.neurons[l]) * columns);
            n.pre[l].release();
        }
        n.jet_scratch.release();
        n.dz[0].release();
        n.dz[1].release();
        n.dy.release();
        n.capacity = columns;
        n.loaded_id = 0;
    }
    if (backward && n.dz[0].count < size_t(widest) * n.capacity) {
        n.dz[0].resize(size_t(widest) * n.capacity);
        n.dz[1].resize(size_t(widest) * n.capacity);
    }
}

// Slabs only the generic tier uses (pre-activations, the jet scratch and the
// backward's dE/dY), allocated on its first use so the fused tiers, which
// keep Z and dE/dY on chip, leave that memory to larger chunks.
static void ensure_generic_storage(NetRecord& n, bool backward) {
    const int widest = *std::max_element(n.neurons.begin(), n.neurons.end());
    for (int l = 0; l <= n.layers; ++l)
        if (n.linear[l] != 1) n.pre[l].reserve(size_t(n.neurons[l]) * n.capacity);
    n.jet_scratch.reserve(size_t(widest) * n.capacity);
    if (backward) n.dy.reserve(size_t(widest) * n.capacity);
}

void Engine::ensure_reductions(NetRecord& n, int count) {
    if (!n.cost_partials.ptr) {
        n.cost_partials.resize(kMaxReduceBlocks);
        n.cost_ticket.resize(1);
        CPDE_CUDA(cudaMemsetAsync(n.cost_ticket.ptr, 0, sizeof(unsigned), stream));
        n.grad_partials.resize(size_t(n.layers) * 256);
        n.grad_tickets.resize(n.layers);
        CPDE_CUDA(cudaMemsetAsync(n.grad_tickets.ptr, 0, n.layers * sizeof(unsigned), stream));
        n.grad_totals.resize(n.layers);
        n.host_grads.reserve(n.layers);
    }
    if (count > n.cost_capacity) {
        n.cost_totals.resize(count);
        n.host_costs.reserve(count);
        n.cost_capacity = count;
    }
}

void Engine::begin_costs(NetRecord& n, int count) {
    std::fill(layer_marked.begin(), layer_marked.end(), 0);  // completion marks belong to one epoch
    CPDE_RUN(*this, "clear_costs", k_clear_costs<<<1, 256, 0, stream>>>(n.cost_totals.ptr, count));
}

// ---------------------------------------------------------------------------
// chunk forward/backward (network::feedforward/backprop,
// cuda/cpde_engine.cuh:889-991, with the jet combine of
// cuda/derivative_kernels_v4.cu:349-745 replaced by the Leibniz tables)

void Engine::activate(NetRecord& n, uint64_t data_id, Context& ctx, int width, int offset, int valid) {
    auto& record = dat(data_id);
    if (n.loaded_id == data_id && n.loaded_version == record.version && n.loaded_width == width &&
        n.loaded_offset == offset && n.loaded_valid == valid && n.loaded_rows == ctx.rows)
        return;
    n.loaded_id = data_id;
    n.loaded_version = record.version;
    n.loaded_width = width;
    n.loaded_offset = offset;
    n.loaded_valid = valid;
    n.loaded_rows = ctx.rows;
    long total = long(valid) * ctx.R() * record.h;
    CPDE_RUN(*this, "stage_input",
             k_stage_input<<<grid_for(total), 256, 0, stream>>>(record.values.ptr, record.h, record.w,
                                                                 ctx.rows_dev.ptr, ctx.R(), offset, valid,
                                                                 n.act[0].ptr));
}

template <bool TA, bool TB, bool BIAS, bool IND>
static void launch_gemm(Engine& e, int M, int N, int K, const float* A, int lda, const float* B, int ldb, float* C,
                        int ldc, const float* bias, int R) {
    dim3 grid(gemm::column_tiles(N, IND), (M + gemm::BM - 1) / gemm::BM, 1);
    CPDE_RUN(e, "gemm", (k_gemm<TA, TB, BIAS, IND><<<grid, gemm::THREADS, 0, e.stream>>>(M, N, K, A, lda, B, ldb, C,
                                                                                          ldc, bias, R, K)));
}

void Engine::forward(NetRecord& n, Context& ctx, int points) {
    if (fast_ok(n, ctx)) return fast_forward(n, ctx, points, false);
    ensure_generic_storage(n, false);
    const int R = ctx.R();
    const int cols = points * R;
    for (int l = 1; l <= n.layers; ++l) {
        const int np = n.neurons[l - 1], nl = n.neurons[l];
        const float* W = n.weights(l - 1);
        const bool nonlin = n.linear[l] != 1;
        float* Z = nonlin ? n.pre[l].ptr : n.act[l].ptr;
        launch_gemm<false, false, true, false>(*this, nl, cols, np, W, nl, n.act[l - 1].ptr, np, Z, nl,
                                               W + long(nl) * np, R);
        if (!nonlin) continue;
        long total = long(nl) * points;
        const int sg = grid_for(total, kJetStagedThreads);
        const size_t sm = jet_staged_smem(R);
        if (R <= kJetStagedRows && n.linear[l] == kSigmoid)
            CPDE_RUN(*this, "jet_forward",
                     k_jet_forward_staged<Sigmoid><<<sg, kJetStagedThreads, sm, stream>>>(
                         Z, n.act[l].ptr, nl, points, R, ctx.tables.ptr));
        else if (R <= kJetStagedRows)
            CPDE_RUN(*this, "jet_forward",
                     k_jet_forward_staged<Tanh><<<sg, kJetStagedThreads, sm, stream>>>(
                         Z, n.act[l].ptr, nl, points, R, ctx.tables.ptr));
        else if (n.linear[l] == kSigmoid)
            CPDE_RUN(*this, "jet_forward",
                     k_jet_forward_dyn<Sigmoid><<<grid_for(total), 256, 0, stream>>>(
                         Z, n.act[l].ptr, n.jet_scratch.ptr, nl, points, R, ctx.tables.ptr));
        else
            CPDE_RUN(*this, "jet_forward",
                     k_jet_forward_dyn<Tanh><<<grid_for(total), 256, 0, stream>>>(Z, n.act[l].ptr, n.jet_scratch.ptr,
                                                                                  nl, points, R, ctx.tables.ptr));
    }
}

void Engine::backward(NetRecord& n, Context& ctx, int points, float* target) {
    if (fast_ok(n, ctx)) return fast_backward(n, ctx, points, target, false);
    ensure_generic_storage(n, true);
    const int R = ctx.R();
    const long cols = long(points) * R;
    float* cur = n.dz[0].ptr;
    for (int l = n.layers; l >= 1; --l) {
        const int np = n.neurons[l - 1], nl = n.neurons[l];
        // weight gradient with the bias column appended: (nl x np+1) += dZ (nl x cols) . [A; 1_value]^T
        const int M = nl, N = np + 1;
        long base = long((M + gemm::BM - 1) / gemm::BM) * gemm::column_tiles(N, true);
        long splits = std::max(1L, std::min((2L * 148 + base - 1) / base, (cols + 255) / 256));
        long per = ((cols + splits - 1) / splits + gemm::BK - 1) / gemm::BK * gemm::BK;
        splits = (cols + per - 1) / per;
        n.partial.reserve(size_t(splits) * M * N);
        dim3 grid(gemm::column_tiles(N, true), (M + gemm::BM - 1) / gemm::BM, unsigned(splits));
        CPDE_RUN(*this, "gemm_wgrad",
                 (k_gemm<false, true, false, true><<<grid, gemm::THREADS, 0, stream>>>(
                     M, N, int(cols), cur, nl, n.act[l - 1].ptr, np, n.partial.ptr, M, nullptr, R, int(per))));
        CPDE_RUN(*this, "splitk_reduce",
                 k_splitk_reduce<<<grid_for(long(M) * N), 256, 0, stream>>>(
                     n.partial.ptr, int(splits), M, N, n.gradient_base(l - 1, target), nl, 1));
        layer_done(l - 1);
        if (l == 1) break;
        float* next = cur == n.dz[0].ptr ? n.dz[1].ptr : n.dz[0].ptr;
        const float* W = n.weights(l - 1);
        if (n.linear[l - 1] == 1) {
            launch_gemm<true, false, false, false>(*this, np, int(cols), nl, W, nl, cur, nl, next, np, nullptr, R);
        } else {
            launch_gemm<true, false, false, false>(*this, np, int(cols), nl, W, nl, cur, nl, n.dy.ptr, np, nullptr, R);
            long total = long(np) * points;
            const int sg = grid_for(total, kJetStagedThreads);
            const size_t sm = jet_staged_smem(R);
            if (R <= kJetStagedRows && n.linear[l - 1] == kSigmoid)
                CPDE_RUN(*this, "jet_adjoint",
                         k_jet_adjoint_staged<Sigmoid><<<sg, kJetStagedThreads, sm, stream>>>(
                             n.dy.ptr, n.act[l - 1].ptr, next, np, points, R, ctx.tables.ptr));
            else if (R <= kJetStagedRows)
                CPDE_RUN(*this, "jet_adjoint",
                         k_jet_adjoint_staged<Tanh><<<sg, kJetStagedThreads, sm, stream>>>(
                             n.dy.ptr, n.act[l - 1].ptr, next, np, points, R, ctx.tables.ptr));
            else if (n.linear[l - 1] == kSigmoid)
                CPDE_RUN(*this, "jet_adjoint",
                         k_jet_adjoint_dyn<Sigmoid><<<grid_for(total), 256, 0, stream>>>(
                             n.dy.ptr, n.act[l - 1].ptr, n.jet_scratch.ptr, next, np, points, R, ctx.tables.ptr));
            else
                CPDE_RUN(*this, "jet_adjoint",
                         k_jet_adjoint_dyn<Tanh><<<grid_for(total), 256, 0, stream>>>(
                             n.dy.ptr, n.act[l - 1].ptr, n.jet_scratch.ptr, next, np, points, R, ctx.tables.ptr));
        }
        cur = next;
    }
}


bool Engine::fast_ok(NetRecord& n, Context& ctx) const {
    if (tier == 1 || ctx.static_id < 0) return false;
    const int L = n.layers;
    if (L < 3 || n.neurons[0] > 8 || n.neurons[L] > 8) return false;
    for (int l = 1; l < L; ++l)
        if (n.linear[l] == 1 || n.linear[l] != n.linear[1] || n.neurons[l] % 32 != 0) return false;
    return true;
}

// The fused head serves matching costs with 1 or 2 outputs after a 128-wide
// last hidden layer, or 1 output after a 256-wide one.
bool Engine::fused_head_ok(NetRecord& n, CostRecord& c, Context& ctx) const {
    const int K = n.neurons[n.layers - 1], O = n.neurons.back();
    return c.kind == 0 && fast_ok(n, ctx) && ((O <= 2 && K == 128) || (O == 1 && K == 256));
}

// The point-tile epoch (kernels_small.cuh) takes chunks whose forward is not
// reused, when the fused head applies, the gradient banks of all layers are
// one contiguous range, and the chunk is small enough (tier 0) or tier 3 asks.
bool Engine::point_epoch_ok(NetRecord& n, Context& ctx, long points, float* target) const {
    if (tier != 0 && tier != 3) return false;
    if (n.layers > small::kMaxLayers) return false;
    if (!target)
        for (int l = 1; l < n.layers; ++l)
            if (n.active[l] != n.active[0]) return false;
    // tensor-core layers overtake it sooner than FFMA layers (measured on the
    // 2->128^4->1 published workload: orders 4-6 favour tensor cores from ~8K columns)
    const long limit = use_tensor_cores(tier, ctx, n) ? point_epoch_columns / 4 : point_epoch_columns;
    return tier == 3 || points * ctx.R() <= limit;
}


void Engine::run_cost(NetRecord& n, CostRecord& c, int cost_index, int points, int offset, bool collect,
                      bool gradient, const double* multiplier) {
    const int outputs = n.neurons.back();
    const int R = c.context ? c.context->R() : 0;
    const float* y = n.act[n.layers].ptr;
    float* g = gradient ? n.dz[0].ptr : nullptr;
    CostReduce red{n.cost_partials.ptr, n.cost_ticket.ptr, n.cost_totals.ptr + cost_index};
    const int blocks = std::max(1, std::min(1024, (points + kReduceThreads - 1) / kReduceThreads));
    if (c.kind == 0) {
        auto& t = dat(c.target_id);
        CPDE_RUN(*this, "cost_matching",
                 k_cost_matching<<<blocks, kReduceThreads, 0, stream>>>(y, g, t.values.ptr, t.w, c.target_rows.ptr,
                                                                        c.weights.ptr, c.weight_samples, outputs, R,
                                                                        points, offset, collect, gradient, red));
    } else if (c.kind == 1) {
        CPDE_RUN(*this, "cost_polynomial",
                 k_cost_polynomial<<<blocks, kReduceThreads, 0, stream>>>(
                     y, g, c.terms.ptr, c.coefficients.ptr, c.term_count, c.rhs.ptr, c.weights.ptr, outputs, R,
                     c.equations, dat(c.input_id).w, points, offset, collect, gradient, red));
    } else {
        c.program->compile();
        int RO = R * outputs, samples = c.samples, col = collect, grad = gradient;
        const double* fields = c.fields.ptr;
        const double* weights = c.quadrature_weights.ptr;
        float* gp = g ? g : n.dz[0].ptr;
        if (!gp) gp = n.act[n.layers].ptr;  // never written when gradient == 0
        void* args[] = {(void*)&y,       (void*)&gp,      (void*)&fields, (void*)&weights, &RO,
                        &samples,        &points,         &offset,        (void*)&multiplier, &col,
                        &grad,           (void*)&red.partials, (void*)&red.ticket, (void*)&red.total};
        CPDE_RUN(*this, "cost_integral",
                 driver_check(driver_api().launch(c.program->kernel, blocks, 1, 1, kReduceThreads, 1, 1, 0, stream, args,
                                             nullptr),
                              "cuLaunchKernel"));
    }
    if (gradient && multiplier && c.kind != 2) {
        long count = long(points) * R * outputs;
        CPDE_RUN(*this, "scale", k_scale<<<grid_for(count), 256, 0, stream>>>(g, count, multiplier));
    }
}

// One cost over its chunks (Server::pass, cuda/cpde_server.cu:223-257).
void Engine::pass(NetRecord& n, CostRecord& c, int cost_index, bool bwd, bool collect, const double* multiplier,
                  int begin, int end, bool reuse_forward, bool backward_storage, float* target) {
    if (!c.input_id) return;
    bwd = bwd && c.has_gradient;
    backward_storage = backward_storage && c.has_gradient;
    auto& input = dat(c.input_id);
    end = std::min(end, input.w);
    require(begin >= 0 && begin % c.width == 0 && (!reuse_forward || long(end) - begin <= c.width),
            "invalid cost pass range");
    Context& ctx = *c.context;
    require(n.capacity >= long(c.width) * long(c.rows.size()) && n.dz[0].ptr && n.cost_totals.ptr,
            "internal error: network storage was not prepared for this cost");
    const bool fused = bwd && fused_head_ok(n, c, ctx);
    const bool expr_head = bwd && !fused && c.has_components && expression_head_ok(n, c, ctx);
    for (int offset = begin; offset < end; offset += c.width) {
        int valid = std::min(c.width, input.w - offset);
        const bool tile_epoch = fused && !reuse_forward && c.has_components && point_epoch_ok(n, ctx, valid, target);
        if (reuse_forward) {
            require(n.loaded_id == c.input_id && n.loaded_version == input.version && n.loaded_width == c.width &&
                        n.loaded_offset == offset && n.loaded_valid == valid && n.loaded_rows == c.rows,
                    "forward context is no longer current");
        } else {
            activate(n, c.input_id, ctx, c.width, offset, valid);
            if (tile_epoch) {
                point_epoch(n, c, ctx, valid, offset, collect, multiplier, cost_index, target);
                continue;
            }
            if (c.has_components) {
                if (fused || expr_head) fast_forward(n, ctx, valid, true);
                else forward(n, ctx, valid);
            }
        }
        if (expr_head) {
            CostReduce red{n.cost_partials.ptr, n.cost_ticket.ptr, n.cost_totals.ptr + cost_index};
            expression_head(n, c, ctx, valid, offset, collect, multiplier, red, target);
            fast_backward(n, ctx, valid, target, true);
            continue;
        }
        if (fused) {
            CostReduce red{n.cost_partials.ptr, n.cost_ticket.ptr, n.cost_totals.ptr + cost_index};
            fused_head(n, c, ctx, valid, offset, collect, multiplier, red, target);
            fast_backward(n, ctx, valid, target, true);
            continue;
        }
        run_cost(n, c, cost_index, valid, offset, collect, bwd, multiplier);
        if (bwd) backward(n, ctx, valid, target);
    }
}

void Engine::prepare_costs(NetRecord& n, const std::vector<uint64_t>& ids, uint64_t ni, bool bwd) {
    long columns = 1;
    for (auto id : ids) {
        auto& c = cost(id);
        require(c.network_id == ni, "cost belongs to another network");
        if (c.input_id) columns = std::max(columns, long(c.width) * long(c.rows.size()));
        if (c.program) c.program->compile();
    }
    (void)bwd;
    ensure_arena(n, columns, true);  // output adjoints are written even by value-only integral passes
    ensure_reductions(n, int(ids.size()));
}

// ---------------------------------------------------------------------------
// evaluation (cuda/cpde_server.cu:171-183)

uint64_t Engine::evaluate(uint64_t ni, uint64_t di, int chunk) {
    auto& n = net(ni);
    auto& input = dat(di);
    require(input.h == n.neurons.front(), "input channel mismatch");
    require((chunk ? std::min(chunk, input.total) : input.total) > 0, "invalid chunk size");
    int width = std::max(1, chunk ? std::min(chunk, input.w) : input.w);
    auto rows = all_rows(input);
    auto ctx = make_context(input, rows, nonlinear_net(n));
    ensure_arena(n, long(width) * ctx->R(), false);
    auto out = std::unique_ptr<DataRecord>(new DataRecord);
    out->d = input.d;
    out->h = n.neurons.back();
    out->w = input.w;
    out->total = input.total;
    out->lo = input.lo;
    out->v = input.v;
    out->table = input.table;
    out->values.resize(size_t(out->d) * out->h * out->w);
    for (int offset = 0; offset < input.w; offset += width) {
        int valid = std::min(width, input.w - offset);
        activate(n, di, *ctx, width, offset, valid);
        forward(n, *ctx, valid);
        long total = long(valid) * ctx->R() * out->h;
        CPDE_RUN(*this, "scatter_output",
                 k_scatter_output<<<grid_for(total), 256, 0, stream>>>(n.act[n.layers].ptr, out->h, ctx->R(),
                                                                        ctx->rows_dev.ptr, offset, valid, out->w,
                                                                        out->values.ptr));
    }
    check_device_errors();
    uint64_t id = next_id++;
    data[id] = std::move(out);
    return id;
}

// ---------------------------------------------------------------------------
// costs (cuda/cpde_server.cu:477-482, 489-533)

// Chunk width in samples of this rank's shard (at least 1, so an empty shard
// runs no chunks); the reference's "invalid chunk size" check applies to the
// whole data.
static int chunk_width(const DataRecord& d, int chunk) {
    require((chunk ? std::min(chunk, d.total) : d.total) > 0, "invalid chunk size");
    return std::max(1, chunk ? std::min(chunk, d.w) : d.w);
}

// [rows][samples][inner] host array -> the rows restricted to one shard's samples.
template <class T>
static std::vector<T> shard_rows(const std::vector<T>& a, size_t rows, long samples, long inner, Shard part) {
    std::vector<T> out(rows * size_t(part.count) * inner);
    for (size_t r = 0; r < rows; ++r)
        std::copy(a.begin() + (r * samples + part.lo) * inner, a.begin() + (r * samples + part.lo + part.count) * inner,
                  out.begin() + r * part.count * inner);
    return out;
}

uint64_t Engine::cost_matching(uint64_t ni, uint64_t in, uint64_t tgt, int chunk, std::vector<int> rows,
                               std::vector<int> tr, int ws, std::vector<float> w) {
    auto c = std::unique_ptr<CostRecord>(new CostRecord);
    c->network_id = ni;
    c->input_id = in;
    c->target_id = tgt;
    c->kind = 0;
    c->rows = rows;
    auto& n = net(ni);
    auto& d = dat(in);
    require(d.h == n.neurons.front(), "input channel mismatch");
    c->width = chunk_width(d, chunk);
    c->context = make_context(d, rows, nonlinear_net(n));
    auto& t = dat(tgt);
    require(t.h == n.neurons.back() && t.total == d.total, "target shape mismatch");
    require(tr.size() == rows.size() && (ws == 1 || ws == d.total) && w.size() == rows.size() * size_t(ws) * t.h,
            "matching weight shape mismatch");
    for (int r : tr) require(r >= 0 && r < t.d, "target derivative mismatch");
    for (float x : w) require(std::isfinite(x) && x >= 0, "invalid matching weight");
    if (ws > 1 && world > 1) {
        // per-sample weights follow the samples into the shards; a rank whose
        // shard is empty (more ranks than samples) keeps no weights and runs
        // no chunk of this cost, so its weight_samples of 0 is never read
        w = shard_rows(w, rows.size(), ws, t.h, shard(ws));
        ws = d.w;
    }
    c->weight_samples = ws;
    c->target_rows.upload(tr, stream);
    c->weights.upload(w, stream);
    CPDE_CUDA(cudaStreamSynchronize(stream));
    uint64_t id = next_id++;
    costs[id] = std::move(c);
    return id;
}

uint64_t Engine::cost_polynomial(uint64_t ni, uint64_t in, int chunk, std::vector<int> rows, int equations,
                                 std::vector<int> raw, std::vector<float> co, std::vector<float> rhs,
                                 std::vector<float> w) {
    auto c = std::unique_ptr<CostRecord>(new CostRecord);
    c->network_id = ni;
    c->input_id = in;
    c->kind = 1;
    c->rows = rows;
    auto& n = net(ni);
    auto& d = dat(in);
    require(d.h == n.neurons.front(), "input channel mismatch");
    c->width = chunk_width(d, chunk);
    c->context = make_context(d, rows, nonlinear_net(n));
    c->equations = equations;
    require(equations > 0 && raw.size() % 3 == 0 && co.size() == raw.size() / 3 * size_t(d.total) &&
                rhs.size() == size_t(equations) * d.total && w.size() == rhs.size(),
            "equation data shape mismatch");
    const long limit = long(rows.size()) * n.neurons.back();
    std::vector<PolyTerm> terms;
    for (size_t i = 0; i < raw.size(); i += 3) {
        require(raw[i] >= 0 && raw[i] < equations && raw[i + 1] >= 0 && raw[i + 1] < limit && raw[i + 2] >= -1 &&
                    raw[i + 2] < limit,
                "invalid polynomial term");
        terms.push_back({raw[i], raw[i + 1], raw[i + 2]});
    }
    for (float x : w) require(std::isfinite(x) && x >= 0, "invalid equation weight");
    for (float x : co) require(std::isfinite(x), "invalid coefficient");
    for (float x : rhs) require(std::isfinite(x), "invalid right-hand side");
    c->term_count = int(terms.size());
    if (world > 1) {
        const Shard part = shard(d.total);
        co = shard_rows(co, terms.size(), d.total, 1, part);
        rhs = shard_rows(rhs, size_t(equations), d.total, 1, part);
        w = shard_rows(w, size_t(equations), d.total, 1, part);
    }
    c->terms.upload(terms, stream);
    c->coefficients.upload(co, stream);
    c->rhs.upload(rhs, stream);
    c->weights.upload(w, stream);
    CPDE_CUDA(cudaStreamSynchronize(stream));
    uint64_t id = next_id++;
    costs[id] = std::move(c);
    return id;
}

uint64_t Engine::cost_integral(uint64_t ni, uint64_t in, int chunk, int samples, std::vector<int> raw,
                               std::vector<double> constants, int fields, std::vector<double> numeric,
                               std::vector<double> weights) {
    auto c = std::unique_ptr<CostRecord>(new CostRecord);
    c->kind = 2;
    c->network_id = ni;
    c->input_id = in;
    c->samples = samples;
    auto& n = net(ni);
    const int outputs = n.neurons.back();
    require(samples >= 0 && chunk >= 0 && fields >= 0 && fields <= 512 && weights.size() == size_t(samples) &&
                numeric.size() == size_t(fields) * samples,
            "invalid integral field shape");
    require(!constants.empty() && constants.size() <= 512 && raw.size() == constants.size() * 3,
            "invalid expression IR size");
    if (samples) {
        auto& d = dat(in);
        require(d.h == n.neurons.front() && d.total == samples, "integral input shape mismatch");
        std::vector<int> requested;
        for (size_t i = 0; i < constants.size(); ++i)
            if (raw[3 * i] == 1) {
                int component = raw[3 * i + 1];
                require(component >= 0 && long(component) < long(d.d) * outputs, "component outside derivative schema");
                requested.push_back(component / outputs);
            }
        for (int row : all_rows(d)) {
            bool needed = d.order(row) == 0;
            for (int target : requested) {
                bool dependency = true;
                auto a = d.counts(row), b = d.counts(target);
                for (size_t v = 0; v < a.size(); ++v)
                    if (a[v] > b[v]) {
                        dependency = false;
                        break;
                    }
                needed = needed || dependency;
            }
            if (needed) c->rows.push_back(row);
        }
        c->context = make_context(d, c->rows, nonlinear_net(n));
        c->width = chunk_width(d, chunk);
    } else {
        require(!in, "empty integral must not have input data");
        c->width = 0;
    }
    std::vector<ScalarNode> ir;
    for (int i = 0; i < int(constants.size()); ++i) {
        int op = raw[3 * i], a = raw[3 * i + 1], mask = raw[3 * i + 2];
        require(op >= 0 && op <= 14 && std::isfinite(constants[i]), "invalid expression node");
        if (op == 1) {
            require(a >= 0 && (mask == 0 || mask == 1), "invalid component");
            if (samples) {
                auto row = std::find(c->rows.begin(), c->rows.end(), a / outputs);
                require(row != c->rows.end(), "component outside derivative closure");
                a = int(row - c->rows.begin()) * outputs + a % outputs;
            }
        }
        if (op == 2) require(a >= 0 && a < fields, "invalid field index");
        if (op >= 3) {
            require(a >= 0 && a < i, "invalid expression dependency");
            if (op <= 6) require(mask >= 0 && mask < i, "invalid expression dependency");
        }
        ir.push_back({op, a, mask, constants[i]});
    }
    for (double x : numeric) require(std::isfinite(x), "nonfinite integral field");
    for (double x : weights) require(std::isfinite(x), "nonfinite quadrature weight");
    c->has_components = false;
    c->has_gradient = false;
    for (const auto& node : ir)
        if (node.op == 1) {
            c->has_components = true;
            if (node.b == 0) c->has_gradient = true;
        }
    auto source = expression_source(ir);
    auto found = programs.find(source);
    if (found == programs.end())
        found = programs.emplace(source, std::make_shared<ExpressionProgram>(std::move(ir))).first;
    c->program = found->second;
    if (samples && world > 1) {
        const Shard part = shard(samples);
        numeric = shard_rows(numeric, size_t(fields), samples, 1, part);
        weights = shard_rows(weights, 1, samples, 1, part);
        c->samples = int(part.count);
    }
    c->fields.upload(numeric, stream);
    c->quadrature_weights.upload(weights, stream);
    CPDE_CUDA(cudaStreamSynchronize(stream));
    uint64_t id = next_id++;
    costs[id] = std::move(c);
    return id;
}

void Engine::release(int kind, uint64_t id) {
    if (kind == 0) {
        for (auto& c : costs)
            require(c.second->input_id != id && c.second->target_id != id,
                    "data is retained by a cost; close that cost first");
        data.erase(id);
    } else if (kind == 1) {
        for (auto& c : costs)
            require(c.second->network_id != id, "network is retained by a cost; close that cost first");
        nets.erase(id);
    } else if (kind == 2) {
        costs.erase(id);
    } else {
        require(false, "invalid object kind");
    }
}

// ---------------------------------------------------------------------------
// optimizer state (cuda/cpde_server.cu:184-222; cuda/cpde_engine.cuh:916-945,993-1014)

void Engine::reset_optimizer(NetRecord& n, int method) {
    CPDE_CUDA(cudaStreamSynchronize(stream));
    for (int l = 0; l < n.layers; ++l) n.active[l] = 1;
    for (int b = 1; b < 4; ++b) CPDE_CUDA(cudaMemsetAsync(n.bank[b].ptr, 0, n.params * 4, stream));
    if (method == 0) set_steps(n, n.initial_step);
    n.optimizer = method;
    n.adam_step = 0;
}

static std::vector<OptLayer> opt_table(NetRecord& n) {
    std::vector<OptLayer> t;
    for (int l = 0; l < n.layers; ++l) t.push_back({n.offset[l], n.count[l], n.active[l]});
    return t;
}

void Engine::set_steps(NetRecord& n, float value) {
    CPDE_RUN(*this, "fill", k_fill<<<grid_for(n.params), 256, 0, stream>>>(n.bank[3].ptr, n.params, value));
    CPDE_CUDA(cudaMemsetAsync(n.bank[1].ptr, 0, n.params * 4, stream));
    CPDE_CUDA(cudaMemsetAsync(n.bank[2].ptr, 0, n.params * 4, stream));
}

void Engine::floor_steps(NetRecord& n, float value) {
    int widest = *std::max_element(n.count.begin(), n.count.end());
    dim3 grid(grid_for(widest, 256, 256), n.layers);
    CPDE_RUN(*this, "rprop_floor",
             k_rprop_floor<<<grid, 256, 0, stream>>>(n.bank[1].ptr, n.bank[2].ptr, n.bank[3].ptr, n.opt_layers.ptr,
                                                      value));
}

AdamStep Engine::adam_step(NetRecord& n, int step) {
    return AdamStep{n.learning_rate, 0.9f, 0.999f, std::pow(0.9f, float(step)), std::pow(0.999f, float(step))};
}

// Gradient statistics, the update gate and the optimizer update in one launch
// (k_inspect_update), then one download of the cost totals, the statistics
// and the gate's decision. The caller validates with the reference's rules
// and messages and commits the host side of the update with commit_update.
bool Engine::inspect_and_update(NetRecord& n, int method, int costs, GraphRecord* g) {
    n.opt_layers.upload(opt_table(n), stream);
    n.update_applied.reserve(1);
    n.host_applied.reserve(1);
    require(method == 0 || n.adam_step < uint64_t(INT_MAX), "Adam counter exceeds supported range");
    const int* graph_bad =
        g ? reinterpret_cast<const int*>(reinterpret_cast<const char*>(g->summary.ptr) +
                                         offsetof(GraphRecord::Summary, bad_node))
          : nullptr;
    CPDE_RUN(*this, "inspect_update",
             k_inspect_update<<<1, 1024, 0, stream>>>(n.bank[0].ptr, n.bank[1].ptr, n.bank[2].ptr, n.bank[3].ptr,
                                                      n.opt_layers.ptr, n.layers, n.grad_totals.ptr,
                                                      n.cost_totals.ptr, costs, graph_bad, method,
                                                      adam_step(n, int(n.adam_step + 1)), n.update_applied.ptr));
    CPDE_CUDA(cudaMemcpyAsync(n.host_applied.ptr, n.update_applied.ptr, sizeof(int), cudaMemcpyDeviceToHost, stream));
    download(n, costs, n.layers);
    return n.host_applied.ptr[0] != 0;
}

// Host side of an update that k_inspect_update applied: RPROP's gradient
// history alternates banks, Adam counts its step.
void Engine::commit_update(NetRecord& n, int method) {
    if (method == 0)
        for (int l = 0; l < n.layers; ++l) n.active[l] = 3 - n.active[l];
    else
        ++n.adam_step;
}

Payload Engine::metadata(NetRecord& n) {
    Payload b;
    b.put<uint32_t>(1);
    b.put_array(n.neurons);
    b.put_array(n.linear);
    b.put<int32_t>(n.optimizer);
    b.put<uint64_t>(n.updates);
    b.put<uint64_t>(n.adam_step);
    b.put<uint64_t>(n.stage_done);
    b.put<uint64_t>(n.remaining);
    b.put<float>(n.learning_rate);
    b.put<float>(n.initial_step);
    b.put_string(n.stage);
    return b;
}

Payload Engine::snapshot(NetRecord& n) {
    CPDE_CUDA(cudaStreamSynchronize(stream));
    Payload b = metadata(n);
    std::vector<float> host(n.params);
    std::vector<std::vector<float>> banks(4, std::vector<float>(n.params));
    for (int j = 0; j < 4; ++j)
        CPDE_CUDA(cudaMemcpy(banks[j].data(), n.bank[j].ptr, n.params * 4, cudaMemcpyDeviceToHost));
    for (int l = 0; l < n.layers; ++l) {
        b.put<int32_t>(n.active[l]);
        for (int j = 0; j < 4; ++j) b.put_array(banks[j].data() + n.offset[l], size_t(n.count[l]));
    }
    return b;
}

void Engine::restore(NetRecord& n, Payload& b) {
    require(b.get<uint32_t>() == 1, "unsupported state version");
    require(b.array<int>() == n.neurons && b.array<int>() == n.linear, "state architecture mismatch");
    int optimizer = b.get<int32_t>();
    require(optimizer >= -1 && optimizer <= 1, "invalid optimizer state");
    uint64_t updates = b.get<uint64_t>(), adam = b.get<uint64_t>(), done = b.get<uint64_t>(),
             remaining = b.get<uint64_t>();
    float lr = b.get<float>(), step = b.get<float>();
    auto stage = b.string();
    require(std::isfinite(lr) && lr > 0 && std::isfinite(step) && step > 0, "invalid optimizer settings");
    std::vector<int> active;
    std::vector<std::vector<float>> banks(4, std::vector<float>(n.params));
    for (int l = 0; l < n.layers; ++l) {
        int a = b.get<int32_t>();
        require(a == 1 || a == 2, "invalid active gradient buffer");
        active.push_back(a);
        for (int j = 0; j < 4; ++j) {
            auto v = b.array<float>();
            require(v.size() == size_t(n.count[l]), "state buffer shape mismatch");
            std::copy(v.begin(), v.end(), banks[j].begin() + n.offset[l]);
        }
    }
    b.end();
    CPDE_CUDA(cudaStreamSynchronize(stream));
    n.active = active;
    for (int j = 0; j < 4; ++j)
        CPDE_CUDA(cudaMemcpy(n.bank[j].ptr, banks[j].data(), n.params * 4, cudaMemcpyHostToDevice));
    n.optimizer = optimizer;
    n.updates = updates;
    n.adam_step = adam;
    n.stage_done = done;
    n.remaining = remaining;
    n.learning_rate = lr;
    n.initial_step = step;
    n.stage = stage;
}

// ---------------------------------------------------------------------------
// reductions and validation (cuda/cpde_server.cu:323-352; cuda/reduction_kernels.cuh:252-267)

void Engine::inspect_gradients(NetRecord& n, float* target) {
    std::vector<const float*> ptrs;
    for (int l = 0; l < n.layers; ++l) ptrs.push_back(n.gradient_base(l, target));
    n.grad_ptrs.upload(ptrs, stream);
    int widest = *std::max_element(n.count.begin(), n.count.end());
    dim3 grid(grid_for(widest, 256, 256), n.layers);
    GradReduce red{n.grad_partials.ptr, n.grad_tickets.ptr, n.grad_totals.ptr};
    std::vector<GradStats> empty(n.layers, grad_empty());
    CPDE_CUDA(cudaMemcpyAsync(n.grad_totals.ptr, empty.data(), n.layers * sizeof(GradStats), cudaMemcpyHostToDevice,
                              stream));
    CPDE_RUN(*this, "inspect_gradients",
             k_inspect_gradients<<<grid, 256, 0, stream>>>(n.grad_ptrs.ptr, n.grad_counts.ptr, red));
    CPDE_CUDA(cudaStreamSynchronize(stream));  // keeps `empty` alive until the copy completes
}

void Engine::download(NetRecord& n, int count, int layers) {
    check_device_errors();
    if (count)
        CPDE_CUDA(cudaMemcpyAsync(n.host_costs.ptr, n.cost_totals.ptr, count * sizeof(CostStats),
                                  cudaMemcpyDeviceToHost, stream));
    if (layers)
        CPDE_CUDA(cudaMemcpyAsync(n.host_grads.ptr, n.grad_totals.ptr, layers * sizeof(GradStats),
                                  cudaMemcpyDeviceToHost, stream));
    CPDE_CUDA(cudaStreamSynchronize(stream));
}

void Engine::validate_costs(NetRecord& n, size_t count, std::vector<double>& values, bool before_update) {
    const std::string phase = before_update ? "; no optimizer update performed for this iteration"
                                            : " during objective evaluation";
    for (size_t i = 0; i < count; ++i) {
        const auto& c = n.host_costs.ptr[i];
        values[i] = c.value;
        if (c.bad_sample != INT_MAX) {
            std::string what = c.bad_component < 0 ? "objective" : "dE/dY component " + std::to_string(c.bad_component);
            throw RequestError("non-finite " + what + " at cost index " + std::to_string(i) + ", sample " +
                               std::to_string(c.bad_sample) + phase);
        }
        if (!std::isfinite(c.value)) throw RequestError("non-finite reduced objective" + phase);
    }
}

// ---------------------------------------------------------------------------
// cost graphs (cuda/cpde_server.cu:38-70, cuda/cost_graph.cuh:6-27,
// cuda/graph_schedule.hpp:18-55)

__global__ void k_graph_execute(const ScalarNode* nodes, int count, int root, const CostStats* integrals, int leaves,
                                double* values, double* adjoints, double* multipliers, int* active,
                                GraphRecord::Summary* summary, int gradient) {
    if (blockIdx.x || threadIdx.x) return;
    int bad = -1;
    for (int i = 0; i < leaves; ++i) multipliers[i] = 0;
    for (int i = 0; i < count; ++i) {
        ScalarNode n = nodes[i];
        adjoints[i] = 0;
        active[i] = n.op == kLeaf;
        if (n.op == kLeaf) {
            values[i] = integrals[n.a].value;
        } else {
            values[i] = scalar_value(n.op, n.a < 0 ? 0 : values[n.a], n.b < 0 ? 0 : values[n.b], n.parameter);
            if (n.op > kField)
                active[i] = active[n.a] || ((n.op <= kDiv || n.op == kAttach) && active[n.b]);
        }
        if (!isfinite(values[i]) && bad < 0) bad = i;
    }
    summary->value = values[root];
    summary->bad_node = bad;
    if (!gradient || bad >= 0) return;
    adjoints[root] = 1;
    for (int i = count - 1; i >= 0; --i) {
        ScalarNode n = nodes[i];
        double seed = adjoints[i];
        if (seed == 0 || !active[i]) continue;
        if (n.op == kLeaf) {
            multipliers[n.a] += seed;
        } else if (n.op > kField) {
            double da, db;
            scalar_partials(n.op, values[n.a], n.b < 0 ? 0 : values[n.b], values[i], n.parameter, da, db);
            if (active[n.a]) adjoints[n.a] += seed * da;
            if ((n.op <= kDiv || n.op == kAttach) && active[n.b]) adjoints[n.b] += seed * db;
        }
        if (!isfinite(seed) && bad < 0) bad = i;
    }
    for (int i = 0; i < leaves; ++i)
        if (!isfinite(multipliers[i])) bad = root;
    summary->bad_node = bad;
}

// Which leaf multipliers are known before any integral is evaluated.
static std::vector<GraphRecord::Known> graph_schedule(const std::vector<ScalarNode>& nodes, int root, int leaves) {
    using K = GraphRecord::Known;
    auto known = [](double v) { return K{std::isfinite(v), v}; };
    const K unknown{false, 0};
    auto sum = [&](K a, K b) { return a.known && b.known ? known(a.value + b.value) : unknown; };
    auto product = [&](K a, K b) {
        if ((a.known && a.value == 0) || (b.known && b.value == 0)) return known(0);
        return a.known && b.known ? known(a.value * b.value) : unknown;
    };
    size_t count = nodes.size();
    std::vector<K> values(count, unknown), da(count, unknown), db(count, unknown);
    std::vector<bool> active(count, false);
    for (size_t i = 0; i < count; ++i) {
        auto n = nodes[i];
        if (n.op == kConstant) {
            values[i] = known(n.parameter);
            continue;
        }
        if (n.op == kLeaf) {
            active[i] = true;
            continue;
        }
        bool binary = n.op <= kDiv || n.op == kAttach;
        K a = values[n.a], b = binary ? values[n.b] : known(0);
        active[i] = active[n.a] || (binary && active[n.b]);
        if (a.known && (b.known || n.op == kAttach)) values[i] = known(scalar_value(n.op, a.value, b.value, n.parameter));
        if (n.op == kAdd || n.op == kAttach) {
            da[i] = db[i] = known(1);
        } else if (n.op == kSub) {
            da[i] = known(1);
            db[i] = known(-1);
        } else if (n.op == kMul) {
            da[i] = b;
            db[i] = a;
        } else if (n.op == kDiv) {
            if (b.known && b.value != 0) {
                da[i] = known(1 / b.value);
                if (a.known) db[i] = known(-(a.value / b.value) / b.value);
            }
        } else if (n.op == kNeg) {
            da[i] = known(-1);
        } else if (n.op == kPower && (n.parameter == 0 || n.parameter == 1)) {
            da[i] = known(n.parameter);
        } else if (a.known && values[i].known) {
            double x, y;
            scalar_partials(n.op, a.value, b.value, values[i].value, n.parameter, x, y);
            da[i] = known(x);
        }
    }
    std::vector<K> adjoints(count, known(0)), multipliers(leaves, known(0));
    adjoints[root] = known(1);
    for (int i = int(count) - 1; i >= 0; --i) {
        auto n = nodes[i];
        K seed = adjoints[i];
        if (!active[i] || (seed.known && seed.value == 0)) continue;
        if (n.op == kLeaf) {
            multipliers[n.a] = sum(multipliers[n.a], seed);
        } else {
            if (active[n.a]) adjoints[n.a] = sum(adjoints[n.a], product(seed, da[i]));
            if ((n.op <= kDiv || n.op == kAttach) && active[n.b]) adjoints[n.b] = sum(adjoints[n.b], product(seed, db[i]));
        }
    }
    return multipliers;
}

void Engine::read_graph(GraphRecord& g, Payload& b, int leaves) {
    auto raw = b.array<int>();
    auto constants = b.array<double>();
    g.root = b.get<int>();
    require(!constants.empty() && constants.size() <= 4096 && raw.size() == 3 * constants.size() && g.root >= 0 &&
                g.root < int(constants.size()),
            "invalid cost graph size");
    for (int i = 0; i < int(constants.size()); ++i) {
        int op = raw[3 * i], a = raw[3 * i + 1], c = raw[3 * i + 2];
        require(std::isfinite(constants[i]), "nonfinite graph constant");
        require(op == 0 || op == 1 || (op >= 3 && op <= 15), "invalid graph opcode");
        if (op == 1) require(a >= 0 && a < leaves, "invalid graph leaf");
        if (op >= 3) {
            require(a >= 0 && a < i, "graph must be topologically ordered");
            if (op <= 6 || op == 15) require(c >= 0 && c < i, "invalid graph child");
        }
        g.nodes.push_back({op, a, c, constants[i]});
    }
    size_t count = g.nodes.size();
    g.nodes_dev.upload(g.nodes, stream);
    g.values.resize(count);
    g.adjoints.resize(count);
    g.active.resize(count);
    g.multipliers.resize(std::max(1, leaves));
    g.summary.resize(1);
    g.host.reserve(1);
    g.host.ptr[0] = {0, -1, 0};
    g.schedule = graph_schedule(g.nodes, g.root, leaves);
    std::vector<double> fixed(std::max(1, leaves), 0.0);
    for (int i = 0; i < leaves; ++i)
        if (g.schedule[i].known) fixed[i] = g.schedule[i].value;
    g.fixed_multipliers.upload(fixed, stream);
    CPDE_CUDA(cudaStreamSynchronize(stream));
}

void Engine::run_graph(GraphRecord& g, NetRecord& n, int leaves, bool gradient) {
    CPDE_RUN(*this, "graph_execute",
             k_graph_execute<<<1, 1, 0, stream>>>(g.nodes_dev.ptr, int(g.nodes.size()), g.root, n.cost_totals.ptr,
                                                  leaves, g.values.ptr, g.adjoints.ptr, g.multipliers.ptr,
                                                  g.active.ptr, g.summary.ptr, gradient));
}

// Server::graph_pass (cuda/cpde_server.cu:273-318): leaves whose multiplier is
// known run forward+backward at once; the others contribute values first, the
// graph runs on device, then they run backward with device multipliers. The
// most expensive such leaf runs last so its final chunk's forward is reused.
void Engine::graph_pass(NetRecord& n, const std::vector<uint64_t>& ids, GraphRecord& g, bool bwd, float* target) {
    begin_costs(n, int(ids.size()));
    int reuse = -1, last_offset = 0;
    double best_work = -1;
    if (bwd) {
        for (int l = 0; l < n.layers; ++l)
            CPDE_CUDA(cudaMemsetAsync(n.gradient_base(l, target), 0, n.count[l] * 4, stream));
        for (size_t i = 0; i < ids.size(); ++i) {
            if (g.schedule[i].known) continue;
            auto& c = cost(ids[i]);
            if (!c.input_id || !c.has_gradient || !c.has_components) continue;
            auto& d = dat(c.input_id);
            double derivative_work = 0, work = 0;
            for (int r : c.rows) derivative_work += std::ldexp(1.0, d.order(r));
            for (int l = 0; l < n.layers; ++l) {
                work += 2.0 * n.neurons[l] * n.neurons[l + 1] * c.rows.size();
                if (n.linear[l] != 1) work += n.neurons[l] * derivative_work;
            }
            work *= c.width;
            if (work > best_work) {
                best_work = work;
                reuse = int(i);
            }
        }
    }
    for (size_t i = 0; i < ids.size(); ++i) {
        if (int(i) == reuse) continue;
        bool immediate = bwd && g.schedule[i].known && g.schedule[i].value != 0;
        pass(n, cost(ids[i]), int(i), immediate, true, immediate ? g.fixed_multipliers.ptr + i : nullptr, 0, INT_MAX,
             false, bwd, target);
    }
    if (reuse >= 0) {
        auto& c = cost(ids[reuse]);
        last_offset = ((dat(c.input_id).w - 1) / c.width) * c.width;
        pass(n, c, reuse, false, true, nullptr, 0, INT_MAX, false, true, target);
    }
    reduce_costs(n, ids);  // leaf integrals over all ranks before the graph runs
    run_graph(g, n, int(ids.size()), bwd);
    if (bwd) {
        if (reuse >= 0)
            pass(n, cost(ids[reuse]), reuse, true, false, g.multipliers.ptr + reuse, last_offset, INT_MAX, true, true,
                 target);
        for (size_t i = 0; i < ids.size(); ++i)
            if (!g.schedule[i].known)
                pass(n, cost(ids[i]), int(i), true, false, g.multipliers.ptr + i, 0,
                     int(i) == reuse ? last_offset : INT_MAX, false, true, target);
        reduce_gradient(n, target);
    }
    CPDE_CUDA(cudaMemcpyAsync(g.host.ptr, g.summary.ptr, sizeof(GraphRecord::Summary), cudaMemcpyDeviceToHost,
                              stream));
}

static void graph_validate(GraphRecord& g) {
    if (g.host.ptr[0].bad_node >= 0)
        throw RequestError("invalid value or derivative in cost graph node " + std::to_string(g.host.ptr[0].bad_node));
}

void Engine::evaluate_costs(NetRecord& n, const std::vector<uint64_t>& ids, std::vector<double>& values,
                            GraphRecord* g) {
    if (g) {
        graph_pass(n, ids, *g, false, nullptr);
        download(n, int(ids.size()), 0);
        validate_costs(n, ids.size(), values, false);
        graph_validate(*g);
        return;
    }
    begin_costs(n, int(ids.size()));
    for (size_t i = 0; i < ids.size(); ++i)
        pass(n, cost(ids[i]), int(i), false, true, nullptr, 0, INT_MAX, false, false, nullptr);
    reduce_costs(n, ids);
    download(n, int(ids.size()), 0);
    validate_costs(n, ids.size(), values, false);
}

void Engine::report_values(NetRecord& n, uint64_t completed, int after, const std::vector<double>& values,
                           GraphRecord* g, const EventSink& emit) {
    Payload r;
    r.put<uint64_t>(completed);
    r.put<uint64_t>(n.updates);
    r.put<int32_t>(after);
    r.put_array(values);
    if (g) r.put<double>(g->host.ptr[0].value);
    emit(g ? 6 : 2, r);
}

void Engine::gradient_report(NetRecord& n, uint64_t epoch, const EventSink& emit) {
    Payload r;
    r.put<uint64_t>(epoch);
    r.put<uint64_t>(n.updates);
    r.put<int32_t>(n.layers);
    for (int i = 0; i < n.layers; ++i) {
        const auto& g = n.host_grads.ptr[i];
        r.put<double>(g.squared_norm);
        r.put<double>(g.max_abs);
        r.put<uint64_t>(g.nonfinite);
        r.put<int32_t>(g.first_nonfinite == INT_MAX ? -1 : g.first_nonfinite);
    }
    emit(5, r);
}

// ---------------------------------------------------------------------------
// training (Server::train, cuda/cpde_server.cu:364-435)

void Engine::train(Payload& b, bool graph_mode, const EventSink& emit, const volatile int32_t* stop) {
    uint64_t ni = b.get<uint64_t>();
    auto& n = net(ni);
    auto ids = b.array<uint64_t>();
    uint64_t epochs = b.get<uint64_t>();
    int method = b.get<int32_t>(), fresh = b.get<int32_t>();
    float steps = b.get<float>();
    int moments = b.get<int32_t>();
    float lr = b.get<float>();
    int verbose = b.get<int32_t>(), log = b.get<int32_t>(), eval = b.get<int32_t>(), outputs = b.get<int32_t>(),
        save = b.get<int32_t>();
    (void)verbose;
    auto stage = b.string();
    int diagnostics = b.get<int32_t>();
    std::unique_ptr<GraphRecord> graph;
    if (graph_mode) {
        graph.reset(new GraphRecord);
        read_graph(*graph, b, int(ids.size()));
    }
    uint64_t restore_every = 0;
    float restore_step = 0;
    if (b.more()) {
        restore_every = b.get<uint64_t>();
        restore_step = b.get<float>();
    }
    b.end();
    require(!ids.empty() && epochs > 0, "training needs costs and positive epochs");
    require(method == 0 || method == 1, "unknown optimizer");
    require(ids.size() <= INT_MAX && log >= 0 && eval >= 0 && save >= 0 && diagnostics >= 0 && std::isfinite(lr) &&
                lr >= 0 && std::isfinite(steps) && steps >= 0,
            "invalid training controls");
    require((restore_every == 0 && restore_step == 0) ||
                (restore_every > 0 && method == 0 && std::isfinite(restore_step) && restore_step >= FLT_MIN),
            "invalid periodic RPROP restoration controls");
    prepare_costs(n, ids, ni, true);
    if (fresh || n.optimizer != method) reset_optimizer(n, method);
    if (lr > 0) n.learning_rate = lr;
    if (steps > 0) {
        require(method == 0, "reset_steps requires RPROP");
        set_steps(n, steps);
    }
    if (moments) {
        require(method == 1, "reset_moments requires Adam");
        reset_optimizer(n, 1);
    }
    if (graph) {
        if (n.stage.substr(0, n.stage.find('|')) != stage.substr(0, stage.find('|'))) n.stage_done = 0;
        n.stage = stage;
    } else if (n.stage != stage) {
        n.stage = stage;
        n.stage_done = 0;
    }
    n.remaining = epochs;
    std::vector<double> values(ids.size());
    uint64_t completed = 0, last_saved = UINT64_MAX, last_eval = UINT64_MAX;
    auto stopped = [&]() { return stop && *stop; };
    while (completed < epochs && !stopped()) {
        const bool collect = (log && (completed + 1) % log == 0) || completed + 1 == epochs;
        if (graph) {
            graph_pass(n, ids, *graph, true, nullptr);
        } else {
            begin_costs(n, int(ids.size()));
            for (int l = 0; l < n.layers; ++l)
                CPDE_CUDA(cudaMemsetAsync(n.gradient(l), 0, n.count[l] * 4, stream));
            for (size_t i = 0; i < ids.size(); ++i)
                pass(n, cost(ids[i]), int(i), true, collect, nullptr, 0, INT_MAX, false, true, nullptr);
            reduce_gradient(n, nullptr);
            reduce_costs(n, ids);
        }
        const bool applied = inspect_and_update(n, method, int(ids.size()), graph.get());
        bool bad_gradient = false;
        for (int i = 0; i < n.layers; ++i) bad_gradient = bad_gradient || n.host_grads.ptr[i].nonfinite != 0;
        if (bad_gradient || (diagnostics && ((completed + 1) % diagnostics == 0 || completed + 1 == epochs)))
            gradient_report(n, completed + 1, emit);
        validate_costs(n, ids.size(), values, true);
        if (graph) graph_validate(*graph);
        if (bad_gradient)
            for (int i = 0; i < n.layers; ++i) {
                const auto& g = n.host_grads.ptr[i];
                if (g.nonfinite)
                    throw RequestError("non-finite weight gradient in layer " + std::to_string(i) +
                                       ", flattened index " + std::to_string(g.first_nonfinite) +
                                       "; no optimizer update performed for this iteration");
            }
        if (!applied) throw DeviceError("internal error: the device update gate refused an update validation accepts");
        commit_update(n, method);
        ++completed;
        ++n.updates;
        ++n.stage_done;
        n.remaining = epochs - completed;
        if (restore_every && n.updates % restore_every == 0) {
            floor_steps(n, restore_step);
            CPDE_CUDA(cudaStreamSynchronize(stream));
        }
        bool last = completed == epochs || stopped();
        if (collect) report_values(n, completed, 0, values, graph.get(), emit);
        if (eval && (completed % eval == 0 || last)) {
            evaluate_costs(n, ids, values, graph.get());
            report_values(n, completed, 1, values, graph.get(), emit);
            last_eval = completed;
            if (outputs)
                for (auto id : ids) {
                    auto& c = cost(id);
                    uint64_t output = evaluate(ni, c.input_id, c.width);
                    auto& d = dat(output);
                    std::vector<float> a(size_t(d.d) * d.h * d.total);
                    gather(d, a.data());
                    Payload r;
                    r.put<uint64_t>(id);
                    r.put_array(a);
                    data.erase(output);
                    emit(4, r);
                }
        }
        if (save && (completed % save == 0 || last)) {
            emit(3, snapshot(n));
            last_saved = completed;
        }
    }
    if (last_eval != completed) {
        evaluate_costs(n, ids, values, graph.get());
        report_values(n, completed, 1, values, graph.get(), emit);
    }
    if (save && last_saved != completed) emit(3, snapshot(n));
    Payload result;
    result.put<uint64_t>(completed);
    result.put<int32_t>(completed < epochs);
    auto meta = metadata(n);
    result.put_array(meta.bytes);
    emit(0, result);
}

// Op 14 (cuda/cpde_server.cu:535-551). Gradients go to a scratch bank, so the
// optimizer state is untouched without a snapshot/restore round trip.
Payload Engine::graph_evaluate(Payload& b) {
    uint64_t ni = b.get<uint64_t>();
    auto& n = net(ni);
    auto ids = b.array<uint64_t>();
    bool gradient = b.get<int>() != 0;
    require(!ids.empty(), "cost graph needs at least one integral");
    GraphRecord graph;
    read_graph(graph, b, int(ids.size()));
    b.end();
    prepare_costs(n, ids, ni, gradient);
    n.eval_gradient.reserve(n.params);
    float* target = gradient ? n.eval_gradient.ptr : nullptr;
    std::vector<double> values(ids.size());
    graph_pass(n, ids, graph, gradient, target);
    if (gradient) inspect_gradients(n, target);
    download(n, int(ids.size()), gradient ? n.layers : 0);
    validate_costs(n, ids.size(), values, false);
    graph_validate(graph);
    Payload out;
    out.put<double>(graph.host.ptr[0].value);
    if (gradient) {
        out.put<int>(n.layers);
        std::vector<float> g(n.params);
        CPDE_CUDA(cudaMemcpy(g.data(), target, n.params * 4, cudaMemcpyDeviceToHost));
        for (int l = 0; l < n.layers; ++l) {
            require(!n.host_grads.ptr[l].nonfinite, "nonfinite weight gradient during evaluation");
            out.put_array(g.data() + n.offset[l], size_t(n.count[l]));
        }
    }
    return out;
}

// One fixed-weight epoch without synchronisation (op 90's step).
void Engine::epoch(uint64_t ni, const std::vector<uint64_t>& ids) {
    auto& n = net(ni);
    prepare_costs(n, ids, ni, true);
    begin_costs(n, int(ids.size()));
    for (int l = 0; l < n.layers; ++l) CPDE_CUDA(cudaMemsetAsync(n.gradient(l), 0, n.count[l] * 4, stream));
    for (size_t i = 0; i < ids.size(); ++i)
        pass(n, cost(ids[i]), int(i), true, true, nullptr, 0, INT_MAX, false, true, nullptr);
    reduce_gradient(n, nullptr);
    reduce_costs(n, ids);
}

Payload Engine::benchmark(uint64_t ni, uint64_t ci, int warm, int iterations, int batches) {
    auto& n = net(ni);
    require(warm >= 0 && iterations > 0 && batches > 0, "invalid benchmark controls");
    std::vector<uint64_t> ids{ci};
    prepare_costs(n, ids, ni, true);
    for (int i = 0; i < warm; ++i) epoch(ni, ids);
    CPDE_CUDA(cudaStreamSynchronize(stream));
    cudaEvent_t start, stop;
    CPDE_CUDA(cudaEventCreate(&start));
    CPDE_CUDA(cudaEventCreate(&stop));
    std::vector<double> wall, gpu;
    for (int batch = 0; batch < batches; ++batch) {
        auto t0 = std::chrono::steady_clock::now();
        CPDE_CUDA(cudaEventRecord(start, stream));
        for (int i = 0; i < iterations; ++i) epoch(ni, ids);
        CPDE_CUDA(cudaEventRecord(stop, stream));
        CPDE_CUDA(cudaEventSynchronize(stop));
        auto t1 = std::chrono::steady_clock::now();
        float ms = 0;
        CPDE_CUDA(cudaEventElapsedTime(&ms, start, stop));
        wall.push_back(std::chrono::duration<double, std::milli>(t1 - t0).count() / iterations);
        gpu.push_back(double(ms) / iterations);
    }
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    Payload out;
    out.put_array(wall);
    out.put_array(gpu);
    inspect_gradients(n, nullptr);
    download(n, 1, n.layers);
    std::vector<double> values(1);
    validate_costs(n, 1, values, false);
    out.put<double>(values[0]);
    std::vector<float> g(n.params);
    for (int l = 0; l < n.layers; ++l) {
        CPDE_CUDA(cudaMemcpy(g.data() + n.offset[l], n.gradient(l), n.count[l] * 4, cudaMemcpyDeviceToHost));
        out.put_array(g.data() + n.offset[l], size_t(n.count[l]));
    }
    return out;
}

}  // namespace cpde
