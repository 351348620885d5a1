// Engine objects: data, networks, costs, cost graphs, and the Engine that owns
// them on one device. The Engine mirrors the reference server's object model
// and command semantics (cuda/cpde_server.cu:26-555) with its own storage and
// kernels.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "collectives.hpp"
#include "common.hpp"
#include "expression.hpp"
#include "kernels_fast.cuh"
#include "kernels_small.cuh"
#include "kernels_tc.cuh"
#include "kernels_ws.cuh"
#include "kernels_generic.cuh"
#include "scalar.hpp"
#include "schema.hpp"
#include "wire.hpp"

namespace cpde {

enum Activation { kSigmoid = 0, kLinear = 1, kTanhAct = 2 };

struct DataRecord {
    int d = 0, h = 0, w = 0, v = 0;  // derivative rows, channels, samples (this rank's shard), variables
    int total = 0, lo = 0;            // samples over all ranks; first sample of this rank's shard
    std::vector<int> table;           // d x (v+1) row-major: order, counts...
    DeviceBuffer<float> values;       // (row, sample, channel)
    uint64_t version = 0;
    int order(int row) const { return table[size_t(row) * (v + 1)]; }
    std::vector<int> counts(int row) const {
        return std::vector<int>(table.begin() + size_t(row) * (v + 1) + 1, table.begin() + size_t(row + 1) * (v + 1));
    }
};

// A derivative context: the data rows a pass propagates, their jet tables.
struct Context {
    std::vector<int> rows;  // data-table rows in propagation order
    JetPlan plan;
    bool planned = false;
    int static_id = -1;  // generated register-resident jet code for exactly these rows, if any
    DeviceBuffer<int> rows_dev;
    DeviceBuffer<int> tables;
    int R() const { return int(rows.size()); }
};

struct CostRecord {
    uint64_t network_id = 0, input_id = 0, target_id = 0;
    int kind = 0, width = 0, equations = 0, weight_samples = 0, samples = 0;
    std::vector<int> rows;
    std::shared_ptr<Context> context;
    DeviceBuffer<int> target_rows;
    DeviceBuffer<float> weights, coefficients, rhs;
    DeviceBuffer<PolyTerm> terms;
    int term_count = 0;
    std::shared_ptr<ExpressionProgram> program;
    std::shared_ptr<RuntimeKernel> head;  // fused expression head for the shape in head_key
    std::string head_key;
    DeviceBuffer<double> fields, quadrature_weights;
    bool has_components = true, has_gradient = true;
};

struct GraphRecord {
    std::vector<ScalarNode> nodes;
    int root = 0;
    struct Known {
        bool known;
        double value;
    };
    std::vector<Known> schedule;
    DeviceBuffer<ScalarNode> nodes_dev;
    DeviceBuffer<double> values, adjoints, multipliers, fixed_multipliers;
    DeviceBuffer<int> active;
    struct Summary {
        double value;
        int bad_node;
        int pad;
    };
    DeviceBuffer<Summary> summary;
    PinnedBuffer<Summary> host;
};

struct NetRecord {
    std::vector<int> neurons, linear;
    int layers = 0;  // weight layers = neurons.size() - 1
    std::vector<long> offset;
    std::vector<int> count;
    long params = 0;
    DeviceBuffer<float> bank[4];  // W, gradient 1, gradient 2, steps or first moment
    std::vector<int> active;      // per layer: 1 or 2
    int optimizer = -1;
    uint64_t updates = 0, adam_step = 0, stage_done = 0, remaining = 0;
    float learning_rate = .001f, initial_step = .002f;
    std::string stage;

    // activation arena (interleaved layout), sized for `capacity` columns
    long capacity = 0;
    std::vector<DeviceBuffer<float>> act;  // act[l]: A_l (l < L) or Z_L
    std::vector<DeviceBuffer<float>> pre;  // pre[l]: Z_l of nonlinear layers
    DeviceBuffer<float> dz[2], dy, jet_scratch, partial, input_partial;
    DeviceBuffer<float> eval_gradient;  // gradient target of op 14 (keeps history intact)
    DeviceBuffer<float> w_hi, w_lo;     // TF32 split of the weights, K-major for the forward (W)
    DeviceBuffer<float> wb_hi, wb_lo;   // TF32 split of the weights as stored (K-major for W^T)

    // which chunk's forward is resident (cuda/cpde_server.cu:163)
    uint64_t loaded_id = 0, loaded_version = 0;
    int loaded_width = 0, loaded_offset = 0, loaded_valid = 0;
    std::vector<int> loaded_rows;

    // reductions
    int cost_capacity = 0;
    DeviceBuffer<CostStats> cost_totals, cost_partials;
    DeviceBuffer<unsigned> cost_ticket;
    DeviceBuffer<GradStats> grad_totals, grad_partials;
    DeviceBuffer<unsigned> grad_tickets;
    DeviceBuffer<const float*> grad_ptrs;
    DeviceBuffer<int> grad_counts;
    PinnedBuffer<CostStats> host_costs;
    PinnedBuffer<GradStats> host_grads;
    DeviceBuffer<OptLayer> opt_layers;
    DeviceBuffer<int> update_applied;  // decision of the fused update's gate
    PinnedBuffer<int> host_applied;

    float* weights(int l) { return bank[0].ptr + offset[l]; }
    float* gradient(int l) { return bank[active[l]].ptr + offset[l]; }
    float* gradient_base(int l, float* target) { return target ? target + offset[l] : gradient(l); }
};

using EventSink = std::function<void(uint32_t, const Payload&)>;

struct KernelTimer;

class Engine {
   public:
    explicit Engine(int device);
    ~Engine();
    int device;
    cudaStream_t stream = nullptr;
    // 0 automatic, 1 generic kernels only, 2 tensor-core GEMMs where eligible,
    // 3 the point-tile epoch wherever it is eligible
    int tier = 0;
    long point_epoch_columns = 16384;  // automatic tier: point-tile epochs up to this many columns per chunk
    std::string last_error;
    DeviceBuffer<int> tc_error;  // nonzero after a tensor-core kernel gave up waiting

    // Point sharding: rank `rank` of `world` engines, one per device, each
    // holding a contiguous shard of every Data object; gradients and cost
    // totals are summed over the group with NCCL on this engine's stream.
    int rank = 0, world = 1;
    ncclComm_t comm = nullptr;
    // The gradient all-reduce runs per layer on its own stream: each layer's
    // reduction waits only for the event its backward recorded when that
    // layer's gradient was complete, so the reductions of the upper layers
    // overlap the backward of the lower ones.
    cudaStream_t comm_stream = nullptr;
    cudaEvent_t comm_done = nullptr;
    std::vector<cudaEvent_t> layer_events;
    std::vector<char> layer_marked;
    void layer_done(int layer);
    void join(int rank, int world, const void* unique_id);
    Shard shard(long total) const { return shard_range(total, rank, world); }
    void reduce_costs(NetRecord& n, const std::vector<uint64_t>& ids);
    void reduce_gradient(NetRecord& n, float* target);
    void gather(DataRecord& d, float* host);  // the whole (row, sample, channel) array on every rank
    void upload_shard(DataRecord& d, const float* values);
    DeviceBuffer<double> shard_values;
    DeviceBuffer<long long> shard_keys;
    DeviceBuffer<int> shard_offsets;
    std::vector<int> shard_offsets_host;  // what shard_offsets holds
    DeviceBuffer<float> gather_send, gather_recv;
    void check_device_errors();

    uint64_t next_id = 1;
    std::unordered_map<uint64_t, std::unique_ptr<DataRecord>> data;
    std::unordered_map<uint64_t, std::unique_ptr<NetRecord>> nets;
    std::unordered_map<uint64_t, std::unique_ptr<CostRecord>> costs;
    std::unordered_map<std::string, std::shared_ptr<ExpressionProgram>> programs;
    std::unordered_map<std::string, std::shared_ptr<RuntimeKernel>> heads;  // by source
    std::map<std::string, std::shared_ptr<Context>> contexts;

    // ops
    uint64_t create_data(int d, int h, int w, int v, const int* table, size_t table_count, const float* values,
                         size_t count);
    void replace_data(uint64_t id, const float* values, size_t count);
    uint64_t create_net(const std::vector<int>& neurons, const std::vector<int>& linear,
                        const std::vector<std::vector<float>>& initial);
    uint64_t evaluate(uint64_t net, uint64_t data, int chunk);
    uint64_t cost_matching(uint64_t net, uint64_t in, uint64_t tgt, int chunk, std::vector<int> rows,
                           std::vector<int> target_rows, int weight_samples, std::vector<float> weights);
    uint64_t cost_polynomial(uint64_t net, uint64_t in, int chunk, std::vector<int> rows, int equations,
                             std::vector<int> raw_terms, std::vector<float> coefficients, std::vector<float> rhs,
                             std::vector<float> weights);
    uint64_t cost_integral(uint64_t net, uint64_t in, int chunk, int samples, std::vector<int> raw,
                           std::vector<double> constants, int fields, std::vector<double> numeric,
                           std::vector<double> weights);
    void release(int kind, uint64_t id);
    Payload snapshot(NetRecord& n);
    void restore(NetRecord& n, Payload& b);
    void train(Payload& b, bool graph_mode, const EventSink& emit, const volatile int32_t* stop);
    Payload graph_evaluate(Payload& b);
    Payload benchmark(uint64_t net, uint64_t cost, int warm, int iterations, int batches);
    void epoch(uint64_t net, const std::vector<uint64_t>& ids);

    DataRecord& dat(uint64_t id);
    NetRecord& net(uint64_t id);
    CostRecord& cost(uint64_t id);

    // timing of kernel classes (off by default)
    std::unique_ptr<KernelTimer> timer;
    void timing(bool enable);
    std::string timing_report();

   private:
    std::shared_ptr<Context> make_context(DataRecord& d, const std::vector<int>& rows, bool need_plan);
    std::vector<int> all_rows(DataRecord& d);
    void ensure_arena(NetRecord& n, long columns, bool backward);
    void ensure_reductions(NetRecord& n, int costs);
    void begin_costs(NetRecord& n, int count);
    void activate(NetRecord& n, uint64_t data_id, Context& ctx, int width, int offset, int valid);
    void forward(NetRecord& n, Context& ctx, int points);
    void backward(NetRecord& n, Context& ctx, int points, float* target);
    bool fast_ok(NetRecord& n, Context& ctx) const;
    bool fused_head_ok(NetRecord& n, CostRecord& c, Context& ctx) const;
    bool point_epoch_ok(NetRecord& n, Context& ctx, long points, float* target) const;
    void fused_head(NetRecord& n, CostRecord& c, Context& ctx, long points, int offset, bool collect,
                    const double* multiplier, CostReduce red, float* target);
    bool expression_head_ok(NetRecord& n, CostRecord& c, Context& ctx) const;
    void expression_head(NetRecord& n, CostRecord& c, Context& ctx, long points, int offset, bool collect,
                         const double* multiplier, CostReduce red, float* target);
    void point_epoch(NetRecord& n, CostRecord& c, Context& ctx, long points, int offset, bool collect,
                     const double* multiplier, int cost_index, float* target);
    void fast_forward(NetRecord& n, Context& ctx, int points, bool hidden_only);
    void fast_backward(NetRecord& n, Context& ctx, int points, float* target, bool skip_output);
    void run_cost(NetRecord& n, CostRecord& c, int cost_index, int points, int offset, bool collect, bool gradient,
                  const double* multiplier);
    void pass(NetRecord& n, CostRecord& c, int cost_index, bool backward, bool collect, const double* multiplier,
              int begin, int end, bool reuse_forward, bool backward_storage, float* target);
    void prepare_costs(NetRecord& n, const std::vector<uint64_t>& ids, uint64_t ni, bool backward);
    void read_graph(GraphRecord& g, Payload& b, int leaves);
    void run_graph(GraphRecord& g, NetRecord& n, int leaves, bool gradient);
    void graph_pass(NetRecord& n, const std::vector<uint64_t>& ids, GraphRecord& g, bool backward, float* target);
    void inspect_gradients(NetRecord& n, float* target);
    void download(NetRecord& n, int costs, int layers);
    void validate_costs(NetRecord& n, size_t count, std::vector<double>& values, bool before_update);
    void evaluate_costs(NetRecord& n, const std::vector<uint64_t>& ids, std::vector<double>& values, GraphRecord* g);
    void reset_optimizer(NetRecord& n, int method);
    void set_steps(NetRecord& n, float value);
    void floor_steps(NetRecord& n, float value);
    AdamStep adam_step(NetRecord& n, int step);
    bool inspect_and_update(NetRecord& n, int method, int costs, GraphRecord* g);
    void commit_update(NetRecord& n, int method);
    Payload metadata(NetRecord& n);
    void gradient_report(NetRecord& n, uint64_t epoch, const EventSink& emit);
    void report_values(NetRecord& n, uint64_t completed, int after, const std::vector<double>& values,
                       GraphRecord* g, const EventSink& emit);
};

}  // namespace cpde
