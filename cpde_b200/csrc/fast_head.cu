// Fused matching head and point-tile epoch dispatch (its own translation
// unit, compiled in parallel with the rest of the library).
#include "engine_internal.hpp"
#include "generated/jets_static_source.cuh"

namespace cpde {

namespace {
struct FastHead {
    Engine& e;
    NetRecord& n;
    CostRecord& c;
    long P;
    int offset;
    bool collect;
    const double* multiplier;
    CostReduce red;
    float* target;
    template <int SID, class Act, int O, int KPT>
    void go() {
        const int L = n.layers, K = n.neurons[L - 1];
        const int grid = int(std::min<long>(148L * 8, std::max(1L, (P + 3) / 4)));
        n.partial.reserve(size_t(grid) * O * (K + 1));
        auto& t = e.dat(c.target_id);
        // two staging slots of a point's values (R rows x K neurons)
        const size_t smem = size_t(2) * StaticJet<SID>::R * KPT * fast::BM * sizeof(float);
        static bool ready[64] = {};
        if (!ready[e.device & 63]) {
            allow_smem(fast::k_head_matching<SID, Act, O, KPT>, smem);
            ready[e.device & 63] = true;
        }
        CPDE_RUN(e, "head_matching",
                 (fast::k_head_matching<SID, Act, O, KPT><<<grid, fast::BM, smem, e.stream>>>(
                     K, P, offset, n.weights(L - 1), n.act[L - 1].ptr, n.dz[1].ptr, t.values.ptr, t.w,
                     c.target_rows.ptr, c.weights.ptr, c.weight_samples, multiplier, collect, red, n.partial.ptr)));
        const long size = long(O) * (K + 1);
        CPDE_RUN(e, "sum_partials", (fast::k_sum_partials<<<fast::sum_grid(size), 256, 0, e.stream>>>(
                                        n.partial.ptr, grid, size, n.gradient_base(L - 1, target))));
        e.layer_done(L - 1);
    }
    template <int SID, class Act, int O>
    void by_width() {
        if (n.neurons[n.layers - 1] == 128) go<SID, Act, O, 1>();
        else go<SID, Act, 1, 2>();  // fused_head_ok admits 256-wide last layers for one output only
    }
    template <int SID, class Act>
    void by_outputs() {
        if (n.neurons.back() == 1) by_width<SID, Act, 1>();
        else by_width<SID, Act, 2>();
    }
    template <int SID>
    void run() {
        if (n.linear[1] == kTanhAct) by_outputs<SID, Tanh>();
        else by_outputs<SID, Sigmoid>();
    }
};

struct PointEpoch {
    Engine& e;
    NetRecord& n;
    CostRecord& c;
    long P;
    int offset;
    bool collect;
    const double* multiplier;
    CostReduce red;
    float* target;
    template <int SID, class Act, int O, int K>
    void go() {
        constexpr int R = StaticJet<SID>::R;
        using T = small::Tiling<R>;
        const size_t smem = small::SmemSize<R, O>::FLOATS * sizeof(float);
        static bool ready[64] = {};
        if (!ready[e.device & 63]) {
            allow_smem(small::k_point_epoch<SID, Act, O, K>, smem);
            ready[e.device & 63] = true;
        }
        // at most one CTA per SM, each over a contiguous run of point tiles
        const long tiles = (P + T::PTS - 1) / T::PTS;
        const int per = int((tiles + 147) / 148);
        const int grid = int((tiles + per - 1) / per);
        small::EpochNet net{};
        net.layers = n.layers;
        for (int l = 0; l <= n.layers; ++l) net.width[l] = n.neurons[l];
        for (int l = 0; l < n.layers; ++l) {
            net.W[l] = n.weights(l);
            net.act[l] = n.act[l].ptr;
            net.offset[l] = n.offset[l];
        }
        net.dz[0] = n.dz[0].ptr;
        net.dz[1] = n.dz[1].ptr;
        net.params = n.params;
        n.partial.reserve(size_t(grid) * n.params);
        net.partials = n.partial.ptr;
        auto& t = e.dat(c.target_id);
        small::EpochHead head{t.values.ptr, t.w,    c.target_rows.ptr, c.weights.ptr, c.weight_samples,
                              multiplier,   collect, offset,           red};
        CPDE_RUN(e, "point_epoch", (small::k_point_epoch<SID, Act, O, K><<<grid, small::THREADS, smem, e.stream>>>(
                                       net, P, per, head)));
        CPDE_RUN(e, "sum_partials", (fast::k_sum_partials<<<fast::sum_grid(n.params), 256, 0, e.stream>>>(
                                        n.partial.ptr, grid, n.params, n.gradient_base(0, target))));
        for (int l = 0; l < n.layers; ++l) e.layer_done(l);
    }
    template <int SID, class Act, int O>
    void by_width() {
        if (n.neurons[n.layers - 1] == 128) go<SID, Act, O, 128>();
        else go<SID, Act, 1, 256>();  // fused_head_ok admits 256-wide last layers for one output only
    }
    template <int SID, class Act>
    void by_outputs() {
        if (n.neurons.back() == 1) by_width<SID, Act, 1>();
        else by_width<SID, Act, 2>();
    }
    template <int SID>
    void run() {
        if (n.linear[1] == kTanhAct) by_outputs<SID, Tanh>();
        else by_outputs<SID, Sigmoid>();
    }
};
}  // namespace

void Engine::fused_head(NetRecord& n, CostRecord& c, Context& ctx, long points, int offset, bool collect,
                        const double* multiplier, CostReduce red, float* target) {
    with_schema(ctx.static_id, FastHead{*this, n, c, points, offset, collect, multiplier, red, target});
}

// The fused expression head (an NVRTC kernel built from the cost's program
// and the schema's jet code, expression.hpp) takes integral costs on fast-tier
// networks whose last hidden layer has 32, 64 or 128 neurons and at most 4
// outputs; other shapes run the output layer, the cost and the output
// backward as three kernels.
bool Engine::expression_head_ok(NetRecord& n, CostRecord& c, Context& ctx) const {
    if (c.kind != 2 || !c.program || !fast_ok(n, ctx)) return false;
    const int K = n.neurons[n.layers - 1], O = n.neurons.back();
    return (K == 32 || K == 64 || K == 128) && O <= 4 && ctx.R() * O <= 128;
}

void Engine::expression_head(NetRecord& n, CostRecord& c, Context& ctx, long points, int offset, bool collect,
                             const double* multiplier, CostReduce red, float* target) {
    const int L = n.layers, K = n.neurons[L - 1], O = n.neurons.back(), R = ctx.R();
    const bool tanh_act = n.linear[1] == kTanhAct;
    const std::string key = std::to_string(ctx.static_id) + "|" + std::to_string(tanh_act) + "|" +
                            std::to_string(O) + "|" + std::to_string(K);
    if (!c.head || c.head_key != key) {
        std::string source = expression_head_source(c.program->nodes, kStaticJetSource[ctx.static_id],
                                                    ctx.static_id, tanh_act, R, O, K);
        auto& h = heads[source];
        if (!h) h = std::make_shared<RuntimeKernel>(std::move(source), "cpde_head");
        c.head = h;
        c.head_key = key;
    }
    c.head->compile();
    const int per_round = (128 / K) * head_points_per_lane(R);  // points a CTA takes per round
    const int grid = int(std::min<long>(148L * 8, std::max(1L, (points + per_round - 1) / per_round)));
    n.partial.reserve(size_t(grid) * O * (K + 1));
    int k = K, p = int(points), off = offset, samples = c.samples, col = collect;
    const float* W = n.weights(L - 1);
    const float* Y = n.act[L - 1].ptr;
    float* dZ = n.dz[1].ptr;
    const double* fields = c.fields.ptr;
    const double* weights = c.quadrature_weights.ptr;
    float* partials = n.partial.ptr;
    void* args[] = {&k,        &p,      &off,          &samples,           (void*)&W,         (void*)&Y,
                    &dZ,       (void*)&fields, (void*)&weights, (void*)&multiplier, &col, &partials,
                    (void*)&red.partials, (void*)&red.ticket, (void*)&red.total};
    CPDE_RUN(*this, "head_expression",
             driver_check(driver_api().launch(c.head->kernel, unsigned(grid), 1, 1, 128, 1, 1, 0, stream, args, nullptr),
                          "cuLaunchKernel"));
    const long size = long(O) * (K + 1);
    CPDE_RUN(*this, "sum_partials", (fast::k_sum_partials<<<fast::sum_grid(size), 256, 0, stream>>>(
                                        n.partial.ptr, grid, size, n.gradient_base(L - 1, target))));
    layer_done(L - 1);
}

void Engine::point_epoch(NetRecord& n, CostRecord& c, Context& ctx, long points, int offset, bool collect,
                         const double* multiplier, int cost_index, float* target) {
    CostReduce red{n.cost_partials.ptr, n.cost_ticket.ptr, n.cost_totals.ptr + cost_index};
    with_schema(ctx.static_id, PointEpoch{*this, n, c, points, offset, collect, multiplier, red, target});
}

}  // namespace cpde
