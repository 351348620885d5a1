// Fast-tier hidden-layer forward dispatch (its own translation unit so the
// kernels it instantiates compile in parallel with the rest of the library).
#include "engine_internal.hpp"

namespace cpde {

namespace {
struct FastForward {
    Engine& e;
    NetRecord& n;
    long P;
    bool tensor;  // tcgen05 3xTF32 GEMMs where the shapes allow
    bool hidden_only;  // leave the output layer to a fused head
    template <int SID, class Act>
    void layers() {
        using namespace fast;
        constexpr int R = StaticJet<SID>::R;
        using T = Tiling<R>;
        const size_t smem = Smem<T::BN>::FLOATS * sizeof(float);
        const size_t smem64 = Smem<T::BN, 64>::FLOATS * sizeof(float);  // layers of at most 64 neurons
        static bool ready[64] = {};
        if (!ready[e.device & 63]) {
            allow_smem(k_forward<SID, Act>, smem);
            allow_smem(k_forward<SID, Act, 64>, smem64);
            ready[e.device & 63] = true;
        }
        const int L = n.layers;
        for (int l = 1; l < L; ++l) {
            const int M = n.neurons[l], K = n.neurons[l - 1];
            const float* W = n.weights(l - 1);
            const float* b = W + long(M) * K;
            if (l == 1) {
                CPDE_RUN(e, "input_forward",
                         (k_input_forward<SID, Act><<<grid_for(long(M) * P, THREADS, 148 * 32), THREADS, 0,
                                                      e.stream>>>(M, K, P, W, b, n.act[0].ptr, n.act[1].ptr)));
            } else if (tensor && M % 32 == 0 && K % tcg::KS == 0 && K <= ws::kMaxK) {
                // warp-specialised: weights resident in tensor memory, slab ring in shared memory
                using WT = ws::Tiling<R>;
                static bool ws_ready[64] = {};
                if (!ws_ready[e.device & 63]) {
                    allow_smem(ws::k_forward_ws<SID, Act>, WT::SMEM);
                    ws_ready[e.device & 63] = true;
                }
                const CUtensorMap mx = tensor_map(n.act[l - 1].ptr, K, P * R, WT::N);
                const long tiles = (P + WT::PTS - 1) / WT::PTS;
                const int halves = ws::paired_tiles(M, K) ? 2 : 1;  // two column tiles per accumulator
                const long items = (tiles + halves - 1) / halves;
                const int ny = (M + tcg::BM - 1) / tcg::BM;  // a narrower layer fills part of one slice
                dim3 grid(unsigned(std::min<long>(items, std::max(1, 148 / ny))), unsigned(ny));
                CPDE_RUN(e, "forward_ws", (ws::k_forward_ws<SID, Act><<<grid, ws::THREADS, WT::SMEM, e.stream>>>(
                                              mx, M, K, P, W, n.act[l].ptr, e.tc_error.ptr, halves)));
            } else if (tensor && M % tcg::BM == 0 && K % tcg::KS == 0) {
                // wider inputs: the weight slabs stream through the shared-memory ring with the activations
                using WT = ws::WideTiling<R>;
                static bool wide_ready[64] = {};
                if (!wide_ready[e.device & 63]) {
                    allow_smem(ws::k_forward_wide<SID, Act>, WT::SMEM);
                    wide_ready[e.device & 63] = true;
                }
                n.w_hi.reserve(n.params);
                n.w_lo.reserve(n.params);
                float* hi = n.w_hi.ptr + n.offset[l - 1];
                float* lo = n.w_lo.ptr + n.offset[l - 1];
                CPDE_RUN(e, "split_weights", (tcg::k_split_tf32<<<grid_for(long(M) * K), 256, 0, e.stream>>>(
                                                 W, hi, lo, M, K, 1)));
                const CUtensorMap mh = tensor_map(hi, K, M, tcg::BM), ml = tensor_map(lo, K, M, tcg::BM);
                const CUtensorMap mx = tensor_map(n.act[l - 1].ptr, K, P * R, WT::N);
                const long tiles = (P + WT::PTS - 1) / WT::PTS;
                dim3 grid(unsigned(std::min<long>(tiles, std::max(1, 148 / (M / tcg::BM)))), unsigned(M / tcg::BM));
                CPDE_RUN(e, "forward_wide",
                         (ws::k_forward_wide<SID, Act><<<grid, ws::THREADS, WT::SMEM, e.stream>>>(
                             mx, mh, ml, M, K, P, b, n.act[l].ptr, e.tc_error.ptr)));
            } else if (M <= 64) {
                dim3 grid(unsigned((P + T::PTS - 1) / T::PTS), 1);
                CPDE_RUN(e, "forward",
                         (k_forward<SID, Act, 64><<<grid, THREADS, smem64, e.stream>>>(M, K, P, W, b, n.act[l - 1].ptr,
                                                                                        n.act[l].ptr)));
            } else {
                dim3 grid(unsigned((P + T::PTS - 1) / T::PTS), unsigned((M + BM - 1) / BM));
                CPDE_RUN(e, "forward",
                         (k_forward<SID, Act><<<grid, THREADS, smem, e.stream>>>(M, K, P, W, b, n.act[l - 1].ptr,
                                                                                  n.act[l].ptr)));
            }
        }
        if (hidden_only) return;
        const int O = n.neurons[L], K = n.neurons[L - 1];
        const float* W = n.weights(L - 1);
        if (O == 1)
            CPDE_RUN(e, "output_forward",
                     (k_output_forward1<<<grid_for(P * R, THREADS, 148 * 8), THREADS, 0, e.stream>>>(
                         K, P, R, W, W + K, n.act[L - 1].ptr, n.act[L].ptr)));
        else
            CPDE_RUN(e, "output_forward",
                     (k_output_forward<<<grid_for(P * R * 32, THREADS, 148 * 64), THREADS, 0, e.stream>>>(
                         O, K, P, R, W, W + long(O) * K, n.act[L - 1].ptr, n.act[L].ptr)));
    }
    template <int SID>
    void run() {
        if (n.linear[1] == kTanhAct) layers<SID, Tanh>();
        else layers<SID, Sigmoid>();
    }
};

}  // namespace

void Engine::fast_forward(NetRecord& n, Context& ctx, int points, bool hidden_only) {
    with_schema(ctx.static_id, FastForward{*this, n, points, use_tensor_cores(tier, ctx, n), hidden_only});
}

}  // namespace cpde
