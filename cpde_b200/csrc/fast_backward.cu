// Fast-tier backward dispatch: output layer, hidden-layer adjoints and weight
// gradients (its own translation unit, compiled in parallel with the rest).
#include "engine_internal.hpp"

namespace cpde {

namespace {
struct FastBackward {
    Engine& e;
    NetRecord& n;
    long P;
    float* target;
    bool use_tensor;
    bool skip_output;  // a fused head already produced dZ of the last hidden layer
    template <int SID, class Act>
    void layers() {
        using namespace fast;
        constexpr int R = StaticJet<SID>::R;
        using T = Tiling<R>;
        const size_t smem = Smem<T::BN>::FLOATS * sizeof(float);
        const size_t smem64 = Smem<T::BN, 64>::FLOATS * sizeof(float);  // layers of at most 64 neurons
        static bool ready[64] = {};
        if (!ready[e.device & 63]) {
            allow_smem(k_backward<SID, Act, false>, smem);
            allow_smem(k_backward<SID, Act, true>, smem);
            allow_smem(k_backward<SID, Act, false, 64>, smem64);
            allow_smem(k_backward<SID, Act, true, 64>, smem64);
            ready[e.device & 63] = true;
        }
        const int L = n.layers;
        const long cols = P * R;
        // output layer: adjoint into the last hidden layer, output weight gradient
        if (!skip_output) {
            const int O = n.neurons[L], K = n.neurons[L - 1];
            const int bx = int(std::min<long>(148 * 8, std::max(1L, (P + 15) / 16)));
            const int slice = output_slice(K);
            dim3 grid(bx, (K + slice - 1) / slice);
            n.partial.reserve(size_t(bx) * O * (K + 1));
            static bool out_ready[64] = {};
            if (!out_ready[e.device & 63]) {
                allow_smem(k_output_backward<SID, Act>, output_backward_smem<R>());
                out_ready[e.device & 63] = true;
            }
            CPDE_RUN(e, "output_backward",
                     (k_output_backward<SID, Act><<<grid, THREADS, output_backward_smem<R>(), e.stream>>>(
                         O, K, P, n.weights(L - 1), n.dz[0].ptr, n.act[L - 1].ptr, n.dz[1].ptr, n.partial.ptr)));
            long size = long(O) * (K + 1);
            CPDE_RUN(e, "sum_partials", (k_sum_partials<<<fast::sum_grid(size), 256, 0, e.stream>>>(
                                            n.partial.ptr, bx, size, n.gradient_base(L - 1, target))));
        }
        e.layer_done(L - 1);
        float* cur = n.dz[1].ptr;
        const bool tensor = use_tensor;
        if (tensor) {
            n.wb_hi.reserve(n.params);
            n.wb_lo.reserve(n.params);
        }
        for (int l = L - 1; l >= 2; --l) {
            const int M = n.neurons[l], N = n.neurons[l - 1];
            // weight gradient of layer l (M x N plus bias), split over columns
            // enough column splits to fill two CTAs per SM, but at least 64
            // columns (FFMA) or 128 columns (tensor cores) per split
            const int tiles = ((N + BM - 1) / BM) * ((M + BM - 1) / BM);
            const bool tc_wgrad = tensor && M % 32 == 0 && N % 32 == 0;  // slices past a narrow layer's end are zeros
            const long min_cols = tc_wgrad ? 128 : 64, align = tc_wgrad ? tcg::KS : BK;
            long splits = std::max(1L, std::min<long>((2L * 148 + tiles - 1) / tiles, (cols + min_cols - 1) / min_cols));
            long per = ((cols + splits - 1) / splits + align - 1) / align * align;
            splits = (cols + per - 1) / per;
            n.partial.reserve(size_t(splits) * M * (N + 1));
            dim3 wg(unsigned(splits), (N + BM - 1) / BM, (M + BM - 1) / BM);
            if (tc_wgrad) {
                // warp-specialised: dZ through registers into tensor memory, Y_prev MN-major from TMA;
                // one CTA per SM over the (N/128) x (M/128) tiles
                static bool wg_ready[64] = {};
                if (!wg_ready[e.device & 63]) {
                    allow_smem(ws::k_wgrad_ws<128>, ws::kWgSmem);
                    allow_smem(ws::k_wgrad_ws<64>, ws::kWgSmem64);
                    wg_ready[e.device & 63] = true;
                }
                const bool narrow = M <= 64 && N <= 64;  // 64-neuron slices, a deeper ring
                const int nb = narrow ? 64 : 128;
                const int ny = (N + nb - 1) / nb, nz = (M + nb - 1) / nb;
                splits = std::max(1L, std::min<long>(std::max(1, 148 / (ny * nz)), (cols + 31) / 32));
                n.partial.reserve(size_t(splits) * M * (N + 1));
                const CUtensorMap md = mn32_map(cur, M, cols), ma = mn32_map(n.act[l - 1].ptr, N, cols);
                const dim3 wgrid = dim3(unsigned(splits), unsigned(ny), unsigned(nz));
                if (narrow)
                    CPDE_RUN(e, "weight_gradient_ws",
                             (ws::k_wgrad_ws<64><<<wgrid, ws::WgShape<64>::kThreads, ws::kWgSmem64, e.stream>>>(
                                 md, ma, M, N, cols, R, n.partial.ptr, e.tc_error.ptr)));
                else
                    CPDE_RUN(e, "weight_gradient_ws",
                             (ws::k_wgrad_ws<128><<<wgrid, ws::WgShape<128>::kThreads, ws::kWgSmem, e.stream>>>(
                                 md, ma, M, N, cols, R, n.partial.ptr, e.tc_error.ptr)));
            } else if (M <= 64 && N <= 64) {
                // 64 x 64 tiles of 64 threads, about eight CTAs per SM
                splits = std::max(1L, std::min<long>(148L * 8, (cols + 63) / 64));
                per = ((cols + splits - 1) / splits + BK - 1) / BK * BK;
                splits = (cols + per - 1) / per;
                n.partial.reserve(size_t(splits) * M * (N + 1));
                CPDE_RUN(e, "weight_gradient", (k_weight_gradient64<<<dim3(unsigned(splits), 1, 1), 64, 0, e.stream>>>(
                                                   M, N, cols, R, per, cur, n.act[l - 1].ptr, n.partial.ptr)));
            } else {
                CPDE_RUN(e, "weight_gradient", (k_weight_gradient<<<wg, THREADS, 0, e.stream>>>(
                                                   M, N, cols, R, per, cur, n.act[l - 1].ptr, n.partial.ptr)));
            }
            long size = long(M) * (N + 1);
            CPDE_RUN(e, "sum_partials", (k_sum_partials<<<fast::sum_grid(size), 256, 0, e.stream>>>(
                                            n.partial.ptr, int(splits), size, n.gradient_base(l - 1, target))));
            e.layer_done(l - 1);
            // adjoint into layer l-1
            const float* W = n.weights(l - 1);
            const long tiles_p = (P + T::PTS - 1) / T::PTS;
            const bool input = l - 1 == 1;
            float* next = cur == n.dz[0].ptr ? n.dz[1].ptr : n.dz[0].ptr;
            const int K0 = n.neurons[0];
            if (tensor && N % 32 == 0 && M % tcg::KS == 0 && M <= ws::kMaxK) {
                // warp-specialised: W^T resident in tensor memory, dZ slab ring in shared memory
                using WT = ws::Tiling<R>;
                using WTI = ws::Tiling<R, R * StaticJet<SID>::V>;  // with the input-jet rows
                static bool bw_ready[64] = {};
                if (!bw_ready[e.device & 63]) {
                    allow_smem(ws::k_backward_ws<SID, Act, false>, WT::BSMEM);
                    allow_smem(ws::k_backward_ws<SID, Act, true>, WTI::BSMEM);
                    bw_ready[e.device & 63] = true;
                }
                const CUtensorMap mz = tensor_map(cur, M, cols, WT::N);
                const long tt = (P + WT::PTS - 1) / WT::PTS;
                const int halves = ws::paired_tiles(N, M) ? 2 : 1;  // two column tiles per accumulator
                const long items = (tt + halves - 1) / halves;
                const int ny = (N + tcg::BM - 1) / tcg::BM;  // a narrower layer fills part of one slice
                const int bx = int(std::min<long>(items, std::max(1, 148 / ny)));
                dim3 grid(bx, ny);
                if (input) {
                    const int parts = 2 * halves * bx;  // one per epilogue group and tile half of each CTA
                    n.input_partial.reserve(size_t(parts) * N * (K0 + 1));
                    CPDE_RUN(e, "backward_input_ws",
                             (ws::k_backward_ws<SID, Act, true><<<grid, ws::THREADS, WTI::BSMEM, e.stream>>>(
                                 mz, M, N, P, W, n.act[1].ptr, nullptr, n.act[0].ptr, K0, n.input_partial.ptr,
                                 e.tc_error.ptr, halves)));
                    long isize = long(N) * (K0 + 1);
                    CPDE_RUN(e, "sum_partials", (k_sum_partials<<<fast::sum_grid(isize), 256, 0, e.stream>>>(
                                                    n.input_partial.ptr, parts, isize, n.gradient_base(0, target))));
                } else {
                    CPDE_RUN(e, "backward_ws",
                             (ws::k_backward_ws<SID, Act, false><<<grid, ws::THREADS, WT::BSMEM, e.stream>>>(
                                 mz, M, N, P, W, n.act[l - 1].ptr, next, nullptr, 0, nullptr, e.tc_error.ptr,
                                 halves)));
                    cur = next;
                }
                continue;
            }
            if (tensor && N % tcg::BM == 0 && M % tcg::KS == 0) {
                // wider layers: the W^T slabs stream through the shared-memory ring with the dZ slabs
                using WT = ws::WideTiling<R>;
                static bool wide_ready[64] = {};
                if (!wide_ready[e.device & 63]) {
                    allow_smem(ws::k_backward_wide<SID, Act, false>, WT::SMEM);
                    allow_smem(ws::k_backward_wide<SID, Act, true>, WT::SMEM);
                    wide_ready[e.device & 63] = true;
                }
                float* hi = n.wb_hi.ptr + n.offset[l - 1];
                float* lo = n.wb_lo.ptr + n.offset[l - 1];
                CPDE_RUN(e, "split_weights", (tcg::k_split_tf32<<<grid_for(long(M) * N), 256, 0, e.stream>>>(
                                                 W, hi, lo, N, M, 0)));
                const CUtensorMap mh = tensor_map(hi, M, N, tcg::BM), ml = tensor_map(lo, M, N, tcg::BM);
                const CUtensorMap mz = tensor_map(cur, M, cols, WT::N);
                const long tt = (P + WT::PTS - 1) / WT::PTS;
                const int bx = int(std::min<long>(tt, std::max(1, 148 / (N / tcg::BM))));
                dim3 grid(bx, N / tcg::BM);
                if (input) {
                    n.input_partial.reserve(size_t(2 * bx) * N * (K0 + 1));
                    CPDE_RUN(e, "backward_input_wide",
                             (ws::k_backward_wide<SID, Act, true><<<grid, ws::THREADS, WT::SMEM, e.stream>>>(
                                 mz, mh, ml, M, N, P, n.act[1].ptr, nullptr, n.act[0].ptr, K0, n.input_partial.ptr,
                                 e.tc_error.ptr)));
                    long isize = long(N) * (K0 + 1);
                    CPDE_RUN(e, "sum_partials", (k_sum_partials<<<fast::sum_grid(isize), 256, 0, e.stream>>>(
                                                    n.input_partial.ptr, 2 * bx, isize, n.gradient_base(0, target))));
                } else {
                    CPDE_RUN(e, "backward_wide",
                             (ws::k_backward_wide<SID, Act, false><<<grid, ws::THREADS, WT::SMEM, e.stream>>>(
                                 mz, mh, ml, M, N, P, n.act[l - 1].ptr, next, nullptr, 0, nullptr, e.tc_error.ptr)));
                    cur = next;
                }
                continue;
            }
            const bool narrow = N <= 64;  // 64-neuron tiles
            if (input) {
                const int bx = int(std::min<long>(tiles_p, 148 * 2));
                dim3 grid(bx, narrow ? 1 : (N + BM - 1) / BM);
                n.input_partial.reserve(size_t(bx) * N * (K0 + 1));
                if (narrow)
                    CPDE_RUN(e, "backward_input",
                             (k_backward<SID, Act, true, 64><<<grid, THREADS, smem64, e.stream>>>(
                                 N, M, P, W, cur, n.act[1].ptr, nullptr, n.act[0].ptr, K0, n.input_partial.ptr)));
                else
                    CPDE_RUN(e, "backward_input",
                             (k_backward<SID, Act, true><<<grid, THREADS, smem, e.stream>>>(
                                 N, M, P, W, cur, n.act[1].ptr, nullptr, n.act[0].ptr, K0, n.input_partial.ptr)));
                long isize = long(N) * (K0 + 1);
                CPDE_RUN(e, "sum_partials", (k_sum_partials<<<fast::sum_grid(isize), 256, 0, e.stream>>>(
                                                n.input_partial.ptr, bx, isize, n.gradient_base(0, target))));
            } else {
                const int bx = int(std::min<long>(tiles_p, 148 * 8));
                dim3 grid(bx, narrow ? 1 : (N + BM - 1) / BM);
                if (narrow)
                    CPDE_RUN(e, "backward",
                             (k_backward<SID, Act, false, 64><<<grid, THREADS, smem64, e.stream>>>(
                                 N, M, P, W, cur, n.act[l - 1].ptr, next, nullptr, 0, nullptr)));
                else
                    CPDE_RUN(e, "backward",
                             (k_backward<SID, Act, false><<<grid, THREADS, smem, e.stream>>>(
                                 N, M, P, W, cur, n.act[l - 1].ptr, next, nullptr, 0, nullptr)));
                cur = next;
            }
        }
    }
    template <int SID>
    void run() {
        if (n.linear[1] == kTanhAct) layers<SID, Tanh>();
        else layers<SID, Sigmoid>();
    }
};
}  // namespace

void Engine::fast_backward(NetRecord& n, Context& ctx, int points, float* target, bool skip_output) {
    with_schema(ctx.static_id, FastBackward{*this, n, points, target, use_tensor_cores(tier, ctx, n), skip_output});
}

}  // namespace cpde
