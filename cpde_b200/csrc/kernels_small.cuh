// Point-tile epoch: one launch runs a whole fixed-weight epoch of a matching
// cost for point sets too small to fill the GPU layer by layer.
//
// Every sample is independent until the point-axis sums (weight gradients,
// loss), so each CTA takes a contiguous range of points and runs, on that
// range alone: the input layer, the hidden layers with their jet combine, the
// output layer fused with the matching residual, the jet adjoints back to the
// first hidden layer, and every weight gradient restricted to its own columns.
// Each CTA stores a full gradient-shaped partial; one k_sum_partials launch
// folds them in a fixed order. A per-layer epoch (cuda/cpde_engine.cuh:889-991)
// issues two to four launches per layer and leaves most SMs idle at these sizes.
//
// Activations written earlier in the launch are read back by the same CTA
// after __syncthreads with L2 (ld.global.cg) loads; only weights, inputs and
// targets, which no thread writes, go through the read-only path.
#pragma once
#include "kernels_fast.cuh"

namespace cpde {
namespace small {

using fast::BK;
using fast::BM;
using fast::THREADS;

constexpr int kMaxLayers = 16;

// Columns per GEMM tile: whole points, about 32 columns, padded to 16.
template <int R>
struct Tiling {
    static constexpr int PTS = (32 / R) > 0 ? (32 / R) : 1;
    static constexpr int COLS = PTS * R;
    static constexpr int BN = ((COLS + 15) / 16) * 16;
};

// Shared memory: the larger of the GEMM staging area, the weight-gradient
// slabs and the output-layer sums.
template <int R, int O>
struct SmemSize {
    static constexpr int GEMM = fast::Smem<Tiling<R>::BN>::FLOATS;
    static constexpr int WGRAD = 2 * 2 * BK * (BM + 4);
    static constexpr int HEAD = 8 * O * R + 2 * 256 * O + 2 * O;
    static constexpr int A = GEMM > WGRAD ? GEMM : WGRAD;
    static constexpr int FLOATS = A > HEAD ? A : HEAD;
};

struct EpochNet {
    int layers;                      // L: weight layers; hidden layers 1..L-1
    int width[kMaxLayers + 1];       // neurons per layer, inputs first
    const float* W[kMaxLayers];      // W[l]: layer l+1, column-major n_{l+1} x n_l, then bias
    float* act[kMaxLayers];          // act[l], l < L: chunk activations (act[0] = staged inputs)
    long offset[kMaxLayers];         // gradient offset of W[l]
    float* dz[2];                    // adjoint ping-pong buffers
    long params;                     // gradient floats per partial
    float* partials;                 // [gridDim.x][params]
};

struct EpochHead {
    const float* target;
    int target_samples;
    const int* target_rows;
    const float* weights;
    int weight_samples;
    const double* multiplier;
    int collect;
    int offset;  // first sample of the chunk
    CostReduce red;
};

// Column loader over activations produced in this launch.
struct FreshColumns {
    const float* base;
    int K;
    long columns;
    __device__ float4 operator()(int c, int k4) const {
        if (c >= columns || k4 * 4 >= K) return make_float4(0.f, 0.f, 0.f, 0.f);
        return __ldcg(reinterpret_cast<const float4*>(base + (size_t)c * K) + k4);
    }
};

// Y = f(W X + b) for points [q0, q1) of a hidden layer (M x K weights).
template <int SID, class Act>
__device__ __forceinline__ void hidden_forward(int M, int K, const float* W, const float* X, float* Y, long q0,
                                               long q1, float* smem) {
    constexpr int R = StaticJet<SID>::R;
    using T = Tiling<R>;
    using S = fast::Smem<T::BN>;
    const float* bias = W + (size_t)M * K;
    for (long p0 = q0; p0 < q1; p0 += T::PTS) {
        const int points = int(min((long)T::PTS, q1 - p0));
        for (int m_base = 0; m_base < M; m_base += BM) {
            float acc[8][T::BN / 16] = {};
            auto aload = [&](int m, int k) -> float {
                const int mm = m_base + m;
                return (mm < M && k < K) ? __ldg(W + mm + (size_t)k * M) : 0.f;
            };
            fast::gemm_main<T::BN>(acc, smem, K, aload, FreshColumns{X + (size_t)p0 * R * K, K, (long)points * R});
            fast::stage_tile<T::BN>(acc, smem);
            for (int e = threadIdx.x; e < BM * points; e += THREADS) {
                const int m = e % BM, p = e / BM, mm = m_base + m;
                if (mm >= M) continue;
                float z[R], y[R];
#pragma unroll
                for (int r = 0; r < R; ++r) z[r] = smem[(p * R + r) * S::LDZ + m];
                z[0] += __ldg(bias + mm);
                StaticJet<SID>::template forward<Act>(z, y);
                float* out = Y + ((size_t)(p0 + p) * R) * M + mm;
#pragma unroll
                for (int r = 0; r < R; ++r) out[(size_t)r * M] = y[r];
            }
            __syncthreads();
        }
    }
}

// Output layer, matching residual and output adjoint for points [q0, q1):
// z = W_out y + b, g = 2 w (z - t), dY = W_out^T g, jet adjoint with Y into
// dZ. The output weight gradient (O x K, bias last) goes to `part`.
template <int SID, class Act, int O, int K>
__device__ __forceinline__ void matching_head(const float* Wout, const float* Y, float* dZ, long q0, long q1,
                                              const EpochHead& h, float* part, float* smem, CostStats& local) {
    constexpr int R = StaticJet<SID>::R;
    constexpr int GROUPS = THREADS / K, WARPS = K / 32;
    const int t = threadIdx.x, n = t % K, g = t / K, wig = n >> 5, lane = t & 31;
    float* sums = smem;                      // [GROUPS][WARPS][O * R]
    float* fold = smem + 8 * O * R;          // [K][O] group-1 weight sums, then [O] bias sums
    float w[O], gw[O], bias[O], gb[O];
#pragma unroll
    for (int o = 0; o < O; ++o) {
        w[o] = __ldg(Wout + o + (size_t)n * O);
        bias[o] = __ldg(Wout + (size_t)K * O + o);
        gw[o] = 0.f;
        gb[o] = 0.f;
    }
    const double scale = h.multiplier ? *h.multiplier : 1.0;
    for (long base = q0; base < q1; base += GROUPS) {
        const long p = base + g;
        const bool live = p < q1;
        float y[R];
#pragma unroll
        for (int r = 0; r < R; ++r) y[r] = live ? __ldcg(Y + ((size_t)p * R + r) * K + n) : 0.f;
#pragma unroll
        for (int o = 0; o < O; ++o)
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float v = w[o] * y[r];
#pragma unroll
                for (int s = 16; s; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
                if (lane == 0) sums[(g * WARPS + wig) * O * R + o * R + r] = v;
            }
        __syncthreads();
        float gr[O][R];
        float value = 0.f;
        if (live) {
            const int wp = h.weight_samples == 1 ? 0 : h.offset + int(p);
#pragma unroll
            for (int d = 0; d < R; ++d)
#pragma unroll
                for (int o = 0; o < O; ++o) {
                    float z = d == 0 ? bias[o] : 0.f;
#pragma unroll
                    for (int k = 0; k < WARPS; ++k) z += sums[(g * WARPS + k) * O * R + o * R + d];
                    const float wt = __ldg(h.weights + ((size_t)d * h.weight_samples + wp) * O + o);
                    float grad = 0.f;
                    if (wt != 0.f) {
                        const float res =
                            z - __ldg(h.target +
                                      ((size_t)__ldg(h.target_rows + d) * h.target_samples + h.offset + p) * O + o);
                        value += wt * res * res;
                        grad = 2.0f * wt * res;
                    }
                    gr[o][d] = grad;
                }
        }
        __syncthreads();  // sums is rewritten by the next points
        if (!live) continue;
        if (n == 0) {
            if (!isfinite(value)) mark_bad(local, h.offset + int(p), -1);
            if (h.collect) local.value += double(value);
#pragma unroll
            for (int d = 0; d < R; ++d)
#pragma unroll
                for (int o = 0; o < O; ++o)
                    if (!isfinite(gr[o][d])) mark_bad(local, h.offset + int(p), d * O + o);
        }
        if (h.multiplier)
#pragma unroll
            for (int o = 0; o < O; ++o)
#pragma unroll
                for (int d = 0; d < R; ++d) gr[o][d] = scale == 0 ? 0.f : float(gr[o][d] * scale);
#pragma unroll
        for (int o = 0; o < O; ++o) gb[o] += gr[o][0];
        float dy[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            float acc = 0.f;
#pragma unroll
            for (int o = 0; o < O; ++o) {
                acc = fmaf(w[o], gr[o][r], acc);
                gw[o] = fmaf(gr[o][r], y[r], gw[o]);
            }
            dy[r] = acc;
        }
        StaticJet<SID>::template adjoint<Act>(y, dy);
        float* out = dZ + (size_t)p * R * K + n;
#pragma unroll
        for (int r = 0; r < R; ++r) out[(size_t)r * K] = dy[r];
    }
    // fold the point groups (group 0 keeps the sums) and store the partial
    if (GROUPS == 2) {
        if (g == 1) {
#pragma unroll
            for (int o = 0; o < O; ++o) fold[n * O + o] = gw[o];
            if (n == 0)
#pragma unroll
                for (int o = 0; o < O; ++o) fold[K * O + o] = gb[o];
        }
        __syncthreads();
        if (g == 0) {
#pragma unroll
            for (int o = 0; o < O; ++o) gw[o] += fold[n * O + o];
            if (n == 0)
#pragma unroll
                for (int o = 0; o < O; ++o) gb[o] += fold[K * O + o];
        }
        __syncthreads();
    }
    if (g == 0) {
#pragma unroll
        for (int o = 0; o < O; ++o) part[o + (size_t)n * O] = gw[o];
        if (n == 0)
#pragma unroll
            for (int o = 0; o < O; ++o) part[o + (size_t)K * O] = gb[o];
    }
}

// Weight gradient of a hidden layer (M x N, bias column last) over columns
// [c_begin, c_end): out[m + n M] = sum_c dZ[c][m] A[c][n].
__device__ __forceinline__ void hidden_weight_gradient(int M, int N, int R, const float* dZ, const float* A,
                                                       long c_begin, long c_end, float* out, float* smem) {
    constexpr int LD = BM + 4;
    float* As = smem;                 // [2][BK][LD]  dZ slab: [k = column][m]
    float* Bs = smem + 2 * BK * LD;   // [2][BK][LD]  A slab:  [k = column][n]
    const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
    for (int m_base = 0; m_base < M; m_base += BM)
        for (int n_base = 0; n_base < N; n_base += BM) {
            float acc[8][8] = {};
            float bias_acc = 0.f;
            float4 ra[2], rb[2];
            auto fetch = [&](long c0) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int idx = t + j * THREADS, c = idx >> 5, r4 = idx & 31;
                    const long col = c0 + c;
                    const bool ok = col < c_end;
                    const int m = m_base + r4 * 4, nn = n_base + r4 * 4;
                    ra[j] = ok && m < M ? __ldcg(reinterpret_cast<const float4*>(dZ + (size_t)col * M + m))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
                    rb[j] = ok && nn < N ? __ldcg(reinterpret_cast<const float4*>(A + (size_t)col * N + nn))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            };
            auto store = [&](int buf) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int idx = t + j * THREADS, c = idx >> 5, r4 = idx & 31;
                    *reinterpret_cast<float4*>(As + (buf * BK + c) * LD + r4 * 4) = ra[j];
                    *reinterpret_cast<float4*>(Bs + (buf * BK + c) * LD + r4 * 4) = rb[j];
                }
            };
            if (c_begin < c_end) {
                fetch(c_begin);
                store(0);
                __syncthreads();
                int buf = 0;
                for (long c0 = c_begin; c0 < c_end; c0 += BK) {
                    const bool more = c0 + BK < c_end;
                    if (more) fetch(c0 + BK);
                    const float* a = As + buf * BK * LD;
                    const float* b = Bs + buf * BK * LD;
#pragma unroll
                    for (int k = 0; k < BK; ++k) {
                        const float4 a0 = *reinterpret_cast<const float4*>(a + k * LD + ty * 8);
                        const float4 a1 = *reinterpret_cast<const float4*>(a + k * LD + ty * 8 + 4);
                        const float4 b0 = *reinterpret_cast<const float4*>(b + k * LD + tx * 8);
                        const float4 b1 = *reinterpret_cast<const float4*>(b + k * LD + tx * 8 + 4);
                        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                        const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                        for (int i = 0; i < 8; ++i)
#pragma unroll
                            for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
                    }
                    if (n_base == 0 && t < BM) {
                        // value-row columns carry the bias gradient
                        const long first = ((c0 + R - 1) / R) * R;
                        for (long c = first; c < c0 + BK && c < c_end; c += R) bias_acc += a[(c - c0) * LD + t];
                    }
                    __syncthreads();
                    if (more) {
                        store(buf ^ 1);
                        __syncthreads();
                        buf ^= 1;
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int m = m_base + ty * 8 + i;
                if (m >= M) continue;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int nn = n_base + tx * 8 + j;
                    if (nn < N) out[m + (size_t)nn * M] = acc[i][j];
                }
            }
            if (n_base == 0 && t < BM && m_base + t < M) out[m_base + t + (size_t)N * M] = bias_acc;
        }
}

// dZ_prev = adjoint(W^T dZ; Y_prev) for points [q0, q1); W is K x M
// column-major (this layer K neurons, previous layer M). With INPUT_GRAD the
// previous layer is the first hidden one: dZ_prev is not stored and the first
// layer's gradient (M x (K0+1), bias last) goes to `part` instead.
template <int SID, class Act, bool INPUT_GRAD>
__device__ __forceinline__ void hidden_backward(int M, int K, const float* W, const float* dZ, const float* Yprev,
                                                float* dZprev, const float* X0, int K0, float* part, long q0,
                                                long q1, float* smem) {
    constexpr int R = StaticJet<SID>::R;
    using T = Tiling<R>;
    using S = fast::Smem<T::BN>;
    for (int m_base = 0; m_base < M; m_base += BM) {
        float gacc[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) gacc[k] = 0.f;
        for (long p0 = q0; p0 < q1; p0 += T::PTS) {
            const int points = int(min((long)T::PTS, q1 - p0));
            float acc[8][T::BN / 16] = {};
            auto aload = [&](int m, int k) -> float {
                const int mm = m_base + m;
                return (mm < M && k < K) ? __ldg(W + k + (size_t)mm * K) : 0.f;
            };
            fast::gemm_main<T::BN>(acc, smem, K, aload, FreshColumns{dZ + (size_t)p0 * R * K, K, (long)points * R});
            fast::stage_tile<T::BN>(acc, smem);
            for (int e = threadIdx.x; e < BM * points; e += THREADS) {
                const int m = e % BM, p = e / BM, mm = m_base + m;
                if (mm >= M) continue;
                float g[R], y[R];
                const float* yp = Yprev + ((size_t)(p0 + p) * R) * M + mm;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    g[r] = smem[(p * R + r) * S::LDZ + m];
                    y[r] = __ldcg(yp + (size_t)r * M);
                }
                StaticJet<SID>::template adjoint<Act>(y, g);
                if (INPUT_GRAD) {
                    fast::input_gradient<R>(g, X0 + (size_t)(p0 + p) * R * K0, K0, gacc);  // inputs: staged before launch
                } else {
                    float* out = dZprev + ((size_t)(p0 + p) * R) * M + mm;
#pragma unroll
                    for (int r = 0; r < R; ++r) out[(size_t)r * M] = g[r];
                }
            }
            __syncthreads();
        }
        if (INPUT_GRAD) {
            // thread t and t + 128 share neuron t % 128: fold, then store
            float* red = smem;  // [BM][9]
            const int m = threadIdx.x % BM;
            if (threadIdx.x >= BM)
#pragma unroll
                for (int k = 0; k < 9; ++k) red[m * 9 + k] = gacc[k];
            __syncthreads();
            if (threadIdx.x < BM && m_base + m < M) {
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (k < K0) part[m_base + m + (size_t)k * M] = gacc[k] + red[m * 9 + k];
                part[m_base + m + (size_t)K0 * M] = gacc[8] + red[m * 9 + 8];
            }
            __syncthreads();
        }
    }
}

// The epoch of one cost chunk. grid = ceil(tiles / tiles_per_cta); CTA b owns
// points [b * tiles_per_cta * PTS, ...). Hidden widths must be multiples of 4,
// the first layer must have at most 8 inputs and the last hidden layer K
// neurons (128 or 256).
template <int SID, class Act, int O, int K>
__global__ void __launch_bounds__(THREADS, 1) k_point_epoch(EpochNet net, long P, int tiles_per_cta, EpochHead head) {
    constexpr int R = StaticJet<SID>::R;
    using T = Tiling<R>;
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    const int L = net.layers;
    const long q0 = (long)blockIdx.x * tiles_per_cta * T::PTS;
    const long q1 = min(P, q0 + (long)tiles_per_cta * T::PTS);
    float* part = net.partials + (size_t)blockIdx.x * net.params;
    CostStats local = cost_empty();

    // first hidden layer: one thread per (neuron, point)
    {
        const int M = net.width[1], K0 = net.width[0];
        const float* W = net.W[0];
        const float* X = net.act[0];
        float* Y = net.act[1];
        for (long e = threadIdx.x; e < (long)M * (q1 - q0); e += THREADS) {
            const int m = int(e % M);
            const long p = q0 + e / M;
            float z[R], y[R];
            fast::input_rows<R>(W, M, m, K0, X + (size_t)p * R * K0, z);  // inputs: staged before launch
            z[0] += __ldg(W + (size_t)M * K0 + m);
            StaticJet<SID>::template forward<Act>(z, y);
            float* out = Y + (size_t)p * R * M + m;
#pragma unroll
            for (int r = 0; r < R; ++r) out[(size_t)r * M] = y[r];
        }
        __syncthreads();
    }
    for (int l = 2; l < L; ++l)
        hidden_forward<SID, Act>(net.width[l], net.width[l - 1], net.W[l - 1], net.act[l - 1], net.act[l], q0, q1,
                                 smem);
    matching_head<SID, Act, O, K>(net.W[L - 1], net.act[L - 1], net.dz[1], q0, q1, head, part + net.offset[L - 1],
                                  smem, local);
    __syncthreads();
    float* cur = net.dz[1];
    for (int l = L - 1; l >= 2; --l) {
        const int M = net.width[l], N = net.width[l - 1];
        hidden_weight_gradient(M, N, R, cur, net.act[l - 1], q0 * R, q1 * R, part + net.offset[l - 1], smem);
        __syncthreads();
        if (l - 1 == 1) {
            hidden_backward<SID, Act, true>(N, M, net.W[l - 1], cur, net.act[1], nullptr, net.act[0], net.width[0],
                                            part + net.offset[0], q0, q1, smem);
        } else {
            float* next = cur == net.dz[0] ? net.dz[1] : net.dz[0];
            hidden_backward<SID, Act, false>(N, M, net.W[l - 1], cur, net.act[l - 1], next, nullptr, 0, nullptr, q0,
                                             q1, smem);
            cur = next;
        }
        __syncthreads();
    }
    cost_finish(local, head.red);
}

}  // namespace small
}  // namespace cpde
