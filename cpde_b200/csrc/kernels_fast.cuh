// Fast tier: fused kernels for networks whose hidden widths are multiples of
// 32 and whose derivative schema has register-resident jet code
// (generated/jets_static.cuh).
//
// Every GEMM tile covers 128 neurons x Pt whole points, i.e. Pt*R adjacent
// columns of the interleaved activation layout, so the epilogue owns all R
// derivative rows of each (neuron, point) and applies the jet combine (forward)
// or its adjoint (backward) in registers before a single coalesced store.
// The reference instead runs one launch per derivative row for the combine
// and another for the adjoint (cuda/cpde_engine.cuh:852-866,973).
#pragma once
#include "generated/jets_static.cuh"
#include "kernels_generic.cuh"
#include "tc.cuh"

namespace cpde {
namespace fast {

constexpr int THREADS = 256;
constexpr int BM = 128;  // neurons per tile
constexpr int BK = 16;   // K slab

// Points per tile and padded column count for R derivative rows: as many whole
// points as fit in 128 columns, rounded up to a multiple of 16 columns.
template <int R>
struct Tiling {
    static constexpr int PTS = (128 / R) > 0 ? (128 / R) : 1;
    static constexpr int COLS = PTS * R;
    static constexpr int BN = ((COLS + 15) / 16) * 16;
    static constexpr int TN = BN / 16;  // columns per thread
};

// Shared memory of the GEMM main loop, reused by the epilogue as a Z tile
// (BMT neurons: 128, or 64 for layers of at most 64 neurons).
template <int BN, int BMT = BM>
struct Smem {
    static constexpr int LDA = BMT + 4, LDB = BN + 4, LDZ = BMT + 4;
    static constexpr int MAIN = 2 * BK * LDA + 2 * BK * LDB;
    static constexpr int EPI = BN * LDZ;
    static constexpr int FLOATS = MAIN > EPI ? MAIN : EPI;
};

// ---------------------------------------------------------------------------
// Main loop: acc[RM][TN] += A (BMT x K) * B (K x BN), RM = BMT / 16. A and B
// slabs are staged through registers so the next slab's global loads overlap
// the current FMAs.
//   A loader: a(m, k) for m < BMT, k < K (zero outside)
//   B loader: b4(c, k4) returns float4 of b(k4*4 .. k4*4+3, c) (zero outside)
//
// Thread layout (Layout<BN, BMT>). When BN is a multiple of 64 the 8 warps
// form a 2 x 4 grid of (BMT/2) x (BN/4) warp tiles and lane (tm, tn) =
// (lane / 4, lane % 4) owns rows wm BMT/2 + 32 h + 4 tm + i and columns
// wn BN/4 + 16 g + 4 tn + j (i, j < 4): every shared-memory read of a k step
// is a float4, and the lanes of one read cover one contiguous 128-byte (A)
// or 64-byte (B) span, one wavefront each: 3 wavefronts per 32 FMAs of a
// 64-row tile, 4 per 64 of a 128-row tile. (A layout of scalar column reads,
// 16 lanes apart, took 9 wavefronts per 32 FMAs and held the 64-row forward
// at about half of the FMA pipe, bound on shared-memory bandwidth.)
// Otherwise thread (ty, tx) = (t / 16, t % 16) owns rows ty RM + i and
// columns tx + 16 j.
template <int BN, int BMT>
struct Layout {
    static constexpr bool kWide = BN % 64 == 0;
    static constexpr int RM = BMT / 16, TN = BN / 16;
    // first row of the thread's row group h, first column of its column group g (kWide), or the
    // row base and column of index j (otherwise)
    __device__ static int row(int h) {
        const int t = threadIdx.x;
        if constexpr (kWide) return (t >> 7) * (BMT / 2) + 32 * h + 4 * ((t & 31) >> 2);
        else return (t >> 4) * RM + 4 * h;
    }
    __device__ static int column(int g) {
        const int t = threadIdx.x;
        if constexpr (kWide) return ((t >> 5) & 3) * (BN / 4) + 16 * g + 4 * (t & 3);
        else return (t & 15) + 16 * g;
    }
};

template <int BN, int BMT = BM, class ALoad, class BLoad>
__device__ __forceinline__ void gemm_main(float (&acc)[BMT / 16][BN / 16], float* smem, int K, const ALoad& aload,
                                          const BLoad& bload) {
    using S = Smem<BN, BMT>;
    using Lo = Layout<BN, BMT>;
    constexpr int TN = BN / 16, RM = BMT / 16;
    float* As = smem;                   // [2][BK][LDA]
    float* Bs = smem + 2 * BK * S::LDA;  // [2][BK][LDB]
    const int t = threadIdx.x;
    // A slab: 16 x BMT values, RM per thread: k = t/16 (0..15), m = (t%16)*RM + i
    constexpr int BLOADS = (BN * 4 + THREADS - 1) / THREADS;  // float4 loads of the B slab per thread
    float ra[RM];
    float4 rb[BLOADS];
    auto fetch = [&](int k0) {
        const int k = t >> 4, m0 = (t & 15) * RM;
#pragma unroll
        for (int i = 0; i < RM; ++i) ra[i] = aload(m0 + i, k0 + k);
#pragma unroll
        for (int j = 0; j < BLOADS; ++j) {
            int idx = t + j * THREADS;  // (column, k-quad)
            int c = idx >> 2, q = idx & 3;
            rb[j] = c < BN ? bload(c, (k0 >> 2) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store = [&](int buf) {
        float* a = As + buf * BK * S::LDA;
        float* b = Bs + buf * BK * S::LDB;
        const int k = t >> 4, m0 = (t & 15) * RM;
#pragma unroll
        for (int i4 = 0; i4 < RM / 4; ++i4)
            *reinterpret_cast<float4*>(a + k * S::LDA + m0 + 4 * i4) =
                make_float4(ra[4 * i4], ra[4 * i4 + 1], ra[4 * i4 + 2], ra[4 * i4 + 3]);
#pragma unroll
        for (int j = 0; j < BLOADS; ++j) {
            int idx = t + j * THREADS;
            int c = idx >> 2, q = idx & 3;
            if (c < BN) {
                b[(4 * q + 0) * S::LDB + c] = rb[j].x;
                b[(4 * q + 1) * S::LDB + c] = rb[j].y;
                b[(4 * q + 2) * S::LDB + c] = rb[j].z;
                b[(4 * q + 3) * S::LDB + c] = rb[j].w;
            }
        }
    };
    const int slabs = (K + BK - 1) / BK;
    fetch(0);
    store(0);
    __syncthreads();
    // the thread's first row of A and first column of B in slab buffer 0
    const float* a_base = As + Lo::row(0);
    const float* b_base = Bs + Lo::column(0);
    for (int s = 0; s < slabs; ++s) {
        const int buf = s & 1;
        if (s + 1 < slabs) fetch((s + 1) * BK);
        const float* a = a_base + buf * BK * S::LDA;
        const float* b = b_base + buf * BK * S::LDB;
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            float av[RM];
#pragma unroll
            for (int h = 0; h < RM / 4; ++h) {
                // row group h starts 32 rows (kWide) or 4 rows further
                const float4 a4 = *reinterpret_cast<const float4*>(a + k * S::LDA + (Lo::kWide ? 32 : 4) * h);
                av[4 * h] = a4.x;
                av[4 * h + 1] = a4.y;
                av[4 * h + 2] = a4.z;
                av[4 * h + 3] = a4.w;
            }
            float bv[TN];
            if constexpr (Lo::kWide) {
#pragma unroll
                for (int g = 0; g < TN / 4; ++g) {
                    const float4 b4 = *reinterpret_cast<const float4*>(b + k * S::LDB + 16 * g);
                    bv[4 * g] = b4.x;
                    bv[4 * g + 1] = b4.y;
                    bv[4 * g + 2] = b4.z;
                    bv[4 * g + 3] = b4.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < TN; ++j) bv[j] = b[k * S::LDB + 16 * j];
            }
#pragma unroll
            for (int i = 0; i < RM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (s + 1 < slabs) {
            store(buf ^ 1);
            __syncthreads();
        }
    }
    __syncthreads();  // smem is reused by the epilogue
}

template <int BN, int BMT = BM>
__device__ __forceinline__ void stage_tile(const float (&acc)[BMT / 16][BN / 16], float* smem) {
    using S = Smem<BN, BMT>;
    using Lo = Layout<BN, BMT>;
    constexpr int RM = BMT / 16;
#pragma unroll
    for (int j = 0; j < BN / 16; ++j) {
        const int c = Lo::kWide ? Lo::column(j >> 2) + (j & 3) : Lo::column(j);
#pragma unroll
        for (int h = 0; h < RM / 4; ++h)
            *reinterpret_cast<float4*>(smem + c * S::LDZ + Lo::row(h)) =
                make_float4(acc[4 * h][j], acc[4 * h + 1][j], acc[4 * h + 2][j], acc[4 * h + 3][j]);
    }
    __syncthreads();
}

// Column loader of an interleaved activation matrix (K rows per column).
struct ColumnLoad {
    const float* base;  // first column of the tile
    int K;
    long columns;  // valid columns from base
    __device__ float4 operator()(int c, int k4) const {
        if (c >= columns || k4 * 4 >= K) return make_float4(0.f, 0.f, 0.f, 0.f);
        return __ldg(reinterpret_cast<const float4*>(base + (size_t)c * K) + k4);
    }
};

// ---------------------------------------------------------------------------
// Narrow first layer (K <= 8 inputs): one loop nest per input width, so no FMA
// or load is predicated off for the unused inputs (a predicated 8-wide loop
// issues 2.5x the instructions at K = 2).

// Calls f(e, x[e]) for e = 0 .. L-1 in order, reading the row with the
// widest loads its alignment allows: the inputs of point p start at
// X + p L, X 16-byte aligned, so rows of L % 4 == 0 floats are 16-byte
// aligned and rows of even L 8-byte aligned. Every lane of a warp reads the
// same row (one broadcast transaction per load).
template <int L, class F>
__device__ __forceinline__ void for_row(const float* x, F f) {
    if constexpr (L % 4 == 0) {
#pragma unroll
        for (int i = 0; i < L / 4; ++i) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
            f(4 * i, v.x);
            f(4 * i + 1, v.y);
            f(4 * i + 2, v.z);
            f(4 * i + 3, v.w);
        }
    } else if constexpr (L % 2 == 0) {
#pragma unroll
        for (int i = 0; i < L / 2; ++i) {
            const float2 v = __ldg(reinterpret_cast<const float2*>(x) + i);
            f(2 * i, v.x);
            f(2 * i + 1, v.y);
        }
    } else {
#pragma unroll
        for (int i = 0; i < L; ++i) f(i, __ldg(x + i));
    }
}

// for_row over a row in shared memory (plain loads; x 16-byte aligned).
template <int L, class F>
__device__ __forceinline__ void for_row_shared(const float* x, F f) {
    if constexpr (L % 4 == 0) {
#pragma unroll
        for (int i = 0; i < L / 4; ++i) {
            const float4 v = reinterpret_cast<const float4*>(x)[i];
            f(4 * i, v.x);
            f(4 * i + 1, v.y);
            f(4 * i + 2, v.z);
            f(4 * i + 3, v.w);
        }
    } else if constexpr (L % 2 == 0) {
#pragma unroll
        for (int i = 0; i < L / 2; ++i) {
            const float2 v = reinterpret_cast<const float2*>(x)[i];
            f(2 * i, v.x);
            f(2 * i + 1, v.y);
        }
    } else {
#pragma unroll
        for (int i = 0; i < L; ++i) f(i, x[i]);
    }
}

// z[r] = sum_k W[m + k M] x[r K + k]
template <int R, int K>
__device__ __forceinline__ void input_rows_k(const float* __restrict__ W, int M, int m, const float* x,
                                             float (&z)[R]) {
    float w[K];
#pragma unroll
    for (int k = 0; k < K; ++k) w[k] = __ldg(W + m + (size_t)k * M);
#pragma unroll
    for (int r = 0; r < R; ++r) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) acc = fmaf(w[k], __ldg(x + r * K + k), acc);
        z[r] = acc;
    }
}
template <int R>
__device__ __forceinline__ void input_rows(const float* __restrict__ W, int M, int m, int K, const float* x,
                                           float (&z)[R]) {
    switch (K) {
        case 1: input_rows_k<R, 1>(W, M, m, x, z); break;
        case 2: input_rows_k<R, 2>(W, M, m, x, z); break;
        case 3: input_rows_k<R, 3>(W, M, m, x, z); break;
        case 4: input_rows_k<R, 4>(W, M, m, x, z); break;
        default: {
            float w[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) w[k] = k < K ? __ldg(W + m + (size_t)k * M) : 0.f;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (k < K) acc = fmaf(w[k], __ldg(x + r * K + k), acc);
                z[r] = acc;
            }
        }
    }
}

// gacc[k] += sum_r g[r] x[r K + k] (k < K), gacc[8] += g[0] (bias)
template <int R, int K>
__device__ __forceinline__ void input_gradient_k(const float (&g)[R], const float* x, float (&gacc)[9]) {
    for_row<R * K>(x, [&](int e, float v) { gacc[e % K] = fmaf(g[e / K], v, gacc[e % K]); });
    gacc[8] += g[0];
}
// input_gradient_k with the point's row x in shared memory
template <int R, int K>
__device__ __forceinline__ void input_gradient_row(const float (&g)[R], const float* x, float (&gacc)[9]) {
    for_row_shared<R * K>(x, [&](int e, float v) { gacc[e % K] = fmaf(g[e / K], v, gacc[e % K]); });
    gacc[8] += g[0];
}
template <int R>
__device__ __forceinline__ void input_gradient(const float (&g)[R], const float* x, int K, float (&gacc)[9]) {
    switch (K) {
        case 1: input_gradient_k<R, 1>(g, x, gacc); break;
        case 2: input_gradient_k<R, 2>(g, x, gacc); break;
        case 3: input_gradient_k<R, 3>(g, x, gacc); break;
        case 4: input_gradient_k<R, 4>(g, x, gacc); break;
        default:
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (k < K) gacc[k] = fmaf(g[r], __ldg(x + r * K + k), gacc[k]);
            gacc[8] += g[0];
    }
}

// ---------------------------------------------------------------------------
// Hidden layer forward: Y = f(W X + b) with the jet combine in the epilogue.
// grid = (ceil(P / PTS), ceil(M / BMT)). Requires K % 4 == 0. The 64-neuron
// variant is held to 85 registers so that three CTAs share an SM (its tiles
// are short, and the first slab's load latency is exposed in each).

template <int SID, class Act, int BMT = BM>
__global__ void __launch_bounds__(THREADS, BMT == 64 ? 3 : 2) k_forward(int M, int K, long P, const float* __restrict__ W,
                                                     const float* __restrict__ bias, const float* __restrict__ X,
                                                     float* __restrict__ Y) {
    constexpr int R = StaticJet<SID>::R;
    using T = Tiling<R>;
    using S = Smem<T::BN, BMT>;
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    const long p0 = (long)blockIdx.x * T::PTS;
    const int m_base = blockIdx.y * BMT;
    const long points = min((long)T::PTS, P - p0);
    float acc[BMT / 16][T::TN] = {};
    auto aload = [&](int m, int k) -> float {
        int mm = m_base + m;
        return (mm < M && k < K) ? __ldg(W + mm + (size_t)k * M) : 0.f;
    };
    ColumnLoad bload{X + (size_t)p0 * R * K, K, points * R};
    gemm_main<T::BN, BMT>(acc, smem, K, aload, bload);
    stage_tile<T::BN, BMT>(acc, smem);
    for (int e = threadIdx.x; e < BMT * T::PTS; e += THREADS) {
        const int m = e % BMT, p = e / BMT;
        const int mm = m_base + m;
        if (p >= points || mm >= M) continue;
        float z[R], y[R];
#pragma unroll
        for (int r = 0; r < R; ++r) z[r] = smem[(p * R + r) * S::LDZ + m];
        z[0] += __ldg(bias + mm);
        StaticJet<SID>::template forward<Act>(z, y);
        float* out = Y + ((size_t)(p0 + p) * R) * M + mm;
#pragma unroll
        for (int r = 0; r < R; ++r) out[(size_t)r * M] = y[r];
    }
}

// First hidden layer: Y = f(W X + b) for a narrow input (K <= 8); one thread
// per (neuron, point). Memory-bound on the store of Y.
template <int SID, class Act>
__global__ void __launch_bounds__(THREADS) k_input_forward(int M, int K, long P, const float* __restrict__ W,
                                                           const float* __restrict__ bias,
                                                           const float* __restrict__ X, float* __restrict__ Y) {
    constexpr int R = StaticJet<SID>::R;
    const long total = (long)M * P;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)blockDim.x * gridDim.x) {
        const int m = int(e % M);
        const long p = e / M;
        float z[R], y[R];
        input_rows<R>(W, M, m, K, X + (size_t)p * R * K, z);
        z[0] += __ldg(bias + m);
        StaticJet<SID>::template forward<Act>(z, y);
        float* out = Y + (size_t)p * R * M + m;
#pragma unroll
        for (int r = 0; r < R; ++r) out[(size_t)r * M] = y[r];
    }
}

// ---------------------------------------------------------------------------
// Hidden layer backward: dZ_prev = adjoint(W^T dZ; Y_prev) with the jet
// adjoint in the epilogue. M = width of the previous layer, K = this layer's.
// With INPUT_GRAD the previous layer is the first hidden layer: its weight
// gradient partial (M x (K0+1) with K0 input channels, bias last) is
// accumulated per CTA and dZ_prev is not stored.

template <int SID, class Act, bool INPUT_GRAD, int BMT = BM>
__global__ void __launch_bounds__(THREADS, BMT == 64 && !INPUT_GRAD ? 3 : 2) k_backward(int M, int K, long P, const float* __restrict__ W,
                                                      const float* __restrict__ dZ, const float* __restrict__ Yprev,
                                                      float* __restrict__ dZprev, const float* __restrict__ X0,
                                                      int K0, float* __restrict__ input_partials) {
    constexpr int R = StaticJet<SID>::R;
    using T = Tiling<R>;
    using S = Smem<T::BN, BMT>;
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    const int m_base = blockIdx.y * BMT;
    // INPUT_GRAD: up to 8 input channels + bias of this thread's neuron (every
    // role of a thread has the same neuron because THREADS is a multiple of BM)
    float gacc[9];
#pragma unroll
    for (int b = 0; b < 9; ++b) gacc[b] = 0.f;
    // Grid-stride over point tiles so INPUT_GRAD partials stay per CTA.
    for (long tile = blockIdx.x; tile * T::PTS < P; tile += gridDim.x) {
        const long p0 = tile * T::PTS;
        const long points = min((long)T::PTS, P - p0);
        float acc[BMT / 16][T::TN] = {};
        // A = W^T: a(m, k) = W[k + m*K] (W is K x M column-major)
        auto aload = [&](int m, int k) -> float {
            int mm = m_base + m;
            return (mm < M && k < K) ? __ldg(W + k + (size_t)mm * K) : 0.f;
        };
        ColumnLoad bload{dZ + (size_t)p0 * R * K, K, points * R};
        gemm_main<T::BN, BMT>(acc, smem, K, aload, bload);
        stage_tile<T::BN, BMT>(acc, smem);
        for (int e = threadIdx.x; e < BMT * T::PTS; e += THREADS) {
            const int m = e % BMT, p = e / BMT;
            const int mm = m_base + m;
            if (p >= points || mm >= M) continue;
            float g[R], y[R];
            const float* yp = Yprev + ((size_t)(p0 + p) * R) * M + mm;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                g[r] = smem[(p * R + r) * S::LDZ + m];
                y[r] = yp[(size_t)r * M];
            }
            StaticJet<SID>::template adjoint<Act>(y, g);
            if (INPUT_GRAD) {
                input_gradient<R>(g, X0 + (size_t)(p0 + p) * R * K0, K0, gacc);
            } else {
                float* out = dZprev + ((size_t)(p0 + p) * R) * M + mm;
#pragma unroll
                for (int r = 0; r < R; ++r) out[(size_t)r * M] = g[r];
            }
        }
        __syncthreads();
    }
    if (INPUT_GRAD) {
        // Fold this thread's roles into per-neuron sums in smem, then store the
        // CTA partial: input_partials[cta][m][k], k = 0..K0 (bias last).
        float* red = smem;  // [BMT][9]
        for (int i = threadIdx.x; i < BMT * 9; i += THREADS) red[i] = 0.f;
        __syncthreads();
        const int m = threadIdx.x % BMT;
        for (int turn = 0; turn < THREADS / BMT; ++turn) {
            if (threadIdx.x / BMT == turn)
#pragma unroll
                for (int k = 0; k < 9; ++k) red[m * 9 + k] += gacc[k];
            __syncthreads();
        }
        // partial of CTA column x: full M x (K0+1) column-major; y-blocks write disjoint neuron slices
        float* out = input_partials + (size_t)blockIdx.x * M * (K0 + 1);
        for (int i = threadIdx.x; i < BMT * (K0 + 1); i += THREADS) {
            int ml = i % BMT, k = i / BMT;
            if (m_base + ml < M) out[(m_base + ml) + (size_t)k * M] = red[ml * 9 + (k == K0 ? 8 : k)];
        }
    }
}

// ---------------------------------------------------------------------------
// Weight gradient of a hidden layer, split over columns: each CTA sums
// dZ[:, c] A[:, c]^T over its column range into a TILE x TILE tile (plus the
// bias column: sum of dZ over value-row columns) and stores a partial
// partials[cta][m + n*M] (n = N is the bias). grid = (splits, ceil(N/TILE),
// ceil(M/TILE)), (TILE/8)^2 threads.

template <int TILE>
__device__ __forceinline__ void weight_gradient_tile(int M, int N, long columns, int R, long per_split,
                                                     const float* __restrict__ dZ, const float* __restrict__ A,
                                                     float* __restrict__ partials) {
    constexpr int TT = TILE / 8, NT = TT * TT;  // threads per tile side, per CTA (8 x 8 outputs each)
    constexpr int LOADS = 4 * TILE / NT;        // float4 loads of each slab per thread
    constexpr int LD = TILE + 4;
    __shared__ __align__(16) float As[2][BK][LD];  // dZ slab: [k = column][m]
    __shared__ __align__(16) float Bs[2][BK][LD];  // A slab:  [k = column][n]
    const int t = threadIdx.x, tx = t % TT, ty = t / TT;
    const int n_base = blockIdx.y * TILE, m_base = blockIdx.z * TILE;
    const long c_begin = (long)blockIdx.x * per_split;
    const long c_end = min(columns, c_begin + per_split);
    float acc[8][8] = {};
    float bias_acc = 0.f;  // thread t < TILE: neuron m_base + t
    float4 ra[LOADS], rb[LOADS];
    // slab loads: 16 columns x TILE rows = 4 TILE float4 of each operand
    auto fetch = [&](long c0) {
#pragma unroll
        for (int j = 0; j < LOADS; ++j) {
            int idx = t + j * NT;
            int c = idx / (TILE / 4), r4 = idx % (TILE / 4);  // column in slab, float4 index along rows
            long col = c0 + c;
            bool ok = col < c_end;
            int m = m_base + r4 * 4, n = n_base + r4 * 4;
            ra[j] = ok && m < M ? __ldg(reinterpret_cast<const float4*>(dZ + (size_t)col * M + m))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
            rb[j] = ok && n < N ? __ldg(reinterpret_cast<const float4*>(A + (size_t)col * N + n))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int j = 0; j < LOADS; ++j) {
            int idx = t + j * NT;
            int c = idx / (TILE / 4), r4 = idx % (TILE / 4);
            *reinterpret_cast<float4*>(&As[buf][c][r4 * 4]) = ra[j];
            *reinterpret_cast<float4*>(&Bs[buf][c][r4 * 4]) = rb[j];
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
#pragma unroll
            for (int k = 0; k < BK; ++k) {
                const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 8]);
                const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 8 + 4]);
                const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 8]);
                const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 8 + 4]);
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            }
            if (blockIdx.y == 0 && t < TILE) {
                // value-row columns of this slab carry the bias gradient
                long first = ((c0 + R - 1) / R) * R;
                for (long c = first; c < c0 + BK && c < c_end; c += R) bias_acc += As[buf][c - c0][t];
            }
            if (more) {
                __syncthreads();
                store(buf ^ 1);
                __syncthreads();
                buf ^= 1;
            }
        }
    }
    float* out = partials + (size_t)blockIdx.x * M * (N + 1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        int m = m_base + ty * 8 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int n = n_base + tx * 8 + j;
            if (n < N) out[m + (size_t)n * M] = acc[i][j];
        }
    }
    if (blockIdx.y == 0 && t < TILE && m_base + t < M) out[m_base + t + (size_t)N * M] = bias_acc;
}

static __global__ void __launch_bounds__(THREADS, 2) k_weight_gradient(int M, int N, long columns, int R, long per_split,
                                                             const float* __restrict__ dZ,
                                                             const float* __restrict__ A,
                                                             float* __restrict__ partials) {
    weight_gradient_tile<BM>(M, N, columns, R, per_split, dZ, A, partials);
}

// The same with 64 x 64 tiles and 64 threads, for layers of at most 64 x 64
// (a 128 x 128 tile would compute three quarters zeros there). (Held to 128
// registers for eight CTAs per SM instead of six it measured slower: 0.333 ->
// 0.348 ms on config 3's layers.)
static __global__ void __launch_bounds__(64) k_weight_gradient64(int M, int N, long columns, int R, long per_split,
                                                          const float* __restrict__ dZ, const float* __restrict__ A,
                                                          float* __restrict__ partials) {
    weight_gradient_tile<64>(M, N, columns, R, per_split, dZ, A, partials);
}

// ---------------------------------------------------------------------------
// Output layer (n_out <= 8 linear outputs): Z_out[o, p, r] = W_out Y + b.
// One warp per (point, row) column group: lanes split the K inputs.

static __global__ void k_output_forward(int O, int K, long P, int R, const float* __restrict__ W,
                                 const float* __restrict__ bias, const float* __restrict__ Y,
                                 float* __restrict__ Z) {
    // a warp per column, four columns in flight (their loads issued together)
    constexpr int U = 4;
    const int lane = threadIdx.x & 31;
    const long warps = ((long)gridDim.x * blockDim.x) >> 5;
    const long columns = P * R;
    for (long c0 = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; c0 < columns; c0 += U * warps) {
        float acc[U][8];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int o = 0; o < 8; ++o) acc[u][o] = 0.f;
        for (int k = lane; k < K; k += 32) {
            float v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const long c = c0 + u * warps;
                v[u] = c < columns ? __ldg(Y + (size_t)c * K + k) : 0.f;
            }
#pragma unroll
            for (int o = 0; o < 8; ++o)
                if (o < O) {
                    const float w = __ldg(W + o + (size_t)k * O);
#pragma unroll
                    for (int u = 0; u < U; ++u) acc[u][o] = fmaf(w, v[u], acc[u][o]);
                }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const long c = c0 + u * warps;
#pragma unroll
            for (int o = 0; o < 8; ++o) {
                if (o >= O) break;
                float v = acc[u][o];
                for (int s = 16; s; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
                if (lane == 0 && c < columns) Z[(size_t)c * O + o] = v + ((c % R) == 0 ? __ldg(bias + o) : 0.f);
            }
        }
    }
}

// Output layer backward: dY = W_out^T dZ_out, adjoint with Y -> dZ of the
// last hidden layer; weight gradient of the output layer accumulated per CTA
// (partials[cta][o + k*O], bias at k = K). One thread per (neuron, point):
// a CTA covers output_slice(K) neurons (K itself when it divides 128, so no
// thread idles at widths 32 and 64) and THREADS / slice point lanes; each
// thread copies the values of its next point into shared memory while it
// works on the current one.
__host__ __device__ constexpr int output_slice(int K) { return K <= BM && BM % K == 0 ? K : BM; }
template <int R>
constexpr size_t output_backward_smem() { return size_t(2) * R * THREADS * sizeof(float); }

template <int SID, class Act>
__global__ void __launch_bounds__(THREADS) k_output_backward(int O, int K, long P, const float* __restrict__ W,
                                                             const float* __restrict__ dZout,
                                                             const float* __restrict__ Y, float* __restrict__ dZ,
                                                             float* __restrict__ partials) {
    constexpr int R = StaticJet<SID>::R;
    extern __shared__ float ystage[];  // [2][R][THREADS], output_backward_smem<R>() bytes
    __shared__ float red[THREADS];
    const int NB = output_slice(K), lanes = THREADS / NB;
    float gw[8], gb[8];
#pragma unroll
    for (int o = 0; o < 8; ++o) gw[o] = gb[o] = 0.f;
    const int t = threadIdx.x, ml = t % NB, m = blockIdx.y * NB + ml;
    const int lane_p = t / NB;  // 0 .. lanes - 1 (threads beyond lanes * NB idle)
    const bool active = m < K && lane_p < lanes;
    float w[8];
#pragma unroll
    for (int o = 0; o < 8; ++o) w[o] = (o < O && active) ? __ldg(W + o + (size_t)m * O) : 0.f;
    const long stride = (long)gridDim.x * lanes;
    auto stage = [&](long q, int slot) {
        if (active && q < P)
#pragma unroll
            for (int r = 0; r < R; ++r)
                tc::copy_async4(ystage + (slot * R + r) * THREADS + t, Y + ((size_t)q * R + r) * K + m);
        tc::copy_async_commit();
    };
    int slot = 0;
    long p = (long)blockIdx.x * lanes + lane_p;
    stage(p, 0);
    for (; p < P; p += stride) {
        stage(p + stride, slot ^ 1);
        tc::copy_async_wait<1>();
        if (!active) continue;
        const float* dzo = dZout + (size_t)p * R * O;
        float g[R], y[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            y[r] = ystage[(slot * R + r) * THREADS + t];
            float acc = 0.f;
#pragma unroll
            for (int o = 0; o < 8; ++o)
                if (o < O) {
                    const float d = __ldg(dzo + r * O + o);
                    acc = fmaf(w[o], d, acc);
                    gw[o] = fmaf(d, y[r], gw[o]);
                    if (r == 0) gb[o] += d;
                }
            g[r] = acc;
        }
        slot ^= 1;
        StaticJet<SID>::template adjoint<Act>(y, g);
        float* out = dZ + (size_t)p * R * K + m;
#pragma unroll
        for (int r = 0; r < R; ++r) out[(size_t)r * K] = g[r];
    }
    tc::copy_async_wait<0>();
    // fold the point lanes of each neuron, lane order
    float* out = partials + (size_t)blockIdx.x * O * (K + 1);
    for (int o = 0; o < O && o < 8; ++o) {
        red[t] = gw[o];
        __syncthreads();
        if (lane_p == 0 && active) {
            float sum = red[ml];
            for (int l = 1; l < lanes; ++l) sum += red[l * NB + ml];
            out[o + (size_t)m * O] = sum;
        }
        __syncthreads();
    }
    // bias: every neuron saw the same output adjoints; neuron 0 of each lane
    if (blockIdx.y == 0)
        for (int o = 0; o < O && o < 8; ++o) {
            red[t] = gb[o];
            __syncthreads();
            if (t == 0) {
                float sum = 0.f;
                for (int l = 0; l < lanes; ++l) sum += red[l * NB];
                out[o + (size_t)K * O] = sum;
            }
            __syncthreads();
        }
}

// Sum over the 32 lanes of a warp of each of 32 per-lane values, transposed:
// afterwards lane i holds the warp sum of v[i] in v[0] (31 shuffles in all,
// recursive halving: the lanes of each pair keep the half their index bit
// selects and add the partner's copy of it).
__device__ __forceinline__ float warp_transpose_sum(float (&v)[32]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const bool upper = lane & off;
#pragma unroll
        for (int j = 0; j < off; ++j) {
            const float send = upper ? v[j] : v[j + off];
            const float keep = upper ? v[j + off] : v[j];
            v[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    return v[0];
}

// Output layer with one linear output: a warp takes 32 columns at a time, each
// lane sums its slice k = lane + 32 j of every column's dot product (loads
// coalesced along k), and one transposed butterfly leaves column c0 + lane's
// sum in lane `lane`: 31 shuffles per 32 columns instead of 5 per column.
static __global__ void k_output_forward1(int K, long P, int R, const float* __restrict__ W,
                                         const float* __restrict__ bias, const float* __restrict__ Y,
                                         float* __restrict__ Z) {
    const int lane = threadIdx.x & 31;
    const long warps = ((long)gridDim.x * blockDim.x) >> 5;
    const long columns = P * R;
    const float b = __ldg(bias);
    for (long c0 = (((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 32; c0 < columns; c0 += warps * 32) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
        for (int k = lane; k < K; k += 32) {
            const float w = __ldg(W + k);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const long c = c0 + i;
                v[i] = fmaf(w, c < columns ? __ldg(Y + (size_t)c * K + k) : 0.f, v[i]);
            }
        }
        const float sum = warp_transpose_sum(v);
        const long c = c0 + lane;
        if (c < columns) Z[c] = sum + ((c % R) == 0 ? b : 0.f);
    }
}

// Fused output head for a matching cost: Z_out = W_out Y + b for O linear
// outputs, the squared-error loss and its adjoints (the arithmetic and order of
// k_cost_matching, cuda/cost_kernels.cuh:6-35), the output layer's weight
// gradient, dY = W_out^T dZ_out and the jet adjoint into the last hidden layer,
// all from one read of that layer's jets. One thread owns neurons
// t + 128 j (j < KPT, K = 128 KPT); a CTA walks points. Per point the O x R
// output dot products are reduced within each warp by transposed butterflies
// and across the 4 warps in shared memory; thread v < O R then owns output
// component v (row v % R, output v / R): its residual, loss term and gradient,
// which every thread reads back for the adjoint.
// partials[cta][o + m O] (bias at m = K) are summed by k_sum_partials.
template <int SID, class Act, int O, int KPT>
__global__ void __launch_bounds__(BM) k_head_matching(int K, long P, int offset, const float* __restrict__ W,
                                                      const float* __restrict__ Y, float* __restrict__ dZ,
                                                      const float* __restrict__ target, int target_samples,
                                                      const int* __restrict__ target_rows,
                                                      const float* __restrict__ weights, int weight_samples,
                                                      const double* __restrict__ multiplier, int collect,
                                                      CostReduce red, float* __restrict__ partials) {
    constexpr int R = StaticJet<SID>::R;
    constexpr int V = O * R;              // output components of a point, at most BM
    constexpr int GROUPS = (V + 31) / 32;
    static_assert(V <= BM, "one thread per output component");
    __shared__ float sums[4][GROUPS * 32];
    __shared__ float grads[V];
    __shared__ float values[4];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float w[KPT][O], gw[KPT][O];
#pragma unroll
    for (int j = 0; j < KPT; ++j)
#pragma unroll
        for (int o = 0; o < O; ++o) {
            w[j][o] = __ldg(W + o + (size_t)(t + BM * j) * O);
            gw[j][o] = 0.f;
        }
    // thread t < V: output component (row d, output o); its bias and target row
    const int d_own = t % R, o_own = t / R;
    const float bias_own = t < V ? __ldg(W + (size_t)K * O + o_own) : 0.f;
    const int trow = t < V ? __ldg(target_rows + d_own) : 0;
    float gb[O];
#pragma unroll
    for (int o = 0; o < O; ++o) gb[o] = 0.f;
    const double scale = multiplier ? *multiplier : 1.0;
    CostStats local = cost_empty();
    // The thread's values of its next point go into a shared-memory staging
    // slot (per-thread asynchronous copies) while it works on the current one.
    extern __shared__ float ystage[];  // [2][R][KPT * BM]
    auto stage = [&](long q, int slot) {
        if (q < P)
#pragma unroll
            for (int j = 0; j < KPT; ++j)
#pragma unroll
                for (int r = 0; r < R; ++r)
                    tc::copy_async4(ystage + (slot * R + r) * KPT * BM + t + BM * j,
                                    Y + ((size_t)q * R + r) * K + t + BM * j);
        tc::copy_async_commit();
    };
    int slot = 0;
    stage(blockIdx.x, 0);
    for (long p = blockIdx.x; p < P; p += gridDim.x) {
        stage(p + gridDim.x, slot ^ 1);
        tc::copy_async_wait<1>();
        float y[KPT][R];
#pragma unroll
        for (int j = 0; j < KPT; ++j)
#pragma unroll
            for (int r = 0; r < R; ++r) y[j][r] = ystage[(slot * R + r) * KPT * BM + t + BM * j];
        slot ^= 1;
#pragma unroll
        for (int g = 0; g < GROUPS; ++g) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int c = g * 32 + i, o = c / R, r = c % R;
                float a = 0.f;
                if (c < V)
#pragma unroll
                    for (int j = 0; j < KPT; ++j) a = fmaf(w[j][o], y[j][r], a);
                v[i] = a;
            }
            sums[warp][g * 32 + lane] = warp_transpose_sum(v);
        }
        __syncthreads();
        float value = 0.f;
        if (t < V) {
            const float z = sums[0][t] + sums[1][t] + sums[2][t] + sums[3][t] + (d_own == 0 ? bias_own : 0.f);
            const int wp = weight_samples == 1 ? 0 : offset + int(p);
            const float wt = __ldg(weights + ((size_t)d_own * weight_samples + wp) * O + o_own);
            float grad = 0.f;
            if (wt != 0.f) {
                const float res = z - __ldg(target + ((size_t)trow * target_samples + offset + p) * O + o_own);
                value = wt * res * res;
                grad = 2.0f * wt * res;
            }
            if (!isfinite(grad)) mark_bad(local, offset + int(p), d_own * O + o_own);
            if (multiplier) grad = scale == 0 ? 0.f : float(grad * scale);
            grads[t] = grad;
        }
#pragma unroll
        for (int sft = 16; sft; sft >>= 1) value += __shfl_xor_sync(0xffffffffu, value, sft);
        if (lane == 0) values[warp] = value;
        __syncthreads();
        if (t == 0) {
            const float total = values[0] + values[1] + values[2] + values[3];
            if (!isfinite(total)) mark_bad(local, offset + int(p), -1);
            if (collect) local.value += double(total);
        }
        float gr[O][R];
#pragma unroll
        for (int o = 0; o < O; ++o)
#pragma unroll
            for (int r = 0; r < R; ++r) gr[o][r] = grads[o * R + r];
#pragma unroll
        for (int o = 0; o < O; ++o) gb[o] += gr[o][0];
#pragma unroll
        for (int j = 0; j < KPT; ++j) {
            float dy[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float acc = 0.f;
#pragma unroll
                for (int o = 0; o < O; ++o) {
                    acc = fmaf(w[j][o], gr[o][r], acc);
                    gw[j][o] = fmaf(gr[o][r], y[j][r], gw[j][o]);
                }
                dy[r] = acc;
            }
            StaticJet<SID>::template adjoint<Act>(y[j], dy);
            float* out = dZ + (size_t)p * R * K + t + BM * j;
#pragma unroll
            for (int r = 0; r < R; ++r) out[(size_t)r * K] = dy[r];
        }
    }
    tc::copy_async_wait<0>();
    float* out = partials + (size_t)blockIdx.x * O * (K + 1);
#pragma unroll
    for (int j = 0; j < KPT; ++j)
#pragma unroll
        for (int o = 0; o < O; ++o) out[o + (size_t)(t + BM * j) * O] = gw[j][o];
    if (t == 0)
#pragma unroll
        for (int o = 0; o < O; ++o) out[o + (size_t)K * O] = gb[o];
    cost_finish(local, red);
}

// Sum CTA partials (fixed order) into a layer gradient (accumulating). A block
// of 256 threads takes 32 consecutive elements; its 8 warps sum interleaved
// subsets of the partials, which are then folded in warp order.
static __global__ void __launch_bounds__(256) k_sum_partials(const float* __restrict__ partials, int count, long size,
                                                      float* __restrict__ out) {
    __shared__ float part[8][33];
    const int x = threadIdx.x & 31, y = threadIdx.x >> 5;
    for (long base = (long)blockIdx.x * 32; base < size; base += (long)gridDim.x * 32) {
        const long i = base + x;
        float acc = 0.f;
        if (i < size)
            for (int c = y; c < count; c += 8) acc += partials[(size_t)c * size + i];
        part[y][x] = acc;
        __syncthreads();
        if (y == 0 && i < size) {
            float t = part[0][x];
#pragma unroll
            for (int k = 1; k < 8; ++k) t += part[k][x];
            out[i] += t;
        }
        __syncthreads();
    }
}

// Blocks for k_sum_partials (256 threads each) over `size` elements.
inline int sum_grid(long size) { return int(std::min<long>((size + 31) / 32, 148L * 16)); }

}  // namespace fast
}  // namespace cpde
