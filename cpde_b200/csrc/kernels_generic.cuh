// Generic-tier kernels: correct for every network shape and derivative schema.
//
// Activation layout (engine-internal, per layer): column c = p*R + r holds the
// n values of neuron 0..n-1 for point p and derivative row r, so element
// (neuron m, point p, row r) lives at (p*R + r)*n + m. A point's R rows are
// adjacent columns, which lets a tile of whole points carry every derivative a
// jet combine needs. The reference stores rows channel-major instead
// (cuda/cpde_engine.cuh:365); conversion happens only at copy-in/copy-out.
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace cpde {

constexpr int kReduceThreads = 256;
constexpr int kMaxReduceBlocks = 4096;  // capacity of the per-block partial arrays

struct CostStats {
    double value;
    int bad_sample;     // INT_MAX when none
    int bad_component;  // -1: objective; otherwise row*outputs+output
};

struct GradStats {
    double squared_norm;
    double max_abs;
    unsigned long long nonfinite;
    int first_nonfinite;  // INT_MAX when none
    int pad;
};

__host__ __device__ inline CostStats cost_empty() { return {0.0, INT_MAX, INT_MAX}; }
__host__ __device__ inline CostStats cost_combine(CostStats a, const CostStats& b) {
    a.value += b.value;
    if (b.bad_sample < a.bad_sample || (b.bad_sample == a.bad_sample && b.bad_component < a.bad_component)) {
        a.bad_sample = b.bad_sample;
        a.bad_component = b.bad_component;
    }
    return a;
}
__host__ __device__ inline GradStats grad_empty() { return {0.0, 0.0, 0ull, INT_MAX, 0}; }
__host__ __device__ inline GradStats grad_combine(GradStats a, const GradStats& b) {
    a.squared_norm += b.squared_norm;
    if (b.max_abs > a.max_abs) a.max_abs = b.max_abs;
    a.nonfinite += b.nonfinite;
    if (b.first_nonfinite < a.first_nonfinite) a.first_nonfinite = b.first_nonfinite;
    return a;
}

__device__ inline void mark_bad(CostStats& s, int sample, int component) {
    s = cost_combine(s, CostStats{0.0, sample, component});
}

// ---------------------------------------------------------------------------
// Block-wide reductions with warp shuffles, then a deterministic last-block
// finish: every block stores its partial; the block that arrives last (atomic
// ticket) combines all partials in block order and folds them into *total.

__device__ inline CostStats warp_reduce(CostStats v) {
    for (int o = 16; o; o >>= 1) {
        CostStats w;
        w.value = __shfl_down_sync(0xffffffffu, v.value, o);
        w.bad_sample = __shfl_down_sync(0xffffffffu, v.bad_sample, o);
        w.bad_component = __shfl_down_sync(0xffffffffu, v.bad_component, o);
        v = cost_combine(v, w);
    }
    return v;
}
__device__ inline GradStats warp_reduce(GradStats v) {
    for (int o = 16; o; o >>= 1) {
        GradStats w;
        w.squared_norm = __shfl_down_sync(0xffffffffu, v.squared_norm, o);
        w.max_abs = __shfl_down_sync(0xffffffffu, v.max_abs, o);
        w.nonfinite = __shfl_down_sync(0xffffffffu, v.nonfinite, o);
        w.first_nonfinite = __shfl_down_sync(0xffffffffu, v.first_nonfinite, o);
        v = grad_combine(v, w);
    }
    return v;
}

template <class T, class Empty>
__device__ T block_reduce(T v, Empty empty) {
    __shared__ T lanes[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_reduce(v);
    if (lane == 0) lanes[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (int)(blockDim.x >> 5) ? lanes[lane] : empty();
        v = warp_reduce(v);
    }
    __syncthreads();
    return v;
}

// Folds this block's value into *total once all blocks have arrived.
// Loads that bypass L1: partials are written by other SMs during this launch.
__device__ inline CostStats load_cg(const CostStats* p) {
    return {__ldcg(&p->value), __ldcg(&p->bad_sample), __ldcg(&p->bad_component)};
}
__device__ inline GradStats load_cg(const GradStats* p) {
    return {__ldcg(&p->squared_norm), __ldcg(&p->max_abs), __ldcg(&p->nonfinite), __ldcg(&p->first_nonfinite), 0};
}

template <class T, class Combine, class Empty>
__device__ void finish_blocks(T mine, T* partials, unsigned* ticket, T* total, Combine combine, Empty empty) {
    __shared__ bool last;
    if (threadIdx.x == 0) {
        partials[blockIdx.x] = mine;
        __threadfence();
        unsigned arrived = atomicAdd(ticket, 1u);
        last = arrived == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // the last block folds the partials with all its threads (fixed order)
    T acc = empty();
    for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) acc = combine(acc, load_cg(partials + b));
    acc = block_reduce(acc, empty);
    if (threadIdx.x == 0) {
        *total = combine(*total, acc);
        *ticket = 0;
    }
}

static __global__ void k_clear_costs(CostStats* totals, int count) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += blockDim.x * gridDim.x)
        totals[i] = cost_empty();
}

// ---------------------------------------------------------------------------
// Activation jets: value and derivative at the value row.

struct Sigmoid {
    static constexpr int id = 0;
    // y = sigma(z), s = sigma'(z) evaluated without cancellation on both tails.
    __device__ static void value(float z, float& y, float& s) {
        float e = __expf(-fabsf(z));
        float big = 1.0f / (1.0f + e);  // sigma(|z|) >= 1/2
        float small = e * big;          // 1 - sigma(|z|)
        y = z >= 0.f ? big : small;
        s = big * small;
    }
    __device__ static float slope_from_value(float y) { return y * (1.0f - y); }
    __device__ static float lead(float y) { return 1.0f - 2.0f * y; }
};

struct Tanh {
    static constexpr int id = 1;
    __device__ static void value(float z, float& y, float& s) {
        y = tanhf(z);
        s = (1.0f - y) * (1.0f + y);
    }
    __device__ static float slope_from_value(float y) { return (1.0f - y) * (1.0f + y); }
    __device__ static float lead(float y) { return -2.0f * y; }
};

// ---------------------------------------------------------------------------
// Copy-in: inputs of one chunk from the data record's (row, sample, channel)
// layout into the interleaved layer-0 layout.

static __global__ void k_stage_input(const float* __restrict__ data, int channels, int data_samples,
                              const int* __restrict__ rows, int R, int offset, int points,
                              float* __restrict__ out) {
    long total = (long)points * R * channels;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)blockDim.x * gridDim.x) {
        int c = int(e % channels);
        long col = e / channels;
        int r = int(col % R);
        long p = col / R;
        out[e] = data[((long)rows[r] * data_samples + offset + p) * channels + c];
    }
}

// Copy-out of evaluation outputs into the (row, sample, output) layout.
static __global__ void k_scatter_output(const float* __restrict__ z, int outputs, int R, const int* __restrict__ rows,
                                 int offset, int points, int data_samples, float* __restrict__ out) {
    long total = (long)points * R * outputs;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)blockDim.x * gridDim.x) {
        int o = int(e % outputs);
        long col = e / outputs;
        int r = int(col % R);
        long p = col / R;
        out[((long)rows[r] * data_samples + offset + p) * outputs + o] = z[e];
    }
}

// ---------------------------------------------------------------------------
// Generic FP32 GEMM, column-major: C = op(A) * op(B) (+ bias / split-K).
// 128 x 128 tile, 8-deep K slab, 256 threads, 8 x 8 outputs per thread (two
// 4-row by two 4-column blocks: thread (tx, ty) = (t % 16, t / 16) owns rows
// tx 4 + {0..3} and 64 + tx 4 + {0..3}, columns ty 4 + {0..3} and
// 64 + ty 4 + {0..3}), so its A and B fragments are float4 reads of shared
// memory and its stores of four consecutive rows are one float4 where the
// leading dimension allows. The next slab is loaded into registers while the
// current one is multiplied (double-buffered shared memory, one barrier per
// slab). The 64 x 64 tile with 4 x 4 outputs it replaced ran this tier's GEMMs
// at about a tenth of the FP32 rate.
//  * BIAS_ROWS: add bias[m] to columns with n % R == 0 (the value row).
//  * INDICATOR: op(B) has one extra virtual column N-1 equal to 1 where
//    k % R == 0, so the last output column is the bias gradient; it is summed
//    from the A slabs in shared memory by the CTAs of the first column tile,
//    and the grid covers only the N-1 real columns.
//  * split-K (gridDim.z > 1): each z-slice writes its own dense M x N partial.

namespace gemm {
constexpr int BM = 128, BN = 128, BK = 8, THREADS = 256, PAD = 4;
// column tiles of a launch with N output columns
inline int column_tiles(int N, bool indicator) { return ((indicator ? N - 1 : N) + BN - 1) / BN; }
}

template <bool TA, bool TB, bool BIAS_ROWS, bool INDICATOR>
__global__ void __launch_bounds__(gemm::THREADS)
k_gemm(int M, int N, int K, const float* __restrict__ A, int lda, const float* __restrict__ B, int ldb,
       float* __restrict__ C, int ldc, const float* __restrict__ bias, int R, int k_per_split) {
    using namespace gemm;
    __shared__ __align__(16) float As[2][BK][BM + PAD];
    __shared__ __align__(16) float Bs[2][BK][BN + PAD];
    const int t = threadIdx.x, tx = t % 16, ty = t / 16;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;  // N tiles on x: no 65535 limit
    const long k_begin = (long)blockIdx.z * k_per_split;
    const long k_end = min((long)K, k_begin + k_per_split);
    const int nreal = INDICATOR ? N - 1 : N;
    // element e = t + THREADS u (u < 4) of a slab: (row or column index, k index)
    auto a_index = [&](int e, int& mm, int& kk) {
        if (TA) { kk = e % BK; mm = e / BK; } else { mm = e % BM; kk = e / BM; }
    };
    auto b_index = [&](int e, int& nn, int& kk) {
        if (TB) { nn = e % BN; kk = e / BN; } else { kk = e % BK; nn = e / BK; }
    };
    float ra[4], rb[4];
    auto load = [&](long k0) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            int mm, kk;
            a_index(t + THREADS * u, mm, kk);
            const long k = k0 + kk;
            const int m = m0 + mm;
            ra[u] = m < M && k < k_end ? (TA ? A[k + (long)m * lda] : A[m + k * (long)lda]) : 0.f;
            int nn;
            b_index(t + THREADS * u, nn, kk);
            const long kb = k0 + kk;
            const int n = n0 + nn;
            rb[u] = n < nreal && kb < k_end ? (TB ? B[n + kb * (long)ldb] : B[kb + (long)n * ldb]) : 0.f;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            int mm, kk;
            a_index(t + THREADS * u, mm, kk);
            As[buf][kk][mm] = ra[u];
            int nn;
            b_index(t + THREADS * u, nn, kk);
            Bs[buf][kk][nn] = rb[u];
        }
    };
    float acc[8][8] = {};
    float bias_acc[8] = {};  // INDICATOR: the bias column of the thread's rows (ty == 0, first column tile)
    const bool bias_thread = INDICATOR && blockIdx.x == 0 && ty == 0;
    int buf = 0;
    if (k_begin < k_end) {
        load(k_begin);
        store(0);
    }
    __syncthreads();
    for (long k0 = k_begin; k0 < k_end; k0 += BK) {
        const bool more = k0 + BK < k_end;
        if (more) load(k0 + BK);  // in flight during the slab's FMAs
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][tx * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + tx * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][ty * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + ty * 4]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (bias_thread) {
            // the value-row columns k of this slab (k % R == 0), in k order
            for (int kk = int((R - k0 % R) % R); kk < BK && k0 + kk < k_end; kk += R) {
#pragma unroll
                for (int i = 0; i < 8; ++i) bias_acc[i] += As[buf][kk][(i < 4 ? tx * 4 : 64 + tx * 4) + (i & 3)];
            }
        }
        if (more) store(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
    float* out = C + (size_t)blockIdx.z * (gridDim.z > 1 ? (size_t)M * N : 0);
    const int ld = gridDim.z > 1 ? M : ldc;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int n = n0 + (j < 4 ? ty * 4 : 64 + ty * 4) + (j & 3);
        if (n >= nreal) continue;
        const bool value_row = BIAS_ROWS && (n % R) == 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = m0 + (h == 0 ? tx * 4 : 64 + tx * 4);
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = acc[4 * h + i][j] + (value_row && m + i < M ? bias[m + i] : 0.f);
            float* dst = out + m + (size_t)n * ld;
            if (m + 3 < M && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (m + i < M) dst[i] = v[i];
            }
        }
    }
    if (bias_thread) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int m = m0 + (i < 4 ? tx * 4 : 64 + tx * 4) + (i & 3);
            if (m < M) out[m + (size_t)(N - 1) * ld] = bias_acc[i];
        }
    }
}

// out[m + n*ldc] (+)= sum_z partial[z][m + n*M], summed in z order (deterministic).
static __global__ void k_splitk_reduce(const float* __restrict__ partial, int splits, int M, int N, float* __restrict__ out,
                                int ldc, int accumulate) {
    long total = (long)M * N;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)blockDim.x * gridDim.x) {
        float acc = 0.f;
        for (int z = 0; z < splits; ++z) acc += partial[(size_t)z * total + e];
        int m = int(e % M);
        long n = e / M;
        float* dst = out + m + n * ldc;
        *dst = accumulate ? *dst + acc : acc;
    }
}

// ---------------------------------------------------------------------------
// Table-driven jets (any schema). Thread per (neuron, point); the rows of that
// element are strided by n in the interleaved layout, so a warp's accesses
// for one row are contiguous. ``tab`` is JetPlan::pack().

__device__ inline float tcoef(const int* t, int i) { return __int_as_float(t[i]); }

template <class Act>
__global__ void k_jet_forward_dyn(const float* __restrict__ Z, float* __restrict__ Y, float* __restrict__ S, int n,
                                  long points, int R, const int* __restrict__ tab) {
    const int* fwd = tab;
    const int* sq = tab + (R + 1);
    long total = (long)n * points;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)blockDim.x * gridDim.x) {
        int m = int(e % n);
        long p = e / n;
        size_t base = (size_t)p * R * n + m;
        float y0, s0;
        Act::value(Z[base], y0, s0);
        Y[base] = y0;
        S[base] = s0;
        float lead = Act::lead(y0);
        for (int r = 1; r < R; ++r) {
            float acc = 0.f;
            for (int t = fwd[r]; t < fwd[r + 1]; t += 3)
                acc = fmaf(tcoef(tab, t) * S[base + (size_t)tab[t + 1] * n], Z[base + (size_t)tab[t + 2] * n], acc);
            Y[base + (size_t)r * n] = acc;
            float sacc = lead * acc;
            for (int t = sq[r]; t < sq[r + 1]; t += 3)
                sacc = fmaf(-tcoef(tab, t) * Y[base + (size_t)tab[t + 1] * n], Y[base + (size_t)tab[t + 2] * n], sacc);
            S[base + (size_t)r * n] = sacc;
        }
    }
}

template <class Act>
__global__ void k_jet_adjoint_dyn(const float* __restrict__ dY, const float* __restrict__ Y, float* __restrict__ S,
                                  float* __restrict__ dZ, int n, long points, int R, const int* __restrict__ tab) {
    const int* sq = tab + (R + 1);
    const int* adj = tab + 2 * (R + 1);
    long total = (long)n * points;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)blockDim.x * gridDim.x) {
        int m = int(e % n);
        long p = e / n;
        size_t base = (size_t)p * R * n + m;
        float y0 = Y[base];
        S[base] = Act::slope_from_value(y0);
        float lead = Act::lead(y0);
        for (int r = 1; r < R; ++r) {
            float sacc = lead * Y[base + (size_t)r * n];
            for (int t = sq[r]; t < sq[r + 1]; t += 3)
                sacc = fmaf(-tcoef(tab, t) * Y[base + (size_t)tab[t + 1] * n], Y[base + (size_t)tab[t + 2] * n], sacc);
            S[base + (size_t)r * n] = sacc;
        }
        for (int r = 0; r < R; ++r) {
            float acc = 0.f;
            for (int t = adj[r]; t < adj[r + 1]; t += 3)
                acc = fmaf(tcoef(tab, t) * S[base + (size_t)tab[t + 1] * n], dY[base + (size_t)tab[t + 2] * n], acc);
            dZ[base + (size_t)r * n] = acc;
        }
    }
}

// Staged variants for schemas of at most kJetStagedRows rows: each thread
// keeps its element's rows of every jet it works on in its own column of
// shared memory ([jet][row][thread]: consecutive threads, consecutive banks),
// so the terms read shared memory instead of going back to the global arrays,
// and the derivative jet s never leaves the SM. Three jets of 32 rows for 128
// threads are 48 KB, the default shared-memory limit.
constexpr int kJetStagedRows = 32, kJetStagedThreads = 128;
inline size_t jet_staged_smem(int R) { return size_t(3) * R * kJetStagedThreads * sizeof(float); }

template <class Act>
__global__ void __launch_bounds__(kJetStagedThreads)
k_jet_forward_staged(const float* __restrict__ Z, float* __restrict__ Y, int n, long points, int R,
                     const int* __restrict__ tab) {
    extern __shared__ float jet_stage[];
    const int T = blockDim.x;
    float* zs = jet_stage + threadIdx.x;  // row r of the thread's element at [r T]
    float* ys = zs + R * T;
    float* ss = ys + R * T;
    const int* fwd = tab;
    const int* sq = tab + (R + 1);
    const long total = (long)n * points;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)blockDim.x * gridDim.x) {
        const int m = int(e % n);
        const long p = e / n;
        const size_t base = (size_t)p * R * n + m;
        for (int r = 0; r < R; ++r) zs[r * T] = Z[base + (size_t)r * n];
        float y0, s0;
        Act::value(zs[0], y0, s0);
        ys[0] = y0;
        ss[0] = s0;
        Y[base] = y0;
        const float lead = Act::lead(y0);
        for (int r = 1; r < R; ++r) {
            float acc = 0.f;
            for (int t = fwd[r]; t < fwd[r + 1]; t += 3)
                acc = fmaf(tcoef(tab, t) * ss[tab[t + 1] * T], zs[tab[t + 2] * T], acc);
            ys[r * T] = acc;
            Y[base + (size_t)r * n] = acc;
            float sacc = lead * acc;
            for (int t = sq[r]; t < sq[r + 1]; t += 3)
                sacc = fmaf(-tcoef(tab, t) * ys[tab[t + 1] * T], ys[tab[t + 2] * T], sacc);
            ss[r * T] = sacc;
        }
    }
}

template <class Act>
__global__ void __launch_bounds__(kJetStagedThreads)
k_jet_adjoint_staged(const float* __restrict__ dY, const float* __restrict__ Y, float* __restrict__ dZ, int n,
                     long points, int R, const int* __restrict__ tab) {
    extern __shared__ float jet_stage[];
    const int T = blockDim.x;
    float* ys = jet_stage + threadIdx.x;
    float* gs = ys + R * T;
    float* ss = gs + R * T;
    const int* sq = tab + (R + 1);
    const int* adj = tab + 2 * (R + 1);
    const long total = (long)n * points;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)blockDim.x * gridDim.x) {
        const int m = int(e % n);
        const long p = e / n;
        const size_t base = (size_t)p * R * n + m;
        for (int r = 0; r < R; ++r) {
            ys[r * T] = Y[base + (size_t)r * n];
            gs[r * T] = dY[base + (size_t)r * n];
        }
        const float y0 = ys[0];
        ss[0] = Act::slope_from_value(y0);
        const float lead = Act::lead(y0);
        for (int r = 1; r < R; ++r) {
            float sacc = lead * ys[r * T];
            for (int t = sq[r]; t < sq[r + 1]; t += 3)
                sacc = fmaf(-tcoef(tab, t) * ys[tab[t + 1] * T], ys[tab[t + 2] * T], sacc);
            ss[r * T] = sacc;
        }
        for (int r = 0; r < R; ++r) {
            float acc = 0.f;
            for (int t = adj[r]; t < adj[r + 1]; t += 3)
                acc = fmaf(tcoef(tab, t) * ss[tab[t + 1] * T], gs[tab[t + 2] * T], acc);
            dZ[base + (size_t)r * n] = acc;
        }
    }
}

// ---------------------------------------------------------------------------
// Costs. One thread per point of the chunk; every output component of the
// point is handled by that thread, so equations that share components add
// into dE/dY without atomics (same contract as cuda/cost_kernels.cuh:4-5).

struct CostReduce {
    CostStats* partials;
    unsigned* ticket;
    CostStats* total;
};

__device__ inline void cost_finish(CostStats local, const CostReduce& red) {
    CostStats b = block_reduce(local, cost_empty);
    finish_blocks(b, red.partials, red.ticket, red.total, cost_combine, cost_empty);
}

// Squared-error matching: sum over rows d and outputs o of w*(y-t)^2, with
// dE/dy = 2w(y-t) (cuda/cost_kernels.cuh:6-35 semantics). ``y``/``g`` use the
// interleaved layout with n = outputs.
static __global__ void k_cost_matching(const float* __restrict__ y, float* __restrict__ g, const float* __restrict__ target,
                                int target_samples, const int* __restrict__ target_rows,
                                const float* __restrict__ weights, int weight_samples, int outputs, int R, int points,
                                int offset, int collect, int gradient, CostReduce red) {
    CostStats local = cost_empty();
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < points; p += blockDim.x * gridDim.x) {
        float value = 0.f;
        const int wp = weight_samples == 1 ? 0 : offset + p;
        for (int d = 0; d < R; ++d)
            for (int o = 0; o < outputs; ++o) {
                size_t i = ((size_t)p * R + d) * outputs + o;
                float w = weights[((size_t)d * weight_samples + wp) * outputs + o];
                float grad = 0.f;
                if (w != 0.f) {
                    float r = y[i] - target[((size_t)target_rows[d] * target_samples + offset + p) * outputs + o];
                    value += w * r * r;
                    grad = 2.0f * w * r;
                }
                if (gradient) g[i] = grad;
            }
        if (!isfinite(value)) mark_bad(local, offset + p, -1);
        if (collect) local.value += double(value);
        if (gradient)
            for (int d = 0; d < R; ++d)
                for (int o = 0; o < outputs; ++o)
                    if (!isfinite(g[((size_t)p * R + d) * outputs + o])) mark_bad(local, offset + p, d * outputs + o);
    }
    cost_finish(local, red);
}

struct PolyTerm {
    int equation, a, b;  // b = -1: linear term
};

__device__ inline float component(const float* y, int index, int outputs, int R, int p) {
    return y[((size_t)p * R + index / outputs) * outputs + index % outputs];
}

// Polynomial residuals r_e = sum_t c_t y_a (y_b or 1) - rhs_e, loss w r^2
// (cuda/cost_kernels.cuh:37-90 semantics).
static __global__ void k_cost_polynomial(const float* __restrict__ y, float* __restrict__ g, const PolyTerm* __restrict__ terms,
                                  const float* __restrict__ coefficients, int term_count, const float* __restrict__ rhs,
                                  const float* __restrict__ weights, int outputs, int R, int equations, int samples,
                                  int points, int offset, int collect, int gradient, CostReduce red) {
    CostStats local = cost_empty();
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < points; p += blockDim.x * gridDim.x) {
        if (gradient)
            for (int i = 0; i < R * outputs; ++i) g[(size_t)p * R * outputs + i] = 0.f;
        float total = 0.f;
        const int sample = offset + p;
        for (int e = 0; e < equations; ++e) {
            float w = weights[(size_t)e * samples + sample];
            if (w == 0.f) continue;
            float r = -rhs[(size_t)e * samples + sample];
            for (int t = 0; t < term_count; ++t) {
                if (terms[t].equation != e) continue;
                float c = coefficients[(size_t)t * samples + sample];
                if (c == 0.f) continue;
                float a = component(y, terms[t].a, outputs, R, p);
                r += c * a * (terms[t].b < 0 ? 1.0f : component(y, terms[t].b, outputs, R, p));
            }
            total += w * r * r;
            float scale = 2.0f * w * r;
            if (!gradient) continue;
            for (int t = 0; t < term_count; ++t) {
                if (terms[t].equation != e) continue;
                float c = coefficients[(size_t)t * samples + sample];
                if (c == 0.f) continue;
                int ia = terms[t].a, ib = terms[t].b;
                size_t ga = ((size_t)p * R + ia / outputs) * outputs + ia % outputs;
                if (ib < 0) {
                    g[ga] += scale * c;
                } else {
                    size_t gb = ((size_t)p * R + ib / outputs) * outputs + ib % outputs;
                    g[ga] += scale * c * component(y, ib, outputs, R, p);
                    g[gb] += scale * c * component(y, ia, outputs, R, p);
                }
            }
        }
        if (!isfinite(total)) mark_bad(local, sample, -1);
        if (collect) local.value += double(total);
        if (gradient)
            for (int i = 0; i < R * outputs; ++i)
                if (!isfinite(g[(size_t)p * R * outputs + i])) mark_bad(local, sample, i);
    }
    cost_finish(local, red);
}

// dE/dy *= multiplier (graph leaf multiplier), zero when the multiplier is 0
// (cuda/cost_graph.cuh:29-34).
static __global__ void k_scale(float* __restrict__ g, long count, const double* __restrict__ multiplier) {
    double m = *multiplier;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < count; i += (long)blockDim.x * gridDim.x)
        g[i] = m == 0 ? 0.f : float(g[i] * m);
}

// ---------------------------------------------------------------------------
// Gradient inspection: per layer L2^2, max |g|, non-finite count and first
// index (cuda/reduction_kernels.cuh:81-98 semantics). blockIdx.y = layer.

struct GradReduce {
    GradStats* partials;  // [layers][gridDim.x]
    unsigned* tickets;    // [layers]
    GradStats* totals;    // [layers]
};

static __global__ void k_inspect_gradients(const float* const* __restrict__ grads, const int* __restrict__ counts,
                                    GradReduce red) {
    const int layer = blockIdx.y;
    const float* g = grads[layer];
    const int count = counts[layer];
    GradStats local = grad_empty();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += blockDim.x * gridDim.x) {
        double v = g[i];
        if (!isfinite(v)) {
            ++local.nonfinite;
            if (i < local.first_nonfinite) local.first_nonfinite = i;
        } else {
            local.squared_norm += v * v;
            double a = fabs(v);
            if (a > local.max_abs) local.max_abs = a;
        }
    }
    GradStats b = block_reduce(local, grad_empty);
    finish_blocks(b, red.partials + (size_t)layer * gridDim.x, red.tickets + layer, red.totals + layer, grad_combine,
                  grad_empty);
}

// ---------------------------------------------------------------------------
// Optimizers over every layer. Banks hold the flat parameters of all layers:
// 0 weights, 1/2 gradient history, 3 RPROP steps or Adam first moment; an
// OptLayer gives a layer's offset, size and current-gradient bank.

struct OptLayer {
    long offset;
    int count;
    int active;  // 1 or 2: bank holding the current gradient
};

// RPROP (cuda/derivative_kernels_v4.cu:752-778): grow x1.2 on agreeing signs,
// roll back and halve on a sign change, |W| <= 20 guard restarting at 0.1.
// One RPROP element: current gradient cur[i], previous prev[i], step D[i],
// weight W[i].
__device__ __forceinline__ void rprop_element(float* cur, const float* prev, float* D, float* W, int i) {
    float a = cur[i], b = prev[i], d = D[i], wi = W[i];
    if (a * b > 0) d *= 1.2f;
    float nw = wi - copysignf(d, a);
    if (a * b < 0) {
        wi += copysignf(d, b);
        d *= 0.5f;
        cur[i] = 0.0f;
    } else if (a != 0.0f) {
        if (fabsf(nw) <= 20.0f) wi = nw;
        else {
            d = 0.1f;
            cur[i] = 0.0f;
        }
    }
    W[i] = wi;
    D[i] = d;
}

// One Adam element (cuda/derivative_kernels_v4.cu:780-799), including the
// reference's double-precision denominator from the 1e-8 literal.
struct AdamStep {
    float alpha, beta1, beta2, beta1t, beta2t;
};
__device__ __forceinline__ void adam_element(const float* grad, float* V, float* M, float* W, int i, AdamStep s) {
    float g = grad[i];
    float m = __fadd_rn(__fmul_rn(s.beta1, M[i]), __fmul_rn(1 - s.beta1, g));
    float v = __fadd_rn(__fmul_rn(s.beta2, V[i]), __fmul_rn(__fmul_rn(1 - s.beta2, g), g));
    M[i] = m;
    V[i] = v;
    float mh = __fdiv_rn(m, 1 - s.beta1t);
    float vh = __fdiv_rn(v, 1 - s.beta2t);
    double step = double(__fmul_rn(s.alpha, mh)) / (double(sqrtf(vh)) + 1e-8);
    float nw = float(double(W[i]) - step);
    if (fabsf(nw) <= 20.0f) W[i] = nw;
}

// The training update with its gradient diagnostics in one launch (one block
// of 1024 threads): each layer's statistics (squared L2 norm, max |g|,
// non-finite count and first index; cuda/reduction_kernels.cuh:81-98) into
// totals[layer], then the gate the host applies before an update (every
// gradient finite, every cost total finite with no bad sample, no bad graph
// node), then the RPROP or Adam update of every layer only if the gate
// passes. *applied records the decision for the host, which validates the
// downloaded statistics with the same rules and reports the reference's
// messages when the gate failed. method: 0 RPROP, 1 Adam.
static __global__ void __launch_bounds__(1024) k_inspect_update(float* __restrict__ w, float* __restrict__ bank1,
                                                                float* __restrict__ bank2, float* __restrict__ bank3,
                                                                const OptLayer* __restrict__ layers, int count,
                                                                GradStats* __restrict__ totals,
                                                                const CostStats* __restrict__ costs, int cost_count,
                                                                const int* __restrict__ graph_bad, int method,
                                                                AdamStep adam, int* __restrict__ applied) {
    __shared__ int gate;
    if (threadIdx.x == 0) gate = 1;
    __syncthreads();
    for (int l = 0; l < count; ++l) {
        const OptLayer L = layers[l];
        const float* g = (L.active == 1 ? bank1 : bank2) + L.offset;
        GradStats local = grad_empty();
        for (int i = threadIdx.x; i < L.count; i += blockDim.x) {
            double v = g[i];
            if (!isfinite(v)) {
                ++local.nonfinite;
                if (i < local.first_nonfinite) local.first_nonfinite = i;
            } else {
                local.squared_norm += v * v;
                double a = fabs(v);
                if (a > local.max_abs) local.max_abs = a;
            }
        }
        GradStats b = block_reduce(local, grad_empty);
        if (threadIdx.x == 0) {
            totals[l] = b;
            if (b.nonfinite) gate = 0;
        }
    }
    if (threadIdx.x == 0) {
        for (int c = 0; c < cost_count; ++c)
            if (costs[c].bad_sample != INT_MAX || !isfinite(costs[c].value)) gate = 0;
        if (graph_bad && *graph_bad >= 0) gate = 0;
        *applied = gate;
    }
    __syncthreads();
    if (!gate) return;
    for (int l = 0; l < count; ++l) {
        const OptLayer L = layers[l];
        float* cur = (L.active == 1 ? bank1 : bank2) + L.offset;
        float* other = (L.active == 1 ? bank2 : bank1) + L.offset;
        for (int i = threadIdx.x; i < L.count; i += blockDim.x) {
            if (method == 0) rprop_element(cur, other, bank3 + L.offset, w + L.offset, i);
            else adam_element(cur, other, bank3 + L.offset, w + L.offset, i, adam);
        }
    }
}

// Steps below the floor are raised to it and that entry's history cleared
// (cuda/derivative_kernels_v4.cu:801-814).
static __global__ void k_rprop_floor(float* __restrict__ bank1, float* __restrict__ bank2, float* __restrict__ steps,
                              const OptLayer* __restrict__ layers, float floor_value) {
    const OptLayer L = layers[blockIdx.y];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < L.count; i += blockDim.x * gridDim.x) {
        long j = L.offset + i;
        if (steps[j] < floor_value) {
            steps[j] = floor_value;
            bank1[j] = 0.f;
            bank2[j] = 0.f;
        }
    }
}

static __global__ void k_fill(float* __restrict__ dst, long count, float value) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < count; i += (long)blockDim.x * gridDim.x)
        dst[i] = value;
}

}  // namespace cpde
