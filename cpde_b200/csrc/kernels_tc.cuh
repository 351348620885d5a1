// Tensor-core tier: hidden-layer GEMMs on tcgen05 with a 3xTF32 split.
//
// Operands reach shared memory by TMA (128-byte swizzle, K-major). The
// weights are split once per epoch into TF32 hi/lo arrays in global memory;
// activation slabs are split in shared memory after they land (the split is
// elementwise, so the swizzled layout is untouched). Each K-step issues
// lo*hi + hi*lo + hi*hi into one FP32 accumulator in tensor memory, which
// keeps products to about 2^-22 relative error. The accumulator rows are the
// layer's neurons, so each epilogue thread reads its neuron's R derivative
// columns of a point straight from tensor memory into the register jet code.
//
// Every mbarrier wait is bounded (kWaitCycles); on a timeout the CTA records
// an error code, all threads agree through __syncthreads_and, the tensor
// memory is released and the CTA returns. The host checks the code.
#pragma once
#include "generated/jets_static.cuh"
#include "kernels_fast.cuh"
#include "kernels_generic.cuh"
#include "tc.cuh"

namespace cpde {
namespace tcg {

constexpr int THREADS = 128;
constexpr int BM = 128;                       // neurons per tile = TMEM lanes
constexpr int KS = 32;                        // K per slab: 32 fp32 = one 128-byte row
constexpr long long kWaitCycles = 2000000000LL;  // about one second

// Tile = 128 neurons x PTS whole points (N <= kTileColumns MMA columns). The
// B regions are sized to N, so smaller tiles let more CTAs share an SM and
// overlap each other's load / split / MMA / epilogue phases.
constexpr int kTileColumns = 128;

template <int R>
struct Tiling {
    static constexpr int PTS = (kTileColumns / R) > 0 ? (kTileColumns / R) : 1;
    static constexpr int COLS = PTS * R;
    static constexpr int N = ((COLS + 7) / 8) * 8;
    static constexpr int TMEM = N <= 32 ? 32 : N <= 64 ? 64 : N <= 128 ? 128 : 256;
    static constexpr int A_BYTES = BM * KS * 4;                      // 16 KB
    static constexpr int B_BYTES = ((N * KS * 4 + 1023) / 1024) * 1024;  // 1024-aligned
    // smem: a_hi, a_lo, b, b_lo, then barriers; +1024 for alignment
    static constexpr int SMEM = 2 * A_BYTES + 2 * B_BYTES + 64 + 1024;
};

enum : int { kErrTma = 1, kErrMma = 2 };

__device__ __forceinline__ void split_slab(float* b, float* b_lo, int floats) {
    float4* hi4 = reinterpret_cast<float4*>(b);
    float4* lo4 = reinterpret_cast<float4*>(b_lo);
    for (int i = threadIdx.x; i < floats / 4; i += blockDim.x) {
        float4 v = hi4[i], h, l;
        h.x = tc::tf32_round(v.x);
        h.y = tc::tf32_round(v.y);
        h.z = tc::tf32_round(v.z);
        h.w = tc::tf32_round(v.w);
        l.x = tc::tf32_round(v.x - h.x);
        l.y = tc::tf32_round(v.y - h.y);
        l.z = tc::tf32_round(v.z - h.z);
        l.w = tc::tf32_round(v.w - h.w);
        hi4[i] = h;
        lo4[i] = l;
    }
}

// Z tile (128 neurons x N columns) = A (128 x K, K-major, pre-split hi/lo) *
// B (N columns of K, K-major; split here). Leaves the accumulator in TMEM.
// Returns false (all threads) when a wait timed out.
template <int N>
__device__ __forceinline__ bool mma_tile(const CUtensorMap* map_a_hi, const CUtensorMap* map_a_lo,
                                         const CUtensorMap* map_b, int a_row, int b_col, int K, float* a_hi,
                                         float* a_lo, float* b, float* b_lo, uint64_t* tma_bar, uint64_t* mma_bar,
                                         uint32_t tmem, uint32_t& phase, int* error) {
    constexpr uint32_t idesc = tc::idesc_tf32(BM, N);
    constexpr uint32_t bytes = 2 * BM * KS * 4 + N * KS * 4;
    const int slabs = K / KS;
    bool ok = true;
    for (int s = 0; s < slabs; ++s) {
        if (threadIdx.x == 0) {
            tc::mbar_expect_tx(tma_bar, bytes);
            tc::tma_load_2d(a_hi, map_a_hi, tma_bar, s * KS, a_row);
            tc::tma_load_2d(a_lo, map_a_lo, tma_bar, s * KS, a_row);
            tc::tma_load_2d(b, map_b, tma_bar, s * KS, b_col);
        }
        ok = __syncthreads_and(tc::mbar_wait(tma_bar, phase, kWaitCycles));
        if (!ok) {
            if (threadIdx.x == 0) atomicExch(error, kErrTma);
            return false;
        }
        split_slab(b, b_lo, N * KS);
        tc::fence_proxy_async();
        __syncthreads();
        tc::tc_fence_after();
        if (threadIdx.x == 0) {
            const uint32_t ah = tc::smem_u32(a_hi), al = tc::smem_u32(a_lo);
            const uint32_t bh = tc::smem_u32(b), bl = tc::smem_u32(b_lo);
#pragma unroll
            for (int kk = 0; kk < KS / 8; ++kk) {
                const uint32_t off = kk * 32;  // 8 TF32 values along the 128-byte row
                tc::mma_tf32(tmem, tc::desc_k_sw128(al + off), tc::desc_k_sw128(bh + off), idesc,
                             (s | kk) != 0);
                tc::mma_tf32(tmem, tc::desc_k_sw128(ah + off), tc::desc_k_sw128(bl + off), idesc, 1);
                tc::mma_tf32(tmem, tc::desc_k_sw128(ah + off), tc::desc_k_sw128(bh + off), idesc, 1);
            }
            tc::mma_commit(mma_bar);
        }
        ok = __syncthreads_and(tc::mbar_wait(mma_bar, phase, kWaitCycles));
        phase ^= 1;
        if (!ok) {
            if (threadIdx.x == 0) atomicExch(error, kErrMma);
            return false;
        }
    }
    tc::tc_fence_after();
    return true;
}

struct Shared {
    float *a_hi, *a_lo, *b, *b_lo;
    uint64_t *tma_bar, *mma_bar;
    uint32_t* tmem_slot;
};

__device__ __forceinline__ Shared carve(uint8_t* raw, int a_bytes, int b_bytes) {
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    Shared s;
    s.a_hi = reinterpret_cast<float*>(base);
    s.a_lo = reinterpret_cast<float*>(base + a_bytes);
    s.b = reinterpret_cast<float*>(base + 2 * a_bytes);
    s.b_lo = reinterpret_cast<float*>(base + 2 * a_bytes + b_bytes);
    s.tma_bar = reinterpret_cast<uint64_t*>(base + 2 * a_bytes + 2 * b_bytes);
    s.mma_bar = s.tma_bar + 1;
    s.tmem_slot = reinterpret_cast<uint32_t*>(s.tma_bar + 2);
    return s;
}

template <int COLS>
__device__ __forceinline__ void setup(Shared& s, uint32_t& tmem) {
    if (threadIdx.x == 0) {
        tc::mbar_init(s.tma_bar, 1);
        tc::mbar_init(s.mma_bar, 1);
        tc::fence_barrier_init();
    }
    if (threadIdx.x < 32) {
        tc::tmem_alloc(s.tmem_slot, COLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    tmem = *s.tmem_slot;
}

template <int COLS>
__device__ __forceinline__ void teardown(uint32_t tmem) {
    tc::tc_fence_before();
    __syncthreads();
    if (threadIdx.x < 32) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, COLS);
    }
}

// Hidden layer forward on tensor cores: Y = f(W X + b), jets in the epilogue.
// Persistent over point tiles: grid = (min(tiles, resident CTAs), M / 128).
template <int SID, class Act>
__global__ void __launch_bounds__(THREADS) k_forward_tc(const __grid_constant__ CUtensorMap map_w_hi,
                                                        const __grid_constant__ CUtensorMap map_w_lo,
                                                        const __grid_constant__ CUtensorMap map_x, int M, int K,
                                                        long P, const float* __restrict__ bias,
                                                        float* __restrict__ Y, int* error) {
    constexpr int R = StaticJet<SID>::R;
    using T = Tiling<R>;
    extern __shared__ uint8_t smem_raw[];
    Shared s = carve(smem_raw, T::A_BYTES, T::B_BYTES);
    uint32_t tmem;
    setup<T::TMEM>(s, tmem);
    const int m_base = blockIdx.y * BM;
    const int warp = threadIdx.x >> 5;
    const int m = m_base + threadIdx.x;
    const uint32_t lane_addr = tmem + (uint32_t(warp * 32) << 16);
    const float b0 = m < M ? __ldg(bias + m) : 0.f;
    uint32_t phase = 0;
    for (long tile = blockIdx.x; tile * T::PTS < P; tile += gridDim.x) {
        const long p0 = tile * T::PTS;
        if (!mma_tile<T::N>(&map_w_hi, &map_w_lo, &map_x, m_base, int(p0 * R), K, s.a_hi, s.a_lo, s.b, s.b_lo,
                            s.tma_bar, s.mma_bar, tmem, phase, error))
            break;
        for (int p = 0; p < T::PTS; ++p) {
            if (p0 + p >= P) break;
            float z[R], y[R];
            tc::tmem_read<R>(lane_addr + p * R, z);
            if (m < M) {
                z[0] += b0;
                StaticJet<SID>::template forward<Act>(z, y);
                float* out = Y + ((size_t)(p0 + p) * R) * M + m;
#pragma unroll
                for (int r = 0; r < R; ++r) out[(size_t)r * M] = y[r];
            }
        }
        tc::tc_fence_before();
    }
    teardown<T::TMEM>(tmem);
}

// Hidden layer backward on tensor cores: dY = W^T dZ (A = W as stored, which
// is K-major for W^T), jet adjoint with Y_prev in the epilogue. M = width of
// the previous layer, K = this layer's. With INPUT_GRAD the previous layer is
// the first hidden one: its weight-gradient partial (M x (K0+1), bias last) is
// accumulated per CTA into partials[blockIdx.x] and dZ_prev is not stored.
template <int SID, class Act, bool INPUT_GRAD>
__global__ void __launch_bounds__(THREADS) k_backward_tc(const __grid_constant__ CUtensorMap map_w_hi,
                                                         const __grid_constant__ CUtensorMap map_w_lo,
                                                         const __grid_constant__ CUtensorMap map_dz, int M, int K,
                                                         long P, const float* __restrict__ Yprev,
                                                         float* __restrict__ dZprev, const float* __restrict__ X0,
                                                         int K0, float* __restrict__ partials, int* error) {
    constexpr int R = StaticJet<SID>::R;
    using T = Tiling<R>;
    extern __shared__ uint8_t smem_raw[];
    Shared s = carve(smem_raw, T::A_BYTES, T::B_BYTES);
    uint32_t tmem;
    setup<T::TMEM>(s, tmem);
    const int m_base = blockIdx.y * BM;
    const int warp = threadIdx.x >> 5;
    const int m = m_base + threadIdx.x;
    const uint32_t lane_addr = tmem + (uint32_t(warp * 32) << 16);
    float gacc[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) gacc[k] = 0.f;
    uint32_t phase = 0;
    for (long tile = blockIdx.x; tile * T::PTS < P; tile += gridDim.x) {
        const long p0 = tile * T::PTS;
        if (!mma_tile<T::N>(&map_w_hi, &map_w_lo, &map_dz, m_base, int(p0 * R), K, s.a_hi, s.a_lo, s.b, s.b_lo,
                            s.tma_bar, s.mma_bar, tmem, phase, error))
            break;
        for (int p = 0; p < T::PTS; ++p) {
            if (p0 + p >= P) break;
            float g[R], y[R];
            tc::tmem_read<R>(lane_addr + p * R, g);
            if (m < M) {
                const float* yp = Yprev + ((size_t)(p0 + p) * R) * M + m;
#pragma unroll
                for (int r = 0; r < R; ++r) y[r] = yp[(size_t)r * M];
                StaticJet<SID>::template adjoint<Act>(y, g);
                if (INPUT_GRAD) {
                    fast::input_gradient<R>(g, X0 + (size_t)(p0 + p) * R * K0, K0, gacc);
                } else {
                    float* out = dZprev + ((size_t)(p0 + p) * R) * M + m;
#pragma unroll
                    for (int r = 0; r < R; ++r) out[(size_t)r * M] = g[r];
                }
            }
        }
        tc::tc_fence_before();
    }
    if (INPUT_GRAD && m < M) {
        float* out = partials + (size_t)blockIdx.x * M * (K0 + 1);
#pragma unroll
        for (int k = 0; k < 8; ++k)  // constant bound keeps gacc in registers
            if (k < K0) out[m + (size_t)k * M] = gacc[k];
        out[m + (size_t)K0 * M] = gacc[8];
    }
    teardown<T::TMEM>(tmem);
}

// hi/lo TF32 split of a weight matrix. transpose: dst[m*K + k] = src[m + k*M]
// (column-major M x K to K-major rows); otherwise elementwise.
static __global__ void k_split_tf32(const float* __restrict__ src, float* __restrict__ hi, float* __restrict__ lo, int M,
                             int K, int transpose) {
    const long total = (long)M * K;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)blockDim.x * gridDim.x) {
        float v;
        if (transpose) {
            const int m = int(i / K), k = int(i % K);
            v = src[m + (size_t)k * M];
        } else {
            v = src[i];
        }
        const float h = tc::tf32_round(v);
        hi[i] = h;
        lo[i] = tc::tf32_round(v - h);
    }
}

}  // namespace tcg
}  // namespace cpde
