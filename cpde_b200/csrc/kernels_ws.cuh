// Warp-specialised tensor-core layers (tcgen05, 3xTF32) for hidden layers of
// up to 128 inputs: a persistent CTA per SM streams its column tiles through
// a ring of shared-memory stages while the tensor cores and the jet epilogue
// work on earlier tiles.
//
// Roles (14 warps):
//   warp 0 (one lane)  TMA producer: one 32-wide K slab of a tile per stage;
//   warp 1 (one lane)  MMA issuer; the warp also owns the tensor-memory block;
//   warps 2-5          split each landed slab into TF32 hi (in place) and lo;
//   warps 6-13         load the layer's weights (hi and lo) into tensor memory
//                      once (warps 6-9), then run the jet epilogue on each
//                      finished tile: warp w reads TMEM lanes 32 (w % 4) .. +31
//                      and takes every other point of the tile.
// Tensor memory (512 columns): weights hi [0, 128), weights lo [128, 256),
// two accumulators [256, 384) and [384, 512), so the epilogue of tile i
// overlaps the MMAs of tile i + 1. The weights are the A operand straight
// from tensor memory, which leaves all of shared memory to the slab ring.
//
// Every wait is bounded. A role that times out raises a shared abort flag;
// the other roles see it in their waits and leave their loops; the producer
// then waits (bounded) for its loads in flight, the MMA issuer for its MMAs,
// and the CTA releases its tensor memory and reports through `error`.
#pragma once
#include "kernels_tc.cuh"

namespace cpde {
namespace ws {

constexpr int kProducerWarp = 0, kMmaWarp = 1, kSplitWarp = 2, kEpilogueWarp = 6;
constexpr int kEpilogueGroups = 2;  // two warps per TMEM lane quarter, alternating points
constexpr int THREADS = (kEpilogueWarp + 4 * kEpilogueGroups) * 32;
constexpr int STAGES = 6;
constexpr int kMaxK = 128;  // weights resident in tensor memory
constexpr uint32_t kTmemColumns = 512, kAccColumn = 256;

template <int R>
struct Tiling {
    static constexpr int PTS = tcg::Tiling<R>::PTS;                // whole points per tile
    static constexpr int COLS = PTS * R;
    static constexpr int N = ((COLS + 15) / 16) * 16;              // MMA N: multiple of 16 for M = 128
    static constexpr int SLAB = ((N * 128 + 1023) / 1024) * 1024;  // one K slab: N rows of 128 bytes
    static constexpr int SMEM = 2 * STAGES * SLAB + 1024 + 256;
};

// A wait taken by every lane of a warp; the warp leaves together when any
// lane saw an abort.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    const bool ok = tc::mbar_wait_or_abort(bar, parity, tcg::kWaitCycles, abort);
    return __all_sync(0xffffffffu, ok);
}

struct Ring {
    float *hi, *lo;  // [STAGES][SLAB / 4]
    uint64_t *full, *split, *empty, *acc_full, *acc_empty, *a_ready, *drain;
    uint32_t* tmem_slot;
    volatile int* abort;
};

template <int SLAB>
__device__ __forceinline__ Ring carve_ring(uint8_t* raw) {
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    Ring r;
    r.hi = reinterpret_cast<float*>(base);
    r.lo = reinterpret_cast<float*>(base + STAGES * SLAB);
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + 2 * STAGES * SLAB);
    r.full = bars;
    r.split = bars + STAGES;
    r.empty = bars + 2 * STAGES;
    r.acc_full = bars + 3 * STAGES;
    r.acc_empty = r.acc_full + 2;
    r.a_ready = r.acc_empty + 2;
    r.drain = r.a_ready + 1;
    r.tmem_slot = reinterpret_cast<uint32_t*>(r.drain + 1);
    r.abort = reinterpret_cast<volatile int*>(r.tmem_slot + 1);
    return r;
}

__device__ __forceinline__ void ring_init(Ring& r) {
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(r.full + s, 1);
            tc::mbar_init(r.split + s, 4);
            tc::mbar_init(r.empty + s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            tc::mbar_init(r.acc_full + a, 1);
            tc::mbar_init(r.acc_empty + a, 4 * kEpilogueGroups);
        }
        tc::mbar_init(r.a_ready, 4);
        tc::mbar_init(r.drain, 1);
        *r.abort = 0;
        tc::fence_barrier_init();
    }
    if ((threadIdx.x >> 5) == kMmaWarp) {
        tc::tmem_alloc(r.tmem_slot, kTmemColumns);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
}

// Producer: the X slabs of every tile this CTA owns, in order. After the last
// issue (or an abort) it waits for the loads still in flight.
template <int SLAB>
__device__ __forceinline__ void produce(const Ring& r, const CUtensorMap* map, long tiles, int tile_columns, int N,
                                        int slabs) {
    uint32_t it = 0;
    for (long tile = blockIdx.x; tile < tiles && !*r.abort; tile += gridDim.x) {
        const int col0 = int(tile * tile_columns);
        for (int s = 0; s < slabs; ++s) {
            const int st = it % STAGES;
            if (!tc::mbar_wait_or_abort(r.empty + st, ((it / STAGES) & 1) ^ 1, tcg::kWaitCycles, r.abort)) break;
            tc::mbar_expect_tx(r.full + st, uint32_t(N) * 128);
            tc::tma_load_2d(r.hi + st * (SLAB / 4), map, r.full + st, s * 32, col0);
            ++it;
        }
    }
    for (uint32_t k = it > STAGES ? it - STAGES : 0; k < it; ++k)
        tc::mbar_wait(r.full + k % STAGES, (k / STAGES) & 1, tcg::kWaitCycles);
}

// Split warps: TF32 hi in place and lo beside it, for every slab in order.
template <int SLAB>
__device__ __forceinline__ void split_all(const Ring& r, long tiles, int N, int slabs) {
    const int tid = threadIdx.x - kSplitWarp * 32;  // 0..127
    uint32_t it = 0;
    for (long tile = blockIdx.x; tile < tiles; tile += gridDim.x)
        for (int s = 0; s < slabs; ++s, ++it) {
            const int st = it % STAGES;
            if (!warp_wait(r.full + st, (it / STAGES) & 1, r.abort)) return;
            float4* h4 = reinterpret_cast<float4*>(r.hi + st * (SLAB / 4));
            float4* l4 = reinterpret_cast<float4*>(r.lo + st * (SLAB / 4));
            for (int i = tid; i < N * 8; i += 128) {
                float4 v = h4[i], h, l;
                h.x = tc::tf32_round(v.x);
                h.y = tc::tf32_round(v.y);
                h.z = tc::tf32_round(v.z);
                h.w = tc::tf32_round(v.w);
                l.x = tc::tf32_round(v.x - h.x);
                l.y = tc::tf32_round(v.y - h.y);
                l.z = tc::tf32_round(v.z - h.z);
                l.w = tc::tf32_round(v.w - h.w);
                h4[i] = h;
                l4[i] = l;
            }
            tc::fence_proxy_async();
            __syncwarp();
            if ((threadIdx.x & 31) == 0) tc::mbar_arrive(r.split + st);
        }
}

// MMA issuer: per tile, lo*hi + hi*lo + hi*hi over the K slabs into one of the
// two accumulators; each slab's stage is released by a commit once its MMAs
// have read it.
template <int N, int SLAB>
__device__ __forceinline__ void issue_mmas(const Ring& r, uint32_t tmem, long tiles, int slabs) {
    constexpr uint32_t idesc = tc::idesc_tf32(128, N);
    bool ok = tc::mbar_wait_or_abort(r.a_ready, 0, tcg::kWaitCycles, r.abort);
    tc::tc_fence_after();
    uint32_t it = 0, local = 0;
    for (long tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++local) {
        const int a = local & 1;
        ok = tc::mbar_wait_or_abort(r.acc_empty + a, ((local >> 1) & 1) ^ 1, tcg::kWaitCycles, r.abort);
        tc::tc_fence_after();
        const uint32_t d = tmem + kAccColumn + a * 128;
        for (int s = 0; ok && s < slabs; ++s, ++it) {
            const int st = it % STAGES;
            ok = tc::mbar_wait_or_abort(r.split + st, (it / STAGES) & 1, tcg::kWaitCycles, r.abort);
            if (!ok) break;
            tc::tc_fence_after();
            const uint32_t bh = tc::smem_u32(r.hi + st * (SLAB / 4)), bl = tc::smem_u32(r.lo + st * (SLAB / 4));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint32_t ah = tmem + s * 32 + kk * 8, al = ah + 128;
                tc::mma_tf32_ts(d, al, tc::desc_k_sw128(bh + kk * 32), idesc, (s | kk) != 0);
                tc::mma_tf32_ts(d, ah, tc::desc_k_sw128(bl + kk * 32), idesc, 1);
                tc::mma_tf32_ts(d, ah, tc::desc_k_sw128(bh + kk * 32), idesc, 1);
            }
            tc::mma_commit(r.empty + st);
        }
        if (ok) tc::mma_commit(r.acc_full + a);
    }
    // every MMA issued so far has completed once this commit arrives
    tc::mma_commit(r.drain);
    tc::mbar_wait(r.drain, 0, tcg::kWaitCycles);
}

// Epilogue warps 6-9: this CTA's 128 weight rows (column-major W with leading
// dimension M) split into TF32 hi and lo, into tensor memory columns [0, K)
// and [128, 128 + K) of the thread's lane.
__device__ __forceinline__ void load_weights(const Ring& r, uint32_t tmem, const float* __restrict__ W, int M,
                                             int K, int m) {
    const int quarter = (threadIdx.x >> 5) & 3;
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    for (int c0 = 0; c0 < K; c0 += 8) {
        float h[8], l[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float v = __ldg(W + m + (size_t)(c0 + j) * M);
            h[j] = tc::tf32_round(v);
            l[j] = tc::tf32_round(v - h[j]);
        }
        tc::tmem_st8(lane_base + c0, h);
        tc::tmem_st8(lane_base + 128 + c0, l);
    }
    tc::tmem_wait_st();
    tc::tc_fence_before();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) tc::mbar_arrive(r.a_ready);
}

__device__ __forceinline__ void teardown(const Ring& r, uint32_t tmem, int* error) {
    tc::tc_fence_before();
    __syncthreads();
    if ((threadIdx.x >> 5) == kMmaWarp) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kTmemColumns);
    }
    if (threadIdx.x == 0 && *r.abort) atomicExch(error, tcg::kErrMma);
}

// Hidden layer forward: Y = f(W X + b) with the jet combine in the epilogue.
// grid = (CTAs over column tiles, M / 128); K a multiple of 32, at most 128.
template <int SID, class Act>
__global__ void __launch_bounds__(THREADS, 1) k_forward_ws(const __grid_constant__ CUtensorMap map_x, int M, int K,
                                                           long P, const float* __restrict__ W,
                                                           float* __restrict__ Y, int* error) {
    constexpr int R = StaticJet<SID>::R;
    using T = Tiling<R>;
    extern __shared__ uint8_t smem_raw[];
    Ring r = carve_ring<T::SLAB>(smem_raw);
    ring_init(r);
    const uint32_t tmem = *r.tmem_slot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long tiles = (P + T::PTS - 1) / T::PTS;
    const int slabs = K / 32;
    if (warp == kProducerWarp) {
        if (lane == 0) produce<T::SLAB>(r, &map_x, tiles, T::COLS, T::N, slabs);
    } else if (warp == kMmaWarp) {
        if (lane == 0) issue_mmas<T::N, T::SLAB>(r, tmem, tiles, slabs);
    } else if (warp < kEpilogueWarp) {
        split_all<T::SLAB>(r, tiles, T::N, slabs);
    } else {
        const int quarter = warp & 3, group = (warp - kEpilogueWarp) >> 2;
        const int m = blockIdx.y * 128 + quarter * 32 + lane;
        if (group == 0) load_weights(r, tmem, W, M, K, m);
        const float b0 = __ldg(W + (size_t)M * K + m);
        const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
        uint32_t local = 0;
        for (long tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            const int a = local & 1;
            if (!warp_wait(r.acc_full + a, (local >> 1) & 1, r.abort)) break;
            tc::tc_fence_after();
            const long p0 = tile * T::PTS;
            for (int p = group; p < T::PTS; p += kEpilogueGroups) {
                if (p0 + p >= P) break;
                float z[R], y[R];
                tc::tmem_read<R>(lane_base + kAccColumn + a * 128 + p * R, z);
                z[0] += b0;
                StaticJet<SID>::template forward<Act>(z, y);
                float* out = Y + ((size_t)(p0 + p) * R) * M + m;
#pragma unroll
                for (int q = 0; q < R; ++q) out[(size_t)q * M] = y[q];
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(r.acc_empty + a);
        }
    }
    teardown(r, tmem, error);
}

}  // namespace ws
}  // namespace cpde
