// Warp-specialised tensor-core layers (tcgen05, 3xTF32) for hidden layers of
// up to 128 inputs: a persistent CTA per SM streams its column tiles through
// a ring of shared-memory stages while the tensor cores and the jet epilogue
// work on earlier tiles.
//
// Roles (15 warps):
//   warp 0 (one lane)  TMA producer: one 32-wide K slab of a tile per stage;
//   warps 1, 6 (lane 0) MMA issuers for the even and the odd tiles of the CTA
//                      (local tile index), each into its own accumulator;
//                      warp 1 also owns the tensor-memory block;
//   warps 2-5          write the TF32 lo part of each landed slab beside it
//                      (the raw slab is the hi part);
//   warps 7-14         load the layer's weights (hi and lo) into tensor memory
//                      once (warps 7-10), then run the jet epilogue on each
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

// Two MMA issuers take alternate tiles (each always into its own accumulator):
// one thread alone leaves the tensor pipe idle while it waits on a stage or an
// accumulator, and at these tile sizes that idle time was about a third of
// the layer.
constexpr int kProducerWarp = 0, kMmaWarp = 1, kSplitWarp = 2, kSecondMmaWarp = 6, kEpilogueWarp = 7;
constexpr int kMmaIssuers = 2;
constexpr int kEpilogueGroups = 2;  // two warps per TMEM lane quarter, alternating points
constexpr int THREADS = (kEpilogueWarp + 4 * kEpilogueGroups) * 32;
constexpr int STAGES = 6;
constexpr int kMaxK = 128;  // weights resident in tensor memory
constexpr uint32_t kTmemColumns = 512, kAccColumn = 256;
constexpr int kSmemLimit = 232448;  // dynamic shared memory of one CTA (227 KB)
constexpr int kStagingSlots = 3;    // backward: Y_prev staged two work items ahead

// XV: input-jet floats of one point (R x inputs) that the backward into the
// first hidden layer keeps per epilogue warp (0 elsewhere).
template <int R, int XV = 0>
struct Tiling {
    static constexpr int PTS = tcg::Tiling<R>::PTS;                // whole points per tile
    static constexpr int COLS = PTS * R;
    static constexpr int N = ((COLS + 15) / 16) * 16;              // MMA N: multiple of 16 for M = 128
    static constexpr int SLAB = ((N * 128 + 1023) / 1024) * 1024;  // one K slab: N rows of 128 bytes
    static constexpr int SMEM = 2 * STAGES * SLAB + 1024 + 256;
    // backward: kStagingSlots R-float staging slots per epilogue thread for
    // the previous layer's values, copied asynchronously kStagingSlots - 1 work
    // items ahead; the slab ring gives up stages where both do not fit
    static constexpr int YBUF = kStagingSlots * R * 4 * 32 * 4 * kEpilogueGroups;
    static constexpr int XROW = (XV + 3) / 4 * 4;                    // floats, 16-byte rows
    static constexpr int XBUF = 4 * kEpilogueGroups * XROW * 4;      // one row per epilogue warp
    static constexpr int BSTAGES = (kSmemLimit - 1024 - 256 - YBUF - XBUF) / (2 * SLAB) < STAGES
                                       ? (kSmemLimit - 1024 - 256 - YBUF - XBUF) / (2 * SLAB)
                                       : STAGES;
    static constexpr int BSMEM = 2 * BSTAGES * SLAB + 1024 + 256 + YBUF + XBUF;
    static_assert(BSTAGES >= 3, "slab ring too shallow beside the staging slots");
};

// A wait taken by every lane of a warp; the warp leaves together when any
// lane saw an abort.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    const bool ok = tc::mbar_wait_or_abort(bar, parity, tcg::kWaitCycles, abort);
    return __all_sync(0xffffffffu, ok);
}

struct Ring {
    float *hi, *lo;  // [stages][SLAB / 4]
    float* staging;   // after the barriers: backward staging slots
    uint64_t *full, *split, *empty, *acc_full, *acc_empty, *a_ready, *drain;  // drain: one per MMA issuer
    uint32_t* tmem_slot;
    volatile int* abort;
};

template <int SLAB, int S = STAGES>
__device__ __forceinline__ Ring carve_ring(uint8_t* raw) {
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    Ring r;
    r.hi = reinterpret_cast<float*>(base);
    r.lo = reinterpret_cast<float*>(base + S * SLAB);
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + 2 * S * SLAB);
    r.full = bars;
    r.split = bars + S;
    r.empty = bars + 2 * S;
    r.acc_full = bars + 3 * S;
    r.acc_empty = r.acc_full + 2;
    r.a_ready = r.acc_empty + 2;
    r.drain = r.a_ready + 1;
    r.tmem_slot = reinterpret_cast<uint32_t*>(r.drain + kMmaIssuers);
    r.abort = reinterpret_cast<volatile int*>(r.tmem_slot + 1);
    r.staging = reinterpret_cast<float*>(base + 2 * S * SLAB + 256);
    return r;
}

template <int S = STAGES>
__device__ __forceinline__ void ring_init(Ring& r) {
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(r.full + s, 1);
            tc::mbar_init(r.split + s, 4);
            tc::mbar_init(r.empty + s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            tc::mbar_init(r.acc_full + a, 1);
            tc::mbar_init(r.acc_empty + a, 4 * kEpilogueGroups);
        }
        tc::mbar_init(r.a_ready, 4);
        for (int i = 0; i < kMmaIssuers; ++i) tc::mbar_init(r.drain + i, 1);
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

// Producer: the X slabs of every work item this CTA owns, in order. A work
// item is one column tile, or with halves = 2 two adjacent tiles 2w, 2w + 1
// whose K slabs follow one another (the layers of at most 64 neurons and 64
// inputs, see PairedTiles); the second tile of the last pair may lie past the
// end, and its load then reads the fill value (zeros). After the last issue
// (or an abort) it waits for the loads still in flight.
template <int SLAB, int S = STAGES>
__device__ __forceinline__ void produce(const Ring& r, const CUtensorMap* map, long items, int tile_columns, int N,
                                        int kslabs, int halves = 1) {
    uint32_t it = 0;
    for (long w = blockIdx.x; w < items && !*r.abort; w += gridDim.x) {
        for (int s = 0; s < kslabs * halves; ++s) {
            const int half = s >= kslabs, ks = s - half * kslabs;
            const int col0 = int((w * halves + half) * tile_columns);
            const int st = it % S;
            if (!tc::mbar_wait_or_abort(r.empty + st, ((it / S) & 1) ^ 1, tcg::kWaitCycles, r.abort)) break;
            tc::mbar_expect_tx(r.full + st, uint32_t(N) * 128);
            tc::tma_load_2d(r.hi + st * (SLAB / 4), map, r.full + st, ks * 32, col0);
            ++it;
        }
    }
    // a load that never lands must not go unnoticed: the CTA then reports an error
    for (uint32_t k = it > S ? it - S : 0; k < it; ++k)
        if (!tc::mbar_wait(r.full + k % S, (k / S) & 1, tcg::kWaitCycles)) *r.abort = 1;
}

// lo parts of float4 elements [0, count) of x4 into l4, strided over `threads`
// threads, eight loads in flight per thread. The tensor core reads an fp32
// operand of a kind::tf32 MMA as its top 19 bits (sign, exponent, 10 mantissa
// bits), so the raw slab already is the hi part, hi = trunc(x), and
// lo = RN_tf32(x - trunc(x)) leaves x - hi - lo below 2^-21 |x|, the accuracy
// of a split that rounds both parts.
__device__ __forceinline__ void split_lo_range(const float4* x4, float4* l4, int count, int tid, int threads = 128) {
    constexpr int U = 8;
    auto lo = [](float x) { return tc::tf32_round(x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u)); };
    for (int base = 0; base < count; base += threads * U) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = base + tid + threads * u;
            v[u] = i < count ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = base + tid + threads * u;
            if (i >= count) break;
            l4[i] = make_float4(lo(v[u].x), lo(v[u].y), lo(v[u].z), lo(v[u].w));
        }
    }
}

// Split warps: the TF32 lo part of every slab, in order, beside the raw slab.
template <int SLAB, int S = STAGES>
__device__ __forceinline__ void split_all(const Ring& r, long tiles, int N, int slabs) {
    const int tid = threadIdx.x - kSplitWarp * 32;  // 0..127
    uint32_t it = 0;
    for (long tile = blockIdx.x; tile < tiles; tile += gridDim.x)
        for (int s = 0; s < slabs; ++s, ++it) {
            const int st = it % S;
            if (!warp_wait(r.full + st, (it / S) & 1, r.abort)) return;
            split_lo_range(reinterpret_cast<const float4*>(r.hi + st * (SLAB / 4)),
                           reinterpret_cast<float4*>(r.lo + st * (SLAB / 4)), N * 8, tid);
            tc::fence_proxy_async();
            __syncwarp();
            if ((threadIdx.x & 31) == 0) tc::mbar_arrive(r.split + st);
        }
}

// How many MMA issuers a ring of S stages supports for tiles of `slabs` K
// slabs. An issuer that skips the other issuer's tile waits on a stage's
// split barrier by phase parity; that is exact only if the stage's previous
// phase (slab it - S) is already complete when the wait starts, which the
// split warps' in-order progress guarantees when S > slabs (that slab then
// precedes everything this issuer consumed before). With fewer stages one
// issuer takes every tile, in ring order.
__host__ __device__ constexpr int mma_issuers(int S, int slabs) { return S > slabs ? kMmaIssuers : 1; }

// MMA issuer `which` of `issuers`: for the CTA's tiles of local index
// which, which + issuers, ..., lo*hi + hi*hi + hi*lo over the K slabs into
// accumulator (local tile index) & 1, once the split warps have written the
// slab's lo part (issuing the two terms of the raw slab before that wait
// measured slower); each slab's stage is released by a commit once its MMAs
// have read it. Slab counter `it` runs over all the CTA's slabs in ring
// order, the other issuer's included.
//
// Term order. The tensor core's FP32 accumulation truncates, so every MMA
// into an accumulator that already holds the large hi*hi sum costs up to an
// ulp of it, whatever it adds. With `group` = 0 each K step issues
// lo*hi, hi*lo, hi*hi in turn (3 K/8 such adds). With `group` = g > 0 the
// tile's slabs go in groups of g: first the two lo terms of all the group's
// slabs, then its hi*hi terms, and only then are its stages released, so in
// the first group the lo terms land on a small accumulator (K/8 adds at full
// size when one group covers the tile). lo_first_group() uses one group per
// tile (or per tile half: the slabs of the two halves of a paired work item
// touch disjoint accumulator lanes) for layers of at most 64 inputs, whose
// one or two slabs per group leave the rest of the ring to the loads ahead.
// Measured on 96 order-2/3 cost cases of 32- and 64-neuron networks: the
// worst gradient error against the float64 oracle went 5.1e-6 -> 1.1e-6, for
// about 8% more time in the paired forward (the stages are held longer).

// The term-order group of a layer with kslabs K slabs per tile (or tile half).
__device__ __forceinline__ int lo_first_group(int kslabs) { return kslabs <= 2 ? kslabs : 0; }

template <int N, int SLAB, int S = STAGES>
__device__ __forceinline__ void issue_mmas(const Ring& r, uint32_t tmem, long tiles, int slabs, int which,
                                           int group = 0) {
    constexpr uint32_t idesc = tc::idesc_tf32(128, N);
    const int issuers = mma_issuers(S, slabs);
    bool ok = tc::mbar_wait_or_abort(r.a_ready, 0, tcg::kWaitCycles, r.abort);
    tc::tc_fence_after();
    uint32_t it = which * slabs, local = which;
    for (long tile = blockIdx.x + which * gridDim.x; ok && which < issuers && tile < tiles;
         tile += issuers * gridDim.x, local += issuers, it += (issuers - 1) * slabs) {
        const int a = local & 1;
        ok = tc::mbar_wait_or_abort(r.acc_empty + a, ((local >> 1) & 1) ^ 1, tcg::kWaitCycles, r.abort);
        tc::tc_fence_after();
        const uint32_t d = tmem + kAccColumn + a * 128;
        const uint32_t first = it;
        if (group == 0) {
            for (int s = 0; ok && s < slabs; ++s) {
                const int st = (first + s) % S;
                ok = tc::mbar_wait_or_abort(r.split + st, ((first + s) / S) & 1, tcg::kWaitCycles, r.abort);
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
        } else {
            for (int g0 = 0; ok && g0 < slabs; g0 += group) {
                const int g1 = min(g0 + group, slabs);
                for (int s = g0; ok && s < g1; ++s) {  // the lo terms of the group
                    const int st = (first + s) % S;
                    ok = tc::mbar_wait_or_abort(r.split + st, ((first + s) / S) & 1, tcg::kWaitCycles, r.abort);
                    if (!ok) break;
                    tc::tc_fence_after();
                    const uint32_t bh = tc::smem_u32(r.hi + st * (SLAB / 4)),
                                   bl = tc::smem_u32(r.lo + st * (SLAB / 4));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t ah = tmem + s * 32 + kk * 8, al = ah + 128;
                        tc::mma_tf32_ts(d, al, tc::desc_k_sw128(bh + kk * 32), idesc, (s | kk) != 0);
                        tc::mma_tf32_ts(d, ah, tc::desc_k_sw128(bl + kk * 32), idesc, 1);
                    }
                }
                for (int s = g0; ok && s < g1; ++s) {  // its hi*hi terms; then the stage is free
                    const int st = (first + s) % S;
                    const uint32_t bh = tc::smem_u32(r.hi + st * (SLAB / 4));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc::mma_tf32_ts(d, tmem + s * 32 + kk * 8, tc::desc_k_sw128(bh + kk * 32), idesc, 1);
                    tc::mma_commit(r.empty + st);
                }
            }
        }
        it = first + slabs;
        if (ok) tc::mma_commit(r.acc_full + a);
    }
    // every MMA this thread issued has completed once this commit arrives
    tc::mma_commit(r.drain + which);
    if (!tc::mbar_wait(r.drain + which, 0, tcg::kWaitCycles)) *r.abort = 1;
}

// Epilogue warps 6-9: the A operand's row `m` (K values) split into TF32 hi
// and lo, into tensor memory columns [0, K) and [128, 128 + K) of the thread's
// lane. The forward's A is W (column-major, leading dimension M: row m holds
// W[m + k M]); the backward's is W^T (row n holds W[k + n K], contiguous).
// Rows m >= M (a layer narrower than the tile's 128 rows) are zero, so those
// accumulator lanes stay zero and the epilogue skips them.
// Paired tiles (halves = 2): the A operand is the block diagonal diag(W, W)
// of 2K columns; lanes of half h (0: lanes 0-63, 1: lanes 64-127) hold row m
// of W in columns [h K, h K + K) and zeros elsewhere.
__device__ __forceinline__ void load_weights(const Ring& r, uint32_t tmem, const float* __restrict__ W, int M,
                                             int K, int m, bool transposed = false, int halves = 1, int half = 0) {
    const int quarter = (threadIdx.x >> 5) & 3;
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    const bool live = m < M;
    for (int c0 = 0; c0 < K * halves; c0 += 8) {
        const int k0 = c0 - (c0 >= K ? K : 0);  // column within W's block (K is a multiple of 8)
        const bool block = live && (c0 >= K) == (half == 1);
        float h[8], l[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float v = !block ? 0.f
                            : transposed ? __ldg(W + (size_t)m * K + k0 + j)
                                         : __ldg(W + m + (size_t)(k0 + j) * M);
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

// Paired tiles: a layer of at most 64 neurons fills only half of the 128
// accumulator lanes, and half of the epilogue warps (those of lane quarters
// 2 and 3) would idle. With halves = 2 one MMA chain computes two adjacent
// column tiles at once: A = diag(W, W) (2K columns, K <= 64) against the K
// slabs of tile 2w followed by those of tile 2w + 1, so lanes 0-63 hold
// tile 2w and lanes 64-127 tile 2w + 1, and every epilogue warp has a tile.
// The tensor cores do twice the (cheap) work; the epilogue, which sets the
// pace of these layers, covers twice the columns per accumulator.
__host__ __device__ constexpr bool paired_tiles(int rows, int K) { return rows <= 64 && K <= 64; }

struct PairedTiles {
    int halves;  // 1, or 2 for paired tiles
    // lane quarter -> (half, first row of the quarter within the layer's 128-row slice)
    __device__ int half(int quarter) const { return halves == 2 ? quarter >> 1 : 0; }
    __device__ int row(int quarter) const { return (halves == 2 ? quarter & 1 : quarter) * 32; }
};

// Hidden layer forward: Y = f(W X + b) with the jet combine in the epilogue.
// grid = (CTAs over work items, M / 128); K a multiple of 32, at most 128;
// halves = 2 (paired tiles) needs M <= 64 and K <= 64.
template <int SID, class Act>
__global__ void __launch_bounds__(THREADS, 1) k_forward_ws(const __grid_constant__ CUtensorMap map_x, int M, int K,
                                                           long P, const float* __restrict__ W,
                                                           float* __restrict__ Y, int* error, int halves) {
    constexpr int R = StaticJet<SID>::R;
    using T = Tiling<R>;
    extern __shared__ uint8_t smem_raw[];
    Ring r = carve_ring<T::SLAB>(smem_raw);
    ring_init(r);
    const uint32_t tmem = *r.tmem_slot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long tiles = (P + T::PTS - 1) / T::PTS, items = (tiles + halves - 1) / halves;
    const int kslabs = K / 32;
    const PairedTiles pt{halves};
    if (warp == kProducerWarp) {
        if (lane == 0) produce<T::SLAB>(r, &map_x, items, T::COLS, T::N, kslabs, halves);
    } else if (warp == kMmaWarp || warp == kSecondMmaWarp) {
        if (lane == 0)
            issue_mmas<T::N, T::SLAB>(r, tmem, items, kslabs * halves, warp == kMmaWarp ? 0 : 1,
                                      lo_first_group(kslabs));
    } else if (warp < kEpilogueWarp) {
        split_all<T::SLAB>(r, items, T::N, kslabs * halves);
    } else {
        const int quarter = warp & 3, group = (warp - kEpilogueWarp) >> 2, half = pt.half(quarter);
        const int m = blockIdx.y * 128 + pt.row(quarter) + lane;
        const bool live = m < M;  // the same for the whole warp: M is a multiple of 32
        if (group == 0) load_weights(r, tmem, W, M, K, m, false, halves, half);
        const float b0 = live ? __ldg(W + (size_t)M * K + m) : 0.f;
        const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
        uint32_t local = 0;
        for (long w = blockIdx.x; w < items; w += gridDim.x, ++local) {
            const int a = local & 1;
            if (!warp_wait(r.acc_full + a, (local >> 1) & 1, r.abort)) break;
            tc::tc_fence_after();
            const long p0 = (w * halves + half) * T::PTS;
            for (int p = group; live && p < T::PTS; p += kEpilogueGroups) {
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

// Hidden layer backward: dZ_prev = adjoint(W^T dZ; Y_prev), the jet adjoint
// in the epilogue. The GEMM is the forward's with A = W^T (rows = the N
// previous-layer neurons of this CTA's slice, K = Ml neurons of this layer)
// and B = the dZ slabs. With INPUT_GRAD the previous layer is the first hidden
// one: dZ_prev is not stored and the first layer's gradient is accumulated
// per thread into input_partials[(halves blockIdx.x + half) 2 + group]
// [n + k N] (bias at k = K0), one partial per epilogue group and tile half.
// The epilogue's reads of Y_prev (and, with INPUT_GRAD, of the inputs) do not
// depend on the accumulator, so each thread copies those of the work item
// (tile, point) two ahead of its current one into a shared-memory staging
// slot, and the DRAM latency of the loads leaves the critical path.
// grid = (CTAs over work items, N / 128); Ml a multiple of 32, at most 128;
// halves = 2 (paired tiles, as in the forward) needs N <= 64 and Ml <= 64.
template <int SID, class Act, bool INPUT_GRAD>
__global__ void __launch_bounds__(THREADS, 1) k_backward_ws(const __grid_constant__ CUtensorMap map_dz, int Ml, int N,
                                                            long P, const float* __restrict__ W,
                                                            const float* __restrict__ Yprev,
                                                            float* __restrict__ dZprev, const float* __restrict__ X0,
                                                            int K0, float* __restrict__ input_partials, int* error,
                                                            int halves) {
    constexpr int R = StaticJet<SID>::R, V = StaticJet<SID>::V;
    constexpr int XV = INPUT_GRAD ? R * V : 0;  // input-jet floats of a point
    using T = Tiling<R, XV>;
    constexpr int S = T::BSTAGES;
    extern __shared__ uint8_t smem_raw[];
    Ring r = carve_ring<T::SLAB, S>(smem_raw);
    ring_init<S>(r);
    const uint32_t tmem = *r.tmem_slot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long tiles = (P + T::PTS - 1) / T::PTS, items = (tiles + halves - 1) / halves;
    const int kslabs = Ml / 32;
    const PairedTiles pt{halves};
    if (warp == kProducerWarp) {
        if (lane == 0) produce<T::SLAB, S>(r, &map_dz, items, T::COLS, T::N, kslabs, halves);
    } else if (warp == kMmaWarp || warp == kSecondMmaWarp) {
        if (lane == 0)
            issue_mmas<T::N, T::SLAB, S>(r, tmem, items, kslabs * halves, warp == kMmaWarp ? 0 : 1,
                                         lo_first_group(kslabs));
    } else if (warp < kEpilogueWarp) {
        split_all<T::SLAB, S>(r, items, T::N, kslabs * halves);
    } else {
        const int quarter = warp & 3, group = (warp - kEpilogueWarp) >> 2, half = pt.half(quarter);
        const int et = threadIdx.x - kEpilogueWarp * 32;  // epilogue thread 0 .. 32 * 4 * groups - 1
        const int n = blockIdx.y * 128 + pt.row(quarter) + lane;
        const bool live = n < N;  // the same for the whole warp: N is a multiple of 32
        if (group == 0) load_weights(r, tmem, W, N, Ml, n, true, halves, half);
        const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
        constexpr int SLOT = R * 32 * 4 * kEpilogueGroups;  // floats of one slot: [q][epilogue thread]
        float* staging = r.staging + et;
        // With INPUT_GRAD the epilogue also needs the point's input jets
        // (R x K0 floats, the same for every lane of the warp). When K0 is the
        // schema's variable count they are loaded at staging time, one element
        // per lane (xq, a three-deep queue that shifts with the slots), and
        // shared through the warp's row of shared memory when consumed;
        // reading them from global memory only then left an L2 round trip on
        // the path of every work item.
        constexpr int XR = XV > 0 ? (XV + 31) / 32 : 1;
        const bool x_queue = INPUT_GRAD && K0 == V;
        float xq[3][XR];
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int c = 0; c < XR; ++c) xq[i][c] = 0.f;
        float* xrow = r.staging + T::YBUF / 4 + (warp - kEpilogueWarp) * T::XROW;
        // The thread's work items in order: points group, group + groups, ...
        // of its tile (half) of each of the CTA's work items. (ft, fp) is the
        // next item to stage. Only the last work item can hold a partial (or,
        // paired, an empty) tile, so the slots a thread stages past its last
        // real item are never read.
        long ft = blockIdx.x;
        int fp = group;
        auto stage = [&](int slot) {
            const long first = (ft * halves + half) * T::PTS;  // first point of the thread's tile
            const bool valid = ft < items && first + fp < P;
            if (valid) {
                const long point = first + fp;
                const float* yp = Yprev + ((size_t)point * R) * N + n;
#pragma unroll
                for (int q = 0; q < R; ++q)
                    tc::copy_async4(staging + slot * SLOT + q * 32 * 4 * kEpilogueGroups, yp + (size_t)q * N);
                if (INPUT_GRAD && !x_queue && lane * 32 < R * K0)
                    tc::prefetch_l2(X0 + (size_t)point * R * K0 + lane * 32);
            }
            if (INPUT_GRAD) {
#pragma unroll
                for (int c = 0; c < XR; ++c) {
                    const int e = lane + 32 * c;
                    xq[0][c] = xq[1][c];
                    xq[1][c] = xq[2][c];
                    xq[2][c] = x_queue && valid && e < XV ? __ldg(X0 + (size_t)(first + fp) * XV + e) : 0.f;
                }
            }
            tc::copy_async_commit();
            fp += kEpilogueGroups;
            if (fp >= T::PTS || first + fp >= P) {
                fp = group;
                ft += gridDim.x;
            }
        };
        if (live)
#pragma unroll
            for (int k = 0; k < kStagingSlots - 1; ++k) stage(k);
        int slot = 0;
        float gacc[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) gacc[k] = 0.f;
        uint32_t local = 0;
        for (long w = blockIdx.x; w < items; w += gridDim.x, ++local) {
            const int a = local & 1;
            if (!warp_wait(r.acc_full + a, (local >> 1) & 1, r.abort)) break;
            tc::tc_fence_after();
            const long p0 = (w * halves + half) * T::PTS;
            for (int p = group; live && p < T::PTS; p += kEpilogueGroups) {
                if (p0 + p >= P) break;
                stage(slot == 0 ? kStagingSlots - 1 : slot - 1);  // the slot read one item ago
                float g[R], y[R];
                tc::tmem_read<R>(lane_base + kAccColumn + a * 128 + p * R, g);
                tc::copy_async_wait<kStagingSlots - 1>();
#pragma unroll
                for (int q = 0; q < R; ++q) y[q] = staging[slot * SLOT + q * 32 * 4 * kEpilogueGroups];
                slot = slot + 1 == kStagingSlots ? 0 : slot + 1;
                StaticJet<SID>::template adjoint<Act>(y, g);
                if (INPUT_GRAD && x_queue) {
                    // the item's input jets: staged two items ago, now the queue's head
                    __syncwarp();  // the previous item's reads of the row are done
#pragma unroll
                    for (int c = 0; c < XR; ++c)
                        if (lane + 32 * c < XV) xrow[lane + 32 * c] = xq[0][c];
                    __syncwarp();
                    fast::input_gradient_row<R, V>(g, xrow, gacc);
                } else if (INPUT_GRAD) {
                    fast::input_gradient<R>(g, X0 + (size_t)(p0 + p) * R * K0, K0, gacc);
                } else {
                    float* out = dZprev + ((size_t)(p0 + p) * R) * N + n;
#pragma unroll
                    for (int q = 0; q < R; ++q) out[(size_t)q * N] = g[q];
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(r.acc_empty + a);
        }
        tc::copy_async_wait<0>();  // no copy may land after the CTA ends
        if (INPUT_GRAD && live) {
            float* out = input_partials +
                         (size_t)((blockIdx.x * halves + half) * kEpilogueGroups + group) * N * (K0 + 1);
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (k < K0) out[n + (size_t)k * N] = gacc[k];
            out[n + (size_t)K0 * N] = gacc[8];
        }
    }
    teardown(r, tmem, error);
}

// ---------------------------------------------------------------------------
// Layers of more than kMaxK inputs (the 256- and 512-neuron layers of configs
// 4 and 5). The weights of a 128-neuron slice no longer fit in tensor memory
// beside the two accumulators, so every stage of the ring carries the K slab
// of the weights (TF32 hi and lo, split once per pass into K-major arrays in
// global memory, where they stay in L2) beside the activation slab, and the
// MMAs read A from shared memory. The roles are the kernels' above; the
// epilogue warps load no weights, and the backward's epilogue reads Y_prev
// directly instead of staging it (at these widths the layer is bound by the
// tensor cores: a tile's MMAs take longer than its epilogue, which runs
// while the other accumulator fills).

constexpr int kWeightSlab = 128 * 128;  // bytes: 128 neurons x 32 fp32 of K

template <int R>
struct WideTiling {
    using T = Tiling<R>;
    static constexpr int PTS = T::PTS, COLS = T::COLS, N = T::N, SLAB = T::SLAB;
    static constexpr int STAGE = 2 * SLAB + 2 * kWeightSlab;
    static constexpr int S = (kSmemLimit - 1024 - 256) / STAGE;
    static constexpr int SMEM = S * STAGE + 1024 + 256;
    static_assert(S >= 3, "wide-layer ring too shallow");
};

// The ring of carve_ring<SLAB, S> with the weight slabs between the
// activation slabs and the barriers: a_hi[S][kWeightSlab], a_lo[S][...].
template <int SLAB, int S>
__device__ __forceinline__ Ring carve_wide(uint8_t* raw, float*& a_hi, float*& a_lo) {
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    a_hi = reinterpret_cast<float*>(base + 2 * S * SLAB);
    a_lo = reinterpret_cast<float*>(base + 2 * S * SLAB + S * kWeightSlab);
    // carve_ring places its barriers right after 2 S SLAB bytes: hand it a base
    // moved back by the weight slabs' size so they land after those instead
    Ring r = carve_ring<SLAB, S>(base + 2 * S * kWeightSlab);
    r.hi = reinterpret_cast<float*>(base);
    r.lo = reinterpret_cast<float*>(base + S * SLAB);
    return r;
}

// Producer of the wide layers: per K slab, the activation slab of the tile
// and the weight slabs (hi, lo) of this CTA's neurons `a_row`..+127.
template <int SLAB, int S>
__device__ __forceinline__ void produce_wide(const Ring& r, float* a_hi, float* a_lo, const CUtensorMap* map,
                                             const CUtensorMap* map_a_hi, const CUtensorMap* map_a_lo, int a_row,
                                             long tiles, int tile_columns, int N, int slabs) {
    // The ring is only S stages deep and a slab's MMAs are short, so an
    // activation slab fetched from HBM when its stage frees would arrive late:
    // each slab's L2 prefetch goes out kPrefetch slabs ahead of its load (the
    // weight slabs are L2-resident already).
    constexpr int kPrefetch = 2 * S;
    auto prefetch = [&](long tile, int s) {  // the slab kPrefetch after (tile, s)
        s += kPrefetch;
        while (s >= slabs) {
            s -= slabs;
            tile += gridDim.x;
        }
        if (tile < tiles) tc::tma_prefetch_2d(map, s * 32, int(tile * tile_columns));
    };
    for (int k = 0; k < kPrefetch && k < slabs; ++k) prefetch(blockIdx.x, k - kPrefetch);
    uint32_t it = 0;
    for (long tile = blockIdx.x; tile < tiles && !*r.abort; tile += gridDim.x) {
        const int col0 = int(tile * tile_columns);
        for (int s = 0; s < slabs; ++s) {
            const int st = it % S;
            if (!tc::mbar_wait_or_abort(r.empty + st, ((it / S) & 1) ^ 1, tcg::kWaitCycles, r.abort)) break;
            tc::mbar_expect_tx(r.full + st, uint32_t(N) * 128 + 2 * kWeightSlab);
            tc::tma_load_2d(r.hi + st * (SLAB / 4), map, r.full + st, s * 32, col0);
            tc::tma_load_2d(a_hi + st * (kWeightSlab / 4), map_a_hi, r.full + st, s * 32, a_row);
            tc::tma_load_2d(a_lo + st * (kWeightSlab / 4), map_a_lo, r.full + st, s * 32, a_row);
            prefetch(tile, s);
            ++it;
        }
    }
    // a load that never lands must not go unnoticed: the CTA then reports an error
    for (uint32_t k = it > S ? it - S : 0; k < it; ++k)
        if (!tc::mbar_wait(r.full + k % S, (k / S) & 1, tcg::kWaitCycles)) *r.abort = 1;
}

// MMA issuer of the wide layers: issue_mmas with A (hi, lo) from the stage's
// weight slabs in shared memory. With no weights in tensor memory each tile
// has two accumulators: hi*hi in columns [256 a, 256 a + 128) and the two
// small lo terms in the next 128. The tensor core's FP32 accumulation does
// not round to nearest, so each add costs up to an ulp of the accumulator;
// the large accumulator then takes a third of the adds, and the epilogue sums
// the pair in IEEE FP32 (measured: the wide layers' output error falls with
// it).
__host__ __device__ constexpr uint32_t wide_accumulator(int a) { return uint32_t(a) * 256u; }

template <int N, int SLAB, int S>
__device__ __forceinline__ void issue_mmas_wide(const Ring& r, const float* a_hi, const float* a_lo, uint32_t tmem,
                                                long tiles, int slabs, int which) {
    constexpr uint32_t idesc = tc::idesc_tf32(128, N);
    const int issuers = mma_issuers(S, slabs);
    bool ok = true;
    uint32_t it = which * slabs, local = which;
    for (long tile = blockIdx.x + which * gridDim.x; ok && which < issuers && tile < tiles;
         tile += issuers * gridDim.x, local += issuers, it += (issuers - 1) * slabs) {
        const int a = local & 1;
        ok = tc::mbar_wait_or_abort(r.acc_empty + a, ((local >> 1) & 1) ^ 1, tcg::kWaitCycles, r.abort);
        tc::tc_fence_after();
        const uint32_t d = tmem + wide_accumulator(a), d_lo = d + 128;
        for (int s = 0; ok && s < slabs; ++s, ++it) {
            const int st = it % S;
            ok = tc::mbar_wait_or_abort(r.split + st, (it / S) & 1, tcg::kWaitCycles, r.abort);
            if (!ok) break;
            tc::tc_fence_after();
            const uint32_t bh = tc::smem_u32(r.hi + st * (SLAB / 4)), bl = tc::smem_u32(r.lo + st * (SLAB / 4));
            const uint32_t ah = tc::smem_u32(a_hi + st * (kWeightSlab / 4));
            const uint32_t al = tc::smem_u32(a_lo + st * (kWeightSlab / 4));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint32_t off = kk * 32;  // 8 TF32 values along the 128-byte rows
                tc::mma_tf32(d_lo, tc::desc_k_sw128(al + off), tc::desc_k_sw128(bh + off), idesc, (s | kk) != 0);
                tc::mma_tf32(d_lo, tc::desc_k_sw128(ah + off), tc::desc_k_sw128(bl + off), idesc, 1);
                tc::mma_tf32(d, tc::desc_k_sw128(ah + off), tc::desc_k_sw128(bh + off), idesc, (s | kk) != 0);
            }
            tc::mma_commit(r.empty + st);
        }
        if (ok) tc::mma_commit(r.acc_full + a);
    }
    tc::mma_commit(r.drain + which);
    if (!tc::mbar_wait(r.drain + which, 0, tcg::kWaitCycles)) *r.abort = 1;
}

// Hidden layer forward of more than kMaxK inputs: Y = f(W X + b). The
// weights come as TF32 hi/lo arrays, row m of K values each (maps with
// 32 x 128 boxes, 128-byte swizzle). grid = (CTAs over column tiles, M / 128).
template <int SID, class Act>
__global__ void __launch_bounds__(THREADS, 1) k_forward_wide(const __grid_constant__ CUtensorMap map_x,
                                                             const __grid_constant__ CUtensorMap map_w_hi,
                                                             const __grid_constant__ CUtensorMap map_w_lo, int M,
                                                             int K, long P, const float* __restrict__ bias,
                                                             float* __restrict__ Y, int* error) {
    constexpr int R = StaticJet<SID>::R;
    using T = WideTiling<R>;
    extern __shared__ uint8_t smem_raw[];
    float *a_hi, *a_lo;
    Ring r = carve_wide<T::SLAB, T::S>(smem_raw, a_hi, a_lo);
    ring_init<T::S>(r);
    const uint32_t tmem = *r.tmem_slot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long tiles = (P + T::PTS - 1) / T::PTS;
    const int slabs = K / 32;
    if (warp == kProducerWarp) {
        if (lane == 0)
            produce_wide<T::SLAB, T::S>(r, a_hi, a_lo, &map_x, &map_w_hi, &map_w_lo, blockIdx.y * 128, tiles, T::COLS,
                                        T::N, slabs);
    } else if (warp == kMmaWarp || warp == kSecondMmaWarp) {
        if (lane == 0) issue_mmas_wide<T::N, T::SLAB, T::S>(r, a_hi, a_lo, tmem, tiles, slabs, warp == kMmaWarp ? 0 : 1);
    } else if (warp < kEpilogueWarp) {
        split_all<T::SLAB, T::S>(r, tiles, T::N, slabs);
    } else {
        const int quarter = warp & 3, group = (warp - kEpilogueWarp) >> 2;
        const int m = blockIdx.y * 128 + quarter * 32 + lane;
        const float b0 = __ldg(bias + m);
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
                tc::tmem_read<R>(lane_base + wide_accumulator(a) + p * R, z);
                tc::tmem_read<R>(lane_base + wide_accumulator(a) + 128 + p * R, y);  // the lo terms
#pragma unroll
                for (int q = 0; q < R; ++q) z[q] += y[q];
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

// Hidden layer backward of more than kMaxK inputs (Ml > kMaxK neurons in this
// layer): dZ_prev = adjoint(W^T dZ; Y_prev), A = W^T from the TF32 hi/lo
// arrays of W as stored (row n holds W[k + n Ml]). INPUT_GRAD as in
// k_backward_ws. grid = (CTAs over column tiles, N / 128).
template <int SID, class Act, bool INPUT_GRAD>
__global__ void __launch_bounds__(THREADS, 1) k_backward_wide(const __grid_constant__ CUtensorMap map_dz,
                                                              const __grid_constant__ CUtensorMap map_w_hi,
                                                              const __grid_constant__ CUtensorMap map_w_lo, int Ml,
                                                              int N, long P, const float* __restrict__ Yprev,
                                                              float* __restrict__ dZprev, const float* __restrict__ X0,
                                                              int K0, float* __restrict__ input_partials, int* error) {
    constexpr int R = StaticJet<SID>::R;
    using T = WideTiling<R>;
    extern __shared__ uint8_t smem_raw[];
    float *a_hi, *a_lo;
    Ring r = carve_wide<T::SLAB, T::S>(smem_raw, a_hi, a_lo);
    ring_init<T::S>(r);
    const uint32_t tmem = *r.tmem_slot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long tiles = (P + T::PTS - 1) / T::PTS;
    const int slabs = Ml / 32;
    if (warp == kProducerWarp) {
        if (lane == 0)
            produce_wide<T::SLAB, T::S>(r, a_hi, a_lo, &map_dz, &map_w_hi, &map_w_lo, blockIdx.y * 128, tiles, T::COLS,
                                        T::N, slabs);
    } else if (warp == kMmaWarp || warp == kSecondMmaWarp) {
        if (lane == 0) issue_mmas_wide<T::N, T::SLAB, T::S>(r, a_hi, a_lo, tmem, tiles, slabs, warp == kMmaWarp ? 0 : 1);
    } else if (warp < kEpilogueWarp) {
        split_all<T::SLAB, T::S>(r, tiles, T::N, slabs);
    } else {
        const int quarter = warp & 3, group = (warp - kEpilogueWarp) >> 2;
        const int n = blockIdx.y * 128 + quarter * 32 + lane;
        const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
        float gacc[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) gacc[k] = 0.f;
        uint32_t local = 0;
        for (long tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            const int a = local & 1;
            if (!warp_wait(r.acc_full + a, (local >> 1) & 1, r.abort)) break;
            tc::tc_fence_after();
            const long p0 = tile * T::PTS;
            for (int p = group; p < T::PTS; p += kEpilogueGroups) {
                if (p0 + p >= P) break;
                float g[R], y[R];
                const float* yp = Yprev + ((size_t)(p0 + p) * R) * N + n;
#pragma unroll
                for (int q = 0; q < R; ++q) y[q] = __ldg(yp + (size_t)q * N);
                {
                    float lo[R];
                    tc::tmem_read<R>(lane_base + wide_accumulator(a) + p * R, g);
                    tc::tmem_read<R>(lane_base + wide_accumulator(a) + 128 + p * R, lo);  // the lo terms
#pragma unroll
                    for (int q = 0; q < R; ++q) g[q] += lo[q];
                }
                StaticJet<SID>::template adjoint<Act>(y, g);
                if (INPUT_GRAD) {
                    fast::input_gradient<R>(g, X0 + (size_t)(p0 + p) * R * K0, K0, gacc);
                } else {
                    float* out = dZprev + ((size_t)(p0 + p) * R) * N + n;
#pragma unroll
                    for (int q = 0; q < R; ++q) out[(size_t)q * N] = g[q];
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(r.acc_empty + a);
        }
        if (INPUT_GRAD) {
            float* out = input_partials + (size_t)(2 * blockIdx.x + group) * N * (K0 + 1);
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (k < K0) out[n + (size_t)k * N] = gacc[k];
            out[n + (size_t)K0 * N] = gacc[8];
        }
    }
    teardown(r, tmem, error);
}

// ---------------------------------------------------------------------------
// Weight gradient of a hidden layer: G (an NB-neuron slice of this layer x an
// NB-neuron slice of the previous layer, plus the bias column) = sum over
// this CTA's columns of dZ[:, c] Y_prev[:, c]^T. Per 32-column stage, TMA brings NB/32
// boxes of 32 neurons x 32 columns of each operand (128-byte swizzle with
// 32-byte atoms, the layout of MN-major TF32 operands). The split warps move
// dZ through registers into tensor memory as the K-major A operand (thread =
// neuron: its 32 columns, TF32 hi and lo, plus its bias sum over value-row
// columns) while the epilogue warps write the lo part of Y_prev beside the
// raw operand (its hi part) as the MN-major B operand, so shared memory
// carries each operand once per MMA term instead of also serving the A side.
// Two MMA issuers take the even and the odd stages, each into its own
// 128 x NB accumulator. The tensor core's FP32 accumulation does not round to
// nearest, so a sum over thousands of column chunks in one accumulator drifts
// (measured: 6e-4 normwise on config 5's gradients against the float64
// oracle); each accumulator therefore sums only kSegment of its issuer's
// chunks before four drain warps fold it into a round-to-nearest FP32 sum in
// shared memory and release it. The second issuer's segments are offset by
// half a segment, so the two drains do not stall both issuers at once.
// grid = (CTAs, N / NB, M / NB): CTAs that share blockIdx.x take the same
// chunks at about the same time, so the slices of dZ and Y_prev that several
// of them read come from L2.
// Slices of NB = 64 neurons (layers of at most 64 x 64): each stage is half
// as large, so the ring holds six stages instead of three; with 128-neuron
// slices of a 64-neuron layer half of every stage was zeros and three
// stages of 32 columns kept too few bytes in flight to cover the HBM
// latency (0.32 ms for 0.67 GB on config 3, 2.1 TB/s). The MMAs keep
// M = 128 (the A lanes 64-127 are never written and their accumulator rows
// never read) with N = 64.

constexpr int kWgBox = 32 * 32 * 4;       // 32 neurons x 32 columns
constexpr int kWgEpilogueWarp = 6, kWgSecondMmaWarp = 10, kWgDrainWarp = 11, kWgSecondSplitWarp = 15;
constexpr uint32_t kWgTmemColumns = 512;

template <int NB>
struct WgShape {
    static_assert(NB == 64 || NB == 128, "weight-gradient slices are 64 or 128 neurons");
    static constexpr int kBoxes = NB / 32;
    static constexpr int kOperand = kBoxes * kWgBox;  // bytes of one operand slice of a chunk
    static constexpr int kStage = 3 * kOperand;       // dZ raw, Y raw (= hi), Y lo
    static constexpr int kStages = NB == 128 ? 3 : 6;
    static constexpr int kSums = NB * NB * 4;         // FP32 sums [column n][neuron m]
    // chunks one accumulator sums before a drain: the 64-neuron slices (the
    // layers of orders <= 3 networks, held to 1e-5) drain twice as often,
    // halving the truncating adds of a segment's sum
    static constexpr int kSegment = NB == 128 ? 16 : 8;
    // split warps: kSplitGroups groups of kSplitWarps (one per TMEM lane quarter
    // the slice uses) take chunks it = group, group + kSplitGroups, ...
    // (a third group of four warps for 128-neuron slices measured no faster)
    static constexpr int kSplitGroups = NB == 128 ? 2 : 3;
    // producer, MMA issuer, 4 split warps, 4 lo warps, second issuer, 4 drain warps, 4 split warps
    static constexpr int kThreads = 608;
    static constexpr int kSplitWarps = NB / 32;
    static constexpr int kLoWarps = NB == 128 ? 4 : 6;
    static constexpr int kBias = kSplitGroups * 128 * 4;  // the split groups' bias sums
    static constexpr int kSmem = kStages * kStage + kSums + kBias + 1024 + 256;
    // tensor memory: accumulator 0 at column 0, accumulator 1 at kSecondAcc, the
    // dZ hi/lo of stage st at kDz + 64 st (+32)
    static constexpr uint32_t kSecondAcc = NB == 128 ? 384 : 64;
    static constexpr uint32_t kDz = 128;
    static_assert(kDz + 64 * kStages <= (NB == 128 ? kSecondAcc : kWgTmemColumns), "tensor memory overlap");
};
constexpr int kWgSmem = WgShape<128>::kSmem;
constexpr int kWgSmem64 = WgShape<64>::kSmem;

// element (mn, k) of such an operand, in floats from its start
__device__ __forceinline__ int mn32_index(int mn, int k) {
    return (mn >> 5) * (kWgBox / 4) + k * 32 + ((((mn & 31) >> 3) ^ (k & 3)) << 3) + (mn & 7);
}

// Segment k of issuer w holds its chunks [start, start + length): issuer 1's
// first segment is half as long.
template <int SEG>
__device__ __forceinline__ int wg_segment_length(int w, int k) { return k == 0 && w ? SEG / 2 : SEG; }
template <int SEG>
__device__ __forceinline__ int wg_segments(int w, int count) {
    if (count <= 0) return 0;
    const int first = wg_segment_length<SEG>(w, 0);
    return count <= first ? 1 : 1 + (count - first + SEG - 1) / SEG;
}
// ring index of the last chunk of segment k of issuer w (of `count` chunks)
template <int SEG>
__device__ __forceinline__ int wg_segment_end(int w, int k, int count) {
    const int first = wg_segment_length<SEG>(w, 0);
    const int last_local = min(count, k == 0 ? first : first + k * SEG) - 1;
    return 2 * last_local + w;
}

// Warp roles of k_wgrad_ws: 0 producer, 1 and 10 MMA issuers, 11-14 drain;
// with 128-neuron slices split groups {2-5} and {15-18} and lo warps 6-9; with
// 64-neuron slices split groups {4, 5}, {16, 17} and {8, 9} (the warps of lane
// quarters 0 and 1) and lo warps 2, 3, 6, 7, 15, 18.
template <int NB>
__device__ __forceinline__ int wg_split_group(int warp) {
    if (NB == 128) return warp >= 2 && warp <= 5 ? 0 : warp >= kWgSecondSplitWarp ? 1 : -1;
    switch (warp) {
        case 4: case 5: return 0;
        case 16: case 17: return 1;
        case 8: case 9: return 2;
        default: return -1;
    }
}
template <int NB>
__device__ __forceinline__ int wg_lo_warp(int warp) {  // index among the lo warps, or -1
    if (NB == 128) return warp >= kWgEpilogueWarp && warp < kWgSecondMmaWarp ? warp - kWgEpilogueWarp : -1;
    switch (warp) {
        case 2: return 0;
        case 3: return 1;
        case 6: return 2;
        case 7: return 3;
        case 15: return 4;
        case 18: return 5;
        default: return -1;
    }
}

template <int NB>
__global__ void __launch_bounds__(WgShape<NB>::kThreads, 1) k_wgrad_ws(const __grid_constant__ CUtensorMap map_dz,
                                                            const __grid_constant__ CUtensorMap map_y, int M, int N,
                                                            long columns, int R, float* __restrict__ partials,
                                                            int* error) {
    using G = WgShape<NB>;
    constexpr int kStages = G::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* sums = reinterpret_cast<float*>(base + kStages * G::kStage);
    float* bias_sums = reinterpret_cast<float*>(base + kStages * G::kStage + G::kSums);  // [split group][neuron]
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + kStages * G::kStage + G::kSums + G::kBias);
    uint64_t *full = bars, *split = bars + kStages, *empty = bars + 2 * kStages, *drain = bars + 3 * kStages;
    uint64_t *acc_full = drain + 1, *acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* split_count = abort + 1;  // split-warp arrivals so far (4 per chunk)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        *split_count = 0;
        for (int s = 0; s < kStages; ++s) {
            tc::mbar_init(full + s, 1);
            tc::mbar_init(split + s, 8);
            tc::mbar_init(empty + s, 1);
        }
        tc::mbar_init(drain, 2);  // one commit per MMA issuer
        for (int w = 0; w < 2; ++w) {
            tc::mbar_init(acc_full + w, 1);   // the issuer's commit at a segment's end
            tc::mbar_init(acc_empty + w, 4);  // the four drain warps
        }
        *abort = 0;
        tc::fence_barrier_init();
    }
    if (warp == kMmaWarp) {
        tc::tmem_alloc(tmem_slot, kWgTmemColumns);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_base = blockIdx.y * NB, m_base = blockIdx.z * NB;
    // 32-column chunks dealt round-robin over the CTAs, so the whole grid
    // streams through one region of both operands at a time
    const long total_chunks = (columns + 31) / 32;
    const int chunks = blockIdx.x < total_chunks ? int((total_chunks - 1 - blockIdx.x) / gridDim.x + 1) : 0;
    const int mine[2] = {(chunks + 1) / 2, chunks / 2};  // chunks of issuer 0 (even) and 1 (odd)
    auto chunk_start = [&](int it) { return 32L * ((long)blockIdx.x + (long)it * gridDim.x); };
    auto stage_ptr = [&](int st, int part) {
        return reinterpret_cast<float*>(base + st * G::kStage + part * G::kOperand);
    };
    auto dz_column = [](int st) { return G::kDz + 64u * uint32_t(st); };
    float* out = partials + (size_t)blockIdx.x * M * (N + 1);
    if (warp == kProducerWarp) {
        if (lane == 0) {
            // L2 prefetches run two ring depths ahead of the loads (the ring
            // alone does not cover the HBM latency of a chunk)
            constexpr int kPrefetch = 2 * kStages;
            auto prefetch = [&](int it) {
                if (it >= chunks) return;
                const int c0 = int(chunk_start(it));
                for (int j = 0; j < G::kBoxes; ++j) {
                    tc::tma_prefetch_2d(&map_dz, m_base + 32 * j, c0);
                    tc::tma_prefetch_2d(&map_y, n_base + 32 * j, c0);
                }
            };
            for (int k = 0; k < kPrefetch; ++k) prefetch(k);
            int it = 0;
            for (; it < chunks && !*abort; ++it) {
                const int st = it % kStages;
                if (!tc::mbar_wait_or_abort(empty + st, ((it / kStages) & 1) ^ 1, tcg::kWaitCycles, abort)) break;
                tc::mbar_expect_tx(full + st, 2 * G::kOperand);
                const int c0 = int(chunk_start(it));
                for (int j = 0; j < G::kBoxes; ++j) {
                    tc::tma_load_2d(stage_ptr(st, 0) + j * (kWgBox / 4), &map_dz, full + st, m_base + 32 * j, c0);
                    tc::tma_load_2d(stage_ptr(st, 1) + j * (kWgBox / 4), &map_y, full + st, n_base + 32 * j, c0);
                }
                prefetch(it + kPrefetch);
            }
            for (int k = it > kStages ? it - kStages : 0; k < it; ++k)
                if (!tc::mbar_wait(full + k % kStages, (k / kStages) & 1, tcg::kWaitCycles)) *abort = 1;
        }
    } else if (warp == kMmaWarp || warp == kWgSecondMmaWarp) {
        // two issuers, the even and the odd chunks, each into its own accumulator
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_tf32(128, NB) | (1u << 16);  // B (Y) MN-major, A (dZ) from TMEM
            const int which = warp == kMmaWarp ? 0 : 1;
            const uint32_t acc = which ? tmem + G::kSecondAcc : tmem;
            int seg = 0, in_seg = 0;
            bool ok = true;
            for (int it = which; ok && it < chunks; it += 2) {
                if (in_seg == wg_segment_length<G::kSegment>(which, seg)) {
                    // the drain warps have folded the previous segment out of the accumulator
                    ok = tc::mbar_wait_or_abort(acc_empty + which, seg & 1, tcg::kWaitCycles, abort);
                    if (!ok) break;
                    ++seg;
                    in_seg = 0;
                }
                const int st = it % kStages;
                if (!tc::mbar_wait_or_abort(split + st, (it / kStages) & 1, tcg::kWaitCycles, abort)) break;
                tc::tc_fence_after();
                const uint32_t yh = tc::smem_u32(stage_ptr(st, 1)), yl = tc::smem_u32(stage_ptr(st, 2));
                const uint32_t ah = tmem + dz_column(st), al = ah + 32;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint32_t off = kk * 1024;  // 8 columns of Y
                    tc::mma_tf32_ts(acc, al + kk * 8, tc::desc_mn32_sw128(yh + off, kWgBox), idesc,
                                    in_seg != 0 || kk != 0);
                    tc::mma_tf32_ts(acc, ah + kk * 8, tc::desc_mn32_sw128(yl + off, kWgBox), idesc, 1);
                    tc::mma_tf32_ts(acc, ah + kk * 8, tc::desc_mn32_sw128(yh + off, kWgBox), idesc, 1);
                }
                tc::mma_commit(empty + st);
                ++in_seg;
                if (in_seg == wg_segment_length<G::kSegment>(which, seg) || it + 2 >= chunks) tc::mma_commit(acc_full + which);
            }
            tc::mma_commit(drain);
            if (!tc::mbar_wait(drain, 0, tcg::kWaitCycles)) *abort = 1;
        }
    } else if (wg_split_group<NB>(warp) >= 0) {
        // split warps, in groups (one warp per TMEM lane quarter of the slice)
        // that take alternate chunks: thread = neuron m (its TMEM lane);
        // the stage's dZ row of that neuron into tensor memory (hi, lo) and its
        // bias over value-row columns (the warps of lanes past the slice only
        // keep the count). A chunk's round (shared-memory reads, conversion,
        // tensor-memory stores and their wait, the barrier) took about 2,000
        // cycles, longer than the chunk's MMAs or its HBM time, so one group
        // alone set the kernel's pace; the groups overlap their rounds (two of
        // four warps for 128-neuron slices, three of two for 64-neuron slices,
        // whose lane quarters 2 and 3 have no split work: 0.218 -> 0.177 ms on
        // config 3's layers against two groups). (Taking
        // two chunks per round in one group instead measured slower: config
        // 2's weight gradient 0.42 -> 0.65 ms, as a batch's first MMAs then
        // wait for its last chunk.) The groups still arrive in chunk order: an
        // MMA issuer waits on a stage's barrier by phase parity, which is exact
        // only if the stage's previous phase (chunk it - kStages, possibly the
        // other group's) is complete when the wait starts; each warp therefore
        // arrives for chunk it only once all kSplitWarps x it arrivals of
        // earlier chunks are in (split_count), while the groups' work overlaps.
        const int group = wg_split_group<NB>(warp);
        const int quarter = warp & 3, m = quarter * 32 + lane;
        const bool mine_lane = quarter * 32 < NB;  // the same for the whole warp
        const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
        float bias = 0.f;
        for (int it = group; it < chunks; it += G::kSplitGroups) {
            const int st = it % kStages;
            if (!warp_wait(full + st, (it / kStages) & 1, abort)) break;
            tc::tc_fence_after();
            if (mine_lane) {
                const long c0 = chunk_start(it);
                const int valid = int(min(32L, columns - c0));
                const int first = int((R - c0 % R) % R);  // first value-row column of the stage
                const float* z = stage_ptr(st, 0);
                for (int c = first; c < valid; c += R) bias += z[mn32_index(m, c)];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float h[8], l[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int c = 8 * q + j;
                        const float v = c < valid ? z[mn32_index(m, c)] : 0.f;
                        h[j] = tc::tf32_round(v);
                        l[j] = tc::tf32_round(v - h[j]);
                    }
                    tc::tmem_st8(lane_base + dz_column(st) + 8 * q, h);
                    tc::tmem_st8(lane_base + dz_column(st) + 32 + 8 * q, l);
                }
                tc::tmem_wait_st();
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                bool in_order = true;
                const long long start = clock64();
                while (*split_count < G::kSplitWarps * it) {
                    if (*abort || clock64() - start > tcg::kWaitCycles) {
                        *abort = 1;
                        in_order = false;
                        break;
                    }
                }
                if (in_order) {
                    tc::mbar_arrive(split + st);
                    __threadfence_block();  // the arrival before the count that releases the next chunk's
                    atomicAdd(const_cast<int*>(split_count), 1);
                }
            }
            if (!__shfl_sync(0xffffffffu, int(!*abort), 0)) break;
        }
        if (mine_lane) bias_sums[group * 128 + m] = bias;
    } else if (wg_lo_warp<NB>(warp) >= 0) {
        // lo warps: the TF32 lo part of Y_prev of every stage (the raw operand
        // is its hi part; the columns past the end of the data arrive as zeros
        // from the tensor map)
        const int tid = wg_lo_warp<NB>(warp) * 32 + lane;
        for (int it = 0; it < chunks; ++it) {
            const int st = it % kStages;
            if (!warp_wait(full + st, (it / kStages) & 1, abort)) break;
            split_lo_range(reinterpret_cast<const float4*>(stage_ptr(st, 1)), reinterpret_cast<float4*>(stage_ptr(st, 2)),
                           G::kOperand / 16, tid, G::kLoWarps * 32);
            tc::fence_proxy_async();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(split + st);
        }
    } else {
        // drain warps: thread = neuron m (its TMEM lane); every finished segment of
        // either accumulator, in the order the segments end, added into sums[n][m]
        const int quarter = warp & 3, m = quarter * 32 + lane;
        const bool mine_lane = quarter * 32 < NB;  // the same for the whole warp
        const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
        if (mine_lane)
            for (int c = 0; c < NB; ++c) sums[c * NB + m] = 0.f;
        const int total[2] = {wg_segments<G::kSegment>(0, mine[0]), wg_segments<G::kSegment>(1, mine[1])};
        int next[2] = {0, 0};
        bool ok = true;
        while (ok && (next[0] < total[0] || next[1] < total[1])) {
            int w;
            if (next[0] >= total[0]) w = 1;
            else if (next[1] >= total[1]) w = 0;
            else w = wg_segment_end<G::kSegment>(0, next[0], mine[0]) <
                                                  wg_segment_end<G::kSegment>(1, next[1], mine[1]) ? 0 : 1;
            ok = warp_wait(acc_full + w, next[w] & 1, abort);
            if (!ok) break;
            tc::tc_fence_after();
            if (mine_lane) {
                const uint32_t acc = lane_base + (w ? G::kSecondAcc : 0u);
                for (int c0 = 0; c0 < NB; c0 += 16) {
                    float v[16];
                    tc::tmem_read<16>(acc + c0, v);
#pragma unroll
                    for (int j = 0; j < 16; ++j) sums[(c0 + j) * NB + m] += v[j];
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(acc_empty + w);
            ++next[w];
        }
        if (ok && mine_lane)
            for (int c = 0; c < NB; ++c)  // the slices of layers narrower than the slice end early
                if (m_base + m < M && n_base + c < N) out[m_base + m + (size_t)(n_base + c) * M] = sums[c * NB + m];
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kWgTmemColumns);
    }
    // the bias column: both split groups' sums (written before the barrier above)
    if (blockIdx.y == 0 && threadIdx.x < NB && m_base + threadIdx.x < M) {
        float b = 0.f;
        for (int g = 0; g < G::kSplitGroups; ++g) b += bias_sums[g * 128 + threadIdx.x];
        out[(size_t)N * M + m_base + threadIdx.x] = b;
    }
    if (threadIdx.x == 0 && *abort) atomicExch(error, tcg::kErrMma);
}

}  // namespace ws
}  // namespace cpde
