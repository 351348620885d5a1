// Shared pieces of the tensor-core layers (kernels_ws.cuh): tile geometry,
// error codes, the wait bound and the TF32 split of a weight matrix.
//
// A layer's GEMM runs on tcgen05 with a 3xTF32 split: each operand is split
// into a TF32 hi part and a TF32 lo part, and every K step issues
// lo*hi + hi*lo + hi*hi into one FP32 accumulator in tensor memory, which
// keeps products to about 2^-22 relative error. The accumulator rows are the
// layer's neurons, so each epilogue thread reads its neuron's R derivative
// columns of a point straight from tensor memory into the register jet code.
//
// Every mbarrier wait is bounded (kWaitCycles); on a timeout the CTA records
// an error code and the host checks it.
#pragma once
#include "generated/jets_static.cuh"
#include "kernels_fast.cuh"
#include "kernels_generic.cuh"
#include "tc.cuh"

namespace cpde {
namespace tcg {

constexpr int BM = 128;                          // neurons per tile = TMEM lanes
constexpr int KS = 32;                           // K per slab: 32 fp32 = one 128-byte row
constexpr long long kWaitCycles = 2000000000LL;  // about one second

// Tile = 128 neurons x PTS whole points (at most kTileColumns MMA columns).
constexpr int kTileColumns = 128;

template <int R>
struct Tiling {
    static constexpr int PTS = (kTileColumns / R) > 0 ? (kTileColumns / R) : 1;
    static constexpr int COLS = PTS * R;
};

enum : int { kErrTma = 1, kErrMma = 2 };

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
