// Launch helpers shared by the engine's translation units: per-kernel event
// timing (CPDE_RUN), grid sizing, tensor-map encoders and the dispatch over
// the generated static schemas.
#pragma once
#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "engine.hpp"

namespace cpde {
// ---------------------------------------------------------------------------
// kernel timing

struct KernelTimer {
    struct Mark {
        const char* name;
        cudaEvent_t start, stop;
    };
    std::vector<Mark> marks;
    std::vector<cudaEvent_t> pool;
    cudaEvent_t get() {
        if (!pool.empty()) {
            auto e = pool.back();
            pool.pop_back();
            return e;
        }
        cudaEvent_t e;
        CPDE_CUDA(cudaEventCreate(&e));
        return e;
    }
    struct Totals {
        long launches = 0;
        double ms = 0;
    };
    std::map<std::string, Totals> totals;
    void collect() {
        for (auto& m : marks) {
            CPDE_CUDA(cudaEventSynchronize(m.stop));
            float ms = 0;
            CPDE_CUDA(cudaEventElapsedTime(&ms, m.start, m.stop));
            auto& t = totals[m.name];
            t.launches += 1;
            t.ms += ms;
            pool.push_back(m.start);
            pool.push_back(m.stop);
        }
        marks.clear();
    }
    ~KernelTimer() {
        for (auto& m : marks) {
            cudaEventDestroy(m.start);
            cudaEventDestroy(m.stop);
        }
        for (auto e : pool) cudaEventDestroy(e);
    }
};

#define CPDE_RUN(engine, name, ...)                                           \
    do {                                                                      \
        KernelTimer* t_ = (engine).timer.get();                               \
        cudaEvent_t a_ = nullptr, b_ = nullptr;                               \
        if (t_) {                                                             \
            a_ = t_->get();                                                   \
            b_ = t_->get();                                                   \
            CPDE_CUDA(cudaEventRecord(a_, (engine).stream));                  \
        }                                                                     \
        __VA_ARGS__;                                                          \
        CPDE_LAUNCHED();                                                      \
        if (t_) {                                                             \
            CPDE_CUDA(cudaEventRecord(b_, (engine).stream));                  \
            t_->marks.push_back({name, a_, b_});                              \
        }                                                                     \
    } while (0)

inline int grid_for(long count, int threads = 256, int cap = 148 * 16) {
    long g = (count + threads - 1) / threads;
    return int(std::max(1L, std::min<long>(g, cap)));
}

// ---------------------------------------------------------------------------
// fast tier dispatch

static_assert(kStaticSchemas == 12, "update CPDE_STATIC_CASES after changing the generated schemas");
#define CPDE_STATIC_CASES(X) X(0) X(1) X(2) X(3) X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11)

template <class F>
static void with_schema(int sid, F&& f) {
    switch (sid) {
#define CPDE_CASE(i) \
    case i:          \
        f.template run<i>(); \
        return;
        CPDE_STATIC_CASES(CPDE_CASE)
#undef CPDE_CASE
    }
    throw DeviceError("unknown static schema");
}

template <class K>
static void allow_smem(K kernel, size_t bytes) {
    CPDE_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes)));
}

inline CUtensorMap tensor_map(const float* base, int inner, long rows, int box_rows) {
    CUtensorMap map;
    cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(inner) * sizeof(float)};
    cuuint32_t box[2] = {cuuint32_t(tcg::KS), cuuint32_t(box_rows)};
    cuuint32_t element_strides[2] = {1, 1};
    driver_check(driver_api().encode_tiled(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims,
                                           strides, box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                 "cuTensorMapEncodeTiled");
    return map;
}

// Box of 32 neurons x 32 columns in the 128-byte swizzle with 32-byte atoms
// (MN-major TF32 operands of the weight-gradient kernel).
inline CUtensorMap mn32_map(const float* base, int inner, long rows) {
    CUtensorMap map;
    cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(inner) * sizeof(float)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t element_strides[2] = {1, 1};
    driver_check(driver_api().encode_tiled(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims,
                                           strides, box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                           CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                 "cuTensorMapEncodeTiled");
    return map;
}

// Tier policy for the fast tier's GEMMs. Tier 2 forces tensor cores
// (3xTF32), tier 4 exact-FP32 FFMA. The automatic tiers (0, and 3 for its
// size limit) use tensor cores at derivative orders 4-6 (tolerance 1e-4). At
// orders 0-3 (tolerance 1e-5) they use them only when every hidden layer has
// at most kNarrowTensorWidth neurons, so that every tensor-core GEMM has at
// most 64 inputs and takes the lo-first term order (ws::issue_mmas): over 96
// integral and polynomial cases of orders 2-3 against the float64 oracle
// (widths 32/64, 517 and 3,000 points) the worst 3xTF32 gradient error is
// then 1.1e-6 (5.1e-6 with the interleaved order), and config 3 (2 -> 64^3
// -> 1, 262,144 points) sits 2.5e-6 from the reference's FP32 gradients.
// Wider layers keep FFMA at orders <= 3: with K = 128 a polynomial cost of
// 517 points (2 -> 128^3 -> 1, order 2), where the residual's gradient
// cancels, came to 2.3e-5 from the oracle, while exact FP32 stays inside 1e-5.
constexpr int kNarrowTensorWidth = 64;
inline bool use_tensor_cores(int tier, const Context& ctx, const NetRecord& n) {
    if (tier == 2) return true;
    if (tier != 0 && tier != 3) return false;
    if (ctx.plan.max_order >= 4) return true;
    for (int l = 1; l + 1 < int(n.neurons.size()); ++l)
        if (n.neurons[l] > kNarrowTensorWidth) return false;
    return true;
}

}  // namespace cpde
