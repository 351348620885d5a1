// Weight gradient of one layer for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc: hosts whose own
// allocator already owns the device's memory (a framework's preallocated
// pool leaves nothing for a second allocator, and an allocation that fails in
// the middle of their step is not recoverable for them), and code on a
// latency-bound path that must not take the implicit device synchronisation
// of cudaMalloc and cudaFree. cpde_layer_gradient_static() serves them: it
// runs the split-column weight-gradient kernel with its per-split partial
// sums in a file-scope static device array instead of engine-allocated
// scratch, and touches no allocator at all. The caller passes device inputs
// and the output.
//
// The array holds kStaticScratchFloats floats (16 MiB); every GPU that loads
// this library keeps it until the process exits. All calls on a device share
// it and it keeps the last call's partials: every partial a call reads is
// written by that call first, so nothing needs clearing (the gradient output,
// which the partial sum accumulates into, is cleared by each call), but two
// calls whose kernels overlap on the GPU (different streams, no ordering
// between them) race on the array and may corrupt each other's results.
#include <mutex>

namespace cpde {

constexpr size_t kStaticScratchFloats = size_t(4) << 20;
static __device__ __align__(256) float g_static_gradient_scratch[kStaticScratchFloats];

// Device address of the array, looked up once per device with that device
// current (the host-side symbol is not a device address) by the first call on
// that device. The cached address belongs to the device's primary context: it
// stays valid for the life of the process unless that context is destroyed
// (cudaDeviceReset), after which this entry point must not be called.
static float* g_static_scratch_address[64] = {};
static std::mutex g_static_scratch_mutex;

static float* static_scratch(int device) {
    require(device >= 0 && device < 64, "device index beyond the static scratch table");
    std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
    if (!g_static_scratch_address[device]) {
        void* address = nullptr;
        CPDE_CUDA(cudaGetSymbolAddress(&address, g_static_gradient_scratch));
        g_static_scratch_address[device] = static_cast<float*>(address);
    }
    return g_static_scratch_address[device];
}

}  // namespace cpde

extern "C" int cpde_layer_gradient_static(cpde_engine* h, const float* dz, const float* activations, int32_t outputs,
                                          int32_t inputs, int64_t points, int32_t rows, float* gradient,
                                          void* stream) {
    return guard(h, [&] {
        using namespace cpde;
        require(dz && activations && gradient, "null device pointer");
        require(outputs > 0 && inputs > 0 && points > 0 && rows > 0, "invalid gradient shape");
        require(outputs % 4 == 0 && inputs % 4 == 0, "outputs and inputs must be multiples of 4");
        require((reinterpret_cast<uintptr_t>(dz) | reinterpret_cast<uintptr_t>(activations)) % 16 == 0,
                "dz and activations must be 16-byte aligned");
        const long size = long(outputs) * (inputs + 1);
        require(size <= long(kStaticScratchFloats),
                "outputs*(inputs+1) exceeds the static scratch of " + std::to_string(kStaticScratchFloats) +
                    " floats");
        const long columns = points * rows;
        require(columns <= INT_MAX, "points*rows exceeds the int32 column range");
        float* partials = static_scratch(h->engine->device);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->engine->stream;
        using namespace cpde::fast;
        const int tiles = ((inputs + BM - 1) / BM) * ((outputs + BM - 1) / BM);
        long splits = std::max(1L, std::min<long>((2L * 148 + tiles - 1) / tiles, (columns + 1023) / 1024));
        splits = std::min<long>(splits, long(kStaticScratchFloats) / size);
        long per = ((columns + splits - 1) / splits + BK - 1) / BK * BK;
        splits = (columns + per - 1) / per;
        CPDE_CUDA(cudaMemsetAsync(gradient, 0, size * sizeof(float), s));
        dim3 grid(unsigned(splits), (inputs + BM - 1) / BM, (outputs + BM - 1) / BM);
        k_weight_gradient<<<grid, THREADS, 0, s>>>(outputs, inputs, columns, rows, per, dz, activations, partials);
        CPDE_LAUNCHED();
        k_sum_partials<<<sum_grid(size), 256, 0, s>>>(partials, int(splits),
                                                                                          size, gradient);
        CPDE_LAUNCHED();
    });
}
