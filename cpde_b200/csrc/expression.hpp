// Compiled integral costs: the scalar IR of a cost is turned into one
// straight-line CUDA kernel (forward values and a reverse sweep in double per
// sample) and compiled at run time with NVRTC for this device's sm_XXXa
// target. The per-sample semantics follow the reference's generated kernel
// (cuda/expression_program.hpp:31-66): zero adjoints for padded or zero-weight
// samples, loss = weight * root, stop-gradient components, aliased components
// summed in double before the float store, and the "bad" code (-1 for a
// non-finite value, else the last non-finite component index). The kernel
// here also folds the per-block loss reduction in (cuda/cost_graph.cuh:35-43
// is a separate launch in the reference) and reads the engine's interleaved
// output layout.
#pragma once
#include <cuda.h>
#include <nvrtc.h>

#include <algorithm>
#include <iomanip>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "common.hpp"
#include "scalar.hpp"

namespace cpde {

inline std::string fmt_double(double x) {
    std::ostringstream s;
    s << std::setprecision(17) << x;
    std::string t = s.str();
    if (t.find_first_of(".eEn") == std::string::npos) t += ".0";
    return t;
}

// Device prelude of every generated kernel: cost statistics and the
// deterministic block/grid reduction (mirrors kernels_generic.cuh).
static const char* kExpressionPrelude = R"PRELUDE(
struct CostStats { double value; int bad_sample; int bad_component; };
__device__ inline CostStats cs_combine(CostStats a, CostStats b) {
  a.value += b.value;
  if (b.bad_sample < a.bad_sample || (b.bad_sample == a.bad_sample && b.bad_component < a.bad_component)) {
    a.bad_sample = b.bad_sample; a.bad_component = b.bad_component; }
  return a; }
__device__ inline CostStats cs_empty() { CostStats e; e.value = 0.0; e.bad_sample = 0x7fffffff; e.bad_component = 0x7fffffff; return e; }
__device__ inline CostStats cs_warp(CostStats v) {
  for (int o = 16; o; o >>= 1) { CostStats w;
    w.value = __shfl_down_sync(0xffffffffu, v.value, o);
    w.bad_sample = __shfl_down_sync(0xffffffffu, v.bad_sample, o);
    w.bad_component = __shfl_down_sync(0xffffffffu, v.bad_component, o);
    v = cs_combine(v, w); }
  return v; }
__device__ inline void cs_finish(CostStats v, CostStats* partials, unsigned* ticket, CostStats* total) {
  __shared__ CostStats lanes[32]; __shared__ bool last;
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = cs_warp(v); if (lane == 0) lanes[warp] = v; __syncthreads();
  if (warp == 0) { v = lane < (int)(blockDim.x >> 5) ? lanes[lane] : cs_empty(); v = cs_warp(v); }
  if (threadIdx.x == 0) { partials[blockIdx.x] = v; __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1; }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // the last block folds the partials with all its threads (fixed order; one
  // thread alone took about a hundred microseconds over a thousand partials,
  // while every other SM idled)
  CostStats acc = cs_empty();
  for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) { volatile CostStats* q = partials + b; CostStats t;
    t.value = q->value; t.bad_sample = q->bad_sample; t.bad_component = q->bad_component; acc = cs_combine(acc, t); }
  acc = cs_warp(acc); __syncthreads(); if (lane == 0) lanes[warp] = acc; __syncthreads();
  if (warp == 0) { acc = lane < (int)(blockDim.x >> 5) ? lanes[lane] : cs_empty(); acc = cs_warp(acc); }
  if (threadIdx.x == 0) { *total = cs_combine(*total, acc); *ticket = 0; } }
)PRELUDE";

// A power with a constant exponent: integer exponents 0-4 as products, the
// rest through pow(). Double pow() is a long dependent chain, and in the fused
// head the few sampling threads run it while the rest of the CTA waits at a
// barrier; pow(x, 0) is 1 for every x (NaN included), as here, and the
// products differ from pow() by at most an ulp or two of double.
inline std::string power_expr(const std::string& a, double p) {
    if (p == 0) return "1.0";
    if (p == 1) return a;
    if (p == 2) return "(" + a + " * " + a + ")";
    if (p == 3) return "(" + a + " * " + a + " * " + a + ")";
    if (p == 4) return "((" + a + " * " + a + ") * (" + a + " * " + a + "))";
    return "pow(" + a + ", " + fmt_double(p) + ")";
}

// The per-sample program as a device function: the output components `yp`
// (RO of them) of sample `sample` in, its loss added to `local` (times the
// quadrature weight w), dE/dY (times w and the graph multiplier `scale`)
// written to `gp`, and a bad entry recorded for a non-finite value or
// adjoint.
inline std::string expression_sample_function(const std::vector<ScalarNode>& nodes) {
    std::ostringstream s;
    s << "__device__ __forceinline__ void cpde_sample(const float* __restrict__ yp, float* __restrict__ gp, int RO, "
         "const double* __restrict__ fields, int samples, int sample, double w, double scale, int collect, "
         "int gradient, CostStats& local) {\n";
    s << "  if (gradient) for (int i = 0; i < RO; ++i) gp[i] = 0.f;\n";
    s << "  if (w == 0) return;\n";
    s << "  if (gradient && scale == 0 && !collect) return;\n";
    s << "  int bad = -2;\n";
    std::vector<bool> active;
    const int count = int(nodes.size());
    for (int i = 0; i < count; ++i) {
        const auto& n = nodes[i];
        std::string a = "v" + std::to_string(n.a), b = "v" + std::to_string(n.b), e;
        switch (n.op) {
            case kConstant: e = fmt_double(n.parameter); break;
            case kLeaf: e = "(double)yp[" + std::to_string(n.a) + "]"; break;
            case kField: e = "fields[(size_t)" + std::to_string(n.a) + " * samples + sample]"; break;
            case kAdd: e = a + " + " + b; break;
            case kSub: e = a + " - " + b; break;
            case kMul: e = a + " * " + b; break;
            case kDiv: e = "(" + b + " == 0 ? nan(\"\") : " + a + " / " + b + ")"; break;
            case kPower: e = power_expr(a, n.parameter); break;
            case kNeg: e = "-" + a; break;
            case kExp: e = "exp(" + a + ")"; break;
            case kLog: e = "log(" + a + ")"; break;
            case kSqrt: e = "sqrt(" + a + ")"; break;
            case kSin: e = "sin(" + a + ")"; break;
            case kCos: e = "cos(" + a + ")"; break;
            case kTanh: e = "tanh(" + a + ")"; break;
            default: throw RequestError("invalid expression node");
        }
        s << "  const double v" << i << " = " << e << "; if (!isfinite(v" << i << ")) bad = -1;\n";
        bool act = n.op == kLeaf ? n.b == 0 : (n.op <= kField ? false : (active[n.a] || (n.op <= kDiv && active[n.b])));
        active.push_back(act);
    }
    s << "  double loss = 0; if (collect) { loss = w * v" << count - 1 << "; if (!isfinite(loss)) bad = -1; }\n";
    s << "  local.value += loss;\n";
    s << "  if (gradient && scale != 0 && bad == -2) {\n";
    for (int i = 0; i < count; ++i) s << "    double d" << i << " = " << (i + 1 == count ? "1.0" : "0.0") << ";\n";
    for (int i = count - 1; i >= 0; --i) {
        const auto& n = nodes[i];
        if (n.op <= kField || !active[i]) continue;
        std::string a = "v" + std::to_string(n.a), b = "v" + std::to_string(n.b), v = "v" + std::to_string(i);
        std::string da = "0", db = "0";
        switch (n.op) {
            case kAdd: da = db = "1.0"; break;
            case kSub: da = "1.0"; db = "-1.0"; break;
            case kMul: da = b; db = a; break;
            case kDiv: da = "1.0 / " + b; db = "-" + v + " / " + b; break;
            case kPower:
                da = n.parameter == 0 ? "0.0"
                                      : (n.parameter == 1 ? "1.0"
                                                          : fmt_double(n.parameter) + " * " +
                                                                power_expr(a, n.parameter - 1));
                break;
            case kNeg: da = "-1.0"; break;
            case kExp: da = v; break;
            case kLog: da = "1.0 / " + a; break;
            case kSqrt: da = "0.5 / " + v; break;
            case kSin: da = "cos(" + a + ")"; break;
            case kCos: da = "-sin(" + a + ")"; break;
            case kTanh: da = "1.0 - " + v + " * " + v; break;
            default: break;
        }
        s << "    if (d" << i << " != 0) {";
        if (active[n.a]) s << " d" << n.a << " += d" << i << " * (" << da << ");";
        if (n.op <= kDiv && active[n.b]) s << " d" << n.b << " += d" << i << " * (" << db << ");";
        s << " }\n";
    }
    std::map<int, std::vector<int>> components;
    for (int i = 0; i < count; ++i)
        if (nodes[i].op == kLeaf && nodes[i].b == 0) components[nodes[i].a].push_back(i);
    for (const auto& entry : components) {
        s << "    { double t = 0";
        for (int i : entry.second) s << " + d" << i;
        s << "; const float o = (float)(t * w * scale); gp[" << entry.first << "] = o; if (!isfinite(o)) bad = "
          << entry.first << "; }\n";
    }
    s << "  }\n";
    s << "  if (bad != -2) { CostStats e; e.value = 0.0; e.bad_sample = sample; e.bad_component = bad; "
         "local = cs_combine(local, e); }\n";
    s << "}\n";
    return s.str();
}

// The standalone cost kernel: one thread per sample over the engine's
// interleaved output layout (point p's RO components at y + p RO), with the
// block and grid reduction of the loss folded in.
inline std::string expression_source(const std::vector<ScalarNode>& nodes) {
    std::ostringstream s;
    s << kExpressionPrelude << expression_sample_function(nodes);
    s << "extern \"C\" __global__ void __launch_bounds__(256) cpde_integral(const float* __restrict__ y, "
         "float* __restrict__ g, const double* __restrict__ fields, const double* __restrict__ weights, "
         "int RO, int samples, int points, int offset, const double* __restrict__ multiplier, int collect, "
         "int gradient, CostStats* partials, unsigned* ticket, CostStats* total) {\n"
         "  CostStats local = cs_empty();\n"
         "  const double scale = multiplier ? *multiplier : 1.0;\n"
         "  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < points; p += blockDim.x * gridDim.x)\n"
         "    cpde_sample(y + (size_t)p * RO, g + (size_t)p * RO, RO, fields, samples, offset + p, "
         "weights[offset + p], scale, collect, gradient, local);\n"
         "  cs_finish(local, partials, ticket, total);\n"
         "}\n";
    return s.str();
}

// Activation structs of the NVRTC-compiled head: the same arithmetic as
// Sigmoid and Tanh in kernels_generic.cuh (the jet adjoint uses only
// slope_from_value and lead).
static const char* kHeadActivations = R"ACT(
struct Sigmoid {
  __device__ static void value(float z, float& y, float& s) {
    float e = __expf(-fabsf(z)); float big = 1.0f / (1.0f + e); float small = e * big;
    y = z >= 0.f ? big : small; s = big * small; }
  __device__ static float slope_from_value(float y) { return y * (1.0f - y); }
  __device__ static float lead(float y) { return 1.0f - 2.0f * y; }
};
struct Tanh {
  __device__ static void value(float z, float& y, float& s) { y = tanhf(z); s = (1.0f - y) * (1.0f + y); }
  __device__ static float slope_from_value(float y) { return (1.0f - y) * (1.0f + y); }
  __device__ static float lead(float y) { return -2.0f * y; }
};
template <int SID> struct StaticJet;
)ACT";

// The fused expression head (last hidden layer of K = NB neurons, K dividing
// 128, O linear outputs): per point, the output jets Z = W_out Y + b from one
// read of the layer's jets (warp butterflies, then a sum over the lane's
// warps in shared memory), the per-sample program on them, dY = W_out^T
// dE/dZ, the jet adjoint into dE/dZ of the last hidden layer, the output
// layer's weight gradient (a partial per CTA) and the loss reduction. A CTA
// of 128 threads has 128 / NB point lanes; each lane takes PB consecutive
// points per round, whose programs PB threads of the lane evaluate at once,
// so a round's two barriers serve LANES * PB points.
static const char* kHeadKernel = R"HEAD(
extern "C" __global__ void __launch_bounds__(128, 4) cpde_head(
    int K, int points, int offset, int samples, const float* __restrict__ W, const float* __restrict__ Y,
    float* __restrict__ dZ, const double* __restrict__ fields, const double* __restrict__ weights,
    const double* __restrict__ multiplier, int collect, float* __restrict__ partials,
    CostStats* cost_partials, unsigned* ticket, CostStats* total) {
  constexpr int R = HEAD_R, O = HEAD_O, NB = HEAD_NB, PB = HEAD_PB, LANES = 128 / NB, WPL = NB / 32, RO = R * O;
  __shared__ float zsum[LANES][WPL][PB][RO];
  __shared__ float comp[LANES][PB][RO];
  __shared__ float gsh[LANES][PB][RO];
  __shared__ float red[128];
  // The last hidden layer's values of the next round are copied asynchronously
  // into ybuf while this round runs (each thread copies and later reads only
  // its own elements, so its own wait_group orders them; no barrier): one
  // round's loads alone left the head bound on DRAM latency.
  __shared__ float ybuf[2][PB][R][128];
  const int t = threadIdx.x, ml = t % NB, lp = t / NB, wl = ml >> 5, lane = t & 31;
  float w[O], gw[O], gb[O];
#pragma unroll
  for (int o = 0; o < O; ++o) { w[o] = W[o + (size_t)ml * O]; gw[o] = 0.f; gb[o] = 0.f; }
  const float* bias = W + (size_t)O * K;
  const double scale = multiplier ? *multiplier : 1.0;
  CostStats local = cs_empty();
  const long stride = (long)gridDim.x * LANES * PB;
  auto prefetch = [&](long base, int b) {
    const long q0 = base + (long)lp * PB;
#pragma unroll
    for (int j = 0; j < PB; ++j)
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (q0 + j < points) {
          const unsigned dst = (unsigned)__cvta_generic_to_shared(&ybuf[b][j][r][t]);
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst),
                       "l"(Y + ((size_t)(q0 + j) * R + r) * K + ml) : "memory");
        }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  int b = 0;
  prefetch((long)blockIdx.x * LANES * PB, 0);
  for (long base = (long)blockIdx.x * LANES * PB; base < points; base += stride, b ^= 1) {
    const long p0 = base + (long)lp * PB;  // this lane's first point of the round
    prefetch(base + stride, b ^ 1);
    asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    float y[PB][R];
#pragma unroll
    for (int j = 0; j < PB; ++j)
#pragma unroll
      for (int r = 0; r < R; ++r) y[j][r] = p0 + j < points ? ybuf[b][j][r][t] : 0.f;
    // the warp's partial output dot products of its PB points (component
    // c = j RO + i), reduced over its 32 neurons by transposed butterflies: lane
    // l ends with component g 32 + l, 31 shuffles per 32 components instead of
    // 5 per component
    constexpr int PV = PB * RO;
#pragma unroll
    for (int g = 0; g < (PV + 31) / 32; ++g) {
      float v[32];
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const int c = g * 32 + q, i = c % RO;
        v[q] = c < PV ? w[i % O] * y[c / RO][i / O] : 0.f;
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const bool upper = lane & off;
#pragma unroll
        for (int q = 0; q < off; ++q) {
          const float send = upper ? v[q] : v[q + off];
          const float keep = upper ? v[q + off] : v[q];
          v[q] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      const int c = g * 32 + lane;
      if (c < PV) (&zsum[lp][wl][0][0])[c] = v[0];
    }
    __syncthreads();
    if (ml < PB && p0 + ml < points) {
      const int j = ml;
      for (int i = 0; i < RO; ++i) {
        float z = 0.f;
        for (int q = 0; q < WPL; ++q) z += zsum[lp][q][j][i];
        comp[lp][j][i] = z + (i < O ? bias[i] : 0.f);
      }
      const long p = p0 + j;
      cpde_sample(comp[lp][j], gsh[lp][j], RO, fields, samples, offset + (int)p, weights[offset + p], scale, collect,
                  1, local);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < PB; ++j) {
      if (p0 + j >= points) break;
      float dy[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float acc = 0.f;
#pragma unroll
        for (int o = 0; o < O; ++o) {
          const float d = gsh[lp][j][r * O + o];
          acc = fmaf(w[o], d, acc);
          gw[o] = fmaf(d, y[j][r], gw[o]);
        }
        dy[r] = acc;
      }
      if (ml == 0)
#pragma unroll
        for (int o = 0; o < O; ++o) gb[o] += gsh[lp][j][o];
      StaticJet<HEAD_SID>::template adjoint<HEAD_ACT>(y[j], dy);
      float* out = dZ + (size_t)(p0 + j) * R * K + ml;
#pragma unroll
      for (int r = 0; r < R; ++r) out[(size_t)r * K] = dy[r];
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");  // no copy lands after the CTA ends
  float* out = partials + (size_t)blockIdx.x * O * (K + 1);
  for (int o = 0; o < O; ++o) {
    red[t] = gw[o];
    __syncthreads();
    if (lp == 0) { float s = 0.f; for (int l = 0; l < LANES; ++l) s += red[l * NB + ml]; out[o + (size_t)ml * O] = s; }
    __syncthreads();
    red[t] = gb[o];
    __syncthreads();
    if (t == 0) { float s = 0.f; for (int l = 0; l < LANES; ++l) s += red[l * NB]; out[o + (size_t)K * O] = s; }
    __syncthreads();
  }
  cs_finish(local, cost_partials, ticket, total);
}
)HEAD";

// Points per lane and round of the head: up to 4, while PB * R jet values
// stay within about 20 registers, so that four CTAs fit an SM (at 8 points
// per lane the head took 255 registers and ran at 12% of the SM's warps).
inline int head_points_per_lane(int R) { return std::max(1, std::min(4, 20 / R)); }

inline std::string expression_head_source(const std::vector<ScalarNode>& nodes, const char* jet_source, int sid,
                                          bool tanh_act, int R, int O, int K) {
    std::ostringstream s;
    s << kExpressionPrelude << kHeadActivations << jet_source << "\n" << expression_sample_function(nodes);
    s << "#define HEAD_R " << R << "\n#define HEAD_O " << O << "\n#define HEAD_NB " << K << "\n#define HEAD_PB "
      << head_points_per_lane(R) << "\n#define HEAD_SID " << sid << "\n#define HEAD_ACT "
      << (tanh_act ? "Tanh" : "Sigmoid") << "\n";
    s << kHeadKernel;
    return s.str();
}

// Driver-API entry points are fetched through the runtime, so the library has
// no link-time dependency on libcuda (it loads on machines without a driver).
struct DriverApi {
    decltype(&cuModuleLoadData) module_load = nullptr;
    decltype(&cuModuleUnload) module_unload = nullptr;
    decltype(&cuModuleGetFunction) get_function = nullptr;
    decltype(&cuLaunchKernel) launch = nullptr;
    decltype(&cuGetErrorString) error_string = nullptr;
    decltype(&cuTensorMapEncodeTiled) encode_tiled = nullptr;
};

inline DriverApi& driver_api() {
    static DriverApi api = [] {
        DriverApi d;
        auto get = [](const char* name, void** fn) {
            cudaDriverEntryPointQueryResult status;
            if (cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &status) != cudaSuccess ||
                status != cudaDriverEntryPointSuccess)
                throw DeviceError(std::string("CUDA driver entry point unavailable: ") + name);
        };
        get("cuModuleLoadData", (void**)&d.module_load);
        get("cuModuleUnload", (void**)&d.module_unload);
        get("cuModuleGetFunction", (void**)&d.get_function);
        get("cuLaunchKernel", (void**)&d.launch);
        get("cuGetErrorString", (void**)&d.error_string);
        get("cuTensorMapEncodeTiled", (void**)&d.encode_tiled);
        return d;
    }();
    return api;
}

inline void driver_check(CUresult r, const char* what) {
    if (r == CUDA_SUCCESS) return;
    const char* msg = nullptr;
    driver_api().error_string(r, &msg);
    throw DeviceError(std::string(what) + ": " + (msg ? msg : "CUDA driver error"));
}

// A kernel compiled at run time with NVRTC for this device's sm_XXa target.
struct RuntimeKernel {
    std::string code, name, log;
    CUmodule module = nullptr;
    CUfunction kernel = nullptr;

    RuntimeKernel(std::string source, std::string entry) : code(std::move(source)), name(std::move(entry)) {}
    RuntimeKernel(const RuntimeKernel&) = delete;
    ~RuntimeKernel() {
        if (module) driver_api().module_unload(module);
    }

    void compile() {
        if (module) return;
        int device = 0;
        CPDE_CUDA(cudaGetDevice(&device));
        cudaDeviceProp prop;
        CPDE_CUDA(cudaGetDeviceProperties(&prop, device));
        std::string arch = "--gpu-architecture=sm_" + std::to_string(prop.major) + std::to_string(prop.minor) +
                           (prop.major >= 9 ? "a" : "");
        const char* options[] = {"--std=c++17", arch.c_str()};
        nvrtcProgram program;
        nvrtcResult r = nvrtcCreateProgram(&program, code.c_str(), (name + ".cu").c_str(), 0, nullptr, nullptr);
        if (r != NVRTC_SUCCESS) throw DeviceError(nvrtcGetErrorString(r));
        r = nvrtcCompileProgram(program, 2, options);
        size_t size = 0;
        nvrtcGetProgramLogSize(program, &size);
        log.assign(size, '\0');
        if (size) nvrtcGetProgramLog(program, &log[0]);
        while (!log.empty() && log.back() == '\0') log.pop_back();
        if (r != NVRTC_SUCCESS) {
            nvrtcDestroyProgram(&program);
            throw RequestError("expression compile failed: " + log);
        }
        nvrtcGetCUBINSize(program, &size);
        std::vector<char> cubin(size);
        nvrtcGetCUBIN(program, cubin.data());
        nvrtcDestroyProgram(&program);
        driver_check(driver_api().module_load(&module, cubin.data()), "cuModuleLoadData");
        driver_check(driver_api().get_function(&kernel, module, name.c_str()), "cuModuleGetFunction");
    }
};

// An integral cost's program: its IR and the standalone cost kernel.
struct ExpressionProgram : RuntimeKernel {
    std::vector<ScalarNode> nodes;
    explicit ExpressionProgram(std::vector<ScalarNode> ir)
        : RuntimeKernel(expression_source(ir), "cpde_integral"), nodes(std::move(ir)) {}
};

}  // namespace cpde
