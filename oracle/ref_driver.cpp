// TEST INFRASTRUCTURE ONLY - never linked into the cpde_b200 engine.
//
// Driver around the unmodified reference server, compiled from the reference's
// own sources where they lie (see oracle/Makefile). It exists for two reasons:
//   * the reference's published timings use a benchmark-only opcode 90 that is
//     distributed as a patch (docs/benchmarks/fourier-timing.patch:13-35) rather
//     than in the server; this driver provides the same request/reply layout by
//     calling the reference Server's own public members (prepare_costs, pass,
//     inspect_gradients, reductions.download, validate_costs) without editing
//     any reference file;
//   * it runs commands on one thread, so a CPU build needs no extra shims.
// Every other opcode goes to the reference's Server::command unchanged
// (cuda/cpde_server.cu:436-555). Opcode 99 (stop) is accepted and ignored,
// because this driver never trains concurrently with reading.
#define main cpde_reference_server_main
#include "cpde_server.cu"
#undef main
#include <chrono>

namespace {
// Timestamps for the op-90 reply: wall clock always; device events when CUDA.
struct Clock {
#if defined(CPDE_CPU_BACKEND)
    std::chrono::steady_clock::time_point t0, t1;
    void start(cudaStream_t) { t0 = std::chrono::steady_clock::now(); }
    double stop(cudaStream_t) {
        t1 = std::chrono::steady_clock::now();
        return std::chrono::duration<double, std::milli>(t1 - t0).count();
    }
#else
    cudaEvent_t a{}, b{};
    Clock() { checkCudaErrors(cudaEventCreate(&a)); checkCudaErrors(cudaEventCreate(&b)); }
    ~Clock() { cudaEventDestroy(a); cudaEventDestroy(b); }
    void start(cudaStream_t s) { checkCudaErrors(cudaEventRecord(a, s)); }
    double stop(cudaStream_t s) {
        checkCudaErrors(cudaEventRecord(b, s)); checkCudaErrors(cudaEventSynchronize(b));
        float ms = 0; checkCudaErrors(cudaEventElapsedTime(&ms, a, b)); return ms;
    }
#endif
};

// Opcode 90: u64 net, u64 cost, i32 warm, i32 iterations, i32 batches ->
// f64[] wall ms/epoch, f64[] device ms/epoch, f64 loss, f32[] gradient per layer.
void benchmark(Server& server, wire::Buffer& b) {
    uint64_t ni = b.get<uint64_t>(); auto& n = server.net(ni); uint64_t ci = b.get<uint64_t>();
    int warm = b.get<int>(), iterations = b.get<int>(), batches = b.get<int>(); b.end();
    require(warm >= 0 && iterations > 0 && batches > 0, "invalid benchmark controls");
    std::vector<uint64_t> ids{ci}; server.prepare_costs(n, ids, ni);
    auto stream = *n.gpu->str->exec;
    auto step = [&]() {
        n.reductions.begin(1, stream); bool first = true;
        server.pass<true>(n, Server::lookup(server.costs, ci), 0, true, first);
    };
    for (int i = 0; i < warm; ++i) step();
    checkCudaErrors(cudaStreamSynchronize(stream));
    std::vector<double> wall, device;
    Clock clock;
    for (int batch = 0; batch < batches; ++batch) {
        auto begin = std::chrono::steady_clock::now(); clock.start(stream);
        for (int i = 0; i < iterations; ++i) step();
        double elapsed = clock.stop(stream);
        auto done = std::chrono::steady_clock::now();
        wall.push_back(std::chrono::duration<double, std::milli>(done - begin).count() / iterations);
        device.push_back(elapsed / iterations);
    }
    wire::Buffer out; out.array(wall); out.array(device);
    server.inspect_gradients(n); n.reductions.download(1, n.neurons.size() - 1, stream);
    std::vector<double> values(1); server.validate_costs(n, ids, values, false); out.put<double>(values[0]);
    for (layer* l = n.gpu->layers; l->W_plus; l = l->next) {
        auto& w = *l->W_plus; std::vector<float> g(size_t(w.Wh) * (w.Ww + 1));
        checkCudaErrors(cudaMemcpy(g.data(), w.act_grad_W()->mem->vals, g.size() * sizeof(float),
                                   cudaMemcpyDeviceToHost));
        out.array(g);
    }
    wire::send(0, out);
}
}  // namespace

int main(int argc, char** argv) {
    std::cout.rdbuf(std::cerr.rdbuf());
    int device = 0;
    if (argc == 3 && std::string(argv[1]) == "--device") device = std::stoi(argv[2]);
    std::atomic<bool> stop(false);
    try {
        Server server(device);
        for (;;) {
            wire::Buffer b;
            if (!wire::read(b)) break;
            uint32_t op = b.get<uint32_t>();
            if (op == 0) { wire::send(0); break; }
            if (op == 99) continue;
            try {
                if (op == 90) benchmark(server, b);
                else server.command(op, b, stop);
            } catch (const std::exception& e) {
                wire::Buffer err; err.string(e.what()); wire::send(1, err);
            }
            stop.store(false);
        }
    } catch (const std::exception& e) {
        std::cerr << e.what() << std::endl;
        return 1;
    }
    return 0;
}
