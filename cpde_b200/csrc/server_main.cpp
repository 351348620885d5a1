// cpde_server: drop-in replacement for the reference executable.
//
// Speaks the reference's framed stdin/stdout protocol (frame = u64 length,
// u32 kind, payload; cuda/protocol.hpp:10-51) and its process model: one
// reader thread that handles the out-of-band stop request (op 99) and one
// executor that runs commands in order (cuda/cpde_server.cu:557-576). Every
// command is decoded here and executed through the C ABI of
// include/cpde_b200.h. Replies are kind 0 (ok) or kind 1 (error string); the
// process stays alive after rejected commands.
#include <atomic>
#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <deque>
#include <iostream>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/cpde_b200.h"
#include "wire.hpp"

namespace {

using cpde::Payload;

bool read_frame(Payload& b) {
    uint64_t n;
    if (std::fread(&n, 1, sizeof(n), stdin) != sizeof(n)) return false;
    if (n < 4 || n > uint64_t(4) * 1024 * 1024 * 1024) throw std::runtime_error("invalid frame size");
    b.bytes.resize(n);
    b.pos = 0;
    size_t got = 0;
    while (got < n) {
        size_t k = std::fread(b.bytes.data() + got, 1, n - got, stdin);
        if (!k) throw std::runtime_error("truncated frame");
        got += k;
    }
    return true;
}

std::mutex out_mutex;
void send(uint32_t kind, const void* payload, size_t len) {
    std::lock_guard<std::mutex> lock(out_mutex);
    uint64_t n = 4 + len;
    if (std::fwrite(&n, 1, 8, stdout) != 8 || std::fwrite(&kind, 1, 4, stdout) != 4 ||
        (len && std::fwrite(payload, 1, len, stdout) != len))
        throw std::runtime_error("response pipe closed");
    std::fflush(stdout);
}
void send(uint32_t kind, const Payload& p = Payload()) { send(kind, p.bytes.data(), p.bytes.size()); }

struct Failure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

struct Server {
    cpde_engine* engine = nullptr;

    void check(int status) {
        if (status != CPDE_OK) throw Failure(cpde_last_error(engine));
    }

    static void to_payload(void* ctx, const void* bytes, size_t len) {
        auto* p = static_cast<Payload*>(ctx);
        p->bytes.insert(p->bytes.end(), (const uint8_t*)bytes, (const uint8_t*)bytes + len);
    }
    static void as_string(void* ctx, const void* bytes, size_t len) {
        static_cast<Payload*>(ctx)->put_array((const char*)bytes, len);
    }
    static void event(void*, uint32_t kind, const void* payload, size_t len) { send(kind, payload, len); }

    // Returns false when the reply has already been sent (streaming commands).
    bool command(uint32_t op, Payload& b, Payload& out, std::atomic<int32_t>& stop) {
        switch (op) {
            case 1: {
                b.end();
                check(cpde_hello(engine, to_payload, &out));
                return true;
            }
            case 2: {
                int d = b.get<int32_t>(), h = b.get<int32_t>(), w = b.get<int32_t>(), v = b.get<int32_t>();
                auto rows = b.array<int>();
                auto a = b.array<float>();
                b.end();
                uint64_t id;
                check(cpde_data_create(engine, d, h, w, v, rows.data(), rows.size(), a.data(), a.size(), &id));
                out.put<uint64_t>(id);
                return true;
            }
            case 3: {
                auto ns = b.array<int>(), ls = b.array<int>();
                std::vector<std::vector<float>> initial;
                while (b.more() && initial.size() + 1 < ns.size()) initial.push_back(b.array<float>());
                b.end();
                std::vector<const float*> ptrs;
                std::vector<size_t> counts;
                for (auto& a : initial) {
                    ptrs.push_back(a.data());
                    counts.push_back(a.size());
                }
                uint64_t id;
                if (initial.size() + 1 != ns.size() && !initial.empty())
                    throw Failure("initial weight shape mismatch");
                check(cpde_net_create(engine, ns.data(), ls.data(), int(std::min(ns.size(), ls.size())),
                                      initial.empty() ? nullptr : ptrs.data(),
                                      initial.empty() ? nullptr : counts.data(), &id));
                out.put<uint64_t>(id);
                return true;
            }
            case 4: {
                uint64_t ni = b.get<uint64_t>(), di = b.get<uint64_t>();
                int chunk = b.get<int32_t>();
                b.end();
                uint64_t id;
                check(cpde_net_evaluate(engine, ni, di, chunk, &id));
                out.put<uint64_t>(id);
                return true;
            }
            case 5: {
                uint64_t id = b.get<uint64_t>();
                b.end();
                int32_t d, c, s;
                check(cpde_data_shape(engine, id, &d, &c, &s));
                std::vector<float> a(size_t(d) * c * s);
                check(cpde_data_download(engine, id, a.data(), a.size()));
                out.put_array(a);
                return true;
            }
            case 6: {
                uint64_t id = b.get<uint64_t>();
                auto a = b.array<float>();
                b.end();
                check(cpde_data_replace(engine, id, a.data(), a.size()));
                return true;
            }
            case 7: {
                uint64_t ni = b.get<uint64_t>(), in = b.get<uint64_t>(), tg = b.get<uint64_t>();
                int kind = b.get<int32_t>(), chunk = b.get<int32_t>();
                auto rows = b.array<int>();
                uint64_t id;
                if (kind == 0) {
                    auto tr = b.array<int>();
                    int ws = b.get<int32_t>();
                    auto w = b.array<float>();
                    b.end();
                    check(cpde_cost_matching(engine, ni, in, tg, chunk, rows.data(), rows.size(), tr.data(), tr.size(),
                                             ws, w.data(), w.size(), &id));
                } else if (kind == 1) {
                    int equations = b.get<int32_t>();
                    auto raw = b.array<int>();
                    auto co = b.array<float>(), rhs = b.array<float>(), w = b.array<float>();
                    b.end();
                    check(cpde_cost_polynomial(engine, ni, in, chunk, rows.data(), rows.size(), equations, raw.data(),
                                               raw.size(), co.data(), co.size(), rhs.data(), rhs.size(), w.data(),
                                               w.size(), &id));
                } else {
                    throw Failure("unknown cost kind");
                }
                out.put<uint64_t>(id);
                return true;
            }
            case 8:
            case 15: {
                const int32_t* flag = reinterpret_cast<const int32_t*>(&stop);
                check(cpde_train(engine, op == 15, b.bytes.data() + b.pos, b.bytes.size() - b.pos, event, nullptr,
                                 flag));
                return false;
            }
            case 9: {
                uint64_t id = b.get<uint64_t>();
                b.end();
                check(cpde_net_snapshot(engine, id, to_payload, &out));
                return true;
            }
            case 10: {
                uint64_t id = b.get<uint64_t>();
                check(cpde_net_restore(engine, id, b.bytes.data() + b.pos, b.bytes.size() - b.pos));
                return true;
            }
            case 11: {
                int kind = b.get<int32_t>();
                uint64_t id = b.get<uint64_t>();
                b.end();
                check(cpde_release(engine, kind, id));
                return true;
            }
            case 12: {
                uint64_t ni = b.get<uint64_t>(), in = b.get<uint64_t>();
                int chunk = b.get<int32_t>(), samples = b.get<int32_t>();
                auto raw = b.array<int>();
                auto constants = b.array<double>();
                int fields = b.get<int32_t>();
                auto numeric = b.array<double>(), weights = b.array<double>();
                b.end();
                uint64_t id;
                check(cpde_cost_integral(engine, ni, in, chunk, samples, raw.data(), raw.size(), constants.data(),
                                         constants.size(), fields, numeric.data(), numeric.size(), weights.data(),
                                         weights.size(), &id));
                out.put<uint64_t>(id);
                return true;
            }
            case 13: {
                uint64_t id = b.get<uint64_t>();
                bool compile = b.get<int32_t>() != 0;
                b.end();
                check(cpde_cost_source(engine, id, compile, as_string, as_string, &out));
                return true;
            }
            case 14: {
                check(cpde_graph_evaluate(engine, b.bytes.data() + b.pos, b.bytes.size() - b.pos, to_payload, &out));
                return true;
            }
            case 90: {
                uint64_t ni = b.get<uint64_t>(), ci = b.get<uint64_t>();
                int warm = b.get<int32_t>(), iterations = b.get<int32_t>(), batches = b.get<int32_t>();
                b.end();
                check(cpde_benchmark(engine, ni, ci, warm, iterations, batches, to_payload, &out));
                return true;
            }
            default:
                throw Failure("unknown command");
        }
    }
};

}  // namespace

int main(int argc, char** argv) {
    std::cout.rdbuf(std::cerr.rdbuf());
    int device = 0;
    if (argc == 3 && std::string(argv[1]) == "--device") device = std::stoi(argv[2]);
    std::mutex mutex;
    std::condition_variable ready;
    std::deque<Payload> queue;
    bool eof = false;
    std::atomic<int32_t> stop(0);
    std::atomic<bool> training(false);
    std::string input_error;
    std::thread reader([&] {
        try {
            for (;;) {
                Payload b;
                if (!read_frame(b)) break;
                uint32_t op = b.get<uint32_t>();
                if (op == 99) {
                    if (training.load()) stop.store(1);
                    continue;
                }
                if (op == 8 || op == 15) {
                    stop.store(0);
                    training.store(true);
                }
                bool quit = op == 0;
                b.pos = 0;
                {
                    std::lock_guard<std::mutex> lock(mutex);
                    queue.push_back(std::move(b));
                }
                ready.notify_one();
                if (quit) break;
            }
        } catch (const std::exception& e) {
            input_error = e.what();
        }
        {
            std::lock_guard<std::mutex> lock(mutex);
            eof = true;
        }
        stop.store(1);
        ready.notify_one();
    });
    int status = 0;
    Server server;
    if (cpde_engine_create(device, &server.engine) != CPDE_OK) {
        std::cerr << "cpde_server: " << cpde_last_error(server.engine) << std::endl;
        status = 1;
    }
    try {
        for (;;) {
            Payload b;
            {
                std::unique_lock<std::mutex> lock(mutex);
                ready.wait(lock, [&] { return eof || !queue.empty(); });
                if (queue.empty()) break;
                b = std::move(queue.front());
                queue.pop_front();
            }
            uint32_t op = b.get<uint32_t>();
            if (op == 0) {
                send(0);
                break;
            }
            try {
                if (status) throw Failure("engine unavailable");
                Payload out;
                if (server.command(op, b, out, stop)) send(0, out);
            } catch (const std::exception& e) {
                Payload err;
                err.put_string(e.what());
                send(1, err);
            }
            if (op == 8 || op == 15) training.store(false);
            stop.store(0);
        }
    } catch (const std::exception& e) {
        std::cerr << e.what() << std::endl;
    }
    reader.join();
    cpde_engine_destroy(server.engine);
    return input_error.empty() ? status : 1;
}
