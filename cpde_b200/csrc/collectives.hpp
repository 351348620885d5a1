// Point sharding across ranks and the NCCL calls of a sharded epoch.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2), so a single-device
// engine never needs it; inside a process that already loaded NCCL (PyTorch)
// the same library instance is reused. Only the types come from nccl.h.
#pragma once
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>

#include "common.hpp"

namespace cpde {

// Contiguous shard of `total` samples for `rank` of `world`; the remainder is
// spread over the first ranks (total = 10, world = 4: 3, 3, 2, 2).
struct Shard {
    long lo = 0, count = 0;
};
inline Shard shard_range(long total, int rank, int world) {
    const long base = total / world, extra = total % world;
    Shard s;
    s.lo = rank * base + std::min<long>(rank, extra);
    s.count = base + (rank < extra ? 1 : 0);
    return s;
}

// Lexicographic (sample, component) key of a cost's first bad entry, so that
// one integer minimum over ranks picks the same entry a single device would.
// component >= -1, INT_MAX when there is none; sample INT_MAX when none.
__host__ __device__ inline long long bad_entry_key(int sample, int component) {
    return (static_cast<long long>(sample) << 32) + (static_cast<long long>(component) + 2147483648LL);
}
__host__ __device__ inline void bad_entry_unkey(long long key, int& sample, int& component) {
    sample = static_cast<int>(key >> 32);
    component = static_cast<int>((key & 0xFFFFFFFFLL) - 2147483648LL);
}

class Nccl {
   public:
    static Nccl& get() {
        static Nccl instance;
        return instance;
    }
    bool available() const { return handle_ != nullptr; }
    const std::string& load_error() const { return error_; }

    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclCommAbort) comm_abort = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;

    void check(ncclResult_t r, const char* what) const {
        if (r != ncclSuccess)
            throw DeviceError(std::string(what) + " failed: " + (error_string ? error_string(r) : "NCCL error"));
    }

   private:
    Nccl() {
        handle_ = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!handle_) {
            const char* e = dlerror();
            error_ = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown error");
            return;
        }
        bool ok = bind(get_unique_id, "ncclGetUniqueId") && bind(comm_init_rank, "ncclCommInitRank") &&
                  bind(comm_destroy, "ncclCommDestroy") && bind(comm_abort, "ncclCommAbort") &&
                  bind(all_reduce, "ncclAllReduce") && bind(all_gather, "ncclAllGather") &&
                  bind(group_start, "ncclGroupStart") && bind(group_end, "ncclGroupEnd") &&
                  bind(error_string, "ncclGetErrorString");
        if (!ok) {
            error_ = "libnccl.so.2 lacks a required entry point";
            handle_ = nullptr;
        }
    }
    template <class F>
    bool bind(F& f, const char* name) {
        f = reinterpret_cast<F>(dlsym(handle_, name));
        return f != nullptr;
    }
    void* handle_ = nullptr;
    std::string error_;
};

}  // namespace cpde
