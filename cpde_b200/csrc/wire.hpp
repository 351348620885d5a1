// Little-endian payload reader/writer for the cPDE wire protocol: scalars,
// arrays as u64 count + elements, strings as byte arrays
// (cuda/protocol.hpp:10-51 defines the same contract).
#pragma once
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "common.hpp"

namespace cpde {

struct Payload {
    std::vector<uint8_t> bytes;
    size_t pos = 0;

    Payload() = default;
    Payload(const void* data, size_t len) : bytes((const uint8_t*)data, (const uint8_t*)data + len) {}

    template <class T>
    T get() {
        if (pos + sizeof(T) > bytes.size()) throw RequestError("truncated command");
        T x;
        std::memcpy(&x, bytes.data() + pos, sizeof(T));
        pos += sizeof(T);
        return x;
    }
    template <class T>
    std::vector<T> array() {
        uint64_t n = get<uint64_t>();
        if (n > (bytes.size() - pos) / sizeof(T)) throw RequestError("truncated array");
        std::vector<T> v(n);
        if (n) std::memcpy(v.data(), bytes.data() + pos, n * sizeof(T));
        pos += n * sizeof(T);
        return v;
    }
    std::string string() {
        auto a = array<char>();
        return std::string(a.begin(), a.end());
    }
    void end() const {
        if (pos != bytes.size()) throw RequestError("unexpected command fields");
    }
    bool more() const { return pos < bytes.size(); }

    template <class T>
    Payload& put(T x) {
        const uint8_t* p = reinterpret_cast<const uint8_t*>(&x);
        bytes.insert(bytes.end(), p, p + sizeof(T));
        return *this;
    }
    template <class T>
    Payload& put_array(const T* a, size_t n) {
        put<uint64_t>(n);
        if (n) {
            const uint8_t* p = reinterpret_cast<const uint8_t*>(a);
            bytes.insert(bytes.end(), p, p + n * sizeof(T));
        }
        return *this;
    }
    template <class T>
    Payload& put_array(const std::vector<T>& a) {
        return put_array(a.data(), a.size());
    }
    Payload& put_string(const std::string& s) { return put_array(s.data(), s.size()); }
};

}  // namespace cpde
