#include "safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <filesystem>
#include <stdexcept>

namespace hyb {
namespace {

// Minimal JSON reader for the safetensors header: an object of objects holding
// strings, integer arrays and (ignored) nested metadata.
struct Json {
    const char* p;
    const char* end;

    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    void expect(char c) {
        ws();
        if (p >= end || *p != c) throw std::runtime_error(std::string("safetensors header: expected '") + c + "'");
        ++p;
    }
    bool peek(char c) {
        ws();
        return p < end && *p == c;
    }
    std::string str() {
        expect('"');
        std::string out;
        while (p < end && *p != '"') {
            if (*p == '\\' && p + 1 < end) {
                ++p;
                out.push_back(*p == 'n' ? '\n' : *p);
            } else {
                out.push_back(*p);
            }
            ++p;
        }
        expect('"');
        return out;
    }
    int64_t integer() {
        ws();
        bool neg = false;
        if (p < end && *p == '-') {
            neg = true;
            ++p;
        }
        int64_t v = 0;
        if (p >= end || *p < '0' || *p > '9') throw std::runtime_error("safetensors header: expected integer");
        while (p < end && *p >= '0' && *p <= '9') v = v * 10 + (*p++ - '0');
        return neg ? -v : v;
    }
    std::vector<int64_t> int_array() {
        std::vector<int64_t> v;
        expect('[');
        if (peek(']')) {
            ++p;
            return v;
        }
        for (;;) {
            v.push_back(integer());
            if (peek(',')) {
                ++p;
                continue;
            }
            expect(']');
            return v;
        }
    }
    void skip_value() {
        ws();
        if (p >= end) throw std::runtime_error("safetensors header: truncated");
        if (*p == '"') {
            str();
        } else if (*p == '{' || *p == '[') {
            const char open = *p, close = open == '{' ? '}' : ']';
            int depth = 0;
            bool in_str = false;
            for (; p < end; ++p) {
                if (in_str) {
                    if (*p == '\\') ++p;
                    else if (*p == '"') in_str = false;
                } else if (*p == '"') {
                    in_str = true;
                } else if (*p == open) {
                    ++depth;
                } else if (*p == close) {
                    if (--depth == 0) {
                        ++p;
                        return;
                    }
                }
            }
        } else {
            while (p < end && *p != ',' && *p != '}' && *p != ']') ++p;
        }
    }
};

}  // namespace

Checkpoint::Checkpoint(const std::string& dir) {
    namespace fs = std::filesystem;
    std::vector<fs::path> shards;
    for (const auto& e : fs::directory_iterator(dir)) {
        if (e.is_regular_file() && e.path().extension() == ".safetensors") shards.push_back(e.path());
    }
    std::sort(shards.begin(), shards.end());
    if (shards.empty()) throw std::runtime_error("no .safetensors shards found in " + dir);
    for (const auto& path : shards) {
        const int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) throw fs::filesystem_error("cannot open shard", path, std::error_code(errno, std::generic_category()));
        struct stat st {};
        if (::fstat(fd, &st) != 0 || st.st_size < 8) {
            ::close(fd);
            throw std::runtime_error("shard too small: " + path.string());
        }
        void* addr = ::mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (addr == MAP_FAILED) throw std::runtime_error("mmap failed: " + path.string());
        maps_.push_back({addr, static_cast<size_t>(st.st_size)});
        const auto* base = static_cast<const uint8_t*>(addr);
        uint64_t hlen = 0;
        std::memcpy(&hlen, base, 8);
        if (8 + hlen > static_cast<uint64_t>(st.st_size)) throw std::runtime_error("bad header length: " + path.string());
        const uint8_t* data = base + 8 + hlen;
        const size_t data_len = static_cast<size_t>(st.st_size) - 8 - hlen;
        Json j{reinterpret_cast<const char*>(base + 8), reinterpret_cast<const char*>(base + 8 + hlen)};
        j.expect('{');
        if (j.peek('}')) continue;
        for (;;) {
            const std::string name = j.str();
            j.expect(':');
            if (name == "__metadata__") {
                j.skip_value();
            } else {
                TensorView tv;
                int64_t lo = -1, hi = -1;
                j.expect('{');
                for (;;) {
                    const std::string key = j.str();
                    j.expect(':');
                    if (key == "dtype") {
                        tv.dtype = j.str();
                    } else if (key == "shape") {
                        tv.shape = j.int_array();
                    } else if (key == "data_offsets") {
                        auto v = j.int_array();
                        if (v.size() != 2) throw std::runtime_error("bad data_offsets for " + name);
                        lo = v[0];
                        hi = v[1];
                    } else {
                        j.skip_value();
                    }
                    if (j.peek(',')) {
                        ++j.p;
                        continue;
                    }
                    j.expect('}');
                    break;
                }
                if (lo < 0 || hi < lo || static_cast<size_t>(hi) > data_len)
                    throw std::runtime_error("tensor data out of range: " + name);
                tv.data = data + lo;
                tv.nbytes = static_cast<size_t>(hi - lo);
                tensors_[name] = tv;
            }
            if (j.peek(',')) {
                ++j.p;
                continue;
            }
            j.expect('}');
            break;
        }
    }
}

Checkpoint::~Checkpoint() {
    for (auto& m : maps_) ::munmap(m.addr, m.len);
}

const TensorView& Checkpoint::get(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) throw std::runtime_error("weight manifest is missing tensor: " + name);
    return it->second;
}

}  // namespace hyb
