// Read-only safetensors access: the file is mmap'd, the JSON header parsed,
// and each tensor exposed as (dtype, shape, pointer into the mapping).
// Format: 8-byte little-endian header length, JSON header, raw data.
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "json.hpp"

namespace hk {

struct TensorView {
    std::string dtype;  // "F32", "BF16", "F16", "I8", ...
    std::vector<int64_t> shape;
    const uint8_t *data = nullptr;
    size_t nbytes = 0;
    int64_t numel() const {
        int64_t n = 1;
        for (auto d : shape) n *= d;
        return n;
    }
};

class SafeTensors {
  public:
    explicit SafeTensors(const std::string &path) : path_(path) {
        fd_ = ::open(path.c_str(), O_RDONLY);
        if (fd_ < 0) throw std::runtime_error("cannot open " + path);
        struct stat st;
        if (fstat(fd_, &st) != 0) throw std::runtime_error("cannot stat " + path);
        size_ = static_cast<size_t>(st.st_size);
        if (size_ < 8) throw std::runtime_error("truncated safetensors file " + path);
        map_ = static_cast<uint8_t *>(mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0));
        if (map_ == MAP_FAILED) throw std::runtime_error("cannot mmap " + path);
        uint64_t hlen = 0;
        std::memcpy(&hlen, map_, 8);
        if (hlen > size_ - 8) throw std::runtime_error("bad safetensors header length in " + path);
        json::Value h = json::parse(std::string(reinterpret_cast<const char *>(map_ + 8), hlen));
        const uint8_t *base = map_ + 8 + hlen;
        const size_t data_size = size_ - 8 - hlen;
        for (auto &kv : h.obj) {
            if (kv.first == "__metadata__") continue;
            const json::Value &info = kv.second;
            const json::Value *dt = info.get("dtype");
            const json::Value *sh = info.get("shape");
            const json::Value *off = info.get("data_offsets");
            if (!dt || !sh || !off || off->arr.size() != 2)
                throw std::runtime_error("bad tensor entry " + kv.first + " in " + path);
            TensorView t;
            t.dtype = dt->str;
            for (auto &d : sh->arr) t.shape.push_back(static_cast<int64_t>(d.num));
            const size_t a = static_cast<size_t>(off->arr[0].num), b = static_cast<size_t>(off->arr[1].num);
            if (b < a || b > data_size) throw std::runtime_error("bad data offsets for " + kv.first);
            t.data = base + a;
            t.nbytes = b - a;
            tensors_[kv.first] = t;
        }
    }
    ~SafeTensors() {
        if (map_ && map_ != MAP_FAILED) munmap(map_, size_);
        if (fd_ >= 0) ::close(fd_);
    }
    SafeTensors(const SafeTensors &) = delete;
    SafeTensors &operator=(const SafeTensors &) = delete;

    const std::map<std::string, TensorView> &tensors() const { return tensors_; }
    const std::string &path() const { return path_; }

  private:
    std::string path_;
    int fd_ = -1;
    size_t size_ = 0;
    uint8_t *map_ = nullptr;
    std::map<std::string, TensorView> tensors_;
};

// Widen a tensor to fp32 (F32, F16, BF16, F64 supported).
inline std::vector<float> to_f32(const TensorView &t) {
    const int64_t n = t.numel();
    std::vector<float> out(static_cast<size_t>(n));
    if (t.dtype == "F32") {
        if (t.nbytes != static_cast<size_t>(n) * 4) throw std::runtime_error("size mismatch");
        std::memcpy(out.data(), t.data, t.nbytes);
    } else if (t.dtype == "BF16") {
        if (t.nbytes != static_cast<size_t>(n) * 2) throw std::runtime_error("size mismatch");
        const uint16_t *p = reinterpret_cast<const uint16_t *>(t.data);
        for (int64_t i = 0; i < n; ++i) {
            uint32_t u = static_cast<uint32_t>(p[i]) << 16;
            std::memcpy(&out[static_cast<size_t>(i)], &u, 4);
        }
    } else if (t.dtype == "F16") {
        if (t.nbytes != static_cast<size_t>(n) * 2) throw std::runtime_error("size mismatch");
        const uint16_t *p = reinterpret_cast<const uint16_t *>(t.data);
        for (int64_t i = 0; i < n; ++i) {
            const uint16_t h = p[i];
            const uint32_t sign = (h & 0x8000u) << 16;
            uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF, u;
            if (exp == 0) {
                if (man == 0) {
                    u = sign;
                } else {  // subnormal
                    exp = 127 - 15 + 1;
                    while (!(man & 0x400)) {
                        man <<= 1;
                        --exp;
                    }
                    man &= 0x3FF;
                    u = sign | (exp << 23) | (man << 13);
                }
            } else if (exp == 31) {
                u = sign | 0x7F800000u | (man << 13);
            } else {
                u = sign | ((exp + 127 - 15) << 23) | (man << 13);
            }
            std::memcpy(&out[static_cast<size_t>(i)], &u, 4);
        }
    } else if (t.dtype == "F64") {
        const double *p = reinterpret_cast<const double *>(t.data);
        for (int64_t i = 0; i < n; ++i) out[static_cast<size_t>(i)] = static_cast<float>(p[i]);
    } else {
        throw std::runtime_error("unsupported tensor dtype " + t.dtype);
    }
    return out;
}

}  // namespace hk
