// Read-only GGUF (version 2/3) container for Kev packed backbones: string
// metadata and the F32 / Q8_0 / Q4_0 tensors the reference's converter writes
// (crates/huncho-backend/src/qwen_quantized.rs:91-193). Layout: magic "GGUF",
// u32 version, u64 tensor count, u64 metadata count; metadata entries (string
// key, u32 value type, value); tensor infos (string name, u32 n_dims, u64 dims
// innermost first, u32 type, u64 offset); tensor data at the next multiple of
// the alignment (`general.alignment`, default 32). Strings are u64 length +
// bytes. Every read is bounds-checked against the mapped file.
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace hk {

enum : uint32_t { kGgufF32 = 0, kGgufF16 = 1, kGgufQ4_0 = 2, kGgufQ8_0 = 8 };

struct GgufTensor {
    uint32_t type = 0;
    std::vector<int64_t> shape;  // outermost first (rows, cols)
    const uint8_t *data = nullptr;
    size_t nbytes = 0;
};

class GgufFile {
  public:
    explicit GgufFile(const std::string &path) : path_(path) {
        fd_ = ::open(path.c_str(), O_RDONLY);
        if (fd_ < 0) throw std::runtime_error("cannot open " + path);
        struct stat st;
        if (fstat(fd_, &st) != 0) throw std::runtime_error("cannot stat " + path);
        size_ = static_cast<size_t>(st.st_size);
        if (size_ < 24) throw std::runtime_error("truncated GGUF file " + path);
        map_ = static_cast<const uint8_t *>(mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0));
        if (map_ == MAP_FAILED) throw std::runtime_error("cannot mmap " + path);
        parse();
    }
    ~GgufFile() {
        if (map_ && map_ != MAP_FAILED) munmap(const_cast<uint8_t *>(map_), size_);
        if (fd_ >= 0) ::close(fd_);
    }
    GgufFile(const GgufFile &) = delete;
    GgufFile &operator=(const GgufFile &) = delete;

    const std::map<std::string, std::string> &strings() const { return strings_; }
    const std::map<std::string, GgufTensor> &tensors() const { return tensors_; }
    std::string meta(const std::string &k) const {
        auto it = strings_.find(k);
        if (it == strings_.end()) throw std::runtime_error("GGUF metadata `" + k + "` missing in " + path_);
        return it->second;
    }

    // Bytes of a tensor of `shape` and `type`.
    static size_t nbytes_of(uint32_t type, const std::vector<int64_t> &shape) {
        int64_t n = 1;
        for (int64_t d : shape) {
            if (d < 0 || (d > 0 && n > (int64_t(1) << 40) / d)) throw std::runtime_error("GGUF tensor too large");
            n *= d;
        }
        switch (type) {
            case kGgufF32: return static_cast<size_t>(n) * 4;
            case kGgufF16: return static_cast<size_t>(n) * 2;
            case kGgufQ8_0:
            case kGgufQ4_0:
                if (shape.empty() || shape.back() % 32) throw std::runtime_error("GGUF block rows must be 32-aligned");
                return static_cast<size_t>(n / 32) * (type == kGgufQ8_0 ? 34 : 18);
            default: throw std::runtime_error("unsupported GGUF tensor type " + std::to_string(type));
        }
    }

  private:
    size_t pos_ = 0;
    const uint8_t *need(size_t n) {
        if (n > size_ || pos_ > size_ - n) throw std::runtime_error("truncated GGUF file " + path_);
        const uint8_t *p = map_ + pos_;
        pos_ += n;
        return p;
    }
    template <typename T>
    T rd() {
        T v;
        std::memcpy(&v, need(sizeof(T)), sizeof(T));
        return v;
    }
    std::string rstr() {
        const uint64_t n = rd<uint64_t>();
        if (n > size_) throw std::runtime_error("bad GGUF string length in " + path_);
        const uint8_t *p = need(static_cast<size_t>(n));
        return std::string(reinterpret_cast<const char *>(p), static_cast<size_t>(n));
    }
    // Skips (or, for strings and integers, records) one metadata value.
    std::string rvalue(uint32_t vt, int depth = 0) {
        if (depth > 4) throw std::runtime_error("GGUF metadata nested too deeply");
        switch (vt) {
            case 0: case 1: case 7: return std::to_string(static_cast<int>(*need(1)));
            case 2: case 3: return std::to_string(rd<uint16_t>());
            case 4: return std::to_string(rd<uint32_t>());
            case 5: return std::to_string(rd<int32_t>());
            case 6: need(4); return {};
            case 8: return rstr();
            case 9: {
                const uint32_t et = rd<uint32_t>();
                const uint64_t n = rd<uint64_t>();
                if (n > size_) throw std::runtime_error("bad GGUF array length");
                for (uint64_t i = 0; i < n; ++i) rvalue(et, depth + 1);
                return {};
            }
            case 10: return std::to_string(rd<uint64_t>());
            case 11: return std::to_string(rd<int64_t>());
            case 12: need(8); return {};
            default: throw std::runtime_error("unknown GGUF metadata type " + std::to_string(vt));
        }
    }
    void parse() {
        if (std::memcmp(need(4), "GGUF", 4) != 0) throw std::runtime_error("not a GGUF file: " + path_);
        const uint32_t version = rd<uint32_t>();
        if (version != 2 && version != 3) throw std::runtime_error("unsupported GGUF version " + std::to_string(version));
        const uint64_t n_t = rd<uint64_t>(), n_kv = rd<uint64_t>();
        if (n_t > (1u << 20) || n_kv > (1u << 20)) throw std::runtime_error("implausible GGUF counts in " + path_);
        for (uint64_t i = 0; i < n_kv; ++i) {
            std::string k = rstr();
            const uint32_t vt = rd<uint32_t>();
            std::string v = rvalue(vt);
            if (vt == 8 || vt == 4 || vt == 5 || vt == 10 || vt == 11) strings_[k] = v;
        }
        struct Info {
            std::string name;
            uint32_t type;
            std::vector<int64_t> shape;
            uint64_t off;
        };
        std::vector<Info> infos;
        for (uint64_t i = 0; i < n_t; ++i) {
            Info f;
            f.name = rstr();
            const uint32_t nd = rd<uint32_t>();
            if (nd > 4) throw std::runtime_error("GGUF tensor `" + f.name + "` has too many dims");
            std::vector<int64_t> dims(nd);
            for (uint32_t d = 0; d < nd; ++d) dims[d] = static_cast<int64_t>(rd<uint64_t>());
            f.shape.assign(dims.rbegin(), dims.rend());
            f.type = rd<uint32_t>();
            f.off = rd<uint64_t>();
            infos.push_back(std::move(f));
        }
        size_t align = 32;
        auto al = strings_.find("general.alignment");
        if (al != strings_.end()) align = static_cast<size_t>(std::stoull(al->second));
        if (align == 0 || align > 4096) throw std::runtime_error("bad GGUF alignment");
        const size_t base = (pos_ + align - 1) / align * align;
        for (auto &f : infos) {
            GgufTensor t;
            t.type = f.type;
            t.shape = f.shape;
            t.nbytes = nbytes_of(f.type, f.shape);
            if (f.off > size_ || base > size_ - f.off || t.nbytes > size_ - base - f.off)
                throw std::runtime_error("GGUF tensor `" + f.name + "` exceeds the file");
            t.data = map_ + base + f.off;
            if (tensors_.count(f.name)) throw std::runtime_error("duplicate GGUF tensor `" + f.name + "`");
            tensors_[f.name] = t;
        }
    }

    std::string path_;
    int fd_ = -1;
    size_t size_ = 0;
    const uint8_t *map_ = nullptr;
    std::map<std::string, std::string> strings_;
    std::map<std::string, GgufTensor> tensors_;
};

}  // namespace hk
